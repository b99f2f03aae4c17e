// Per-device runtime of the B200 library (see runtime.hpp).
#include "runtime.hpp"

#include <cstring>
#include <map>
#include <memory>
#include <string>

#include "kq_b200.h"

namespace kqb {

void diag_set(kq_diagnostic *d, kq_status s, const char *fmt, ...) {
    if (d == nullptr) return;
    d->status = s;
    d->message[0] = '\0';
    if (fmt == nullptr) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(d->message, sizeof(d->message), fmt, ap);
    va_end(ap);
    d->message[sizeof(d->message) - 1] = '\0';
}

kq_status cuda_fail(kq_diagnostic *d, cudaError_t e, const char *what) {
    kq_status s = (e == cudaErrorMemoryAllocation) ? KQ_STATUS_OUT_OF_MEMORY
                                                   : KQ_STATUS_INVALID_ARGUMENT;
    diag_set(d, s, "%s: CUDA error %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return s;
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (a != 0 && b > UINT64_MAX / a) return false;
    *out = a * b;
    return true;
}

bool add_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (UINT64_MAX - a < b) return false;
    *out = a + b;
    return true;
}

bool ranges_overlap(const void *a, uint64_t an, const void *b, uint64_t bn) {
    if (a == nullptr || b == nullptr || an == 0 || bn == 0) return false;
    uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    if (x > UINTPTR_MAX - an || y > UINTPTR_MAX - bn) return true;
    return x < y + bn && y < x + an;
}

cudaError_t copy_sync(void *dst, const void *src, size_t bytes, cudaMemcpyKind kind, cudaStream_t stream) {
    if (bytes == 0) return cudaSuccess;
    cudaError_t e = cudaMemcpyAsync(dst, src, bytes, kind, stream);
    return e != cudaSuccess ? e : cudaStreamSynchronize(stream);
}

bool is_device_pointer(const void *p) {
    if (p == nullptr) return false;
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, p);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

namespace {
std::mutex g_ctx_mu;
std::map<int, std::unique_ptr<DeviceContext>> g_ctx;
thread_local int g_device = -1;
}  // namespace

int current_device() {
    if (g_device < 0) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess) {
            cudaGetLastError();
            dev = 0;
        }
        g_device = dev;
    }
    return g_device;
}

void set_current_device(int device) { g_device = device; }

DeviceContext *context_for(int device) {
    std::lock_guard<std::mutex> lk(g_ctx_mu);
    auto it = g_ctx.find(device);
    if (it != g_ctx.end()) return it->second.get();
    auto c = std::make_unique<DeviceContext>();
    c->device = device;
    if (cudaSetDevice(device) != cudaSuccess) return nullptr;
    if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) return nullptr;
    c->stream = c->own_stream;
    if (cudaMalloc(&c->err_word, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
    if (cudaMallocHost(&c->err_host, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
    if (cudaMemset(c->err_word, 0, sizeof(unsigned long long)) != cudaSuccess) return nullptr;
    if (cudaDeviceSynchronize() != cudaSuccess) return nullptr;
    DeviceContext *raw = c.get();
    g_ctx.emplace(device, std::move(c));
    return raw;
}

kq_status context(DeviceContext **out, kq_diagnostic *d) {
    int dev = current_device();
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0) {
        cudaGetLastError();
        diag_set(d, KQ_STATUS_UNSUPPORTED_MODEL,
                 "no CUDA device available: the B200 operators have no CPU fallback (%s)",
                 cudaGetErrorString(e));
        return KQ_STATUS_UNSUPPORTED_MODEL;
    }
    DeviceContext *c = context_for(dev);
    if (c == nullptr) {
        cudaError_t le = cudaGetLastError();
        return cuda_fail(d, le == cudaSuccess ? cudaErrorInitializationError : le,
                         "device context initialisation");
    }
    KQB_CUDA(cudaSetDevice(dev), d, "cudaSetDevice");
    *out = c;
    return KQ_STATUS_OK;
}

ErrorWord DeviceContext::begin_call() {
    ErrorWord w;
    w.word = err_word;
    w.call_id = next_call++;
    if (next_call == 0) next_call = 1;
    return w;
}

kq_status DeviceContext::workspace(size_t bytes, void **out, kq_diagnostic *d) {
    if (bytes > arena_bytes) {
        KQB_CUDA(cudaStreamSynchronize(stream), d, "workspace growth sync");
        if (arena) cudaFree(arena);
        arena = nullptr;
        arena_bytes = 0;
        size_t want = bytes + bytes / 4 + (1u << 20);
        KQB_CUDA(cudaMalloc(&arena, want), d, "workspace allocation");
        arena_bytes = want;
    }
    *out = arena;
    return KQ_STATUS_OK;
}

static const char *error_text(uint32_t code) {
    switch (code & 0xFFu) {
    case kErrNonFinite: return "a non-finite input, state or intermediate value";
    case kErrDecay: return "GDN log decay must be finite and non-positive";
    case kErrSelection: return "QSA selected-token count is invalid";
    case kErrTimeout: return "a tensor-core pipeline wait that timed out";
    case kErrRange: return "a projection input is beyond the tensor-core range (|x| >= 2^18)";
    default: return "device error";
    }
}

kq_status DeviceContext::synchronize(kq_diagnostic *d) {
    cudaError_t e = cudaStreamSynchronize(stream);
    if (e != cudaSuccess) {
        for (Rollbackable *r : dirty) r->on_error(0);
        dirty.clear();
        return cuda_fail(d, e, "stream synchronize");
    }
    KQB_CUDA(cudaMemcpy(err_host, err_word, sizeof(unsigned long long), cudaMemcpyDeviceToHost),
             d, "error word read");
    unsigned long long word = *err_host;
    if (word != 0ull) {
        uint32_t failing = (uint32_t)(word & 0xffffffffull);
        uint32_t code = (uint32_t)(word >> 32);
        for (Rollbackable *r : dirty) r->on_error(failing);
        dirty.clear();
        KQB_CUDA(cudaMemsetAsync(err_word, 0, sizeof(unsigned long long), stream), d, "error word reset");
        kq_status s = code == kErrSelection ? KQ_STATUS_INVALID_QSA_STATE : KQ_STATUS_NUMERIC_DOMAIN;
        diag_set(d, s, "device reported %s (code 0x%x, call %u); state rolled back", error_text(code), code,
                 failing);
        return s;
    }
    for (Rollbackable *r : dirty) r->on_success();
    dirty.clear();
    return KQ_STATUS_OK;
}

kq_status DeviceContext::staging(size_t bytes, void **out, kq_diagnostic *d) {
    if (bytes > stage_bytes) {
        KQB_CUDA(cudaStreamSynchronize(stream), d, "staging growth sync");
        if (stage_arena) cudaFree(stage_arena);
        stage_arena = nullptr;
        stage_bytes = 0;
        const size_t want = bytes + bytes / 4 + (1u << 20);
        KQB_CUDA(cudaMalloc(&stage_arena, want), d, "staging allocation");
        stage_bytes = want;
    }
    *out = stage_arena;
    return KQ_STATUS_OK;
}

uint64_t hash_bytes(const void *p, size_t bytes) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    uint64_t h = 0x243F6A8885A308D3ull ^ bytes;
    size_t i = 0;
    for (; i + 8 <= bytes; i += 8) {
        uint64_t w;
        std::memcpy(&w, b + i, 8);
        h = (h ^ w) * 0x9E3779B97F4A7C15ull;
        h ^= h >> 29;
    }
    for (; i < bytes; ++i) h = (h ^ b[i]) * 0x100000001B3ull;
    return h ^ (h >> 32);
}

kq_status DeviceContext::upload_cached(const float *host, uint64_t count, const float **out, kq_diagnostic *d) {
    const size_t bytes = count * sizeof(float);
    const uint64_t h = hash_bytes(host, bytes);
    ++upload_clock;
    for (auto &u : uploads) {
        if (u.host == host && u.count == count) {
            if (u.hash != h) {
                // same array, new contents: refresh the device copy in place
                KQB_CUDA(copy_sync(u.dev, host, bytes, cudaMemcpyHostToDevice, stream), d, "weight upload");
                u.hash = h;
            }
            u.last_use = upload_clock;
            *out = u.dev;
            return KQ_STATUS_OK;
        }
    }
    // make room: least recently used arrays leave first
    while (!uploads.empty() && upload_bytes + bytes > kUploadCacheBytes) {
        size_t oldest = 0;
        for (size_t i = 1; i < uploads.size(); ++i)
            if (uploads[i].last_use < uploads[oldest].last_use) oldest = i;
        KQB_CUDA(cudaStreamSynchronize(stream), d, "upload cache eviction sync");
        cudaFree(uploads[oldest].dev);
        upload_bytes -= uploads[oldest].count * sizeof(float);
        uploads.erase(uploads.begin() + (std::ptrdiff_t)oldest);
    }
    CachedUpload u;
    u.host = host;
    u.count = count;
    u.hash = h;
    u.last_use = upload_clock;
    KQB_CUDA(cudaMalloc(&u.dev, bytes), d, "weight upload allocation");
    const cudaError_t e = copy_sync(u.dev, host, bytes, cudaMemcpyHostToDevice, stream);
    if (e != cudaSuccess) {
        cudaFree(u.dev);
        return cuda_fail(d, e, "weight upload");
    }
    uploads.push_back(u);
    upload_bytes += bytes;
    *out = u.dev;
    return KQ_STATUS_OK;
}

// ---------------------------------------------------------------- profiler
namespace {
struct TimerState {
    std::mutex mu;
    std::string name;     // kernel family being timed ("" = off)
    std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
    std::vector<cudaEvent_t> pool;
    double total_ms = 0.0;
    uint64_t count = 0;
};
TimerState g_timer;

cudaEvent_t timer_event() {
    if (!g_timer.pool.empty()) {
        cudaEvent_t e = g_timer.pool.back();
        g_timer.pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

void timer_drain(bool wait) {
    size_t keep = 0;
    for (size_t i = 0; i < g_timer.pending.size(); ++i) {
        auto pr = g_timer.pending[i];
        if (wait) cudaEventSynchronize(pr.second);
        if (cudaEventQuery(pr.second) == cudaSuccess) {
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, pr.first, pr.second);
            g_timer.total_ms += ms;
            g_timer.count += 1;
            g_timer.pool.push_back(pr.first);
            g_timer.pool.push_back(pr.second);
        } else {
            cudaGetLastError();
            g_timer.pending[keep++] = pr;
        }
    }
    g_timer.pending.resize(keep);
}
thread_local cudaEvent_t t_start = nullptr;
}  // namespace

KernelTimer::KernelTimer(const char *name, cudaStream_t s) : slot(0), stream(s) {
    std::lock_guard<std::mutex> lk(g_timer.mu);
    if (g_timer.name.empty() || g_timer.name != name) return;
    slot = 1;
    t_start = timer_event();
    cudaEventRecord(t_start, stream);
}

KernelTimer::~KernelTimer() {
    if (!slot) return;
    std::lock_guard<std::mutex> lk(g_timer.mu);
    cudaEvent_t end = timer_event();
    cudaEventRecord(end, stream);
    g_timer.pending.push_back({t_start, end});
    if (g_timer.pending.size() > 4096) timer_drain(false);
}

}  // namespace kqb

using namespace kqb;

extern "C" {

kq_status kq_b200_set_device(int device, kq_diagnostic *diagnostic) {
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
        cudaGetLastError();
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "device index is not available");
    }
    set_current_device(device);
    KQB_CUDA(cudaSetDevice(device), diagnostic, "cudaSetDevice");
    if (diagnostic) { diagnostic->status = KQ_STATUS_OK; diagnostic->message[0] = '\0'; }
    return KQ_STATUS_OK;
}

kq_status kq_b200_set_stream(void *cuda_stream, kq_diagnostic *diagnostic) {
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "stream switch sync");
    c->stream = cuda_stream ? static_cast<cudaStream_t>(cuda_stream) : c->own_stream;
    return KQ_STATUS_OK;
}

void *kq_b200_get_stream(void) {
    DeviceContext *c;
    if (context(&c, nullptr) != KQ_STATUS_OK) return nullptr;
    return c->stream;
}

kq_status kq_b200_synchronize(kq_diagnostic *diagnostic) {
    if (diagnostic) { diagnostic->status = KQ_STATUS_OK; diagnostic->message[0] = '\0'; }
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    return c->synchronize(diagnostic);
}

uint64_t kq_b200_kernel_launch_count(void) { return launches_total(); }

void kq_b200_profile_kernel(const char *kernel_family) {
    std::lock_guard<std::mutex> lk(g_timer.mu);
    timer_drain(true);
    g_timer.name = kernel_family ? kernel_family : "";
    g_timer.total_ms = 0.0;
    g_timer.count = 0;
}

void kq_b200_profile_read(uint64_t *launches, double *total_ms) {
    std::lock_guard<std::mutex> lk(g_timer.mu);
    timer_drain(true);
    if (launches) *launches = g_timer.count;
    if (total_ms) *total_ms = g_timer.total_ms;
}

}  // extern "C"
