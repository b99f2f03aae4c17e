// Allocation-free batched linear: kq_b200_provider_linear_batch_f32_static.
//
// Some callers cannot call cudaMalloc: a serving loop that has handed every
// free byte of HBM to its KV cache and runs with a fixed memory budget, a
// host framework whose own caching allocator owns the device memory and
// forbids side allocations, or a latency-bound loop where cudaMalloc /
// cudaFree would synchronise the device and stall the other streams.  The
// allocating entry point (kq_b200_provider_linear_batch_f32) grows a
// per-device work-space arena on first use; this one takes its scratch from
// a fixed array compiled into the library instead.
//
// Scratch: one file-scope __device__ array of kStaticScratchBytes (4 MiB),
// [error word | pad to 256 B | activation tiles of the tensor-core GEMM].
// Every GPU that loads the library holds it until the process exits.  The
// activation tiles of a call need ceil(batch/64) * ceil(columns/64) * 16 KiB
// (batches above 8); larger calls are rejected with KQ_STATUS_LIMIT_EXCEEDED.
// Every call on a device shares the array and it keeps the last call's
// contents: the error word is cleared at the start of each call, the tiles
// are fully rewritten before they are read.  Calls whose kernels overlap on
// the GPU (different streams, or several host threads) race on it.
//
// The device address of the array is looked up once per device, with that
// device current, when a provider is created on it (kq_b200_provider_create
// calls static_scratch_prepare).  The lookup is what makes the driver load
// the array, so it happens at provider creation, before the host commits the
// rest of HBM, and not on a later call: under lazy module loading the first
// use of this file's code would otherwise allocate the 4 MiB then.
//
// The limit applies to the tensor-core path only (batches above 8 on a
// weight type the tensor-core GEMM covers); the warp GEMV and the CUDA-core
// tiles use no scratch.
#include "kernels.hpp"
#include "provider.hpp"
#include "runtime.hpp"

#include <cstdio>
#include <mutex>

#include "kq_b200.h"

namespace kqb {
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;
constexpr size_t kErrorBytes = 256;   // error word, padded to keep the tiles aligned
constexpr int kMaxStaticDevices = 64;

static __device__ __align__(256) uint8_t g_linear_scratch[kStaticScratchBytes];

std::mutex g_scratch_mu;
uint8_t *g_scratch_addr[kMaxStaticDevices];   // device address of g_linear_scratch, per device

}  // namespace

// Device address of the scratch array on the current device `device`.
kq_status static_scratch(int device, uint8_t **out, kq_diagnostic *d) {
    if (device < 0 || device >= kMaxStaticDevices)
        return fail(d, KQ_STATUS_LIMIT_EXCEEDED, "device index beyond the static scratch table");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (g_scratch_addr[device] == nullptr) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_linear_scratch);
        if (e != cudaSuccess) return cuda_fail(d, e, "cudaGetSymbolAddress(static scratch)");
        g_scratch_addr[device] = static_cast<uint8_t *>(p);
    }
    *out = g_scratch_addr[device];
    return KQ_STATUS_OK;
}

kq_status static_scratch_prepare(int device, kq_diagnostic *d) {
    uint8_t *p = nullptr;
    return static_scratch(device, &p, d);
}

namespace {

// Runs on `device`, then restores the caller's current device.
struct DeviceScope {
    int previous = -1;
    bool active = false;
    cudaError_t enter(int device) {
        cudaError_t e = cudaGetDevice(&previous);
        if (e != cudaSuccess) return e;
        e = cudaSetDevice(device);
        active = e == cudaSuccess;
        return e;
    }
    ~DeviceScope() {
        if (active && previous >= 0) cudaSetDevice(previous);
    }
};

}  // namespace
}  // namespace kqb

using namespace kqb;

kq_status kq_b200_provider_linear_batch_f32_static(kq_weight_provider *provider,
                                                   const kq_semantic_tensor *semantic, uint64_t rows,
                                                   uint64_t columns, const float *x, uint32_t batch, float *y,
                                                   void *cuda_stream, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    ProviderTensor *t = provider_lookup(provider, semantic);
    if (t == nullptr || x == nullptr || y == nullptr || batch == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, semantic and buffers are required");
    if (t->is_vector) return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH, "semantic is not a matrix");
    if (t->parts[0] != nullptr || !t->col_heads.empty())
        return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH,
                    "the allocation-free linear takes whole tensors with canonical columns");
    if (rows != t->m.rows || columns != t->m.cols)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "linear shape does not match the semantic");
    if (!is_device_pointer(x) || !is_device_pointer(y))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "batched linear takes device buffers");
    if (ranges_overlap(x, (uint64_t)batch * columns * 4, y, (uint64_t)batch * rows * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "linear input and output overlap");
    const bool umma_path = batch > 8 && !force_simt_projection() && umma_supported(t->m);
    const size_t tiles = umma_path ? umma_xtile_bytes(batch, (uint32_t)columns, /*allow_wide=*/false) : 0;
    if (tiles > kStaticScratchBytes - kErrorBytes) {
        char msg[160];
        snprintf(msg, sizeof msg, "batch %u x %llu columns needs %zu bytes of activation tiles; the static scratch "
                 "holds %zu", batch, (unsigned long long)columns, tiles, kStaticScratchBytes - kErrorBytes);
        return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, msg);
    }
    DeviceScope scope;
    KQB_CUDA(scope.enter(provider->device), diagnostic, "cudaSetDevice");
    uint8_t *scratch = nullptr;
    kq_status st = static_scratch(provider->device, &scratch, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
    unsigned long long *err_word = reinterpret_cast<unsigned long long *>(scratch);
    KQB_CUDA(cudaMemsetAsync(err_word, 0, sizeof(unsigned long long), stream), diagnostic, "error word clear");
    const ErrorWord err{err_word, 1u};
    launch_check_finite(x, (uint64_t)batch * columns, err, stream);
    ProjSegments segs{};
    segs.count = 1;
    segs.m[0] = t->m;
    const bool tensor_cores = umma_path &&
                              launch_projection_umma(segs, x, (uint32_t)columns, y, (uint32_t)rows, batch,
                                                     scratch + kErrorBytes, kStaticScratchBytes - kErrorBytes,
                                                     err, stream, /*cache_maps=*/false, /*allow_wide=*/false);
    if (!tensor_cores)   // warp GEMV / SIMT tiles: no scratch
        launch_projection(segs, x, (uint32_t)columns, y, (uint32_t)rows, batch, err, stream, nullptr, 0);
    KQB_CUDA(cudaGetLastError(), diagnostic, "linear launch");
    // the call completes before it returns, so it can report its own errors
    unsigned long long word = 0;
    KQB_CUDA(cudaMemcpyAsync(&word, err_word, sizeof word, cudaMemcpyDeviceToHost, stream), diagnostic,
             "error word read");
    KQB_CUDA(cudaStreamSynchronize(stream), diagnostic, "linear synchronize");
    if (word != 0ull) {
        const uint32_t code = (uint32_t)(word >> 32);
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN,
                    code == kErrNonFinite ? "device reported a non-finite input or result"
                                          : "device reported an error in the tensor-core projection");
    }
    provider->metrics.linear_requests += 1;
    return KQ_STATUS_OK;
}
