// Host-side runtime shared by the C-ABI translation units: per-device
// context (stream, device error word, workspace arena), diagnostics, CUDA
// error mapping and the roll-back bookkeeping of asynchronous calls.
#pragma once

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <functional>
#include <mutex>
#include <unordered_set>
#include <vector>

#include <cuda_runtime.h>

#include "kernels.hpp"
#include "kq_status.h"

namespace kqb {

void diag_set(kq_diagnostic *diagnostic, kq_status status, const char *fmt, ...);
inline kq_status fail(kq_diagnostic *d, kq_status s, const char *msg) {
    diag_set(d, s, "%s", msg);
    return s;
}

// Maps a CUDA runtime error onto the ABI's status codes.
kq_status cuda_fail(kq_diagnostic *d, cudaError_t e, const char *what);

#define KQB_CUDA(call, diag, what)                                   \
    do {                                                             \
        cudaError_t kqb_e_ = (call);                                 \
        if (kqb_e_ != cudaSuccess) return ::kqb::cuda_fail((diag), kqb_e_, (what)); \
    } while (0)

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out);
bool add_ok(uint64_t a, uint64_t b, uint64_t *out);
bool ranges_overlap(const void *a, uint64_t a_bytes, const void *b, uint64_t b_bytes);

// True when `p` is device memory (or managed memory) of any device.
bool is_device_pointer(const void *p);

// A copy ordered on `stream` (the library's streams do not synchronise with
// the legacy default stream), complete when it returns.
cudaError_t copy_sync(void *dst, const void *src, size_t bytes, cudaMemcpyKind kind, cudaStream_t stream);

// An object whose device-resident value can be rolled back when an
// asynchronous call fails (GDN and QSA states).
struct Rollbackable {
    virtual ~Rollbackable() = default;
    // record that call `id` advanced this object (called at enqueue time)
    virtual void on_step(uint32_t id) = 0;
    // restore the value after the last successful call (< failing id)
    virtual void on_error(uint32_t failing_id) = 0;
    // all calls since the previous sync succeeded
    virtual void on_success() = 0;
};

// A host F32 array uploaded by a synchronous entry point and kept on the
// device for later calls with the same array (same address, length and
// contents, checked by a hash of the bytes on every call).
struct CachedUpload {
    const float *host = nullptr;
    uint64_t count = 0;
    uint64_t hash = 0;
    float *dev = nullptr;
    uint64_t last_use = 0;
};

struct DeviceContext {
    int device = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    unsigned long long *err_word = nullptr;   // device
    unsigned long long *err_host = nullptr;   // pinned
    uint32_t next_call = 1;
    void *arena = nullptr;
    size_t arena_bytes = 0;
    void *stage_arena = nullptr;
    size_t stage_bytes = 0;
    std::vector<CachedUpload> uploads;
    size_t upload_bytes = 0;
    uint64_t upload_clock = 0;
    std::recursive_mutex mu;
    std::unordered_set<Rollbackable *> dirty;

    ErrorWord begin_call();
    // grow-only device workspace (synchronises when it has to grow)
    kq_status workspace(size_t bytes, void **out, kq_diagnostic *d);
    // grow-only device staging for the synchronous entry points' host inputs
    // and outputs, separate from the operators' workspace (synchronises when
    // it has to grow; a call of a size seen before allocates nothing)
    kq_status staging(size_t bytes, void **out, kq_diagnostic *d);
    // device copy of the host F32 array [count], uploaded only when the
    // array is new or its contents changed since the last call; the cache
    // keeps up to kUploadCacheBytes, least recently used first out
    kq_status upload_cached(const float *host, uint64_t count, const float **out, kq_diagnostic *d);
    // waits for the stream and resolves errors of the calls since the last
    // synchronize (rolling back dirty objects on failure)
    kq_status synchronize(kq_diagnostic *d);
};

// Context of the current device (creating it on first use).
kq_status context(DeviceContext **out, kq_diagnostic *d);
DeviceContext *context_for(int device);
int current_device();
void set_current_device(int device);

// Bump allocator over a workspace region (256-byte aligned slices).
struct Carve {
    char *base;
    size_t used = 0;
    explicit Carve(void *p) : base(static_cast<char *>(p)) {}
    template <typename T>
    T *take(size_t count) {
        size_t bytes = (count * sizeof(T) + 255) & ~size_t(255);
        T *p = reinterpret_cast<T *>(base + used);
        used += bytes;
        return p;
    }
    static size_t round(size_t bytes) { return (bytes + 255) & ~size_t(255); }
};

// Bytes of uploaded F32 weight arrays a device context keeps for the
// synchronous F32 entry points.
constexpr size_t kUploadCacheBytes = size_t(8) << 30;

// 64-bit hash of a byte range (multiply-xorshift over 8-byte words).
uint64_t hash_bytes(const void *p, size_t bytes);

}  // namespace kqb
