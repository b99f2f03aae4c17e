// Gated residual of the decoder layer: the read that mixes B residual
// branches into the mixer's (or the MoE's) input, and the write that adds
// the block's output back into every branch with its own gate.
//
// Replaces kq_layer_gr_read_common and kq_layer_gr_write_f32
// (src/kq_layer_qwen38.c:37-209 of Kestrel-Q), which run one token at a
// time; here every step runs over all T tokens of a call:
//
//   norm     one CTA per (token, branch): (1 + w) RMSNorm of the branch
//   down     [rank x W] and inject [B x W] projections of the normalised
//            branches in one projection launch (kernels_proj.cu)
//   gate     rank = silu(down / B), write gate = 2 sigmoid(inject / B)
//   up       [W x rank] projection of the rank activations
//   mix      read gate = sigmoid(up), mixed = sum_b gate * normalised / B
//   write    out[b] = branch[b] + block * write_gate[b]
//
// The reference's products and sums of the per-token steps are kept in its
// order (sums over the B branches sequential, each product and sum rounded
// separately); the norm's sum of squares and the projections' dot products
// are parallel reductions (tolerance-level differences).
#include "kernels.hpp"

#include <cmath>

namespace kqb {

namespace {

constexpr int kGrThreads = 256;

__device__ __forceinline__ bool gr_err_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}

__device__ __forceinline__ void gr_raise(const ErrorWord &e, uint32_t code) {
    atomicCAS(e.word, 0ull, ((unsigned long long)code << 32) | e.call_id);
}

// kq_sigmoid_scalar (src/kq_numeric.c:628-638): the branch-stable form.
__device__ __forceinline__ float gr_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

}  // namespace

// One CTA per (token, branch): kq_f32_rms_norm (src/kq_numeric.c:730-774)
// with the (1 + w) weight of the branch's H features.
__global__ void __launch_bounds__(kGrThreads)
gr_norm_kernel(GrDims d, const float *__restrict__ norm, const float *__restrict__ br, float *__restrict__ nm,
               ErrorWord err) {
    __shared__ float red[kGrThreads / 32];
    pdl_wait();
    if (gr_err_raised(err)) return;
    const uint32_t H = d.hidden, W = d.hidden * d.branches;
    const uint32_t t = blockIdx.x / d.branches, b = blockIdx.x % d.branches;
    const float *x = br + (size_t)t * W + (size_t)b * H;
    float *y = nm + (size_t)t * W + (size_t)b * H;
    const float *w = norm + (size_t)b * H;
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < H; i += kGrThreads) s = fmaf(x[i], x[i], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        float v = threadIdx.x < kGrThreads / 32 ? red[threadIdx.x] : 0.0f;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    const float mean = __fdiv_rn(red[0], (float)H);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, d.eps)));
    bool ok = isfinite(inv);
    for (uint32_t i = threadIdx.x; i < H; i += kGrThreads) {
        const float v = __fmul_rn(__fmul_rn(x[i], inv), __fadd_rn(1.0f, w[i]));
        y[i] = v;
        if (!isfinite(v)) ok = false;
    }
    if (!ok) gr_raise(err, kErrNonFinite);
}

// rank[t][i] = silu(proj[t][i] / B) for i < R; write_gate[t][b] =
// 2 sigmoid(proj[t][R + b] / B) (src/kq_layer_qwen38.c:109-116,155-163).
// Grid (column blocks, tokens).
__global__ void gr_gate_kernel(GrDims d, uint32_t T, const float *__restrict__ proj, float *__restrict__ rank,
                               float *__restrict__ wg, ErrorWord err) {
    pdl_wait();
    if (gr_err_raised(err)) return;
    const uint32_t R = d.rank, B = d.branches, per = R + B;
    const float fb = (float)B;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y)
        for (uint32_t c = blockIdx.x * blockDim.x + threadIdx.x; c < per; c += gridDim.x * blockDim.x) {
            const float v = __fdiv_rn(proj[(size_t)t * per + c], fb);
            if (c < R)
                rank[(size_t)t * R + c] = __fmul_rn(v, gr_sigmoid(v));
            else
                wg[(size_t)t * B + (c - R)] = __fmul_rn(2.0f, gr_sigmoid(v));
        }
}

// read[t][*] = sigmoid(read logits) in place; mixed[t][h] =
// (sum_b read[t][b][h] * nm[t][b][h]) / B (src/kq_layer_qwen38.c:129-143).
// Grid (feature blocks, tokens).
__global__ void gr_mix_kernel(GrDims d, uint32_t T, float *__restrict__ read, const float *__restrict__ nm,
                              float *__restrict__ mixed, ErrorWord err) {
    pdl_wait();
    if (gr_err_raised(err)) return;
    const uint32_t H = d.hidden, B = d.branches;
    const size_t W = (size_t)H * B;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y)
        for (uint32_t h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x) {
            float s = 0.0f;
            for (uint32_t b = 0; b < B; ++b) {
                const size_t o = (size_t)t * W + (size_t)b * H + h;
                const float g = gr_sigmoid(read[o]);
                read[o] = g;
                s = __fadd_rn(s, __fmul_rn(g, nm[o]));
            }
            mixed[(size_t)t * H + h] = __fdiv_rn(s, (float)B);
        }
}

// out[t][b][h] = br[t][b][h] + block[t][h] * wg[t][b]
// (src/kq_layer_qwen38.c:196-209).  Grid (feature blocks, tokens); a thread
// reads block[t][h] once for every branch.
__global__ void gr_write_kernel(GrDims d, uint32_t T, const float *__restrict__ br, const float *__restrict__ block,
                                const float *__restrict__ wg, float *__restrict__ out, ErrorWord err) {
    pdl_wait();
    if (gr_err_raised(err)) return;
    const uint32_t H = d.hidden, B = d.branches;
    const size_t W = (size_t)H * B;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y)
        for (uint32_t h = blockIdx.x * blockDim.x + threadIdx.x; h < H; h += gridDim.x * blockDim.x) {
            const float v = block[(size_t)t * H + h];
            for (uint32_t b = 0; b < B; ++b) {
                const size_t o = (size_t)t * W + (size_t)b * H + h;
                out[o] = __fadd_rn(br[o], __fmul_rn(v, wg[(size_t)t * B + b]));
            }
        }
}

// Grid of the per-token kernels: blocks of 256 over `n` columns, one row of
// blocks per token (at most 65535 rows; the kernels stride over the rest).
static dim3 grid_tokens(uint32_t n, uint32_t T) {
    return dim3((n + 255) / 256, std::min<uint32_t>(std::max<uint32_t>(T, 1u), 65535u));
}

size_t gr_workspace_bytes(const GrDims &d, uint32_t T) {
    const uint64_t W = (uint64_t)d.hidden * d.branches;
    auto r = [](uint64_t b) { return (b + 255) & ~uint64_t(255); };
    return r(T * W * 4) + r(T * (uint64_t)(d.rank + d.branches) * 4) + r(T * (uint64_t)d.rank * 4) +
           r(T * W * 4) + r(projection_workspace_floats(T, d.rank + d.branches, (uint32_t)W) * 4) +
           r(projection_workspace_floats(T, (uint32_t)W, d.rank) * 4);
}

void gr_carve(const GrDims &d, uint32_t T, void *ws, GrBuffers &b) {
    const uint64_t W = (uint64_t)d.hidden * d.branches;
    char *p = static_cast<char *>(ws);
    auto take = [&](uint64_t bytes) {
        char *q = p;
        p += (bytes + 255) & ~uint64_t(255);
        return reinterpret_cast<float *>(q);
    };
    b.normalized = take(T * W * 4);
    b.proj = take(T * (uint64_t)(d.rank + d.branches) * 4);
    b.rank = take(T * (uint64_t)d.rank * 4);
    b.read = take(T * W * 4);
    b.ws_down_floats = projection_workspace_floats(T, d.rank + d.branches, (uint32_t)W);
    b.ws_down = take(b.ws_down_floats * 4);
    b.ws_up_floats = projection_workspace_floats(T, (uint32_t)W, d.rank);
    b.ws_up = take(b.ws_up_floats * 4);
}

void launch_gr_read(const GrDims &d, const GrWeightsDev &w, const float *br, uint32_t T, float *mixed, float *wg,
                    GrBuffers &b, ErrorWord err, cudaStream_t stream) {
    KernelTimer timer("gr_read", stream);
    const uint32_t W = d.hidden * d.branches;
    launch_pdl(gr_norm_kernel, T * d.branches, kGrThreads, 0, stream, d, w.norm, br, b.normalized, err);
    count_launch();
    ProjSegments s{};
    s.count = 2;
    s.m[0] = w.down;
    s.out_offset[0] = 0;
    s.m[1] = w.inject;
    s.out_offset[1] = d.rank;
    launch_projection(s, b.normalized, W, b.proj, d.rank + d.branches, T, err, stream, b.ws_down, b.ws_down_floats);
    launch_pdl(gr_gate_kernel, grid_tokens(d.rank + d.branches, T), 256, 0, stream, d, T, b.proj, b.rank, wg, err);
    count_launch();
    ProjSegments u{};
    u.count = 1;
    u.m[0] = w.up;
    u.out_offset[0] = 0;
    launch_projection(u, b.rank, d.rank, b.read, W, T, err, stream, b.ws_up, b.ws_up_floats);
    launch_pdl(gr_mix_kernel, grid_tokens(d.hidden, T), 256, 0, stream, d, T, b.read, b.normalized, mixed, err);
    count_launch();
}

void launch_gr_write(const GrDims &d, const float *br, const float *block, const float *wg, uint32_t T, float *out,
                     ErrorWord err, cudaStream_t stream) {
    launch_pdl(gr_write_kernel, grid_tokens(d.hidden, T), 256, 0, stream, d, T, br, block, wg, out, err);
    count_launch();
}

}  // namespace kqb
