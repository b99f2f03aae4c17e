// Chunked (WY-form) gated delta-net prefill for dk = dv = 128.
//
// The reference runs the delta rule token by token (src/kq_gdn_qwen38.c:
// 705-761): S <- e^g S; delta = beta (v - S^T k); S <- S + k delta^T;
// o = S^T q.  Over a chunk of C tokens with S0 the state at its start and
// G_i = g_1 + ... + g_i (log decays, all <= 0), the same recurrence is
//   delta = U - W S0,                  (I + diag(beta) L) W = diag(beta e^G) K
//                                      (I + diag(beta) L) U = diag(beta) V
//   O     = diag(e^G) Q S0 + P delta,  P_ij  = (q_i . k_j) e^(G_i - G_j), j <= i
//   S_C   = e^(G_C) S0 + (diag(e^(G_C - G)) K)^T delta,
// with L_ij = (k_i . k_j) e^(G_i - G_j) for j < i.  Every decay factor is a
// difference G_i - G_j <= 0, so nothing overflows however strong the decay.
//
// Phase 1 (gdn_chunk_prep_kernel), one CTA per (value head, chunk): the
// chunk's L and P (64 x 64 dot products of 128-vectors), then W and U by
// forward substitution (one thread per column), written to work space.
// Phase 2 (gdn_chunk_state_kernel), one CTA per (value head, column slice
// of S): walks the chunks in order with its S slice in shared memory and
// produces delta, O and the next S with three small matrix products per
// chunk.  The state columns are independent, so the slices of a head run in
// parallel.  Phase 3 (gdn_gate_norm_kernel): gated RMSNorm of every
// token, as the recurrence kernel's epilogue.
//
// Arithmetic is F32 (FMA); the result differs from the token-by-token order
// only by rounding.
#include "kernels.hpp"

#include <cmath>

namespace kqb {

namespace {

constexpr int kC = 64;       // tokens per chunk
constexpr int kD = 128;      // dk = dv

__device__ __forceinline__ bool chunk_error_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}
__device__ __forceinline__ void chunk_raise(const ErrorWord &e, uint32_t code) {
    atomicCAS(e.word, 0ull, ((unsigned long long)code << 32) | e.call_id);
}

__device__ __forceinline__ float chunk_sigmoid(float x) {
    if (x >= 0.0f) {
        const float e = expf(-x);
        return 1.0f / (1.0f + e);
    }
    const float e = expf(x);
    return e / (1.0f + e);
}

}  // namespace

// Work-space layout per (value head, chunk), in floats.
constexpr size_t kChunkW = 0;                       // W [64][128]
constexpr size_t kChunkU = kChunkW + kC * kD;       // U [64][128]
constexpr size_t kChunkP = kChunkU + kC * kD;       // P [64][64]
constexpr size_t kChunkEG = kChunkP + kC * kC;      // e^G_i [64]
constexpr size_t kChunkEGC = kChunkEG + kC;         // e^(G_C - G_i) [64]
constexpr size_t kChunkTot = kChunkEGC + kC;        // e^G_C at [0], padding
constexpr size_t kChunkFloats = kChunkTot + 64;

size_t gdn_chunk_workspace_floats(const GdnDims &d, uint32_t tokens) {
    const size_t chunks = (tokens + kC - 1) / kC;
    return chunks * d.value_heads * kChunkFloats + (size_t)tokens * d.value_width;   // + O
}

bool gdn_chunked_supported(const GdnDims &d) { return d.key_dim == kD && d.value_dim == kD; }

// ---------------------------------------------------------------- phase 1
__global__ void __launch_bounds__(256, 2)
gdn_chunk_prep_kernel(GdnDims d, uint32_t tokens, const float *__restrict__ qk, const float *__restrict__ vin,
                      const float *__restrict__ beta, const float *__restrict__ logdecay,
                      float *__restrict__ work, ErrorWord err) {
    pdl_wait();
    // 112.5 KB: two CTAs per SM.  K and Q are [64][128] with their 16-byte
    // chunks XOR-swizzled by row (8 consecutive rows hit 8 bank groups); the
    // Q tile is dead after L and P and then holds W.
    extern __shared__ __align__(16) float cs[];
    float *Ks = cs;                        // [64][128] swizzled
    float *Qs = Ks + kC * kD;              // [64][128] swizzled, then W [64][128]
    float *Us = Qs + kC * kD;              // U [64][128]
    float *Ls = Us + kC * kD;              // [64][64]
    float *Gs = Ls + kC * kC;              // [64]
    float *Bs = Gs + kC;                   // [64]
    auto sw = [](int r, int c4) { return r * kD + ((((c4 >> 2) ^ (r & 7))) << 2); };
    if (chunk_error_raised(err)) return;
    const uint32_t h = blockIdx.x, c = blockIdx.y;
    const uint32_t kh = h / d.repeat;
    const uint32_t t0 = c * kC;
    const uint32_t n = min((uint32_t)kC, tokens - t0);
    const int tid = threadIdx.x;
    float *wk = work + ((size_t)c * d.value_heads + h) * kChunkFloats;

    // q, k rows of key head kh (zero past the end of the sequence)
    for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
        const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
        float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f), k4 = q4;
        if ((uint32_t)r < n) {
            const size_t item = t0 + r;
            q4 = *reinterpret_cast<const float4 *>(qk + (item * 2 + 0) * d.key_width + kh * kD + c4);
            k4 = *reinterpret_cast<const float4 *>(qk + (item * 2 + 1) * d.key_width + kh * kD + c4);
        }
        *reinterpret_cast<float4 *>(Qs + sw(r, c4)) = q4;
        *reinterpret_cast<float4 *>(Ks + sw(r, c4)) = k4;
    }
    if (tid < kC) {
        const bool in = (uint32_t)tid < n;
        Bs[tid] = in ? beta[(size_t)(t0 + tid) * d.value_heads + h] : 0.0f;
        Gs[tid] = in ? logdecay[(size_t)(t0 + tid) * d.value_heads + h] : 0.0f;
    }
    __syncthreads();
    if (tid == 0) {   // cumulative log decay, in token order
        float acc = 0.0f;
        for (int i = 0; i < kC; ++i) {
            acc += Gs[i];
            Gs[i] = acc;
        }
    }
    __syncthreads();
    // L (strictly lower) and P (lower incl. diagonal): thread -> row i,
    // columns j = (tid & 3) + 4 r (the four column groups of a warp read
    // four consecutive K rows: different banks)
    {
        const int i = tid >> 2, j0 = tid & 3;
        float lk[16], pq[16];
#pragma unroll
        for (int r = 0; r < 16; ++r) { lk[r] = 0.f; pq[r] = 0.f; }
        for (int kk = 0; kk < kD; kk += 4) {
            const float4 ki = *reinterpret_cast<const float4 *>(Ks + sw(i, kk));
            const float4 qi = *reinterpret_cast<const float4 *>(Qs + sw(i, kk));
#pragma unroll
            for (int r = 0; r < 16; ++r) {
                const float4 kj = *reinterpret_cast<const float4 *>(Ks + sw(j0 + 4 * r, kk));
                lk[r] = fmaf(ki.x, kj.x, fmaf(ki.y, kj.y, fmaf(ki.z, kj.z, fmaf(ki.w, kj.w, lk[r]))));
                pq[r] = fmaf(qi.x, kj.x, fmaf(qi.y, kj.y, fmaf(qi.z, kj.z, fmaf(qi.w, kj.w, pq[r]))));
            }
        }
        const float gi = Gs[i];
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            const int j = j0 + 4 * r;
            const float f = j <= i ? expf(gi - Gs[j]) : 0.0f;
            Ls[i * kC + j] = j < i ? lk[r] * f : 0.0f;
            wk[kChunkP + i * kC + j] = pq[r] * f;
        }
    }
    const float gc = Gs[n - 1];
    if (tid < kC) {
        wk[kChunkEG + tid] = expf(Gs[tid]);
        wk[kChunkEGC + tid] = (uint32_t)tid < n ? expf(gc - Gs[tid]) : 0.0f;
    }
    if (tid == 0) wk[kChunkTot] = expf(gc);
    __syncthreads();
    // right-hand sides, staged before the sequential solve: W rows start as
    // e^G_i k_i (in the Q tile, dead now), U rows as v_i
    float *Ws = Qs;
    for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
        const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
        const float eg = expf(Gs[r]);
        const float4 k4 = *reinterpret_cast<const float4 *>(Ks + sw(r, c4));
        *reinterpret_cast<float4 *>(Ws + r * kD + c4) = make_float4(eg * k4.x, eg * k4.y, eg * k4.z, eg * k4.w);
        float4 v4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if ((uint32_t)r < n) v4 = *reinterpret_cast<const float4 *>(vin + (size_t)(t0 + r) * d.value_width + h * kD + c4);
        *reinterpret_cast<float4 *>(Us + r * kD + c4) = v4;
    }
    __syncthreads();
    // forward substitution in place, one column per thread: threads 0..127 W,
    // 128..255 U; row i = beta_i (rhs_i - sum_{j<i} L_ij row_j)
    {
        float *X = tid < kD ? Ws : Us;
        const int f = tid & (kD - 1);
        for (int i = 0; i < kC; ++i) {
            const float *Li = Ls + i * kC;
            float acc = 0.0f;
            int j = 0;
            for (; j + 4 <= i; j += 4) {
                const float4 l4 = *reinterpret_cast<const float4 *>(Li + j);
                acc = fmaf(l4.x, X[j * kD + f], acc);
                acc = fmaf(l4.y, X[(j + 1) * kD + f], acc);
                acc = fmaf(l4.z, X[(j + 2) * kD + f], acc);
                acc = fmaf(l4.w, X[(j + 3) * kD + f], acc);
            }
            for (; j < i; ++j) acc = fmaf(Li[j], X[j * kD + f], acc);
            X[i * kD + f] = Bs[i] * (X[i * kD + f] - acc);
        }
    }
    __syncthreads();
    for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
        *reinterpret_cast<float4 *>(wk + kChunkW + 4 * i) = *reinterpret_cast<const float4 *>(Ws + 4 * i);
        *reinterpret_cast<float4 *>(wk + kChunkU + 4 * i) = *reinterpret_cast<const float4 *>(Us + 4 * i);
    }
}

// ---------------------------------------------------------------- phase 2
// CW state columns per CTA (32, 16 or 8: fewer value heads per GPU take
// narrower slices, so that the grid still covers the SMs); NT threads =
// CW columns x G = NT / CW row groups.  The tiles are read as 16-byte
// vectors along their rows (broadcast within a row group), four K steps per
// vector.  Tile loads are cp.async copies issued ahead of use: the next
// chunk's W during the whole current chunk (two W buffers), the current
// chunk's Q, P and decay factors during its delta phase, its K during the
// O phase.  Q and K are stored unscaled; e^G scales a row's Q . S dot and
// e^(G_C - G) scales delta in the state update.

__device__ __forceinline__ void chunk_cp16(float *smem, const float *gmem, bool valid) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    const unsigned n = valid ? 16u : 0u;   // 0: zero fill
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void chunk_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void chunk_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

template <int CW, int NT>
__global__ void __launch_bounds__(NT, 1)
gdn_chunk_state_kernel(GdnDims d, GdnBatchPtrs p, uint32_t tokens, const float *__restrict__ qk,
                       const float *__restrict__ work, float *__restrict__ obuf, ErrorWord err) {
    constexpr int G = NT / CW;       // row groups
    constexpr int RD = kC / G;       // delta / O rows per thread
    constexpr int RS = kD / G;       // state rows per thread
    constexpr int LT = kD + 4;       // row stride of the W / Q / K tiles
    constexpr int LP = kC + 4;       // row stride of P
    static_assert(RS % 4 == 0, "state rows in 16-byte groups");
    pdl_wait();
    extern __shared__ __align__(16) float cs[];
    float *S = cs;                   // [128][CW]
    float *Wb = S + kD * CW;         // [2][64][LT]
    float *Qs = Wb + 2 * kC * LT;    // [64][LT]
    float *Ks = Qs + kC * LT;        // [64][LT]
    float *Ps = Ks + kC * LT;        // [64][LP]
    float *Ds = Ps + kC * LP;        // delta [64][CW]
    float *Eg = Ds + kC * CW;        // e^G_i [64], e^(G_C - G_i) [64], e^G_C [4]
    if (chunk_error_raised(err)) return;
    const uint32_t h = blockIdx.x, sl = blockIdx.y;
    const uint32_t kh = h / d.repeat;
    const uint32_t col0 = sl * CW;
    const int tid = threadIdx.x, f = tid % CW, grp = tid / CW;
    const float *sin_ = p.rec_in[0] + (size_t)h * kD * kD;
    float *sout = p.rec_out[0] + (size_t)h * kD * kD;
    const uint32_t nchunks = (tokens + kC - 1) / kC;
    auto chunk_work = [&](uint32_t c) { return work + ((size_t)c * d.value_heads + h) * kChunkFloats; };
    auto load_w = [&](uint32_t c) {
        const float *wk = chunk_work(c);
        float *dst = Wb + (c & 1u) * kC * LT;
        for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
            const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
            chunk_cp16(dst + r * LT + c4, wk + kChunkW + r * kD + c4, true);
        }
    };
    for (int i = tid; i < kD * CW; i += blockDim.x) S[i] = sin_[(size_t)(i / CW) * kD + col0 + i % CW];
    if (nchunks > 0) load_w(0);
    chunk_commit();
    bool bad = false;
    for (uint32_t c = 0; c < nchunks; ++c) {
        const float *wk = chunk_work(c);
        const uint32_t t0 = c * kC, n = min((uint32_t)kC, tokens - t0);
        __syncthreads();   // the previous chunk is done with Q, K, P, D and its W buffer
        // group A: Q, P, decay factors of this chunk
        for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
            const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
            const bool in = (uint32_t)r < n;
            const size_t item = t0 + (in ? r : 0);
            chunk_cp16(Qs + r * LT + c4, qk + (item * 2 + 0) * d.key_width + kh * kD + c4, in);
        }
        for (int i = tid; i < kC * (kC / 4); i += blockDim.x) {
            const int r = i / (kC / 4), c4 = (i % (kC / 4)) * 4;
            chunk_cp16(Ps + r * LP + c4, wk + kChunkP + r * kC + c4, true);
        }
        if (tid < 32) chunk_cp16(Eg + tid * 4, wk + kChunkEG + tid * 4, true);   // e^G, e^(G_C - G)
        if (tid == 32) chunk_cp16(Eg + 128, wk + kChunkTot, true);                // e^G_C (+ padding)
        chunk_commit();
        // group B: K of this chunk
        for (int i = tid; i < kC * (kD / 4); i += blockDim.x) {
            const int r = i / (kD / 4), c4 = (i % (kD / 4)) * 4;
            const bool in = (uint32_t)r < n;
            const size_t item = t0 + (in ? r : 0);
            chunk_cp16(Ks + r * LT + c4, qk + (item * 2 + 1) * d.key_width + kh * kD + c4, in);
        }
        chunk_commit();
        // group C: W of the next chunk
        if (c + 1 < nchunks) load_w(c + 1);
        chunk_commit();
        chunk_wait<3>();   // this chunk's W (committed one chunk earlier)
        __syncthreads();
        const float *Ws = Wb + (c & 1u) * kC * LT;
        // delta = U - W S : thread -> column f, rows RD grp .. RD grp + RD - 1
        {
            float acc[RD];
#pragma unroll
            for (int r = 0; r < RD; ++r) acc[r] = 0.f;
#pragma unroll 2
            for (int k = 0; k < kD; k += 4) {
                const float s0 = S[k * CW + f], s1 = S[(k + 1) * CW + f], s2 = S[(k + 2) * CW + f],
                            s3 = S[(k + 3) * CW + f];
#pragma unroll
                for (int r = 0; r < RD; ++r) {
                    const float4 w4 = *reinterpret_cast<const float4 *>(Ws + (RD * grp + r) * LT + k);
                    acc[r] = fmaf(w4.w, s3, fmaf(w4.z, s2, fmaf(w4.y, s1, fmaf(w4.x, s0, acc[r]))));
                }
            }
#pragma unroll
            for (int r = 0; r < RD; ++r) {
                const int i = RD * grp + r;
                Ds[i * CW + f] = wk[kChunkU + i * kD + col0 + f] - acc[r];
            }
        }
        chunk_wait<2>();   // Q, P, decay factors
        __syncthreads();
        // O = e^G (Q S) + P delta for the same rows / column
        {
            float acc[RD];
#pragma unroll
            for (int r = 0; r < RD; ++r) acc[r] = 0.f;
#pragma unroll 2
            for (int k = 0; k < kD; k += 4) {
                const float s0 = S[k * CW + f], s1 = S[(k + 1) * CW + f], s2 = S[(k + 2) * CW + f],
                            s3 = S[(k + 3) * CW + f];
#pragma unroll
                for (int r = 0; r < RD; ++r) {
                    const float4 q4 = *reinterpret_cast<const float4 *>(Qs + (RD * grp + r) * LT + k);
                    acc[r] = fmaf(q4.w, s3, fmaf(q4.z, s2, fmaf(q4.y, s1, fmaf(q4.x, s0, acc[r]))));
                }
            }
#pragma unroll
            for (int r = 0; r < RD; ++r) acc[r] *= Eg[RD * grp + r];
#pragma unroll 2
            for (int j = 0; j < kC; j += 4) {
                const float d0 = Ds[j * CW + f], d1 = Ds[(j + 1) * CW + f], d2 = Ds[(j + 2) * CW + f],
                            d3 = Ds[(j + 3) * CW + f];
#pragma unroll
                for (int r = 0; r < RD; ++r) {
                    const float4 p4 = *reinterpret_cast<const float4 *>(Ps + (RD * grp + r) * LP + j);
                    acc[r] = fmaf(p4.w, d3, fmaf(p4.z, d2, fmaf(p4.y, d1, fmaf(p4.x, d0, acc[r]))));
                }
            }
#pragma unroll
            for (int r = 0; r < RD; ++r) {
                const uint32_t i = RD * grp + r;
                if (i < n) {
                    bad |= !isfinite(acc[r]);
                    obuf[(size_t)(t0 + i) * d.value_width + h * kD + col0 + f] = acc[r];
                }
            }
        }
        chunk_wait<1>();   // K
        __syncthreads();   // every read of the old S is done; K visible
        // S = e^(G_C) S + K^T (e^(G_C - G) delta) : thread -> column f, rows RS grp .. RS grp + RS - 1
        {
            const float eg_c = Eg[128];
            float acc[RS];
#pragma unroll
            for (int r = 0; r < RS; ++r) acc[r] = eg_c * S[(RS * grp + r) * CW + f];
#pragma unroll 2
            for (int i = 0; i < kC; ++i) {
                const float dv = Eg[64 + i] * Ds[i * CW + f];
#pragma unroll
                for (int r = 0; r < RS; r += 4) {
                    const float4 k4 = *reinterpret_cast<const float4 *>(Ks + i * LT + RS * grp + r);
                    acc[r] = fmaf(k4.x, dv, acc[r]);
                    acc[r + 1] = fmaf(k4.y, dv, acc[r + 1]);
                    acc[r + 2] = fmaf(k4.z, dv, acc[r + 2]);
                    acc[r + 3] = fmaf(k4.w, dv, acc[r + 3]);
                }
            }
#pragma unroll
            for (int r = 0; r < RS; ++r) S[(RS * grp + r) * CW + f] = acc[r];
        }
    }
    chunk_wait<0>();
    __syncthreads();
    for (int i = tid; i < kD * CW; i += blockDim.x) {
        const float v = S[i];
        bad |= !isfinite(v);
        sout[(size_t)(i / CW) * kD + col0 + i % CW] = v;
    }
    if (__syncthreads_or(bad) && tid == 0) chunk_raise(err, kErrNonFinite);
}

constexpr int kStateThreads = 256;   // 512 measured slower (register-limited, one CTA per SM either way)

template <int CW>
static size_t state_smem() {
    return (size_t)(kD * CW + 4 * kC * (kD + 4) + kC * (kC + 4) + kC * CW + 2 * kC + 4) * sizeof(float);
}

// ---------------------------------------------------------------- phase 3
// One warp per (token, value head), 8 per CTA: lane l takes features
// 4l .. 4l+3; o * rsqrt(mean(o^2) + eps) * norm_w * sigmoid(z).
__global__ void __launch_bounds__(256)
gdn_gate_norm_kernel(GdnDims d, GdnWeightsDev w, const float *__restrict__ obuf, const float *__restrict__ proj,
                     uint32_t ldp, float *__restrict__ gated, uint32_t tokens, ErrorWord err) {
    pdl_wait();
    if (chunk_error_raised(err)) return;
    const uint32_t pair = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pair >= tokens * d.value_heads) return;
    const uint32_t t = pair / d.value_heads, h = pair % d.value_heads;
    const int lane = threadIdx.x & 31;
    const float4 o = *reinterpret_cast<const float4 *>(obuf + (size_t)t * d.value_width + h * kD + 4 * lane);
    float v = o.x * o.x + o.y * o.y + o.z * o.z + o.w * o.w;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v += __shfl_xor_sync(0xffffffffu, v, s);
    const float inv = 1.0f / sqrtf(v / (float)kD + d.eps);
    const float4 z = *reinterpret_cast<const float4 *>(proj + (size_t)t * ldp + d.conv_channels + h * kD + 4 * lane);
    const float4 nw = *reinterpret_cast<const float4 *>(w.norm + 4 * lane);
    const float4 g = make_float4((nw.x * (o.x * inv)) * chunk_sigmoid(z.x), (nw.y * (o.y * inv)) * chunk_sigmoid(z.y),
                                 (nw.z * (o.z * inv)) * chunk_sigmoid(z.z), (nw.w * (o.w * inv)) * chunk_sigmoid(z.w));
    if (!isfinite(g.x) || !isfinite(g.y) || !isfinite(g.z) || !isfinite(g.w)) chunk_raise(err, kErrNonFinite);
    *reinterpret_cast<float4 *>(gated + (size_t)t * d.value_width + h * kD + 4 * lane) = g;
}

void launch_gdn_chunked(const GdnDims &d, const GdnWeightsDev &w, const GdnBatchPtrs &p, uint32_t tokens,
                        const float *qk, const float *v, const float *beta, const float *logdecay,
                        const float *proj, uint32_t ldp, float *gated, float *work, ErrorWord err,
                        cudaStream_t stream) {
    KernelTimer timer("gdn_recurrence", stream);
    const uint32_t chunks = (tokens + kC - 1) / kC;
    float *obuf = work + (size_t)chunks * d.value_heads * kChunkFloats;
    const size_t smem1 = (size_t)(3 * kC * kD + kC * kC + 2 * kC) * sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
        cudaFuncSetAttribute(gdn_chunk_state_kernel<32, kStateThreads>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)state_smem<32>());
        cudaFuncSetAttribute(gdn_chunk_state_kernel<16, kStateThreads>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)state_smem<16>());
        cudaFuncSetAttribute(gdn_chunk_state_kernel<8, 256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)state_smem<8>());
        attr = true;
    }
    {
        KernelTimer t1("gdn_chunk_prep", stream);
        launch_pdl(gdn_chunk_prep_kernel, dim3(d.value_heads, chunks), 256, smem1, stream, d, tokens, qk, v, beta,
                   logdecay, work, err);
        count_launch();
    }
    {
        // the sequential pass: (value heads x column slices) CTAs, slices
        // narrow enough that the grid reaches about 128 CTAs
        KernelTimer t2("gdn_chunk_state", stream);
        if (d.value_heads >= 32) {
            launch_pdl(gdn_chunk_state_kernel<32, kStateThreads>, dim3(d.value_heads, kD / 32), kStateThreads,
                       state_smem<32>(), stream, d, p, tokens, qk, work, obuf, err);
        } else if (d.value_heads >= 16) {
            launch_pdl(gdn_chunk_state_kernel<16, kStateThreads>, dim3(d.value_heads, kD / 16), kStateThreads,
                       state_smem<16>(), stream, d, p, tokens, qk, work, obuf, err);
        } else {
            launch_pdl(gdn_chunk_state_kernel<8, 256>, dim3(d.value_heads, kD / 8), 256, state_smem<8>(), stream, d,
                       p, tokens, qk, work, obuf, err);
        }
        count_launch();
    }
    {
        KernelTimer t3("gdn_gate_norm", stream);
        launch_pdl(gdn_gate_norm_kernel, dim3((tokens * d.value_heads + 7) / 8), 256, 0, stream, d, w, obuf, proj,
                   ldp, gated, tokens, err);
        count_launch();
    }
}

}  // namespace kqb
