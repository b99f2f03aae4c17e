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
// chunk's L and P (64 x 64 dot products of 128-vectors) as TF32 warp MMAs
// with a three-term hi / lo split, then W and U by forward substitution in
// F32 (one thread per column), written to work space.
// Phase 2 (gdn_chunk_state_kernel), one CTA per (value head, column slice
// of S): walks the chunks in order with its S slice in the MMA accumulator
// registers and produces delta, O and the next S with three small matrix
// products per chunk (bf16 warp MMAs, three-term split, F32 accumulation).
// The state columns are independent, so the slices of a head run in
// parallel.  Phase 3 (gdn_gate_norm_kernel): gated RMSNorm of every
// token, as the recurrence kernel's epilogue.
//
// The split products carry a relative error of about 2^-21 (TF32) and
// 2^-16 (bf16) per product besides F32 rounding; the result differs from
// the token-by-token order within the tests' tolerance, not bit for bit.
#include "kernels.hpp"

#include <cmath>

#include <cuda_bf16.h>

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

// Work-space layout per (value head, chunk), in floats.  The operands of
// the phase-2 tensor-core products are stored as bf16 hi / lo pairs
// (v = hi + lo, both bf16) in the padded row layouts the MMA fragments are
// read from (rows of 136 or 72 bf16: conflict-free 32-bit fragment loads):
//   W [64 tokens][128 features], Q [64][128], K^T [128 features][64 tokens],
//   P [64][64]; U stays F32 [64][128].
constexpr int kLK = 136;                            // bf16 row stride, K = 128
constexpr int kLT = 72;                             // bf16 row stride, K = 64
constexpr size_t kTileW = (size_t)kC * kLK / 2;     // floats of one bf16 [64][136] tile
constexpr size_t kTileKT = (size_t)kD * kLT / 2;    // [128][72]
constexpr size_t kTileP = (size_t)kC * kLT / 2;     // [64][72]
constexpr size_t kChunkWh = 0;
constexpr size_t kChunkWl = kChunkWh + kTileW;
constexpr size_t kChunkQh = kChunkWl + kTileW;
constexpr size_t kChunkQl = kChunkQh + kTileW;
constexpr size_t kChunkKTh = kChunkQl + kTileW;
constexpr size_t kChunkKTl = kChunkKTh + kTileKT;
constexpr size_t kChunkPh = kChunkKTl + kTileKT;
constexpr size_t kChunkPl = kChunkPh + kTileP;
constexpr size_t kChunkU = kChunkPl + kTileP;       // U [64][128] F32
constexpr size_t kChunkEG = kChunkU + kC * kD;      // e^G_i [64]
constexpr size_t kChunkEGC = kChunkEG + kC;         // e^(G_C - G_i) [64]
constexpr size_t kChunkTot = kChunkEGC + kC;        // e^G_C at [0], padding
constexpr size_t kChunkFloats = kChunkTot + 64;
static_assert(kChunkU % 4 == 0 && kChunkFloats % 64 == 0, "16-byte aligned regions");

__device__ __forceinline__ void split_store(uint16_t *hi, uint16_t *lo, size_t i, float v) {
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    hi[i] = __bfloat16_as_ushort(h);
    lo[i] = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(h)));
}

// TF32 hi (round to nearest, ties away) and lo (the residual, rounded) of x
__device__ __forceinline__ void tf32_split(float x, uint32_t &hi, uint32_t &lo) {
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hi) : "f"(x));
    const float r = x - __uint_as_float(hi);
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(r));
}

__device__ __forceinline__ void mma_tf32(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x0, x1) -> bf16x2 hi and bf16x2 lo of the residuals, x0 in the low half
__device__ __forceinline__ void bf16_split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

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
    // L (strictly lower) and P (lower incl. diagonal) on the tensor cores:
    // warp w computes rows 16 (w & 3) .. +15 and columns 32 (w >> 2) .. +31
    // of both with m16n8k8 TF32 MMAs and the three-term split (hi = tf32(x),
    // lo = tf32(x - hi); a b ~ a_hi b_hi + a_hi b_lo + a_lo b_hi, relative
    // error ~ 2^-22).  Fragments come from the swizzled F32 tiles (the 8
    // rows of a fragment read 8 different 16-byte chunks).
    {
        const int warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
        const int m0 = 16 * (warp & 3), n0 = 32 * (warp >> 2);
        auto at = [&](const float *T, int r, int f) { return T[sw(r, f & ~3) + (f & 3)]; };
        float lacc[4][4], pacc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) lacc[nt][e] = pacc[nt][e] = 0.0f;
#pragma unroll 2
        for (int k0 = 0; k0 < kD; k0 += 8) {
            uint32_t kh[4], kl[4], qh[4], ql[4];
            const int ar[4] = {m0 + g, m0 + g + 8, m0 + g, m0 + g + 8};
            const int ac[4] = {k0 + q, k0 + q, k0 + q + 4, k0 + q + 4};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                tf32_split(at(Ks, ar[e], ac[e]), kh[e], kl[e]);
                tf32_split(at(Qs, ar[e], ac[e]), qh[e], ql[e]);
            }
#pragma unroll
            for (int nt = 0; nt < 4; ++nt) {
                const int j = n0 + 8 * nt + g;
                uint32_t bh0, bl0, bh1, bl1;
                tf32_split(at(Ks, j, k0 + q), bh0, bl0);
                tf32_split(at(Ks, j, k0 + q + 4), bh1, bl1);
                mma_tf32(lacc[nt], kh, bh0, bh1);
                mma_tf32(pacc[nt], qh, bh0, bh1);
                mma_tf32(lacc[nt], kh, bl0, bl1);
                mma_tf32(pacc[nt], qh, bl0, bl1);
                mma_tf32(lacc[nt], kl, bh0, bh1);
                mma_tf32(pacc[nt], ql, bh0, bh1);
            }
        }
        // decay factors; accumulator element e is row m0 + g (+ 8 for e >= 2),
        // column n0 + 8 nt + 2 q + (e & 1)
        uint32_t *ph = reinterpret_cast<uint32_t *>(wk + kChunkPh), *pl = reinterpret_cast<uint32_t *>(wk + kChunkPl);
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int i = m0 + g + 8 * half, j = n0 + 8 * nt + 2 * q;
                const float gi = Gs[i];
                float pv[2];
#pragma unroll
                for (int c = 0; c < 2; ++c) {
                    const int jj = j + c;
                    const float f = jj <= i ? expf(gi - Gs[jj]) : 0.0f;
                    Ls[i * kC + jj] = jj < i ? lacc[nt][2 * half + c] * f : 0.0f;
                    pv[c] = pacc[nt][2 * half + c] * f;
                }
                uint32_t hi, lo;
                bf16_split2(pv[0], pv[1], hi, lo);
                ph[((size_t)i * kLT + j) / 2] = hi;
                pl[((size_t)i * kLT + j) / 2] = lo;
            }
    }
    // Q [64][136] and K^T [128][72] as bf16 pairs for the tensor-core pass
    {
        uint16_t *qh = reinterpret_cast<uint16_t *>(wk + kChunkQh), *ql = reinterpret_cast<uint16_t *>(wk + kChunkQl);
        uint16_t *kh2 = reinterpret_cast<uint16_t *>(wk + kChunkKTh), *kl2 = reinterpret_cast<uint16_t *>(wk + kChunkKTl);
        for (int e = tid; e < kC * kD; e += blockDim.x) {
            const int r = e / kD, f = e % kD;
            split_store(qh, ql, (size_t)r * kLK + f, Qs[sw(r, f & ~3) + (f & 3)]);
            const int fi = e / kC, ti = e % kC;   // K^T row fi, column ti: coalesced along tokens
            split_store(kh2, kl2, (size_t)fi * kLT + ti, Ks[sw(ti, fi & ~3) + (fi & 3)]);
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
            // four independent partial sums: a quarter of the dependent chain
            float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
            int j = 0;
            for (; j + 4 <= i; j += 4) {
                const float4 l4 = *reinterpret_cast<const float4 *>(Li + j);
                a0 = fmaf(l4.x, X[j * kD + f], a0);
                a1 = fmaf(l4.y, X[(j + 1) * kD + f], a1);
                a2 = fmaf(l4.z, X[(j + 2) * kD + f], a2);
                a3 = fmaf(l4.w, X[(j + 3) * kD + f], a3);
            }
            for (; j < i; ++j) a0 = fmaf(Li[j], X[j * kD + f], a0);
            X[i * kD + f] = Bs[i] * (X[i * kD + f] - ((a0 + a1) + (a2 + a3)));
        }
    }
    __syncthreads();
    {
        uint16_t *wh = reinterpret_cast<uint16_t *>(wk + kChunkWh), *wl = reinterpret_cast<uint16_t *>(wk + kChunkWl);
        for (int e = tid; e < kC * kD; e += blockDim.x) split_store(wh, wl, (size_t)(e / kD) * kLK + e % kD, Ws[e]);
    }
    for (int i = tid; i < kC * (kD / 4); i += blockDim.x)
        *reinterpret_cast<float4 *>(wk + kChunkU + 4 * i) = *reinterpret_cast<const float4 *>(Us + 4 * i);
}

// ---------------------------------------------------------------- phase 2
// One CTA per (value head, slice of CW state columns), 256 threads, walking
// the chunks in order.  The three products of a chunk run on the tensor
// cores as warp MMAs (mma.sync m16n8k16, bf16 operands, F32 accumulate),
// each with the three-term split a b ~ a_hi b_hi + a_hi b_lo + a_lo b_hi:
//   delta = U - W S              (64 x CW, K = 128)
//   O     = e^G (Q S) + P delta  (64 x CW, K = 128 and 64)
//   S     = e^G_C S + K^T delta' (128 x CW, K = 64; delta' = e^(G_C - G) delta)
// Warp w keeps rows 16w .. 16w+15 of the F32 state in its accumulator
// registers for the whole pass; after each update the state is written back
// to shared memory as bf16 pairs, transposed ([column][row]), as the B
// operand of the next chunk.  W is prefetched one chunk ahead; Q, P and the
// decay factors load during the delta products, K^T during the O products.

__device__ __forceinline__ void chunk_cp16(void *smem, const void *gmem) {
    const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gmem));
}
__device__ __forceinline__ void chunk_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void chunk_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment (rows m0 .. m0+15, K k0 .. k0+15) of a row-major bf16 tile with
// row stride ld; B fragment (columns n0 .. n0+7) of a [n][k] bf16 tile.
// Four 8x8 bf16 matrices from shared memory (ldmatrix): thread t gives the
// address of row t % 8 of matrix t / 8 and receives, from each matrix, the
// pair (row lane / 4, columns 2 * (lane % 4) ..): the mma.sync m16n8k16
// fragment layout of A (four matrices) and of two B operands (two each).
__device__ __forceinline__ void ldsm_x4(const uint16_t *p, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
}

// acc += A B over K = 16 * KS steps, three-term split (hi.hi, hi.lo, lo.hi
// in that order).  Per step one ldmatrix.x4 for each A part (rows m0.. and
// m0 + 8.., columns k and k + 8) and one for both B parts (hi then lo,
// columns k and k + 8); row strides of 136 or 72 bf16 put the eight rows of
// a matrix in distinct banks.
template <int KS>
__device__ __forceinline__ void mma3(float (&acc)[4], const uint16_t *ah, const uint16_t *al, int lda, int m0,
                                     const uint16_t *bh, const uint16_t *bl, int ldb, int n0, int g, int q) {
    const int lane = 4 * g + q, mi = lane >> 3, r = lane & 7;
    const size_t oa = (size_t)(m0 + r + 8 * (mi & 1)) * lda + 8 * (mi >> 1);
    const uint16_t *pah = ah + oa, *pal = al + oa;
    const uint16_t *pb = (mi < 2 ? bh : bl) + (size_t)(n0 + r) * ldb + 8 * (mi & 1);
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
        uint32_t a[4], b[4];
        ldsm_x4(pah + 16 * kk, a);
        ldsm_x4(pb + 16 * kk, b);
        mma_bf16(acc, a, b[0], b[1]);
        mma_bf16(acc, a, b[2], b[3]);
        ldsm_x4(pal + 16 * kk, a);
        mma_bf16(acc, a, b[0], b[1]);
    }
}

template <int CW>
struct StateSmem {
    static constexpr size_t st = (size_t)CW * kLK;       // bf16 elements of one S^T part
    static constexpr size_t w = (size_t)kC * kLK;        // one W / Q part
    static constexpr size_t kt = (size_t)kD * kLT;       // one K^T part
    static constexpr size_t p = (size_t)kC * kLT;        // one P part
    static constexpr size_t dt = (size_t)CW * kLT;       // one delta^T part
    static constexpr size_t bytes = (2 * st + 4 * w + 2 * w + 2 * kt + 2 * p + 4 * dt) * 2 + (2 * kC + 4) * 4;
};

template <int CW>
__global__ void __launch_bounds__(256, 1)
gdn_chunk_state_kernel(GdnDims d, GdnBatchPtrs p, uint32_t tokens, const float *__restrict__ work,
                       float *__restrict__ obuf, ErrorWord err) {
    constexpr int NT = CW / 8;        // n8 tiles of the slice
    using SM = StateSmem<CW>;
    pdl_wait();
    extern __shared__ __align__(16) uint16_t sm16[];
    uint16_t *STh = sm16, *STl = STh + SM::st;                 // S^T [CW][136]
    uint16_t *Wb = STl + SM::st;                               // [2 buffers][hi, lo][64][136]
    uint16_t *Qh = Wb + 4 * SM::w, *Ql = Qh + SM::w;           // [64][136]
    uint16_t *KTh = Ql + SM::w, *KTl = KTh + SM::kt;           // [128][72]
    uint16_t *Ph = KTl + SM::kt, *Pl = Ph + SM::p;             // [64][72]
    uint16_t *DTh = Pl + SM::p, *DTl = DTh + SM::dt;           // delta^T [CW][72]
    uint16_t *D2h = DTl + SM::dt, *D2l = D2h + SM::dt;         // (e^(G_C - G) delta)^T
    float *Eg = reinterpret_cast<float *>(D2l + SM::dt);       // e^G [64], e^(G_C - G) [64], e^G_C
    if (chunk_error_raised(err)) return;
    const uint32_t h = blockIdx.x, sl = blockIdx.y;
    const uint32_t col0 = sl * CW;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
    const float *sin_ = p.rec_in[0] + (size_t)h * kD * kD;
    float *sout = p.rec_out[0] + (size_t)h * kD * kD;
    const uint32_t nchunks = (tokens + kC - 1) / kC;
    auto chunk_work = [&](uint32_t c) { return work + ((size_t)c * d.value_heads + h) * kChunkFloats; };
    auto copy = [&](void *dst, const float *src, size_t bytes) {
        for (size_t i = tid; i < bytes / 16; i += blockDim.x)
            chunk_cp16(reinterpret_cast<uint8_t *>(dst) + 16 * i, reinterpret_cast<const uint8_t *>(src) + 16 * i);
    };
    auto load_w = [&](uint32_t c) {
        const float *wk = chunk_work(c);
        uint16_t *dst = Wb + (c & 1u) * 2 * SM::w;
        copy(dst, wk + kChunkWh, SM::w * 2);
        copy(dst + SM::w, wk + kChunkWl, SM::w * 2);
    };
    // the state rows of warp w, columns of the slice, in accumulator layout
    float sacc[NT][4];
    const int r0 = 16 * warp + g;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int c = 8 * nt + 2 * q;
        sacc[nt][0] = sin_[(size_t)r0 * kD + col0 + c];
        sacc[nt][1] = sin_[(size_t)r0 * kD + col0 + c + 1];
        sacc[nt][2] = sin_[(size_t)(r0 + 8) * kD + col0 + c];
        sacc[nt][3] = sin_[(size_t)(r0 + 8) * kD + col0 + c + 1];
    }
    auto store_st = [&]() {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
            const int c = 8 * nt + 2 * q;
            split_store(STh, STl, (size_t)c * kLK + r0, sacc[nt][0]);
            split_store(STh, STl, (size_t)(c + 1) * kLK + r0, sacc[nt][1]);
            split_store(STh, STl, (size_t)c * kLK + r0 + 8, sacc[nt][2]);
            split_store(STh, STl, (size_t)(c + 1) * kLK + r0 + 8, sacc[nt][3]);
        }
    };
    store_st();
    if (nchunks > 0) load_w(0);
    chunk_commit();
    bool bad = false;
    for (uint32_t c = 0; c < nchunks; ++c) {
        const float *wk = chunk_work(c);
        const uint32_t t0 = c * kC, n = min((uint32_t)kC, tokens - t0);
        __syncthreads();   // the previous chunk is done with Q, K^T, P, delta, decay factors and its W
        copy(Qh, wk + kChunkQh, SM::w * 2);          // group A: Q, P, decay factors
        copy(Ql, wk + kChunkQl, SM::w * 2);
        copy(Ph, wk + kChunkPh, SM::p * 2);
        copy(Pl, wk + kChunkPl, SM::p * 2);
        copy(Eg, wk + kChunkEG, (2 * kC + 4) * 4);
        chunk_commit();
        copy(KTh, wk + kChunkKTh, SM::kt * 2);       // group B: K^T
        copy(KTl, wk + kChunkKTl, SM::kt * 2);
        chunk_commit();
        if (c + 1 < nchunks) load_w(c + 1);          // group C: the next chunk's W
        chunk_commit();
        chunk_wait<3>();   // this chunk's W (committed one chunk earlier)
        __syncthreads();   // ... and S^T of the previous update, visible to every warp
        const uint16_t *Wh = Wb + (c & 1u) * 2 * SM::w, *Wl = Wh + SM::w;
        // ---- delta = U - W S, and delta' = e^(G_C - G) delta, both stored transposed as bf16 pairs
        for (int tt = warp; tt < 4 * NT; tt += 8) {
            const int mt = tt / NT, nt = tt % NT;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            mma3<kD / 16>(acc, Wh, Wl, kLK, 16 * mt, STh, STl, kLK, 8 * nt, g, q);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 16 * mt + g + (e >> 1) * 8, col = 8 * nt + 2 * q + (e & 1);
                const float dl = wk[kChunkU + row * kD + col0 + col] - acc[e];
                split_store(DTh, DTl, (size_t)col * kLT + row, dl);
                split_store(D2h, D2l, (size_t)col * kLT + row, wk[kChunkEGC + row] * dl);
            }
        }
        chunk_wait<2>();   // Q, P, decay factors
        __syncthreads();   // ... and delta^T from every warp
        // ---- O = e^G (Q S) + P delta
        for (int tt = warp; tt < 4 * NT; tt += 8) {
            const int mt = tt / NT, nt = tt % NT;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            mma3<kD / 16>(acc, Qh, Ql, kLK, 16 * mt, STh, STl, kLK, 8 * nt, g, q);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] *= Eg[16 * mt + g + (e >> 1) * 8];
            mma3<kC / 16>(acc, Ph, Pl, kLT, 16 * mt, DTh, DTl, kLT, 8 * nt, g, q);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const uint32_t row = 16 * mt + g + (e >> 1) * 8, col = 8 * nt + 2 * q + (e & 1);
                if (row < n) {
                    bad |= !isfinite(acc[e]);
                    obuf[(size_t)(t0 + row) * d.value_width + h * kD + col0 + col] = acc[e];
                }
            }
        }
        chunk_wait<1>();   // K^T
        __syncthreads();   // every read of S^T is done; K^T visible
        // ---- S = e^G_C S + K^T delta'
        {
            const float eg_c = Eg[2 * kC];
#pragma unroll
            for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) sacc[nt][e] *= eg_c;
                mma3<kC / 16>(sacc[nt], KTh, KTl, kLT, 16 * warp, D2h, D2l, kLT, 8 * nt, g, q);
            }
            store_st();
        }
    }
    chunk_wait<0>();
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
        const int c = 8 * nt + 2 * q;
        bad |= !isfinite(sacc[nt][0]) || !isfinite(sacc[nt][1]) || !isfinite(sacc[nt][2]) || !isfinite(sacc[nt][3]);
        sout[(size_t)r0 * kD + col0 + c] = sacc[nt][0];
        sout[(size_t)r0 * kD + col0 + c + 1] = sacc[nt][1];
        sout[(size_t)(r0 + 8) * kD + col0 + c] = sacc[nt][2];
        sout[(size_t)(r0 + 8) * kD + col0 + c + 1] = sacc[nt][3];
    }
    if (__syncthreads_or(bad) && tid == 0) chunk_raise(err, kErrNonFinite);
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
    *reinterpret_cast<float4 *>(gated + (size_t)t * d.value_width + gated_head_pos(w, h) * kD + 4 * lane) = g;
}

void launch_gdn_chunked(const GdnDims &d, const GdnWeightsDev &w, const GdnBatchPtrs &p, uint32_t tokens,
                        const float *qk, const float *v, const float *beta, const float *logdecay,
                        const float *proj, uint32_t ldp, float *gated, float *work, ErrorWord err,
                        cudaStream_t stream) {
    KernelTimer timer("gdn_recurrence", stream);
    const uint32_t chunks = (tokens + kC - 1) / kC;
    float *obuf = work + (size_t)chunks * d.value_heads * kChunkFloats;
    const size_t smem1 = (size_t)(3 * kC * kD + kC * kC + 2 * kC) * sizeof(float);
    static DeviceOnce attr;
    attr.run([&] {
        cudaFuncSetAttribute(gdn_chunk_prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem1);
        cudaFuncSetAttribute(gdn_chunk_state_kernel<32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)StateSmem<32>::bytes);
        cudaFuncSetAttribute(gdn_chunk_state_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)StateSmem<16>::bytes);
        cudaFuncSetAttribute(gdn_chunk_state_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)StateSmem<8>::bytes);
    });
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
        if (d.value_heads >= 32)
            launch_pdl(gdn_chunk_state_kernel<32>, dim3(d.value_heads, kD / 32), 256, StateSmem<32>::bytes, stream,
                       d, p, tokens, work, obuf, err);
        else if (d.value_heads >= 16)
            launch_pdl(gdn_chunk_state_kernel<16>, dim3(d.value_heads, kD / 16), 256, StateSmem<16>::bytes, stream,
                       d, p, tokens, work, obuf, err);
        else
            launch_pdl(gdn_chunk_state_kernel<8>, dim3(d.value_heads, kD / 8), 256, StateSmem<8>::bytes, stream,
                       d, p, tokens, work, obuf, err);
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
