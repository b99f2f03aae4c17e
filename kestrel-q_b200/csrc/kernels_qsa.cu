// QSA (gated block-sparse grouped-query attention) kernels: decode batches
// and uniform prefill groups (consecutive tokens of one sequence).
//
// Math follows the per-token loop of kq_qsa_execute_common
// (src/kq_qsa_qwen38.c:524-828 of Kestrel-Q):
//   (1+w) RMSNorm (:231-256) and NeoX partial RoPE (:258-281) of q, k and the
//   index query; KV / raw-index-key append (:603-606); block indexer over all
//   complete blocks (:608-648); stable top-k by (score desc, id asc)
//   (:328-359); token list = selected blocks in rank order then the partial
//   tail (:654-665); softmax attention over the selected tokens (:716-773);
//   sigmoid output gate (:774-782).
//
// Exactness: every step of the indexer (norms, RoPE, block-key mean, scores)
// is evaluated with explicitly rounded F32 operations in the reference's
// order, and the RoPE cos/sin values come from a host table computed with
// the reference's powf/cosf/sinf expression, so candidate scores - and hence
// the selected blocks - are bit-identical to the reference given identical
// inputs.  The block key of a block is computed once, when the block
// completes, and cached feature-major; the reference recomputes the same
// value from the raw keys on every token.  The attention over the selected
// tokens is checked to tolerance instead: for head_dim 256 it runs on the
// tensor cores over bf16 hi / lo copies of the cache rows.
#include "kernels.hpp"

#include <cstdlib>

#include <cuda_bf16.h>

#include <algorithm>
#include <cmath>

namespace kqb {

__device__ __forceinline__ bool qsa_error_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}
__device__ __forceinline__ void qsa_raise(const ErrorWord &e, uint32_t code) {
    atomicCAS(e.word, 0ull, ((unsigned long long)code << 32) | e.call_id);
}

// Sequential (1+w) RMS statistic: returns 1/sqrt(mean(x^2) + eps) computed as
// the reference does (:234-242), or a non-finite value.
__device__ __forceinline__ float exact_rms_inverse(const float *x, uint32_t n, float eps) {
    float sum = 0.0f;
    for (uint32_t i = 0; i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(x[i], x[i]));
    sum = __fdiv_rn(sum, (float)n);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sum, eps)));
}

// Applies (x * inv) * (1 + w) to x[i] (:247-249).
__device__ __forceinline__ float exact_norm_apply(float x, float inv, float w) {
    return __fmul_rn(__fmul_rn(x, inv), __fadd_rn(1.0f, w));
}

// Rotates the pair (i, i + half) of `x` at a table row (:265-274).
__device__ __forceinline__ void exact_rope_pair(float *x, uint32_t i, uint32_t half,
                                                float cs, float sn) {
    float a = x[i], b = x[i + half];
    x[i] = __fsub_rn(__fmul_rn(a, cs), __fmul_rn(b, sn));
    x[i + half] = __fadd_rn(__fmul_rn(b, cs), __fmul_rn(a, sn));
}

// Normalise + rotate a head vector held in shared memory; `scratch_inv` is
// one float of shared memory per head.  Thread `owner` computes the
// statistic sequentially, then the CTA applies it.
__device__ void exact_norm_rope_shared(float *x, uint32_t n, const float *w, float eps,
                                       const QsaWeightsDev &wd, uint32_t rot,
                                       uint32_t pos, float *inv_slot, bool &bad) {
    if (threadIdx.x == 0) *inv_slot = exact_rms_inverse(x, n, eps);
    __syncthreads();
    float inv = *inv_slot;
    if (!isfinite(inv)) bad = true;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) {
        x[i] = exact_norm_apply(x[i], inv, w[i]);
        if (!isfinite(x[i])) bad = true;
    }
    __syncthreads();
    const uint32_t half = rot / 2;
    const float *cs = wd.rope_cos + (size_t)pos * half;
    const float *sn = wd.rope_sin + (size_t)pos * half;
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x) {
        exact_rope_pair(x, i, half, cs[i], sn[i]);
        if (!isfinite(x[i]) || !isfinite(x[i + half])) bad = true;
    }
    __syncthreads();
}

// Key of block `bi` from its raw index keys, exactly as :614-631, by the
// whole CTA: per-feature means in parallel (each a sequential sum over the
// block's rows), the RMS statistic by one thread in the reference's order,
// then norm and RoPE in parallel; written feature-major into s.block_keys.
// `vec` holds di floats of shared memory, `inv_slot` one more.  All threads
// of the CTA must call it; returns false on a non-finite value.
__device__ bool cta_block_key(const QsaDims &d, const QsaWeightsDev &w, const QsaSeq &s,
                              uint32_t bi, float *vec, float *inv_slot) {
    const uint32_t di = d.index_dim;
    bool bad = false;
    for (uint32_t f = threadIdx.x; f < di; f += blockDim.x) {
        float sum = 0.0f;
        for (uint32_t o = 0; o < d.block; ++o)
            sum = __fadd_rn(sum, s.raw[(size_t)(bi * d.block + o) * di + f]);
        vec[f] = __fdiv_rn(sum, (float)d.block);
    }
    __syncthreads();
    if (threadIdx.x == 0) *inv_slot = exact_rms_inverse(vec, di, d.eps);
    __syncthreads();
    const float inv = *inv_slot;
    if (!isfinite(inv)) bad = true;
    for (uint32_t f = threadIdx.x; f < di; f += blockDim.x) vec[f] = exact_norm_apply(vec[f], inv, w.ik_norm[f]);
    __syncthreads();
    const uint32_t half = d.rotary / 2, bpos = bi * d.block;
    for (uint32_t i = threadIdx.x; i < half; i += blockDim.x)
        exact_rope_pair(vec, i, half, w.rope_cos[(size_t)bpos * half + i], w.rope_sin[(size_t)bpos * half + i]);
    __syncthreads();
    const uint32_t ld = block_key_ld(s.capacity, d.block);
    for (uint32_t f = threadIdx.x; f < di; f += blockDim.x) {
        if (!isfinite(vec[f])) bad = true;
        s.block_keys[(size_t)f * ld + bi] = vec[f];
    }
    return !bad;
}

// bf16 hi (round to nearest) and lo (the residual, rounded) of v at
// row[i] and row[width + i].
__device__ __forceinline__ void split_store16(uint16_t *row, uint32_t i, uint32_t width, float v) {
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    row[i] = __bfloat16_as_ushort(hi);
    row[width + i] = __bfloat16_as_ushort(__float2bfloat16_rn(v - __bfloat162float(hi)));
}

__global__ void qsa_split_rows_kernel(const float *__restrict__ src, uint16_t *__restrict__ dst, uint64_t length,
                                      uint32_t kv_heads, uint64_t capacity) {
    const uint64_t n = length * kv_heads * 256u;
    for (uint64_t e = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; e < n; e += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = e / (kv_heads * 256u);
        const uint32_t h = (uint32_t)(e / 256u % kv_heads), i = (uint32_t)(e % 256u);
        split_store16(dst + ((uint64_t)h * capacity + t) * kQsaSplitRow, i, 256u, src[e]);
    }
}

void launch_qsa_split_rows(const float *src, uint16_t *dst, uint64_t length, uint32_t kv_heads, uint64_t capacity,
                           cudaStream_t stream) {
    if (length == 0) return;
    const uint64_t n = length * kv_heads * 256u;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 148ull * 16);
    qsa_split_rows_kernel<<<blocks, 256, 0, stream>>>(src, dst, length, kv_heads, capacity);
    count_launch();
}

// ------------------------------------------------------------ prepare
//
// grid (B, Hq + Hkv + Hi + 1); 128 threads.  blockIdx.y selects one head:
// a query head (-> q_out), a key head (-> key cache row `pos`, with the
// head's values), an index-query head (-> iq_out), or the raw index key
// (-> raw cache row `pos`, then the key of the block this token completes).
// Each head's RMS statistic is a sequential sum in the reference's order.

constexpr int kPrepThreads = 128;

__global__ void __launch_bounds__(kPrepThreads)
qsa_prepare_kernel(QsaDims d, QsaWeightsDev w, QsaBatch bt,
                   const float *__restrict__ proj, uint32_t ldp,
                   const float *__restrict__ iproj, uint32_t ldi,
                   float *__restrict__ q_out, float *__restrict__ iq_out,
                   bool inline_block_key, bool index_queries, bool queries, ErrorWord err) {
    pdl_wait();
    extern __shared__ float sh[];   // max(d, di) floats + 1
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x;
    uint32_t role = blockIdx.y;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t pos = s.length;
    const float *prow = proj + (size_t)b * ldp;
    const float *irow = iproj + (size_t)b * ldi;
    const uint32_t hd = d.head_dim, di = d.index_dim;
    const uint32_t kvw = d.kv_heads * hd;
    float *vec = sh;
    float *inv_slot = sh + max(hd, di);
    bool bad = false;

    if (role < d.q_heads) {
        if (!queries) return;   // whole CTA: this entry's attention runs on another rank
        // query head: q part of the interleaved [q | gate] rows of the head
        const uint32_t h = role;
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) vec[i] = prow[(size_t)h * 2 * hd + i];
        __syncthreads();
        exact_norm_rope_shared(vec, hd, w.q_norm, d.eps, w, d.rotary, pos, inv_slot, bad);
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) q_out[((size_t)b * d.q_heads + h) * hd + i] = vec[i];
    } else if ((role -= d.q_heads) < d.kv_heads) {
        // key head -> key cache; the head's values are copied as projected
        const uint32_t h = role;
        const float *kproj = prow + (size_t)2 * d.q_heads * hd;
        const float *vproj = kproj + kvw;
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) vec[i] = kproj[h * hd + i];
        __syncthreads();
        exact_norm_rope_shared(vec, hd, w.k_norm, d.eps, w, d.rotary, pos, inv_slot, bad);
        const size_t split_row = ((size_t)h * s.capacity + pos) * kQsaSplitRow;   // used when hd == 256
        for (uint32_t i = threadIdx.x; i < hd; i += blockDim.x) {
            s.key[(size_t)pos * kvw + h * hd + i] = vec[i];
            const float v = vproj[h * hd + i];
            if (!isfinite(v)) bad = true;
            s.value[(size_t)pos * kvw + h * hd + i] = v;
            if (s.key_split != nullptr) {
                split_store16(s.key_split + split_row, i, hd, vec[i]);
                split_store16(s.value_split + split_row, i, hd, v);
            }
        }
    } else if ((role -= d.kv_heads) < d.index_heads) {
        if (!index_queries) return;   // whole CTA: this entry is scored elsewhere
        const uint32_t h = role;
        for (uint32_t i = threadIdx.x; i < di; i += blockDim.x) vec[i] = irow[h * di + i];
        __syncthreads();
        exact_norm_rope_shared(vec, di, w.iq_norm, d.eps, w, d.rotary, pos, inv_slot, bad);
        for (uint32_t i = threadIdx.x; i < di; i += blockDim.x) iq_out[((size_t)b * d.index_heads + h) * di + i] = vec[i];
    } else {
        // raw index key -> raw cache row `pos`
        const float *rk = irow + (size_t)d.index_heads * di;
        for (uint32_t i = threadIdx.x; i < di; i += blockDim.x) {
            const float v = rk[i];
            if (!isfinite(v)) bad = true;
            s.raw[(size_t)pos * di + i] = v;
        }
        __syncthreads();
        // the token completes a block: cache that block's key
        if (inline_block_key && (pos + 1) % d.block == 0)
            if (!cta_block_key(d, w, s, pos / d.block, vec, inv_slot)) bad = true;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) qsa_raise(err, kErrNonFinite);
}

void launch_qsa_prepare(const QsaDims &d, const QsaWeightsDev &w,
                        const QsaBatch &b, uint32_t batch, const float *proj,
                        uint32_t ldp, const float *iproj, uint32_t ldi,
                        float *q_out, float *iq_out, bool inline_block_key,
                        bool index_queries, bool queries, ErrorWord err, cudaStream_t stream) {
    size_t smem = (std::max(d.head_dim, d.index_dim) + 1) * sizeof(float);
    dim3 grid(batch, d.q_heads + d.kv_heads + d.index_heads + 1);
    KernelTimer timer("qsa_prepare", stream);
    launch_pdl(qsa_prepare_kernel, grid, kPrepThreads, smem, stream, d, w, b, proj, ldp, iproj, ldi,
               q_out, iq_out, inline_block_key, index_queries, queries, err);
    count_launch();
}

// ------------------------------------------------------------ block keys
//
// grid (end - first); 128 threads; one CTA per block key.
__global__ void __launch_bounds__(kPrepThreads)
qsa_block_keys_kernel(QsaDims d, QsaWeightsDev w, QsaSeq s, uint32_t first, ErrorWord err) {
    pdl_wait();
    extern __shared__ float vec[];   // di floats + 1
    const bool ok = cta_block_key(d, w, s, first + blockIdx.x, vec, vec + d.index_dim);
    if (__syncthreads_or(!ok) && threadIdx.x == 0) qsa_raise(err, kErrNonFinite);
}

void launch_qsa_block_keys(const QsaDims &d, const QsaWeightsDev &w,
                           const QsaSeq &s, uint32_t first_block,
                           uint32_t end_block, ErrorWord err,
                           cudaStream_t stream) {
    if (end_block <= first_block) return;
    const size_t smem = (d.index_dim + 1) * sizeof(float);
    KernelTimer timer("qsa_block_keys", stream);
    launch_pdl(qsa_block_keys_kernel, end_block - first_block, kPrepThreads, smem, stream, d, w, s, first_block,
               err);
    count_launch();
}

// ------------------------------------------------------------ score
//
// Score of block bi for one entry: the sum over index heads of
// max(0, q_h . key_bi) (each dot a sequential F32 sum over the features,
// products and sums rounded separately as in the reference), / sqrt(di).
//
// grid (ceil(max_blocks / 128), ceil(B / E)), 128 threads, one block per
// thread.  E = 4 when the entries are consecutive tokens of one sequence (a
// prefill chunk: the same block keys), so each key value read from memory
// feeds the products of four entries; else 1.  The features go in groups
// of 8: the thread's 8 key values in registers, each (entry, head)'s 8 query
// values as two 16-byte shared-memory loads.  Products and sums use the
// correctly rounded scalar intrinsics in the reference's order (a paired
// f32x2 multiply + add is not guaranteed to stay unfused, and the scores
// decide a discrete selection).

constexpr uint32_t kScoreThreads = 128;
constexpr uint32_t kScoreHeads = 4;      // index heads per pass

template <int E>
__global__ void __launch_bounds__(kScoreThreads)
qsa_score_kernel(QsaDims d, QsaBatch bt, uint32_t batch, const float *__restrict__ iq,
                 float *__restrict__ scores, uint32_t ld_scores, ErrorWord err) {
    pdl_wait();
    extern __shared__ __align__(16) float qsh[];   // [E][Hi * di]
    if (qsa_error_raised(err)) return;
    const uint32_t e0 = blockIdx.y * E;
    const uint32_t ne = min((uint32_t)E, batch - e0);
    uint32_t nb[E];
    uint32_t nb_max = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        nb[e] = (uint32_t)e < ne ? (batch_seq(bt, e0 + e).length + 1) / d.block : 0u;
        nb_max = max(nb_max, nb[e]);
    }
    if (blockIdx.x * kScoreThreads >= nb_max) return;   // uniform over the CTA
    const uint32_t n = d.index_heads * d.index_dim;
    for (uint32_t i = threadIdx.x; i < E * n; i += kScoreThreads)
        qsh[i] = i / n < ne ? iq[(size_t)e0 * n + i] : 0.0f;
    __syncthreads();
    const uint32_t bi = blockIdx.x * kScoreThreads + threadIdx.x;
    if (bi >= nb_max) return;
    const QsaSeq s = batch_seq(bt, e0);   // E > 1: every entry reads this sequence's keys
    const uint32_t ld = block_key_ld(s.capacity, d.block);
    const float *key = s.block_keys + bi;
    float score[E];
#pragma unroll
    for (int e = 0; e < E; ++e) score[e] = 0.0f;
    for (uint32_t h0 = 0; h0 < d.index_heads; h0 += kScoreHeads) {
        const uint32_t nh = min(kScoreHeads, d.index_heads - h0);
        float dot[E][kScoreHeads];
#pragma unroll
        for (int e = 0; e < E; ++e)
#pragma unroll
            for (uint32_t h = 0; h < kScoreHeads; ++h) dot[e][h] = 0.0f;
        const float *q0 = qsh + h0 * d.index_dim;
        // 8-feature groups while the 16-byte query loads stay aligned
        // (index_dim a multiple of 8), then one feature at a time
        const uint32_t fvec = (d.index_dim & 7u) == 0 ? d.index_dim : 0u;
        for (uint32_t f0 = 0; f0 < fvec; f0 += 8) {
            float kv[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) kv[j] = key[(size_t)(f0 + j) * ld];
#pragma unroll
            for (int e = 0; e < E; ++e)
#pragma unroll
                for (uint32_t h = 0; h < kScoreHeads; ++h) {
                    if (h < nh) {
                        const float *qp = q0 + (size_t)e * n + h * d.index_dim + f0;
                        const float4 qa = *reinterpret_cast<const float4 *>(qp);
                        const float4 qb = *reinterpret_cast<const float4 *>(qp + 4);
                        const float qv[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                        float acc = dot[e][h];
#pragma unroll
                        for (int j = 0; j < 8; ++j) acc = __fadd_rn(acc, __fmul_rn(qv[j], kv[j]));
                        dot[e][h] = acc;
                    }
                }
        }
        for (uint32_t f = fvec; f < d.index_dim; ++f) {
            const float kvf = key[(size_t)f * ld];
#pragma unroll
            for (int e = 0; e < E; ++e)
#pragma unroll
                for (uint32_t h = 0; h < kScoreHeads; ++h)
                    if (h < nh)
                        dot[e][h] = __fadd_rn(dot[e][h], __fmul_rn(q0[(size_t)e * n + h * d.index_dim + f], kvf));
        }
        // positive dots, added in head order
#pragma unroll
        for (int e = 0; e < E; ++e)
#pragma unroll
            for (uint32_t h = 0; h < kScoreHeads; ++h)
                if (h < nh && dot[e][h] > 0.0f) score[e] = __fadd_rn(score[e], dot[e][h]);
    }
    bool bad = false;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        if ((uint32_t)e < ne && bi < nb[e]) {
            const float sc = __fdiv_rn(score[e], d.sqrt_index_dim);
            bad |= !isfinite(sc);
            scores[(size_t)(e0 + e) * ld_scores + bi] = sc;
        }
    }
    if (bad) qsa_raise(err, kErrNonFinite);
}

// f32x2 forms of a separately rounded product and sum (two lanes per
// instruction, each lane rounded exactly as __fmul_rn / __fadd_rn; the
// explicit .rn keeps them from being contracted into a fused multiply-add)
__device__ __forceinline__ uint64_t sc_pair(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void sc_unpair(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t sc_mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ uint64_t sc_add2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

// Block scores of E consecutive entries of one sequence (E a multiple of 4)
// for NB blocks per thread (blocks bi + j * kScoreThreads): every block-key
// load serves E entries, every query read from shared memory serves NB
// blocks, and the E dots of one (head, feature) step run as E / 2 paired
// products and sums.  The queries sit in shared memory as
// [head][feature][entry].  Same arithmetic, in the same order, per entry
// and block as qsa_score_kernel.
template <int E, int NB>
__global__ void __launch_bounds__(kScoreThreads)
qsa_score_pair_kernel(QsaDims d, QsaBatch bt, uint32_t batch, const float *__restrict__ iq,
                      float *__restrict__ scores, uint32_t ld_scores, ErrorWord err) {
    static_assert(E % 4 == 0, "entries come in float4 groups");
    pdl_wait();
    extern __shared__ __align__(16) float qsh[];   // [Hi][di][E]
    if (qsa_error_raised(err)) return;
    const uint32_t e0 = blockIdx.y * E;
    const uint32_t ne = min((uint32_t)E, batch - e0);
    uint32_t nb[E];
    uint32_t nb_max = 0;
#pragma unroll
    for (int e = 0; e < E; ++e) {
        nb[e] = (uint32_t)e < ne ? (batch_seq(bt, e0 + e).length + 1) / d.block : 0u;
        nb_max = max(nb_max, nb[e]);
    }
    const uint32_t cta_blocks = NB * kScoreThreads;
    if (blockIdx.x * cta_blocks >= nb_max) return;   // uniform over the CTA
    const uint32_t di = d.index_dim, n = d.index_heads * di;
    for (uint32_t i = threadIdx.x; i < E * n; i += kScoreThreads) {
        const uint32_t e = i % E, hf = i / E;
        qsh[i] = e < ne ? iq[(size_t)(e0 + e) * n + hf] : 0.0f;
    }
    __syncthreads();
    const uint32_t bi0 = blockIdx.x * cta_blocks + threadIdx.x;
    if (bi0 >= nb_max) return;
    const QsaSeq s = batch_seq(bt, e0);
    const uint32_t ld = block_key_ld(s.capacity, d.block);
    bool live[NB];
    const float *key[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        live[j] = bi0 + j * kScoreThreads < nb_max;
        key[j] = s.block_keys + (live[j] ? bi0 + j * kScoreThreads : bi0);
    }
    float score[NB][E];
#pragma unroll
    for (int j = 0; j < NB; ++j)
#pragma unroll
        for (int e = 0; e < E; ++e) score[j][e] = 0.0f;
    for (uint32_t h0 = 0; h0 < d.index_heads; h0 += kScoreHeads) {
        const uint32_t nh = min(kScoreHeads, d.index_heads - h0);
        uint64_t dot[NB][kScoreHeads][E / 2];
#pragma unroll
        for (int j = 0; j < NB; ++j)
#pragma unroll
            for (uint32_t h = 0; h < kScoreHeads; ++h)
#pragma unroll
                for (int p = 0; p < E / 2; ++p) dot[j][h][p] = 0ull;   // (+0.0f, +0.0f)
        auto step = [&](uint32_t f, const float (&kf)[NB]) {
            uint64_t k2[NB];
#pragma unroll
            for (int j = 0; j < NB; ++j) k2[j] = sc_pair(kf[j], kf[j]);
#pragma unroll
            for (uint32_t h = 0; h < kScoreHeads; ++h) {
                if (h < nh) {
                    const float *qp = qsh + ((size_t)(h0 + h) * di + f) * E;
#pragma unroll
                    for (int p = 0; p < E / 4; ++p) {
                        const float4 q4 = *reinterpret_cast<const float4 *>(qp + 4 * p);
                        const uint64_t qa = sc_pair(q4.x, q4.y), qb = sc_pair(q4.z, q4.w);
#pragma unroll
                        for (int j = 0; j < NB; ++j) {
                            dot[j][h][2 * p] = sc_add2(dot[j][h][2 * p], sc_mul2(qa, k2[j]));
                            dot[j][h][2 * p + 1] = sc_add2(dot[j][h][2 * p + 1], sc_mul2(qb, k2[j]));
                        }
                    }
                }
            }
        };
        uint32_t f = 0;
        for (; f + 4 <= di; f += 4) {
            float kv[4][NB];
#pragma unroll
            for (int t = 0; t < 4; ++t)
#pragma unroll
                for (int j = 0; j < NB; ++j) kv[t][j] = key[j][(size_t)(f + t) * ld];
#pragma unroll
            for (int t = 0; t < 4; ++t) step(f + t, kv[t]);
        }
        for (; f < di; ++f) {
            float kv[NB];
#pragma unroll
            for (int j = 0; j < NB; ++j) kv[j] = key[j][(size_t)f * ld];
            step(f, kv);
        }
        // positive dots, added in head order
#pragma unroll
        for (int j = 0; j < NB; ++j)
#pragma unroll
            for (uint32_t h = 0; h < kScoreHeads; ++h) {
                if (h >= nh) continue;
#pragma unroll
                for (int p = 0; p < E / 2; ++p) {
                    float lo, hi;
                    sc_unpair(dot[j][h][p], lo, hi);
                    if (lo > 0.0f) score[j][2 * p] = __fadd_rn(score[j][2 * p], lo);
                    if (hi > 0.0f) score[j][2 * p + 1] = __fadd_rn(score[j][2 * p + 1], hi);
                }
            }
    }
    bool bad = false;
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        const uint32_t bi = bi0 + j * kScoreThreads;
        if (!live[j]) continue;
#pragma unroll
        for (int e = 0; e < E; ++e) {
            if ((uint32_t)e < ne && bi < nb[e]) {
                const float sc = __fdiv_rn(score[j][e], d.sqrt_index_dim);
                bad |= !isfinite(sc);
                scores[(size_t)(e0 + e) * ld_scores + bi] = sc;
            }
        }
    }
    if (bad) qsa_raise(err, kErrNonFinite);
}

void launch_qsa_score(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                      const float *iq, float *scores, uint32_t ld_scores,
                      uint32_t max_blocks, bool shared_sequence, ErrorWord err, cudaStream_t stream) {
    if (max_blocks == 0) return;
    const size_t n = (size_t)d.index_heads * d.index_dim;
    KernelTimer timer("qsa_score", stream);
    // entries of one sequence share each key load four ways, once that
    // still leaves about four waves of CTAs
    const uint32_t xblocks = (max_blocks + kScoreThreads - 1) / kScoreThreads;
    const char *force = getenv("KQ_B200_SCORE_SHARED");   // tests: 1 = always share when possible
    const bool big = xblocks * ((batch + 3) / 4) >= 4u * 148u || (force && atoi(force) == 1);
    const bool big8 = xblocks * ((batch + 7) / 8) >= 4u * 148u || (force && atoi(force) == 1);
    if (shared_sequence && batch > 1 && big8) {
        // eight entries per key load, two blocks per query read, paired products
        dim3 grid((max_blocks + 2 * kScoreThreads - 1) / (2 * kScoreThreads), (batch + 7) / 8);
        launch_pdl(qsa_score_pair_kernel<8, 2>, grid, kScoreThreads, 8 * n * sizeof(float), stream, d, b, batch,
                   iq, scores, ld_scores, err);
    } else if (shared_sequence && batch > 1 && big) {
        dim3 grid(xblocks, (batch + 3) / 4);
        launch_pdl(qsa_score_kernel<4>, grid, kScoreThreads, 4 * n * sizeof(float), stream, d, b, batch, iq, scores,
                   ld_scores, err);
    } else {
        dim3 grid((max_blocks + kScoreThreads - 1) / kScoreThreads, batch);
        launch_pdl(qsa_score_kernel<1>, grid, kScoreThreads, n * sizeof(float), stream, d, b, batch, iq, scores,
                   ld_scores, err);
    }
    count_launch();
}

// ------------------------------------------------------------ select
//
// grid (B); 1024 threads.  Exact stable top-k: radix select (4 passes of 8
// bits over order-preserving score keys) finds the k-th largest key T; all
// keys > T are taken plus the lowest-id keys == T; the k winners are then
// bitonic-sorted by (key desc, id asc), which is the reference's insertion
// order (:328-359).

constexpr int kSelThreads = 1024;
constexpr int kSelMax = 1024;   // power of two >= the selection limit

__device__ __forceinline__ uint32_t order_key(float v) {
    if (v == 0.0f) v = 0.0f;   // -0 and +0 compare equal in the reference
    uint32_t bits = __float_as_uint(v);
    return (bits & 0x80000000u) ? ~bits : (bits | 0x80000000u);
}

__global__ void __launch_bounds__(kSelThreads)
qsa_select_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ scores,
                  uint32_t ld_scores, uint32_t *__restrict__ selected,
                  uint32_t *__restrict__ selected_count, uint32_t rank_order, ErrorWord err) {
    pdl_wait();
    __shared__ uint32_t hist[256];
    __shared__ uint32_t s_prefix, s_need, s_tie_base, s_abv_base;
    __shared__ unsigned long long cand[kSelMax];
    __shared__ uint32_t warp_tot[kSelThreads / 32], warp_abv[kSelThreads / 32];
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t n = (s.length + 1) / d.block;
    const uint32_t k = min(n, d.topk);
    const float *sc = scores + (size_t)b * ld_scores;
    const uint32_t tid = threadIdx.x;
    if (k > kSelMax) {   // configuration guard: host rejects such configs
        if (tid == 0) qsa_raise(err, kErrSelection);
        return;
    }
    if (tid == 0) { s_prefix = 0; s_need = k; s_tie_base = 0; s_abv_base = 0; }
    uint32_t mask = 0;
    __syncthreads();
    if (k > 0 && k < n) {
        for (int pass = 3; pass >= 0; --pass) {
            for (uint32_t i = tid; i < 256; i += blockDim.x) hist[i] = 0;
            __syncthreads();
            const uint32_t prefix = s_prefix;
            const int shift = pass * 8;
            for (uint32_t i = tid; i < n; i += blockDim.x) {
                uint32_t key = order_key(sc[i]);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid < 32) {
                // highest bin whose suffix count reaches `need`: lane l owns
                // bins 255-8l .. 248-8l (descending), a warp scan finds the lane
                const uint32_t need = s_need;
                uint32_t part = 0;
#pragma unroll
                for (int e = 0; e < 8; ++e) part += hist[255 - 8 * tid - e];
                uint32_t incl = part;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const uint32_t up = __shfl_up_sync(0xffffffffu, incl, o);
                    if ((int)tid >= o) incl += up;
                }
                const uint32_t excl = incl - part;
                const unsigned hit = __ballot_sync(0xffffffffu, incl >= need);
                const int lane_hit = hit ? __ffs(hit) - 1 : 31;
                if ((int)tid == lane_hit) {
                    uint32_t acc = excl, bin = 255 - 8 * tid - 7;
                    for (int e = 0; e < 8; ++e) {
                        const uint32_t bb = 255 - 8 * tid - e;
                        if (acc + hist[bb] >= need) { bin = bb; break; }
                        acc += hist[bb];
                    }
                    s_need = need - acc;
                    s_prefix = prefix | (bin << shift);
                }
            }
            mask |= 255u << shift;
            __syncthreads();
        }
    }
    // gather: keys above the threshold, then the s_need lowest-id ties.
    // Every selected id's position in id order is (#above before it) +
    // min(#ties before it, ties needed), from block-wide prefix counts, so
    // the id-ordered output needs no sort; the rank-ordered one is sorted.
    const bool take_all = (k == n);
    const uint32_t thr = s_prefix;
    const uint32_t ties_needed = take_all ? 0 : s_need;
    if (rank_order) {
        for (uint32_t i = tid; i < kSelMax; i += blockDim.x) cand[i] = 0ull;
    }
    __syncthreads();
    const uint32_t lane = tid & 31, warp = tid >> 5;
    const unsigned lt = (1u << lane) - 1u;
    for (uint32_t start = 0; start < n; start += blockDim.x) {
        uint32_t i = start + tid;
        uint32_t key = 0;
        bool valid = i < n;
        if (valid) key = order_key(sc[i]);
        bool above = valid && (take_all || key > thr);
        bool tie = valid && !take_all && key == thr;
        const unsigned tb = __ballot_sync(0xffffffffu, tie), ab = __ballot_sync(0xffffffffu, above);
        if (lane == 0) {
            warp_tot[warp] = __popc(tb);
            warp_abv[warp] = __popc(ab);
        }
        __syncthreads();
        uint32_t tbefore = 0, abefore = 0;
        for (uint32_t w = 0; w < warp; ++w) {
            tbefore += warp_tot[w];
            abefore += warp_abv[w];
        }
        const uint32_t tie_rank = s_tie_base + tbefore + __popc(tb & lt);
        const uint32_t abv_rank = s_abv_base + abefore + __popc(ab & lt);
        if (above || (tie && tie_rank < ties_needed)) {
            if (rank_order) {
                const uint32_t slot = abv_rank + min(tie_rank, ties_needed);
                if (slot < kSelMax) cand[slot] = ((unsigned long long)key << 32) | (uint32_t)(~i);
            } else {
                selected[(size_t)b * d.topk + abv_rank + min(tie_rank, ties_needed)] = i;
            }
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t tt = 0, ta = 0;
            for (uint32_t w = 0; w < blockDim.x / 32; ++w) {
                tt += warp_tot[w];
                ta += warp_abv[w];
            }
            s_tie_base += tt;
            s_abv_base += ta;
        }
        __syncthreads();
    }
    const uint32_t taken = s_abv_base + min(s_tie_base, ties_needed);
    if (rank_order) {
        // bitonic sort, descending by (score, -id): the reference's rank order
        for (uint32_t size = 2; size <= kSelMax; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                for (uint32_t i = tid; i < kSelMax; i += blockDim.x) {
                    uint32_t j = i ^ stride;
                    if (j > i) {
                        bool desc = (i & size) == 0;
                        unsigned long long a = cand[i], c = cand[j];
                        if ((a < c) == desc) { cand[i] = c; cand[j] = a; }
                    }
                }
                __syncthreads();
            }
        }
        for (uint32_t i = tid; i < k; i += blockDim.x)
            selected[(size_t)b * d.topk + i] = ~(uint32_t)(cand[i] & 0xffffffffull);
    }
    if (tid == 0) {
        selected_count[b] = k;
        if (taken != k) qsa_raise(err, kErrSelection);
    }
}

void launch_qsa_select(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                       const float *scores, uint32_t ld_scores,
                       uint32_t *selected, uint32_t *selected_count,
                       bool rank_order, ErrorWord err, cudaStream_t stream) {
    KernelTimer timer("qsa_select", stream);
    launch_pdl(qsa_select_kernel, batch, kSelThreads, 0, stream, d, b, scores, ld_scores, selected,
               selected_count, rank_order ? 1u : 0u, err);
    count_launch();
}

// ------------------------------------------------------------ attend
//
// grid (B, Hkv, splits); 256 threads = 8 warps.  A split owns a contiguous
// range of the selected-token list.  Each warp takes every 8th token of the
// range, one token at a time: its lanes hold FPL features of the K and V
// rows, compute the logits of all query heads sharing the KV head (warp
// shuffle reductions) and keep an online softmax per head.  The warps'
// partial states are merged in shared memory and written per split.

template <int FPL, int HPW>
__global__ void __launch_bounds__(256)
qsa_attend_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ q,
                  const uint32_t *__restrict__ selected,
                  const uint32_t *__restrict__ selected_count,
                  float *__restrict__ part_o, float *__restrict__ part_ml,
                  uint32_t splits, ErrorWord err) {
    pdl_wait();
    extern __shared__ float smem[];   // [8 warps][HPW][hd + 2]
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t pos = s.length;
    const uint32_t nblocks = (pos + 1) / d.block;
    const uint32_t tail = (pos + 1) % d.block;
    const uint32_t ksel = min(selected_count[b], min(nblocks, d.topk));
    const uint32_t ntok = ksel * d.block + tail;
    const uint32_t per = (ntok + splits - 1) / splits;
    const uint32_t t0 = split * per, t1 = min(ntok, t0 + per);
    const uint32_t hd = d.head_dim;
    const uint32_t kvw = d.kv_heads * hd;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t heads = d.repeat;   // query heads of this KV head (<= HPW)

    float qr[HPW][FPL];
    float acc[HPW][FPL];
    float m[HPW], l[HPW];
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.0f;
#pragma unroll
        for (int f = 0; f < FPL; ++f) {
            uint32_t feat = lane * FPL + f;
            acc[h][f] = 0.0f;
            qr[h][f] = ((uint32_t)h < heads && feat < hd)
                           ? q[((size_t)b * d.q_heads + kvh * heads + h) * hd + feat] : 0.0f;
        }
    }
    const float scale = d.sqrt_head_dim;
    for (uint32_t i = t0 + warp; i < t1; i += 8) {
        uint32_t tok;
        if (i < ksel * d.block) {
            const uint32_t blk = selected[(size_t)b * d.topk + i / d.block];
            if (blk >= nblocks) continue;   // never taken: select raises an error first
            tok = blk * d.block + i % d.block;
        } else {
            tok = nblocks * d.block + (i - ksel * d.block);
        }
        const float *krow = s.key + (size_t)tok * kvw + kvh * hd;
        const float *vrow = s.value + (size_t)tok * kvw + kvh * hd;
        float kv[FPL], vv[FPL];
        if (FPL % 4 == 0) {
#pragma unroll
            for (int f = 0; f < FPL; f += 4) {
                float4 k4 = *reinterpret_cast<const float4 *>(krow + lane * FPL + f);
                float4 v4 = *reinterpret_cast<const float4 *>(vrow + lane * FPL + f);
                kv[f] = k4.x; kv[f + 1] = k4.y; kv[f + 2] = k4.z; kv[f + 3] = k4.w;
                vv[f] = v4.x; vv[f + 1] = v4.y; vv[f + 2] = v4.z; vv[f + 3] = v4.w;
            }
        } else {
#pragma unroll
            for (int f = 0; f < FPL; ++f) {
                uint32_t feat = lane * FPL + f;
                kv[f] = feat < hd ? krow[feat] : 0.0f;
                vv[f] = feat < hd ? vrow[feat] : 0.0f;
            }
        }
#pragma unroll
        for (int h = 0; h < HPW; ++h) {
            float dot = 0.0f;
#pragma unroll
            for (int f = 0; f < FPL; ++f) dot = fmaf(qr[h][f], kv[f], dot);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            float logit = dot / scale;
            float mn = fmaxf(m[h], logit);
            float corr = expf(m[h] - mn);
            float p = expf(logit - mn);
            l[h] = l[h] * corr + p;
#pragma unroll
            for (int f = 0; f < FPL; ++f) acc[h][f] = fmaf(p, vv[f], acc[h][f] * corr);
            m[h] = mn;
        }
    }
    // merge the 8 warps
    const uint32_t stride = hd + 2;
    float *mine = smem + (size_t)warp * HPW * stride;
#pragma unroll
    for (int h = 0; h < HPW; ++h) {
#pragma unroll
        for (int f = 0; f < FPL; ++f) {
            uint32_t feat = lane * FPL + f;
            if (feat < hd) mine[h * stride + feat] = acc[h][f];
        }
        if (lane == 0) { mine[h * stride + hd] = m[h]; mine[h * stride + hd + 1] = l[h]; }
    }
    __syncthreads();
    for (uint32_t idx = threadIdx.x; idx < heads * hd; idx += blockDim.x) {
        uint32_t h = idx / hd, feat = idx % hd;
        float mx = -INFINITY;
        for (int wv = 0; wv < 8; ++wv) mx = fmaxf(mx, smem[(size_t)wv * HPW * stride + h * stride + hd]);
        float o = 0.0f, ll = 0.0f;
        for (int wv = 0; wv < 8; ++wv) {
            const float *src = smem + (size_t)wv * HPW * stride + h * stride;
            float mw = src[hd];
            float c = (mw == -INFINITY) ? 0.0f : expf(mw - mx);
            o += src[feat] * c;
            ll += src[hd + 1] * c;
        }
        uint32_t qh = kvh * heads + h;
        size_t slot = ((size_t)b * d.q_heads + qh) * splits + split;
        part_o[slot * hd + feat] = o;
        if (feat == 0) { part_ml[slot * 2] = mx; part_ml[slot * 2 + 1] = ll; }
    }
}

// Tiled variant for head dimensions 128 / 256 (the BASELINE shapes).
// grid (B, Hkv, splits); 256 threads = 8 warps; warp h owns query head
// kvh*repeat + h.  The split's token range is walked in tiles of 16
// selected tokens whose K and V rows are staged with cp.async into
// double-buffered shared memory (the next tile loads while the current one
// is consumed); 73 KB of shared memory lets three CTAs share an SM.
// Logits: lanes l and l+16 each take half of token l's dot product
// (float4 reads of padded K rows, conflict-free) and combine with a shuffle;
// online softmax per warp; P.V: lane l owns features [4l, 4l+4) and
// [HD/2 + 4l, HD/2 + 4l + 4) (consecutive lanes, conflict-free).

constexpr int kAtTile = 16;

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;\n" ::); }

template <int HD>
__global__ void __launch_bounds__(256, 3)
qsa_attend_tiled_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ q,
                        const uint32_t *__restrict__ selected,
                        const uint32_t *__restrict__ selected_count,
                        float *__restrict__ part_o, float *__restrict__ part_ml,
                        uint32_t splits, ErrorWord err) {
    pdl_wait();
    constexpr int KLD = HD + 4;          // padded K row (conflict-free float4 reads)
    constexpr int HALF = HD / 2;
    constexpr int CH = HD / 4;           // 16-byte chunks per row
    extern __shared__ __align__(16) float sm[];
    float *qs = sm;                                  // [8][HD]
    float *ks = qs + 8 * HD;                         // [2][16][KLD]
    float *vs = ks + 2 * kAtTile * KLD;              // [2][16][HD]
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t pos = s.length;
    const uint32_t nblocks = (pos + 1) / d.block;
    const uint32_t tail = (pos + 1) % d.block;
    const uint32_t ksel = min(selected_count[b], min(nblocks, d.topk));
    const uint32_t ntok = ksel * d.block + tail;
    const uint32_t ntiles = (ntok + kAtTile - 1) / kAtTile;
    const uint32_t per = (ntiles + splits - 1) / splits;
    const uint32_t tile0 = split * per, tile1 = min(ntiles, tile0 + per);
    const uint32_t heads = d.repeat;
    const uint32_t kvw = d.kv_heads * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t *selb = selected + (size_t)b * d.topk;

    for (uint32_t i = threadIdx.x; i < heads * HD; i += blockDim.x)
        qs[i] = q[((size_t)b * d.q_heads + kvh * heads) * HD + i];

    auto token_of = [&](uint32_t i, bool &ok) -> uint32_t {
        ok = i < ntok;
        if (!ok) return 0;
        if (i < ksel * d.block) {
            const uint32_t blk = selb[i / d.block];
            ok = blk < nblocks;
            return ok ? blk * d.block + i % d.block : 0;
        }
        return nblocks * d.block + (i - ksel * d.block);
    };
    auto load_tile = [&](uint32_t tile, int buf) {
        float *kd = ks + buf * kAtTile * KLD;
        float *vd = vs + buf * kAtTile * HD;
        for (int c = threadIdx.x; c < kAtTile * CH; c += blockDim.x) {
            const int t = c / CH, col = (c % CH) * 4;
            bool ok;
            const uint32_t tok = token_of(tile * kAtTile + t, ok);
            if (ok) {
                const size_t off = (size_t)tok * kvw + kvh * HD + col;
                cp_async16(kd + t * KLD + col, s.key + off);
                cp_async16(vd + t * HD + col, s.value + off);
            } else {
                *reinterpret_cast<float4 *>(kd + t * KLD + col) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4 *>(vd + t * HD + col) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
        cp_async_commit();
    };

    float m_run = -INFINITY, l_run = 0.0f;
    float acc[8];
#pragma unroll
    for (int f = 0; f < 8; ++f) acc[f] = 0.0f;
    const float scale = d.sqrt_head_dim;
    const bool active = (uint32_t)warp < heads;
    const int tok_lane = lane & 15, part = lane >> 4;
    const float *qh = qs + warp * HD + part * HALF;

    if (tile0 < tile1) load_tile(tile0, 0);
    for (uint32_t tile = tile0; tile < tile1; ++tile) {
        const int buf = (tile - tile0) & 1;
        if (tile + 1 < tile1) {
            load_tile(tile + 1, buf ^ 1);
            cp_async_wait1();
        } else {
            cp_async_wait0();
        }
        __syncthreads();
        if (active) {
            const float *kr = ks + buf * kAtTile * KLD + tok_lane * KLD + part * HALF;
            float dot = 0.0f;
#pragma unroll 8
            for (int f = 0; f < HALF; f += 4) {
                const float4 qv = *reinterpret_cast<const float4 *>(qh + f);
                const float4 kv = *reinterpret_cast<const float4 *>(kr + f);
                dot = fmaf(qv.x, kv.x, dot);
                dot = fmaf(qv.y, kv.y, dot);
                dot = fmaf(qv.z, kv.z, dot);
                dot = fmaf(qv.w, kv.w, dot);
            }
            dot += __shfl_xor_sync(0xffffffffu, dot, 16);
            bool ok;
            token_of(tile * kAtTile + tok_lane, ok);
            const float logit = ok ? dot / scale : -INFINITY;
            float mt = logit;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float m_new = fmaxf(m_run, mt);
            const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
            const float p = ok ? expf(logit - m_new) : 0.0f;
            float ps = p;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l_run = l_run * corr + ps;
            m_run = m_new;
#pragma unroll
            for (int f = 0; f < 8; ++f) acc[f] *= corr;
            // HD = 128: lanes 16..31 own no features; they read an in-bounds
            // column and their sums are never stored
            const bool pv_lane = lane * 4 < HALF;
            const float *vb = vs + buf * kAtTile * HD + (pv_lane ? lane * 4 : 0);
#pragma unroll 4
            for (int t = 0; t < kAtTile; ++t) {
                const float pt = __shfl_sync(0xffffffffu, p, t);   // lanes without features read row 0..3
                const float4 v0 = *reinterpret_cast<const float4 *>(vb + t * HD);
                const float4 v1 = *reinterpret_cast<const float4 *>(vb + t * HD + HALF);
                acc[0] = fmaf(pt, v0.x, acc[0]);
                acc[1] = fmaf(pt, v0.y, acc[1]);
                acc[2] = fmaf(pt, v0.z, acc[2]);
                acc[3] = fmaf(pt, v0.w, acc[3]);
                acc[4] = fmaf(pt, v1.x, acc[4]);
                acc[5] = fmaf(pt, v1.y, acc[5]);
                acc[6] = fmaf(pt, v1.z, acc[6]);
                acc[7] = fmaf(pt, v1.w, acc[7]);
            }
        }
        __syncthreads();
    }
    if (!active) return;
    const uint32_t qhead = kvh * heads + warp;
    const size_t slot = ((size_t)b * d.q_heads + qhead) * splits + split;
    if (lane * 4 < HALF) {
        *reinterpret_cast<float4 *>(part_o + slot * HD + lane * 4) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        *reinterpret_cast<float4 *>(part_o + slot * HD + HALF + lane * 4) =
            make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
    if (lane == 0) {
        part_ml[slot * 2] = m_run;
        part_ml[slot * 2 + 1] = l_run;
    }
}

// Head-blocked form for head_dim 256 and up to 8 query heads per KV head
// (the BASELINE geometry: 16 query heads over 2 KV heads).  Every K and V
// element of a tile is read from shared memory once and used for all the KV
// head's query heads:
//   QK  warp w scores tokens 2w, 2w+1 of the 16-token tile; lane l holds the
//       8 features [8l, 8l+8) of every query head in registers, forms 8
//       partial dots per token and reduces them with a 9-shuffle
//       reduce-scatter (4 lanes end up with each head's sum);
//   softmax  warp h keeps head h's running max / sum (online softmax);
//   PV  warp w owns features [32w, 32w+32), one per lane, for every head.
// K/V tiles stream through a 3-stage cp.async ring (96 KB), two CTAs per SM.
// f32 pairs for the attention arithmetic (fma.rn.f32x2 / mul.rn.f32x2)
__device__ __forceinline__ uint64_t at_pair(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void at_unpair(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t at_fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ uint64_t at_mul2(uint64_t a, uint64_t b) {
    uint64_t r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}

constexpr int kMhStages = 3;
constexpr int kMhHD = 256;
constexpr int kMhMaxTiles = 32;           // tiles per CTA (the launcher sizes splits for it)
constexpr size_t kMhSmem = (size_t)kMhStages * 2 * kAtTile * kMhHD * 4 + 2 * kAtTile * 8 * 4 + 8 * 4 +
                           (size_t)kMhMaxTiles * kAtTile * 4;

__global__ void __launch_bounds__(256, 2)
qsa_attend_mh_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ q,
                     const uint32_t *__restrict__ selected,
                     const uint32_t *__restrict__ selected_count,
                     float *__restrict__ part_o, float *__restrict__ part_ml,
                     uint32_t splits, ErrorWord err) {
    pdl_wait();
    constexpr int HD = kMhHD;
    extern __shared__ __align__(16) float sm[];
    float *kbuf = sm;                                        // [S][16][HD]
    float *vbuf = kbuf + kMhStages * kAtTile * HD;           // [S][16][HD]
    float *lg = vbuf + kMhStages * kAtTile * HD;             // [16][8] logits
    float *pw = lg + kAtTile * 8;                            // [16][8] weights
    float *corr_s = pw + kAtTile * 8;                        // [8]
    uint32_t *tok_s = reinterpret_cast<uint32_t *>(corr_s + 8);   // [kMhMaxTiles * 16] cache rows
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t pos = s.length;
    const uint32_t nblocks = (pos + 1) / d.block;
    const uint32_t tail = (pos + 1) % d.block;
    const uint32_t ksel = min(selected_count[b], min(nblocks, d.topk));
    const uint32_t ntok = ksel * d.block + tail;
    const uint32_t ntiles = (ntok + kAtTile - 1) / kAtTile;
    const uint32_t per = (ntiles + splits - 1) / splits;
    const uint32_t tile0 = split * per, tile1 = min(ntiles, tile0 + per);
    const uint32_t heads = d.repeat;   // <= 8 (checked by the launcher)
    const uint32_t kvw = d.kv_heads * HD;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t *selb = selected + (size_t)b * d.topk;

    auto token_of = [&](uint32_t i, bool &ok) -> uint32_t {
        ok = i < ntok;
        if (!ok) return 0;
        if (i < ksel * d.block) {
            const uint32_t blk = selb[i / d.block];
            ok = blk < nblocks;
            return ok ? blk * d.block + i % d.block : 0;
        }
        return nblocks * d.block + (i - ksel * d.block);
    };
    // cache row of every token this CTA attends to (UINT32_MAX: none); a
    // split past the sequence's last tile has no tiles (tile1 <= tile0)
    const uint32_t my_tiles = tile1 > tile0 ? tile1 - tile0 : 0u;
    if (my_tiles > (uint32_t)kMhMaxTiles) {
        if (threadIdx.x == 0) qsa_raise(err, kErrSelection);
        return;
    }
    for (uint32_t i = threadIdx.x; i < my_tiles * kAtTile; i += blockDim.x) {
        bool ok;
        const uint32_t tok = token_of(tile0 * kAtTile + i, ok);
        tok_s[i] = ok ? tok : 0xFFFFFFFFu;
    }
    __syncthreads();
    auto load_tile = [&](uint32_t tile) {
        const int buf = (tile - tile0) % kMhStages;
        float *kd = kbuf + buf * kAtTile * HD;
        float *vd = vbuf + buf * kAtTile * HD;
        const uint32_t *tt = tok_s + (tile - tile0) * kAtTile;
        // 16 tokens x 64 chunks of 16 bytes, K and V: 4 + 4 per thread
        for (int c = threadIdx.x; c < kAtTile * (HD / 4); c += blockDim.x) {
            const int t = c >> 6, col = (c & 63) * 4;
            const uint32_t tok = tt[t];
            if (tok != 0xFFFFFFFFu) {
                const size_t off = (size_t)tok * kvw + kvh * HD + col;
                cp_async16(kd + t * HD + col, s.key + off);
                cp_async16(vd + t * HD + col, s.value + off);
            } else {
                *reinterpret_cast<float4 *>(kd + t * HD + col) = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4 *>(vd + t * HD + col) = make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };

    // query features [8 lane, 8 lane + 8) of every head, in registers
    // query features as f32 pairs (paired FMAs: two lanes of math per
    // instruction; attention is checked to tolerance, not bit-exact)
    uint64_t qr[8][4];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
        if ((uint32_t)h < heads) {
            const float *qp = q + ((size_t)b * d.q_heads + kvh * heads + h) * HD + 8 * lane;
            const float4 a = *reinterpret_cast<const float4 *>(qp);
            const float4 c = *reinterpret_cast<const float4 *>(qp + 4);
            qr[h][0] = at_pair(a.x, a.y); qr[h][1] = at_pair(a.z, a.w);
            qr[h][2] = at_pair(c.x, c.y); qr[h][3] = at_pair(c.z, c.w);
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) qr[h][j] = 0ull;
        }
    }
    uint64_t acc2[4];   // heads (0,1), (2,3), (4,5), (6,7) of feature f
#pragma unroll
    for (int i = 0; i < 4; ++i) acc2[i] = 0ull;
    float m_run = -INFINITY, l_run = 0.0f;   // head `warp`'s running softmax state
    const float scale = d.sqrt_head_dim;
    // reduce-scatter: after the three exchange steps lanes {4g..4g+3} hold
    // head g's partial sums, with g = bit4*4 + bit3*2 + bit2 of the lane
    const int my_head = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);

    for (uint32_t t = tile0; t < tile0 + kMhStages - 1; ++t) {
        if (t < tile1) load_tile(t);
        cp_async_commit();
    }
    for (uint32_t tile = tile0; tile < tile1; ++tile) {
        if (tile + kMhStages - 1 < tile1) load_tile(tile + kMhStages - 1);
        cp_async_commit();
        asm volatile("cp.async.wait_group %0;\n" ::"n"(kMhStages - 1));
        __syncthreads();
        const int buf = (tile - tile0) % kMhStages;
        const float *kt = kbuf + buf * kAtTile * HD;
        const float *vt = vbuf + buf * kAtTile * HD;
        // ---- QK: tokens 2 warp, 2 warp + 1
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
            const int tk = 2 * warp + tt;
            const float4 k0 = *reinterpret_cast<const float4 *>(kt + tk * HD + 8 * lane);
            const float4 k1 = *reinterpret_cast<const float4 *>(kt + tk * HD + 8 * lane + 4);
            const uint64_t kp[4] = {at_pair(k0.x, k0.y), at_pair(k0.z, k0.w), at_pair(k1.x, k1.y),
                                    at_pair(k1.z, k1.w)};
            float v[8];
#pragma unroll
            for (int h = 0; h < 8; ++h) {
                uint64_t a2 = 0ull;
#pragma unroll
                for (int j = 0; j < 4; ++j) a2 = at_fma2(qr[h][j], kp[j], a2);
                float lo, hi;
                at_unpair(a2, lo, hi);
                v[h] = lo + hi;
            }
            float w4[4], w2[2];
            const bool u16 = (lane & 16) != 0, u8 = (lane & 8) != 0, u4 = (lane & 4) != 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float send = u16 ? v[i] : v[i + 4];
                const float keep = u16 ? v[i + 4] : v[i];
                w4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const float send = u8 ? w4[i] : w4[i + 2];
                const float keep = u8 ? w4[i + 2] : w4[i];
                w2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
            }
            float w1;
            {
                const float send = u4 ? w2[0] : w2[1];
                const float keep = u4 ? w2[1] : w2[0];
                w1 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
            }
            w1 += __shfl_xor_sync(0xffffffffu, w1, 2);
            w1 += __shfl_xor_sync(0xffffffffu, w1, 1);
            if ((lane & 3) == 0)
                lg[tk * 8 + my_head] = tok_s[(tile - tile0) * kAtTile + tk] != 0xFFFFFFFFu ? w1 / scale : -INFINITY;
        }
        __syncthreads();
        // ---- online softmax: warp h for head h, lanes 0..15 one token each
        if ((uint32_t)warp < heads) {
            const float logit = lane < kAtTile ? lg[lane * 8 + warp] : -INFINITY;
            float mt = logit;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
            const float m_new = fmaxf(m_run, mt);
            const float corr = (m_run == -INFINITY) ? 0.0f : expf(m_run - m_new);
            const float p = (logit == -INFINITY) ? 0.0f : expf(logit - m_new);
            float ps = p;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l_run = l_run * corr + ps;
            m_run = m_new;
            if (lane < kAtTile) pw[lane * 8 + warp] = p;
            if (lane == 0) corr_s[warp] = corr;
        }
        __syncthreads();
        // ---- PV: feature 32 warp + lane of every head
        {
            const int f = 32 * warp + lane;
            const float4 c0 = *reinterpret_cast<const float4 *>(corr_s);
            const float4 c1 = *reinterpret_cast<const float4 *>(corr_s + 4);
            acc2[0] = at_mul2(acc2[0], at_pair(c0.x, c0.y));
            acc2[1] = at_mul2(acc2[1], at_pair(c0.z, c0.w));
            acc2[2] = at_mul2(acc2[2], at_pair(c1.x, c1.y));
            acc2[3] = at_mul2(acc2[3], at_pair(c1.z, c1.w));
#pragma unroll 4
            for (int t = 0; t < kAtTile; ++t) {
                const float vv = vt[t * HD + f];
                const uint64_t v2 = at_pair(vv, vv);
                const float4 p0 = *reinterpret_cast<const float4 *>(pw + t * 8);
                const float4 p1 = *reinterpret_cast<const float4 *>(pw + t * 8 + 4);
                acc2[0] = at_fma2(at_pair(p0.x, p0.y), v2, acc2[0]);
                acc2[1] = at_fma2(at_pair(p0.z, p0.w), v2, acc2[1]);
                acc2[2] = at_fma2(at_pair(p1.x, p1.y), v2, acc2[2]);
                acc2[3] = at_fma2(at_pair(p1.z, p1.w), v2, acc2[3]);
            }
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;\n" ::);
    const int f = 32 * warp + lane;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) at_unpair(acc2[i], acc[2 * i], acc[2 * i + 1]);
#pragma unroll
    for (int h = 0; h < 8; ++h) {
        if ((uint32_t)h < heads) {
            const size_t slot = ((size_t)b * d.q_heads + kvh * heads + h) * splits + split;
            part_o[slot * HD + f] = acc[h];
        }
    }
    if ((uint32_t)warp < heads && lane == 0) {
        const size_t slot = ((size_t)b * d.q_heads + kvh * heads + warp) * splits + split;
        part_ml[slot * 2] = m_run;
        part_ml[slot * 2 + 1] = l_run;
    }
}

// ------------------------------------------------ tensor-core attention
//
// head_dim 256, up to 8 query heads per KV head; grid (entries, kv_heads,
// splits), 288 threads: eight consumer warps and one producer warp.  Reads
// the bf16 hi / lo copies of the cache rows (QsaSeq::key_split /
// value_split: rows [hi 256 | lo 256] per token, KV-head major).  Per tile
// of 16 selected tokens:
//   logits^T [16 tokens][8 heads] = K [16][256] . Q^T [256][8]
//   O^T [256][8] += V^T [256][16] . P^T [16][8]
// as warp MMAs (m16n8k16, bf16 operands, F32 accumulate) with the
// three-term split a b ~ a_hi b_hi + a_hi b_lo + a_lo b_hi, each term in
// its own accumulator; the heads are the n = 8 side, so no MMA row is
// padding.  Warp w owns features [32 w, 32 w + 32): its partial logits over
// them are summed across the eight warps through shared memory (in warp
// order, so every warp sees the same logits and takes the same softmax
// decisions), then each warp multiplies its features of V.  One barrier
// of the consumer warps per tile.  The softmax reference point m is raised only when a
// logit exceeds it by more than kTcRescale (the weights then stay below
// 2^12, and O and l are rescaled rarely); O / l is the same quotient for
// any m.  The logits are kept in base-2 units (Q is scaled by
// log2(e) / sqrt(d) before the split, so the weights are exp2(logit - m));
// m is written back in natural units.  P^T reaches the B operand layout by movmatrix
// transposes.  The producer warp refills a stage as soon as the eight
// consumers have released it (an mbarrier per stage each way), with one
// bulk copy per run of consecutive cache rows (the tokens of a selected
// block); rows of a tile past the selection load cache row 0 and get
// weight 0.

namespace {

constexpr int kTcTile = 16;                               // tokens per tile
constexpr int kTcWarps = 8;                               // consumers; warp 8 produces
constexpr int kTcThreads = 32 * (kTcWarps + 1);
constexpr uint32_t kTcRow = 1040;                         // 1 KB row + 16 B: 8 rows hit 8 bank groups
constexpr uint32_t kTcStage = 2 * kTcTile * kTcRow;       // K rows, then V rows
static_assert(kTcRow == 2 * kQsaSplitRow, "shared-memory rows are split-cache rows");
constexpr int kTcMaxTiles = 32;
constexpr float kTcRescale = 12.0f;                       // base-2 units
constexpr float kTcLog2e = 1.44269504088896340736f;
constexpr float kTcLn2 = 0.69314718055994530942f;
// shared memory of the S-stage kernel: stages, partial logits, cache rows,
// full[S], empty[S], abort flag
template <int S>
struct TcLayout {
    static constexpr size_t log_off = (size_t)S * kTcStage;
    static constexpr size_t tok_off = log_off + 2 * kTcWarps * 32 * 4 * 4;
    static constexpr size_t bar_off = tok_off + (size_t)kTcMaxTiles * kTcTile * 4;
    static constexpr size_t bytes = bar_off + 2 * S * 8 + 16;
    static_assert(log_off % 16 == 0 && tok_off % 16 == 0 && bar_off % 8 == 0, "shared-memory alignment");
};
constexpr uint32_t kTcWaitSite = 8;                        // reported as kErrTimeout | 8 << 8
constexpr uint32_t kTcWaitPolls = 1u << 26;
constexpr uint64_t kTcWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t tc_smem(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint64_t tc_now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ bool tc_poll(uint32_t bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    return done != 0;
}

// Bounded wait by lane 0 of the warp, result broadcast.  Gives up at once
// when another warp has raised the CTA's abort flag; raises it itself after
// the poll or time limit.
__device__ __forceinline__ bool tc_wait_warp(uint64_t *bar, uint32_t parity, volatile uint32_t *abort_flag) {
    uint32_t ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t a = tc_smem(bar);
        uint64_t t0 = 0;   // the clock is read only once a wait is slow
        ok = 0;
        for (uint32_t i = 0; i < kTcWaitPolls; ++i) {
            if (tc_poll(a, parity)) {
                ok = 1;
                break;
            }
            if ((i & 63u) == 63u) {
                if (*abort_flag) break;
                const uint64_t now = tc_now();
                if (t0 == 0) t0 = now;
                else if (now - t0 > kTcWaitNs) {
                    atomicCAS(const_cast<uint32_t *>(abort_flag), 0u, kTcWaitSite);
                    break;
                }
            }
        }
        if (!ok) atomicCAS(const_cast<uint32_t *>(abort_flag), 0u, kTcWaitSite);
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

__device__ __forceinline__ void tc_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(tc_smem(bar)), "r"(bytes)
                 : "memory");
}

// 1-D bulk copy global -> shared (no multicast) completing on `bar`
__device__ __forceinline__ void tc_bulk(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(tc_smem(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_ldsm(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void tc_ldsm_t(uint32_t addr, uint32_t (&r)[4]) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void tc_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// (x0, x1) -> bf16x2 hi (round to nearest) and bf16x2 lo of the residuals;
// x0 in the low half (the lower k index of an MMA operand pair)
__device__ __forceinline__ void tc_split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
    const float2 hf = __bfloat1622float2(h);
    const __nv_bfloat162 l = __floats2bfloat162_rn(x0 - hf.x, x1 - hf.y);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// 8x8 b16 transpose of a fragment (row T / 4, columns 2 (T % 4), +1)
__device__ __forceinline__ uint32_t tc_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

}  // namespace

bool qsa_split_cache_used(const QsaDims &d) { return d.head_dim == 256 && d.repeat <= 8; }

// KQ_B200_SIMT_ATTENTION=1 selects the F32 CUDA-core attention kernel for
// head_dim 256 as well (used by the tests to cross-check the two).
bool force_simt_attention() {
    const char *e = getenv("KQ_B200_SIMT_ATTENTION");
    return e != nullptr && e[0] == '1';
}

template <int kTcStages, int kMinBlocks>
__global__ void __launch_bounds__(kTcThreads, kMinBlocks)
qsa_attend_tc_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ q, const uint32_t *__restrict__ selected,
                     const uint32_t *__restrict__ selected_count, float *__restrict__ part_o,
                     float *__restrict__ part_ml, uint32_t splits, ErrorWord err) {
    pdl_wait();
    extern __shared__ __align__(128) uint8_t tsm[];
    using L = TcLayout<kTcStages>;
    float *plog = reinterpret_cast<float *>(tsm + L::log_off);                 // [2][8 warps][32 lanes][4]
    uint32_t *tok_s = reinterpret_cast<uint32_t *>(tsm + L::tok_off);         // cache row per selected token
    uint64_t *full = reinterpret_cast<uint64_t *>(tsm + L::bar_off);
    uint64_t *empty = full + kTcStages;
    volatile uint32_t *abort_flag = reinterpret_cast<volatile uint32_t *>(empty + kTcStages);
    if (qsa_error_raised(err)) return;
    const uint32_t b = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
    const QsaSeq s = batch_seq(bt, b);
    const uint32_t pos = s.length;
    const uint32_t nblocks = (pos + 1) / d.block;
    const uint32_t tail = (pos + 1) % d.block;
    const uint32_t ksel = min(selected_count[b], min(nblocks, d.topk));
    const uint32_t ntok = ksel * d.block + tail;
    const uint32_t ntiles = (ntok + kTcTile - 1) / kTcTile;
    const uint32_t per = (ntiles + splits - 1) / splits;
    const uint32_t tile0 = split * per, tile1 = min(ntiles, tile0 + per);
    const uint32_t heads = d.repeat;   // <= 8 (checked by the launcher)
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, qd = lane & 3;
    const uint32_t *selb = selected + (size_t)b * d.topk;
    const uint32_t my_tiles = tile1 > tile0 ? tile1 - tile0 : 0u;
    if (my_tiles > (uint32_t)kTcMaxTiles) {
        if (tid == 0) qsa_raise(err, kErrSelection);
        return;
    }
    // cache row of every token of this CTA's tiles (UINT32_MAX: none)
    for (uint32_t i = tid; i < my_tiles * kTcTile; i += kTcThreads) {
        const uint32_t t = tile0 * kTcTile + i;
        uint32_t tok = 0xFFFFFFFFu;
        if (t < ksel * d.block) {
            const uint32_t blk = selb[t / d.block];
            if (blk < nblocks) tok = blk * d.block + t % d.block;
        } else if (t < ntok) {
            tok = nblocks * d.block + (t - ksel * d.block);
        }
        tok_s[i] = tok;
    }
    if (tid == 0) {
        for (int st = 0; st < kTcStages; ++st) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem(&full[st])), "r"(1u));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tc_smem(&empty[st])), "r"((uint32_t)kTcWarps));
        }
        *abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const uint16_t *ksplit = s.key_split + (size_t)kvh * s.capacity * kQsaSplitRow;
    const uint16_t *vsplit = s.value_split + (size_t)kvh * s.capacity * kQsaSplitRow;
    // producer: bulk copies of tile j (relative to tile0).  Lane l < 16 takes
    // token l's key row, lane 16 + l its value row; consecutive cache rows
    // (the tokens of one selected block) go as one copy of the whole run,
    // issued by the lane of its first token.  A row past the selection
    // loads cache row 0.
    auto issue = [&](uint32_t j) {
        const uint32_t st = j % kTcStages;
        if (lane == 0) tc_expect_tx(&full[st], 2u * kTcTile * kTcRow);
        __syncwarp();
        const uint32_t r = lane & 15u, which = (uint32_t)lane >> 4;
        const uint32_t *tt = tok_s + j * kTcTile;
        const uint32_t tok = tt[r];
        const bool start = tok == 0xFFFFFFFFu || r == 0 || tt[r - 1] == 0xFFFFFFFFu || tt[r - 1] + 1 != tok;
        if (start) {
            uint32_t n = 1;
            if (tok != 0xFFFFFFFFu)
                while (r + n < (uint32_t)kTcTile && tt[r + n] == tok + n) ++n;
            const uint16_t *src = (which ? vsplit : ksplit) + (size_t)(tok == 0xFFFFFFFFu ? 0u : tok) * kQsaSplitRow;
            const uint32_t dst = tc_smem(tsm + st * kTcStage + which * kTcTile * kTcRow + r * kTcRow);
            tc_bulk(dst, src, n * kTcRow, &full[st]);
        }
    };
    if (warp == kTcWarps) {
        // producer: a stage is refilled once every consumer has released it
        uint32_t j = 0;
        for (; j < my_tiles; ++j) {
            const uint32_t st = j % kTcStages;
            if (j >= (uint32_t)kTcStages && !tc_wait_warp(&empty[st], (j / kTcStages - 1) & 1u, abort_flag)) break;
            issue(j);
        }
        if (*abort_flag && lane == 0) {
            // let the copies in flight land (bounded) before the CTA exits
            for (uint32_t st = 0; st < (uint32_t)kTcStages && st < j; ++st) {
                const uint32_t last = st + ((j - 1 - st) / kTcStages) * kTcStages;
                const uint32_t a = tc_smem(&full[st]);
                const uint64_t t0 = tc_now();
                while (!tc_poll(a, (last / kTcStages) & 1u) && tc_now() - t0 < kTcWaitNs) {
                }
            }
        }
        return;
    }

    // Q^T fragments of this warp's features (B operand: k = feature, n = head g)
    uint32_t qh[2][2], ql[2][2];
    const float qscale = kTcLog2e / d.sqrt_head_dim;
    {
        const bool hv = (uint32_t)g < heads;
        const float *qp = q + ((size_t)b * d.q_heads + kvh * heads + (hv ? g : 0)) * 256u;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            const int f = 32 * warp + 16 * kk + 2 * qd;
            float2 x0 = make_float2(0.f, 0.f), x1 = x0;
            if (hv) {
                x0 = *reinterpret_cast<const float2 *>(qp + f);
                x1 = *reinterpret_cast<const float2 *>(qp + f + 8);
                x0.x *= qscale; x0.y *= qscale; x1.x *= qscale; x1.y *= qscale;
            }
            tc_split2(x0.x, x0.y, qh[kk][0], ql[kk][0]);
            tc_split2(x1.x, x1.y, qh[kk][1], ql[kk][1]);
        }
    }
    // softmax state of heads 2 qd, 2 qd + 1 (l: this lane's tokens only)
    float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.f, 0.f};
    // O^T of m-tile mt, one accumulator per split term:
    // (feature g, head 2qd | 2qd+1), (feature g + 8, ...)
    float o[3][2][4];
#pragma unroll
    for (int a = 0; a < 3; ++a)
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int i = 0; i < 4; ++i) o[a][mt][i] = 0.f;
    bool failed = false;
    const uint32_t base = tc_smem(tsm);
    // ldmatrix row addresses: K as the A operand (rows = tokens), V as the
    // transposed A operand (rows = features)
    const uint32_t k_lane = ((lane & 7) + ((lane >> 3) & 1) * 8) * kTcRow + (32 * warp + (lane >> 4) * 8) * 2;
    const uint32_t v_lane =
        kTcTile * kTcRow + ((lane & 7) + (lane >> 4) * 8) * kTcRow + (32 * warp + ((lane >> 3) & 1) * 8) * 2;

    for (uint32_t j = 0; j < my_tiles; ++j) {
        const uint32_t st = j % kTcStages;
        if (!tc_wait_warp(&full[st], (j / kTcStages) & 1u, abort_flag)) failed = true;
        const uint32_t stage = base + st * kTcStage;
        // ---- partial logits over this warp's features, one accumulator per split term
        float a[3][4];
#pragma unroll
        for (int i = 0; i < 3; ++i) a[i][0] = a[i][1] = a[i][2] = a[i][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            uint32_t ah[4], al[4];
            tc_ldsm(stage + k_lane + kk * 32, ah);
            tc_ldsm(stage + k_lane + kk * 32 + 512, al);
            tc_mma(a[0], ah, qh[kk][0], qh[kk][1]);
            tc_mma(a[1], ah, ql[kk][0], ql[kk][1]);
            tc_mma(a[2], al, qh[kk][0], qh[kk][1]);
        }
        float *pl = plog + (j & 1u) * kTcWarps * 32 * 4;
        float4 mine;
        mine.x = (a[0][0] + a[1][0]) + a[2][0];
        mine.y = (a[0][1] + a[1][1]) + a[2][1];
        mine.z = (a[0][2] + a[1][2]) + a[2][2];
        mine.w = (a[0][3] + a[1][3]) + a[2][3];
        *reinterpret_cast<float4 *>(pl + (warp * 32 + lane) * 4) = mine;
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kTcWarps) : "memory");
        float4 acc = *reinterpret_cast<const float4 *>(pl + lane * 4);
#pragma unroll
        for (int w = 1; w < kTcWarps; ++w) {
            const float4 x = *reinterpret_cast<const float4 *>(pl + (w * 32 + lane) * 4);
            acc.x += x.x; acc.y += x.y; acc.z += x.z; acc.w += x.w;
        }
        const uint32_t *tt = tok_s + j * kTcTile;
        const bool v0 = tt[g] != 0xFFFFFFFFu, v1 = tt[g + 8] != 0xFFFFFFFFu;
        // (token g, head 2qd), (g, 2qd + 1), (g + 8, 2qd), (g + 8, 2qd + 1)
        const float lg[4] = {v0 ? acc.x : -INFINITY, v0 ? acc.y : -INFINITY, v1 ? acc.z : -INFINITY,
                             v1 ? acc.w : -INFINITY};
        const bool high = lg[0] > m_run[0] + kTcRescale || lg[2] > m_run[0] + kTcRescale ||
                          lg[1] > m_run[1] + kTcRescale || lg[3] > m_run[1] + kTcRescale;
        if (__any_sync(0xffffffffu, high)) {
            // new reference point: the running maximum of each head
#pragma unroll
            for (int c = 0; c < 2; ++c) {
                float mt = fmaxf(lg[c], lg[c + 2]);
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 4));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 8));
                mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 16));
                const float m_new = fmaxf(m_run[c], mt);
                const float corr = (m_run[c] == -INFINITY) ? 0.0f : exp2f(m_run[c] - m_new);
                l_part[c] *= corr;
#pragma unroll
                for (int t3 = 0; t3 < 3; ++t3)
#pragma unroll
                    for (int mt2 = 0; mt2 < 2; ++mt2) {
                        o[t3][mt2][c] *= corr;
                        o[t3][mt2][c + 2] *= corr;
                    }
                m_run[c] = m_new;
            }
        }
        float p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = (lg[i] == -INFINITY) ? 0.0f : exp2f(lg[i] - m_run[i & 1]);
        l_part[0] += p[0] + p[2];
        l_part[1] += p[1] + p[3];
        // P^T as the B operand (k = token, n = head): the fragments of P
        // (token g | g + 8, heads 2qd, 2qd + 1) transposed
        uint32_t h01, l01, h23, l23;
        tc_split2(p[0], p[1], h01, l01);
        tc_split2(p[2], p[3], h23, l23);
        const uint32_t pb0h = tc_trans(h01), pb1h = tc_trans(h23);
        const uint32_t pb0l = tc_trans(l01), pb1l = tc_trans(l23);
        // ---- O^T += V^T P^T over this warp's features
#pragma unroll
        for (int mt2 = 0; mt2 < 2; ++mt2) {
            uint32_t ah[4], al[4];
            tc_ldsm_t(stage + v_lane + mt2 * 32, ah);
            tc_ldsm_t(stage + v_lane + mt2 * 32 + 512, al);
            tc_mma(o[0][mt2], ah, pb0h, pb1h);
            tc_mma(o[1][mt2], ah, pb0l, pb1l);
            tc_mma(o[2][mt2], al, pb0h, pb1h);
        }
        // this warp is done with the stage
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(tc_smem(&empty[st])) : "memory");
    }
    if (failed || *abort_flag) {
        if (tid == 0)
            atomicCAS(err.word, 0ull, ((unsigned long long)(kErrTimeout | (kTcWaitSite << 8)) << 32) | err.call_id);
        return;
    }
    // l over the 16 token rows of the lanes with this qd
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        l_part[c] += __shfl_xor_sync(0xffffffffu, l_part[c], 4);
        l_part[c] += __shfl_xor_sync(0xffffffffu, l_part[c], 8);
        l_part[c] += __shfl_xor_sync(0xffffffffu, l_part[c], 16);
    }
    // partial results of this split: O (features 32 w + 16 mt + g (+ 8)) and m, l
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        const uint32_t h = 2 * qd + c;
        if (h >= heads) continue;
        const size_t slot = ((size_t)b * d.q_heads + kvh * heads + h) * splits + split;
        float *po = part_o + slot * 256u + 32 * warp + g;
#pragma unroll
        for (int mt2 = 0; mt2 < 2; ++mt2) {
            po[16 * mt2] = (o[0][mt2][c] + o[1][mt2][c]) + o[2][mt2][c];
            po[16 * mt2 + 8] = (o[0][mt2][c + 2] + o[1][mt2][c + 2]) + o[2][mt2][c + 2];
        }
        if (warp == 0 && g == 0) {
            part_ml[slot * 2] = m_run[c] * kTcLn2;
            part_ml[slot * 2 + 1] = l_part[c];
        }
    }
}

// ------------------------------------------------------------ checkpoint path
//
// grid (Hq), 256 threads; dynamic shared memory: the token list and the
// logits of one head (selected-token capacity each).  The reference's order
// (src/kq_qsa_qwen38.c:716-773): dots over the features in order divided by
// sqrt(d), the maximum, exp(logit - max) summed in token order by one
// thread, the division, then each feature's context summed in token order.
__global__ void __launch_bounds__(256)
qsa_debug_attention_kernel(QsaDims d, QsaBatch bt, const float *__restrict__ q, const uint32_t *__restrict__ selected,
                           const uint32_t *__restrict__ selected_count, float *__restrict__ logits,
                           float *__restrict__ probs, float *__restrict__ context, ErrorWord err) {
    pdl_wait();
    extern __shared__ float dbg_sm[];
    __shared__ float red[8];
    __shared__ float sum_s;
    if (qsa_error_raised(err)) return;
    const QsaSeq s = batch_seq(bt, 0);
    const uint32_t pos = s.length, h = blockIdx.x, hd = d.head_dim;
    const uint32_t kvh = h / d.repeat, kvw = d.kv_heads * hd;
    const uint32_t nblocks = (pos + 1) / d.block, tail = (pos + 1) % d.block;
    const uint32_t ksel = min(selected_count[0], min(nblocks, d.topk));
    const uint32_t ntok = ksel * d.block + tail;
    uint32_t *tok = reinterpret_cast<uint32_t *>(dbg_sm);
    float *lg = dbg_sm + d.sel_capacity;
    for (uint32_t i = threadIdx.x; i < ntok; i += blockDim.x)
        tok[i] = i < ksel * d.block ? selected[i / d.block] * d.block + i % d.block : nblocks * d.block + (i - ksel * d.block);
    __syncthreads();
    const float *qh = q + (size_t)h * hd;
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < ntok; i += blockDim.x) {
        const float *kr = s.key + (size_t)tok[i] * kvw + kvh * hd;
        float dot = 0.0f;
        for (uint32_t f = 0; f < hd; ++f) dot = __fadd_rn(dot, __fmul_rn(qh[f], kr[f]));
        dot = __fdiv_rn(dot, d.sqrt_head_dim);
        lg[i] = dot;
        logits[(size_t)h * ntok + i] = dot;
        mx = fmaxf(mx, dot);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int w = 1; w < 8; ++w) m = fmaxf(m, red[w]);
        float sum = 0.0f;
        for (uint32_t i = 0; i < ntok; ++i) {
            const float p = expf(__fsub_rn(lg[i], m));
            lg[i] = p;
            sum = __fadd_rn(sum, p);
        }
        if (!(sum > 0.0f) || !isfinite(sum)) qsa_raise(err, kErrNonFinite);
        sum_s = sum;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < ntok; i += blockDim.x) {
        const float p = __fdiv_rn(lg[i], sum_s);
        probs[(size_t)h * ntok + i] = p;
    }
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < ntok; i += blockDim.x) lg[i] = __fdiv_rn(lg[i], sum_s);
    __syncthreads();
    for (uint32_t f = threadIdx.x; f < hd; f += blockDim.x) {
        float acc = 0.0f;
        for (uint32_t i = 0; i < ntok; ++i)
            acc = __fadd_rn(acc, __fmul_rn(lg[i], s.value[(size_t)tok[i] * kvw + kvh * hd + f]));
        context[(size_t)h * hd + f] = acc;
    }
}

void launch_qsa_debug_attention(const QsaDims &d, const QsaBatch &b, const float *q, const uint32_t *selected,
                                const uint32_t *selected_count, float *logits, float *probs, float *context,
                                ErrorWord err, cudaStream_t stream) {
    const size_t smem = (size_t)2 * d.sel_capacity * sizeof(float);
    static DeviceOnce attr;
    attr.run([&] {
        cudaFuncSetAttribute(qsa_debug_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
    });
    launch_pdl(qsa_debug_attention_kernel, dim3(d.q_heads), 256, smem, stream, d, b, q, selected, selected_count,
               logits, probs, context, err);
    count_launch();
}

void launch_qsa_attend(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                       const float *q, const uint32_t *selected,
                       const uint32_t *selected_count, float *partial_o,
                       float *partial_ml, uint32_t splits,
                       ErrorWord err, cudaStream_t stream) {
    // entries fastest: the CTAs in flight together take the same split of
    // many entries, which (with selections in block order) read nearby
    // parts of a shared cache
    dim3 grid(batch, d.kv_heads, splits);
    KernelTimer timer("qsa_attend", stream);
    bool split_rows = qsa_split_cache_used(d) && !force_simt_attention();
    for (uint32_t e = 0; split_rows && e < (b.uniform ? 1u : batch); ++e)
        split_rows = b.s[e].key_split != nullptr && b.s[e].value_split != nullptr;
    if (split_rows) {
        // three stages and two CTAs per SM, or (KQ_B200_ATTEND_STAGES=6) six
        // stages and one CTA
        const char *e = getenv("KQ_B200_ATTEND_STAGES");
        if (e != nullptr && e[0] == '6') {
            static DeviceOnce attr6;
            attr6.run([] {
                cudaFuncSetAttribute(qsa_attend_tc_kernel<6, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)TcLayout<6>::bytes);
            });
            launch_pdl(qsa_attend_tc_kernel<6, 1>, grid, kTcThreads, TcLayout<6>::bytes, stream, d, b, q, selected,
                       selected_count, partial_o, partial_ml, splits, err);
        } else {
            static DeviceOnce attr3;
            attr3.run([] {
                cudaFuncSetAttribute(qsa_attend_tc_kernel<3, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int)TcLayout<3>::bytes);
            });
            launch_pdl(qsa_attend_tc_kernel<3, 2>, grid, kTcThreads, TcLayout<3>::bytes, stream, d, b, q, selected,
                       selected_count, partial_o, partial_ml, splits, err);
        }
    } else if (d.head_dim == 256 && d.repeat <= 8) {
        static DeviceOnce attr;
        attr.run([] {
            cudaFuncSetAttribute(qsa_attend_mh_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMhSmem);
        });
        launch_pdl(qsa_attend_mh_kernel, grid, 256, kMhSmem, stream, d, b, q, selected, selected_count, partial_o,
                   partial_ml, splits, err);
    } else if (d.head_dim == 256 || d.head_dim == 128) {
        const int hd = (int)d.head_dim;
        const size_t smem = (size_t)(8 * hd + 2 * kAtTile * (hd + 4) + 2 * kAtTile * hd) * sizeof(float);
        if (hd == 256) {
            cudaFuncSetAttribute(qsa_attend_tiled_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
            launch_pdl(qsa_attend_tiled_kernel<256>, grid, 256, smem, stream, d, b, q, selected, selected_count,
                                                                    partial_o, partial_ml, splits, err);
        } else {
            cudaFuncSetAttribute(qsa_attend_tiled_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)smem);
            launch_pdl(qsa_attend_tiled_kernel<128>, grid, 256, smem, stream, d, b, q, selected, selected_count,
                                                                    partial_o, partial_ml, splits, err);
        }
    } else {
        // small heads (reduced test shapes): warp-per-token kernel
        size_t smem = (size_t)8 * 8 * (d.head_dim + 2) * sizeof(float);
        if (d.head_dim <= 32) {
            launch_pdl(qsa_attend_kernel<1, 8>, grid, 256, smem, stream, d, b, q, selected, selected_count,
                                                               partial_o, partial_ml, splits, err);
        } else {
            launch_pdl(qsa_attend_kernel<2, 8>, grid, 256, smem, stream, d, b, q, selected, selected_count,
                                                               partial_o, partial_ml, splits, err);
        }
    }
    count_launch();
}

// ------------------------------------------------------------ combine + gate
//
// grid (Hq, B); one thread per feature: merge the split partials, then apply
// the simple-form sigmoid gate 1 / (1 + exp(-g)) of :778.

__global__ void qsa_combine_kernel(QsaDims d, const float *__restrict__ part_o,
                                   const float *__restrict__ part_ml, uint32_t splits,
                                   const float *__restrict__ proj, uint32_t ldp,
                                   float *__restrict__ gated, ErrorWord err) {
    pdl_wait();
    if (qsa_error_raised(err)) return;
    const uint32_t h = blockIdx.x, b = blockIdx.y;
    const uint32_t hd = d.head_dim;
    const size_t base = ((size_t)b * d.q_heads + h) * splits;
    float mx = -INFINITY;
    for (uint32_t s = 0; s < splits; ++s) mx = fmaxf(mx, part_ml[(base + s) * 2]);
    bool bad = false;
    for (uint32_t f = threadIdx.x; f < hd; f += blockDim.x) {
        float o = 0.0f, ll = 0.0f;
        for (uint32_t s = 0; s < splits; ++s) {
            float ms = part_ml[(base + s) * 2];
            float c = (ms == -INFINITY) ? 0.0f : expf(ms - mx);
            o += part_o[(base + s) * hd + f] * c;
            ll += part_ml[(base + s) * 2 + 1] * c;
        }
        float ctx = o / ll;
        float g = proj[(size_t)b * ldp + (size_t)h * 2 * hd + hd + f];
        float sg = 1.0f / (1.0f + expf(-g));
        float out = ctx * sg;
        if (!isfinite(out) || !(ll > 0.0f)) bad = true;
        gated[((size_t)b * d.q_heads + h) * hd + f] = out;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) qsa_raise(err, kErrNonFinite);
}

void launch_qsa_combine(const QsaDims &d, uint32_t batch,
                        const float *partial_o, const float *partial_ml,
                        uint32_t splits, const float *proj, uint32_t ldp,
                        float *gated, ErrorWord err, cudaStream_t stream) {
    dim3 grid(d.q_heads, batch);
    KernelTimer timer("qsa_combine", stream);
    launch_pdl(qsa_combine_kernel, grid, 256, 0, stream, d, partial_o, partial_ml, splits, proj, ldp,
                                                 gated, err);
    count_launch();
}

}  // namespace kqb
