// Routed-expert MoE: router, top-k routing, grouped expert GEMV and the
// gated shared expert.
//
// Replaces the per-token loop of kq_moe_execute_common
// (src/kq_moe_qwen38.c:604-867 of Kestrel-Q).  The reference runs, for every
// token, every selected expert's three projections through the provider;
// here the tokens of one call are grouped by expert so that every selected
// expert's weights cross HBM once per call:
//
//   router    exact F32 product (launch_projection_exact: each logit is the
//             reference's sequential kq_f32_dot), the shared gate logit rides
//             along as row E
//   route     one CTA per token: softmax, the reference's top-k rule,
//             renormalised weights; ranks each pick within its expert
//   dispatch  one CTA: per-expert offsets, the list of active experts, the
//             slot of every pick (slots are expert-major)
//   gate_up   grouped gate and up GEMV of the active experts, SwiGLU in the
//             epilogue -> act[slot][I]; Q4_K: persistent streamed kernel on
//             the tensor cores (every selected expert's rows cross HBM once
//             per call)
//   down      grouped down GEMV -> eout[slot][H]; planar Q8_0: streamed, on
//             the tensor cores
//   combine   one CTA per token: the selected experts' weighted outputs
//             summed in ascending expert id (the reference's accumulation
//             order), plus the shared expert scaled by sigmoid(logit)
//
// Every pick's products are computed from its own token only, so the order
// of the picks inside an expert's group (which the atomics of the route
// kernel decide) does not change any value.
#include "kernels.hpp"
#include "quant.cuh"

#include <cuda_fp16.h>

#include <cmath>

namespace kqb {

namespace {

constexpr int kMoeThreads = 256;
constexpr uint32_t kMoeRowsPerCta = 64;
constexpr int kMoeGroup = 8;   // tokens per weight pass
constexpr int kDispatchThreads = 1024;

__device__ __forceinline__ bool moe_err_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}

__device__ __forceinline__ void moe_raise(const ErrorWord &e, uint32_t code) {
    atomicCAS(e.word, 0ull, ((unsigned long long)code << 32) | e.call_id);
}

// kq_sigmoid_scalar (src/kq_numeric.c:628-638): the branch-stable form.
__device__ __forceinline__ float moe_sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

// kq_f32_swiglu element (src/kq_numeric.c:700-728): silu(gate) * up.
__device__ __forceinline__ float moe_swiglu(float g, float u) {
    const float silu = __fmul_rn(g, moe_sigmoid(g));
    return __fmul_rn(silu, u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace

// ------------------------------------------------------------------ route

// One CTA per token.  logits [T][ldl] (experts 0..E-1), probabilities
// [T][E], selected ids / weights [T][K] in the reference's top-k order;
// counts[e] (zeroed before the launch) counts the picks of expert e and
// rank[t*K+p] is pick p's position among them.
__global__ void __launch_bounds__(kMoeThreads)
moe_route_kernel(MoeDims d, const float *__restrict__ logits, uint32_t ldl, float *__restrict__ probs,
                 uint32_t *__restrict__ sel_ids, float *__restrict__ sel_w, uint32_t *__restrict__ counts,
                 uint32_t *__restrict__ rank, ErrorWord err) {
    extern __shared__ float sp[];   // [E]
    __shared__ float red[kMoeThreads / 32];
    __shared__ float total;
    __shared__ int bad;
    __shared__ uint32_t ids[kMoeMaxTopK];
    pdl_wait();
    if (moe_err_raised(err)) return;
    const uint32_t t = blockIdx.x, E = d.experts, K = d.top_k;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float *lg = logits + (size_t)t * ldl;
    if (tid == 0) bad = 0;
    __syncthreads();
    // softmax of src/kq_numeric.c:776-813: maximum, exp(l - max), one
    // sequential sum in index order, division
    float mx = -INFINITY;
    for (uint32_t e = tid; e < E; e += kMoeThreads) {
        const float v = lg[e];
        if (!isfinite(v)) bad = 1;
        mx = fmaxf(mx, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        float m = red[0];
        for (int i = 1; i < kMoeThreads / 32; ++i) m = fmaxf(m, red[i]);
        red[0] = m;
    }
    __syncthreads();
    mx = red[0];
    // the exponential rounded once from double precision: correctly rounded
    // except within 2^-29 of a rounding boundary
    for (uint32_t e = tid; e < E; e += kMoeThreads) sp[e] = (float)exp((double)__fsub_rn(lg[e], mx));
    __syncthreads();
    if (tid == 0) {   // one sequential sum in index order (four values per shared-memory load)
        float s = 0.0f;
        uint32_t e = 0;
#pragma unroll 4
        for (; e + 4u <= E; e += 4u) {
            const float4 v = *reinterpret_cast<const float4 *>(sp + e);
            s = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(s, v.x), v.y), v.z), v.w);
        }
        for (; e < E; ++e) s = __fadd_rn(s, sp[e]);
        if (!isfinite(s) || s <= 0.0f) bad = 1;
        total = s;
    }
    __syncthreads();
    if (bad) {
        if (tid == 0) moe_raise(err, kErrNonFinite);
        return;
    }
    const float s = total;
    for (uint32_t e = tid; e < E; e += kMoeThreads) {
        const float p = __fdiv_rn(sp[e], s);
        sp[e] = p;
        probs[(size_t)t * E + e] = p;
    }
    __syncthreads();
    if (warp == 0) {
        // top-k of src/kq_moe_qwen38.c:211-245, in index order: the set
        // starts as experts 0..K-1; expert i replaces the worst member (lowest
        // value, lowest id among equal values) when its value is strictly
        // greater.  Lane p < K holds member p; a ballot tests 32 experts
        // against the current worst at once, and the hits are inserted one at
        // a time in index order, the rest of the chunk tested again against
        // the new worst.
        uint32_t my_id = (uint32_t)lane < K ? (uint32_t)lane : 0xFFFFFFFFu;
        float my_v = (uint32_t)lane < K ? sp[lane] : INFINITY;
        uint32_t wpos;
        float wv;
        auto find_worst = [&]() {
            float v = my_v;
            uint32_t id = my_id, pos = (uint32_t)lane;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, v, o);
                const uint32_t oid = __shfl_xor_sync(0xffffffffu, id, o);
                const uint32_t opos = __shfl_xor_sync(0xffffffffu, pos, o);
                if (ov < v || (ov == v && oid < id)) v = ov, id = oid, pos = opos;
            }
            wpos = pos, wv = v;
        };
        find_worst();
        for (uint32_t base = K; base < E; base += 32u) {
            const uint32_t i = base + (uint32_t)lane;
            const float v = i < E ? sp[i] : -INFINITY;
            uint32_t m = __ballot_sync(0xffffffffu, v > wv);
            while (m != 0u) {
                const int l = __ffs((int)m) - 1;
                const float nv = __shfl_sync(0xffffffffu, v, l);
                if ((uint32_t)lane == wpos) my_id = base + (uint32_t)l, my_v = nv;
                find_worst();
                m &= ~((2u << l) - 1u);                       // the experts after l in this chunk
                m &= __ballot_sync(0xffffffffu, v > wv);      // still above the new worst
            }
        }
        if ((uint32_t)lane < K) ids[lane] = my_id;
    }
    __syncthreads();
    if (tid == 0) {
        for (uint32_t i = 1; i < K; ++i) {   // value descending, id ascending
            const uint32_t v = ids[i];
            uint32_t pos = i;
            while (pos > 0) {
                const uint32_t prev = ids[pos - 1];
                if (sp[prev] > sp[v] || (sp[prev] == sp[v] && prev < v)) break;
                ids[pos] = prev;
                --pos;
            }
            ids[pos] = v;
        }
        // renormalisation of src/kq_moe_qwen38.c:256-272
        float ssum = 0.0f;
        for (uint32_t p = 0; p < K; ++p) ssum = __fadd_rn(ssum, sp[ids[p]]);
        bool ok = ssum > 0.0f && isfinite(ssum);
        for (uint32_t p = 0; p < K; ++p) {
            const float w = __fdiv_rn(sp[ids[p]], ssum);
            if (!isfinite(w)) ok = false;
            sel_ids[(size_t)t * K + p] = ids[p];
            sel_w[(size_t)t * K + p] = w;
            rank[(size_t)t * K + p] = atomicAdd(&counts[ids[p]], 1u);
        }
        if (!ok) moe_raise(err, kErrNonFinite);
    }
}

// --------------------------------------------------------------- dispatch

// One CTA.  offsets[e] = picks of experts below e (offsets[E] = all picks),
// active = [number of experts with picks, their ids ascending], and the
// slot of every pick: slot[p] = offsets[e] + rank[p], pick_of_slot[slot] = p.
__global__ void __launch_bounds__(kDispatchThreads)
moe_dispatch_kernel(MoeDims d, uint32_t picks, const uint32_t *__restrict__ sel_ids,
                    const uint32_t *__restrict__ counts, const uint32_t *__restrict__ rank,
                    uint32_t *__restrict__ offsets, uint32_t *__restrict__ active, uint32_t *__restrict__ slot,
                    uint32_t *__restrict__ pick_of_slot, ErrorWord err) {
    extern __shared__ uint32_t off_s[];   // [E + 1]
    __shared__ uint32_t wsum[kDispatchThreads / 32], wact[kDispatchThreads / 32];
    pdl_wait();
    if (moe_err_raised(err)) return;
    const uint32_t E = d.experts;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t per = (E + kDispatchThreads - 1) / kDispatchThreads;
    const uint32_t e0 = min(E, tid * per), e1 = min(E, e0 + per);
    uint32_t sum = 0, act = 0;
    for (uint32_t e = e0; e < e1; ++e) {
        sum += counts[e];
        act += counts[e] != 0u;
    }
    // exclusive block scan of (sum, act)
    uint32_t is = sum, ia = act;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t s2 = __shfl_up_sync(0xffffffffu, is, o), a2 = __shfl_up_sync(0xffffffffu, ia, o);
        if (lane >= o) { is += s2; ia += a2; }
    }
    if (lane == 31) { wsum[warp] = is; wact[warp] = ia; }
    __syncthreads();
    if (warp == 0) {
        uint32_t s = lane < kDispatchThreads / 32 ? wsum[lane] : 0u, a = lane < kDispatchThreads / 32 ? wact[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t s2 = __shfl_up_sync(0xffffffffu, s, o), a2 = __shfl_up_sync(0xffffffffu, a, o);
            if (lane >= o) { s += s2; a += a2; }
        }
        if (lane < kDispatchThreads / 32) { wsum[lane] = s; wact[lane] = a; }
    }
    __syncthreads();
    uint32_t run = is - sum + (warp > 0 ? wsum[warp - 1] : 0u);
    uint32_t arun = ia - act + (warp > 0 ? wact[warp - 1] : 0u);
    for (uint32_t e = e0; e < e1; ++e) {
        off_s[e] = run;
        offsets[e] = run;
        if (counts[e] != 0u) active[1 + arun++] = e;
        run += counts[e];
    }
    if (tid == kDispatchThreads - 1) {
        off_s[E] = wsum[kDispatchThreads / 32 - 1];
        offsets[E] = wsum[kDispatchThreads / 32 - 1];
        active[0] = wact[kDispatchThreads / 32 - 1];
    }
    __syncthreads();
    for (uint32_t p = tid; p < picks; p += kDispatchThreads) {
        const uint32_t s = off_s[sel_ids[p]] + rank[p];
        slot[p] = s;
        pick_of_slot[s] = p;
    }
}

// ---------------------------------------------------------------- gate_up

// acc[j] += w[0..count) . x_j[base..base+count) for the group's tokens.
template <int NB>
__device__ __forceinline__ void dot_group(const float (&w)[32], uint32_t count, const float *const (&xp)[NB],
                                          uint32_t nb, bool vec, float (&acc)[NB]) {
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        if ((uint32_t)j >= nb) break;
        float s = acc[j];
        if (vec) {
            const float4 *p = reinterpret_cast<const float4 *>(xp[j]);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const float4 v = p[i];
                s = fmaf(w[4 * i], v.x, s);
                s = fmaf(w[4 * i + 1], v.y, s);
                s = fmaf(w[4 * i + 2], v.z, s);
                s = fmaf(w[4 * i + 3], v.w, s);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 32; ++i)
                if ((uint32_t)i < count) s = fmaf(w[i], xp[j][i], s);
        }
        acc[j] = s;
    }
}

template <int NB>
__device__ __forceinline__ void gate_up_rows(const MoeDims &d, const QMatrix &gate, const QMatrix &up, const float *x,
                                             uint32_t ldx, uint32_t e, uint32_t s0, uint32_t g0, uint32_t nb,
                                             const uint32_t *pick_of_slot, float *act, float *gate_dbg,
                                             float *up_dbg, uint32_t r, int lane) {
    const uint32_t H = d.hidden, I = d.routed;
    const uint8_t *grow = gate.data + ((size_t)e * I + r) * gate.row_bytes;
    const uint8_t *urow = up.data + ((size_t)e * I + r) * up.row_bytes;
    const float *xrow[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        const uint32_t jj = (uint32_t)j < nb ? (uint32_t)j : 0u;
        xrow[j] = x + (size_t)(pick_of_slot[s0 + g0 + jj] / d.top_k) * ldx;
    }
    float ag[NB], au[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) ag[j] = au[j] = 0.0f;
    const bool xal = (ldx & 3u) == 0u && (reinterpret_cast<uintptr_t>(x) & 15u) == 0u;
    for (uint32_t base = (uint32_t)lane * 32u; base < H; base += 1024u) {
        const uint32_t count = min(32u, H - base);
        const bool vec = xal && count == 32u;
        const float *xp[NB];
#pragma unroll
        for (int j = 0; j < NB; ++j) xp[j] = xrow[j] + base;
        float w[32];
        decode32_any(gate, grow, base, w);
        dot_group<NB>(w, count, xp, nb, vec, ag);
        decode32_any(up, urow, base, w);
        dot_group<NB>(w, count, xp, nb, vec, au);
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        if ((uint32_t)j >= nb) break;
        const float g = warp_sum(ag[j]), u = warp_sum(au[j]);
        if (lane == 0) {
            const size_t o = (size_t)(s0 + g0 + j) * I + r;
            act[o] = moe_swiglu(g, u);
            if (gate_dbg) {
                gate_dbg[o] = g;
                up_dbg[o] = u;
            }
        }
    }
}

// grid (max active experts, ceil(I / 64)); 8 warps, a warp per row.
__global__ void __launch_bounds__(kMoeThreads)
moe_gate_up_kernel(MoeDims d, QMatrix gate, QMatrix up, const float *__restrict__ x, uint32_t ldx,
                   const uint32_t *__restrict__ active, const uint32_t *__restrict__ offsets,
                   const uint32_t *__restrict__ pick_of_slot, float *__restrict__ act, float *gate_dbg,
                   float *up_dbg, ErrorWord err) {
    pdl_wait();
    if (moe_err_raised(err) || blockIdx.x >= active[0]) return;
    const uint32_t e = active[1 + blockIdx.x];
    const uint32_t s0 = offsets[e], n = offsets[e + 1] - s0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t r_end = min(d.routed, (blockIdx.y + 1) * kMoeRowsPerCta);
    for (uint32_t r = blockIdx.y * kMoeRowsPerCta + warp; r < r_end; r += kMoeThreads / 32) {
        for (uint32_t g0 = 0; g0 < n; g0 += kMoeGroup) {
            const uint32_t nb = min((uint32_t)kMoeGroup, n - g0);
            if (nb == 1)
                gate_up_rows<1>(d, gate, up, x, ldx, e, s0, g0, nb, pick_of_slot, act, gate_dbg, up_dbg, r, lane);
            else if (nb == 2)
                gate_up_rows<2>(d, gate, up, x, ldx, e, s0, g0, nb, pick_of_slot, act, gate_dbg, up_dbg, r, lane);
            else if (nb <= 4)
                gate_up_rows<4>(d, gate, up, x, ldx, e, s0, g0, nb, pick_of_slot, act, gate_dbg, up_dbg, r, lane);
            else
                gate_up_rows<8>(d, gate, up, x, ldx, e, s0, g0, nb, pick_of_slot, act, gate_dbg, up_dbg, r, lane);
        }
    }
}

// ------------------------------------------------------------------- down

template <int NB>
__device__ __forceinline__ void down_rows(const MoeDims &d, const QMatrix &down, const float *act, uint32_t e,
                                          uint32_t s0, uint32_t g0, uint32_t nb, float *eout, uint32_t row, int q) {
    const uint32_t H = d.hidden, I = d.routed;
    const bool live = row < H;
    const uint8_t *drow = down.data + ((size_t)e * H + (live ? row : 0u)) * down.row_bytes;
    float acc[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) acc[j] = 0.0f;
    const float *arow[NB];
#pragma unroll
    for (int j = 0; j < NB; ++j) arow[j] = act + (size_t)(s0 + g0 + ((uint32_t)j < nb ? j : 0)) * I;
    const bool aal = (I & 3u) == 0u && (reinterpret_cast<uintptr_t>(act) & 15u) == 0u;
    if (live) {
        for (uint32_t base = (uint32_t)q * 32u; base < I; base += 128u) {
            const uint32_t count = min(32u, I - base);
            const float *ap[NB];
#pragma unroll
            for (int j = 0; j < NB; ++j) ap[j] = arow[j] + base;
            float w[32];
            decode32_any(down, drow, base, w);
            dot_group<NB>(w, count, ap, nb, aal && count == 32u, acc);
        }
    }
#pragma unroll
    for (int j = 0; j < NB; ++j) {
        float v = acc[j];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if ((uint32_t)j < nb && q == 0 && live) eout[(size_t)(s0 + g0 + j) * H + row] = v;
    }
}

// grid (max active experts, ceil(H / 64)); a warp owns 8 rows, four lanes
// per row splitting its 32-value runs.
__global__ void __launch_bounds__(kMoeThreads)
moe_down_kernel(MoeDims d, QMatrix down, const float *__restrict__ act, const uint32_t *__restrict__ active,
                const uint32_t *__restrict__ offsets, float *__restrict__ eout, ErrorWord err) {
    pdl_wait();
    if (moe_err_raised(err) || blockIdx.x >= active[0]) return;
    const uint32_t e = active[1 + blockIdx.x];
    const uint32_t s0 = offsets[e], n = offsets[e + 1] - s0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t row = blockIdx.y * kMoeRowsPerCta + (uint32_t)warp * 8u + (uint32_t)(lane >> 2);
    const int q = lane & 3;
    for (uint32_t g0 = 0; g0 < n; g0 += kMoeGroup) {
        const uint32_t nb = min((uint32_t)kMoeGroup, n - g0);
        if (nb == 1)
            down_rows<1>(d, down, act, e, s0, g0, nb, eout, row, q);
        else if (nb == 2)
            down_rows<2>(d, down, act, e, s0, g0, nb, eout, row, q);
        else if (nb <= 4)
            down_rows<4>(d, down, act, e, s0, g0, nb, eout, row, q);
        else
            down_rows<8>(d, down, act, e, s0, g0, nb, eout, row, q);
    }
}

// ------------------------------------------------ streamed (persistent) paths
//
// Q4_K gate/up and planar Q8_0 down.  One CTA per SM walks a contiguous
// range of tiles (tile = one active expert's block of rows; an expert's
// tiles are consecutive, so a CTA changes experts a few times per launch).
// Tiles stream HBM -> shared memory through a ring of stages (bulk copies,
// mbarrier completion); thread 0 refills a stage as soon as the CTA has read
// it, so ring - 1 tiles are in flight while one is decoded.  The activations
// of the expert's tokens stay in registers (as tensor-core B fragments) for
// every tile of the expert: shared memory carries the weights only.
//
// The products run on the tensor cores (mma.sync m16n8k16, f16 operands,
// F32 accumulation) with both operands built in registers:
//   A (16 rows x 16 columns of codes): each code becomes an exact fp16 by
//     OR-ing it into the mantissa of 1024 (Q4_K nibbles moved to mantissa
//     bits 6..9: 1024 + 64 q, one SHF + LOP3 per pair; sign-flipped Q8_0
//     bytes in the low mantissa byte: 1152 + c, one PRMT per pair).  The
//     offset is removed per sub-block with the sum of the activations, which
//     the same MMA computes against an all-ones A.
//   B (16 columns x 8 MMA columns): column 2t holds the high fp16 part of
//     token t's activations, column 2t + 1 the low part (x' - hi rounded to
//     fp16): hi + lo carries about 22 bits of x' = x * 2^k, k chosen per
//     (warp, token) so that max |x'| lies in [2^14, 2^15).  Four tokens per
//     pass.
// Every fp16 product is exact in F32; the error is the split (2^-22 of |x'|)
// and the F32 accumulation.  The K order inside a 16-column step is a
// permutation applied to A and B alike; it does not change the sum.
//
// A warp owns a fixed column range (Q4_K: one super-block of the tile's gate
// or up rows; Q8_0: one or two 32-code blocks of every row) and walks its
// rows in blocks of 16; lane (g = lane / 4, q = lane % 4) holds rows g and
// g + 8 of a block and token q's two accumulator columns.  Per-warp partial
// sums meet in shared memory, where one thread per output finishes the sum.

constexpr uint32_t kStreamThreads = 640;
constexpr uint32_t kStreamRing = 4;
constexpr uint32_t kGuTile = 32;      // gate rows (and as many up rows) per tile: two 16-row MMA blocks
constexpr uint32_t kDnTile = 128;     // down rows per tile
// The dynamic shared memory the streamed kernels may ask for: the 227 KB
// per-block opt-in less the static part and the 1 KB reserved per CTA.
constexpr uint32_t kStreamSmemLimit = 224u * 1024u;
constexpr uint32_t kStageWaitPolls = 1u << 26;
constexpr uint32_t kMmaWarps = kStreamThreads / 32u;
constexpr uint32_t kGuSbMax = kMmaWarps / 2u;   // super-blocks per row the gate/up warps cover
constexpr uint32_t kMmaTokens = 4;              // tokens per pass
constexpr uint32_t kDnMaxBpw = 2;               // Q8_0 blocks per down warp
constexpr uint32_t kH1024 = 0x64006400u;        // fp16 pair (1024, 1024)
constexpr uint32_t kHOnes = 0x3C003C00u;        // fp16 pair (1, 1)

__device__ __forceinline__ uint32_t moe_smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void moe_bulk(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(moe_smem_u32(dst)), "l"(src), "r"(bytes), "r"(moe_smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void moe_expect(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(moe_smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// Bounded wait for the phase of `bar` with the given parity; false when it
// gave up.
__device__ __forceinline__ bool moe_bar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = moe_smem_u32(bar);
    for (uint32_t i = 0; i < kStageWaitPolls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

// The CTA's share [begin, end) of `total` tiles.
__device__ __forceinline__ void tile_range(uint64_t total, uint32_t &begin, uint32_t &end) {
    begin = (uint32_t)(total * blockIdx.x / gridDim.x);
    end = (uint32_t)(total * (blockIdx.x + 1) / gridDim.x);
}

// A cursor over the CTA's tiles: tile (a, j) (active expert a, row block j)
// sits in ring slot `slot`, and its copies complete the phase of that slot's
// barrier with parity `phase`.  It advances without division.
struct TileCursor {
    uint32_t a, j, slot, phase;

    __device__ __forceinline__ void start(uint32_t tau, uint32_t J) { a = tau / J, j = tau % J, slot = 0, phase = 0; }
    __device__ __forceinline__ void next(uint32_t J, uint32_t ring) {
        if (++j == J) j = 0, ++a;
        if (++slot == ring) slot = 0, phase ^= 1u;
    }
};

struct StreamRing {
    uint64_t *full;
    uint8_t *base;
    uint32_t stage_bytes, ring;

    __device__ __forceinline__ uint8_t *stage(uint32_t slot) const { return base + (size_t)slot * stage_bytes; }
    __device__ __forceinline__ uint64_t *bar(uint32_t slot) const { return full + slot; }

    // Thread 0 only: waits (bounded) for the `count` issued tiles from cursor
    // c on, so that no copy lands in shared memory after the CTA has exited.
    __device__ void drain(TileCursor c, uint32_t count, uint32_t J) const {
        for (uint32_t i = 0; i < count; ++i, c.next(J, ring)) moe_bar_wait(bar(c.slot), c.phase);
    }
};

__device__ __forceinline__ void ring_init(uint64_t *full, uint32_t ring) {
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < ring; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(moe_smem_u32(full + s)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
}

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 2^k for |k| <= 126.
__device__ __forceinline__ float pow2i(int k) { return __uint_as_float((uint32_t)(k + 127) << 23); }

// The prescale exponent k of a token whose largest |x| over the warp's
// columns is m: max |x * 2^k| in [2^14, 2^15); 0 for zero or non-finite m.
__device__ __forceinline__ int prescale_exp(float m) {
    if (!(m > 0.0f) || !isfinite(m)) return 0;
    const int e = (int)((__float_as_uint(m) >> 23) & 0xFFu) - 126;   // m < 2^e (subnormal m: e = -126)
    return max(-126, min(126, 15 - e));
}

// The B register of two scaled activation values: their high fp16 parts for
// an even MMA column, their low parts (value - high part) for an odd one.
__device__ __forceinline__ uint32_t b_part(float x0, float x1, bool low) {
    const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
    const __half2 v = low ? __floats2half2_rn(x0 - __half2float(h0), x1 - __half2float(h1)) : __halves2half2(h0, h1);
    return *reinterpret_cast<const uint32_t *>(&v);
}

// Byte i of v as a float (0..255): the byte in the mantissa of 2^23, minus
// 2^23.
__device__ __forceinline__ float byte_f(uint32_t v, uint32_t i) {
    return __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7540u | i)) - 8388608.0f;
}

// ---- Q4_K gate/up: a warp owns one super-block of the tile's gate or up
// rows (H / 256 <= kGuSbMax).  Lane (g, q) reads bytes 8q .. 8q + 7 of each
// 32-byte code group: their low nibbles are values 8q .. 8q + 7 of the
// group's first sub-block, their high nibbles the same values of the second.

// Scale-table entries of one super-block header h (fp16 d, fp16 dmin, 12
// packed 6-bit scale / min bytes) for sub-blocks 4*half .. 4*half + 3: per
// code group (two sub-blocks) (d*sc/64, 16*d*sc + dmin*m) of each, d*sc and
// dmin*m rounded as the reference rounds them (src/kq_numeric.c:161-174
// layout).  The four scales and mins come out one per byte lane: sub-block
// j < 4: scale s[j] & 63, min s[j+4] & 63; j >= 4: scale
// (s[j+4] & 15) | (s[j-4] >> 6) << 4, min (s[j+4] >> 4) | (s[j] >> 6) << 4.
__device__ __forceinline__ void q4k_header_entries(uint4 h, uint32_t half, float4 &e0, float4 &e1) {
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dm = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t sc = half ? (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u) : h.y & 0x3F3F3F3Fu;
    const uint32_t mn = half ? ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u) : h.z & 0x3F3F3F3Fu;
    float a[4], b[4];
#pragma unroll
    for (uint32_t i = 0; i < 4; ++i) {
        const float dl = __fmul_rn(d, byte_f(sc, i));
        a[i] = dl * 0.015625f;
        b[i] = fmaf(16.0f, dl, __fmul_rn(dm, byte_f(mn, i)));
    }
    e0 = make_float4(a[0], b[0], a[1], b[1]);
    e1 = make_float4(a[2], b[2], a[3], b[3]);
}

// The fp16 pairs of code word w (bytes b0..b3): low nibbles of (b0, b2) and
// of (b1, b3), high nibbles of (b0, b2) and of (b1, b3), each nibble moved
// to mantissa bits 6..9: value 1024 + 64 q.
__device__ __forceinline__ uint32_t q4_lo02(uint32_t w) { return ((w << 6) & 0x03C003C0u) | kH1024; }
__device__ __forceinline__ uint32_t q4_lo13(uint32_t w) { return ((w >> 2) & 0x03C003C0u) | kH1024; }
__device__ __forceinline__ uint32_t q4_hi02(uint32_t w) { return ((w << 2) & 0x03C003C0u) | kH1024; }
__device__ __forceinline__ uint32_t q4_hi13(uint32_t w) { return ((w >> 6) & 0x03C003C0u) | kH1024; }

// One warp's B operand for one pass of up to four tokens: per code group gg
// of the super-block, the first sub-block's value pairs (8q, 8q+2),
// (8q+1, 8q+3), (8q+4, 8q+6), (8q+5, 8q+7), then the second's; the sums of
// x' over each sub-block for token q; 2^-k of token q.
struct GuFrags {
    uint32_t b[4][8];
    float xs[4][2];
    float unscale;
};

// xrow: the activation row of this lane's token (MMA column g = lane / 4:
// token g / 2, high part for even g, low part for odd g), null past the
// pass's tokens.
__device__ __forceinline__ void gu_frags(const float *__restrict__ xrow, uint32_t s, uint32_t lane, GuFrags &f) {
    const uint32_t g = lane >> 2, q = lane & 3u;
    const bool low = (g & 1u) != 0u;
    const float *xr = xrow ? xrow + s * 256u + 8u * q : nullptr;
    float m = 0.0f;   // pass 1: the token's largest |x| over the warp's 256 columns
    if (xr) {
#pragma unroll
        for (int o = 0; o < 16; ++o) {   // 4 code groups x 2 sub-blocks x 2 float4
            const float4 v =
                __ldg(reinterpret_cast<const float4 *>(xr + 64 * (o >> 2) + 32 * ((o >> 1) & 1) + 4 * (o & 1)));
            m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int k = prescale_exp(m);
    const float sc = pow2i(k);
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {   // pass 2: scaled values -> fp16 parts
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
            if (xr) {
                a = __ldg(reinterpret_cast<const float4 *>(xr + 64 * gg + 32 * h));
                b = __ldg(reinterpret_cast<const float4 *>(xr + 64 * gg + 32 * h + 4));
            }
            f.b[gg][4 * h] = b_part(a.x * sc, a.z * sc, low);
            f.b[gg][4 * h + 1] = b_part(a.y * sc, a.w * sc, low);
            f.b[gg][4 * h + 2] = b_part(b.x * sc, b.z * sc, low);
            f.b[gg][4 * h + 3] = b_part(b.y * sc, b.w * sc, low);
        }
        float dl[4] = {0.f, 0.f, 0.f, 0.f}, dh[4] = {0.f, 0.f, 0.f, 0.f};
        mma_f16(dl, kHOnes, kHOnes, kHOnes, kHOnes, f.b[gg][0], f.b[gg][1]);
        mma_f16(dl, kHOnes, kHOnes, kHOnes, kHOnes, f.b[gg][2], f.b[gg][3]);
        mma_f16(dh, kHOnes, kHOnes, kHOnes, kHOnes, f.b[gg][4], f.b[gg][5]);
        mma_f16(dh, kHOnes, kHOnes, kHOnes, kHOnes, f.b[gg][6], f.b[gg][7]);
        f.xs[gg][0] = dl[0] + dl[1];
        f.xs[gg][1] = dh[0] + dh[1];
    }
    f.unscale = pow2i(-__shfl_sync(0xffffffffu, k, (int)(8u * q)));
}

// Partial sums over super-block s of rows g, g + 8 of the 16-row block at
// `rows` (pitch rb), token q.  tab: the block's first row of the scale table
// (pitch tp float4).
__device__ __forceinline__ void gu_block(const uint8_t *rows, uint32_t rb, const float4 *tab, uint32_t tp,
                                         uint32_t s, uint32_t lane, const GuFrags &f, float &t0, float &t1) {
    const uint32_t g = lane >> 2, q = lane & 3u;
    const uint8_t *r0 = rows + (size_t)g * rb + s * 144u + 16u + 8u * q, *r1 = r0 + (size_t)8 * rb;
    const float4 *s0 = tab + (size_t)g * tp + s * 4u, *s1 = s0 + (size_t)8 * tp;
#pragma unroll
    for (int gg = 0; gg < 4; ++gg) {
        const uint2 c0 = *reinterpret_cast<const uint2 *>(r0 + 32 * gg);
        const uint2 c1 = *reinterpret_cast<const uint2 *>(r1 + 32 * gg);
        float dl[4] = {0.f, 0.f, 0.f, 0.f}, dh[4] = {0.f, 0.f, 0.f, 0.f};
        mma_f16(dl, q4_lo02(c0.x), q4_lo02(c1.x), q4_lo13(c0.x), q4_lo13(c1.x), f.b[gg][0], f.b[gg][1]);
        mma_f16(dl, q4_lo02(c0.y), q4_lo02(c1.y), q4_lo13(c0.y), q4_lo13(c1.y), f.b[gg][2], f.b[gg][3]);
        mma_f16(dh, q4_hi02(c0.x), q4_hi02(c1.x), q4_hi13(c0.x), q4_hi13(c1.x), f.b[gg][4], f.b[gg][5]);
        mma_f16(dh, q4_hi02(c0.y), q4_hi02(c1.y), q4_hi13(c0.y), q4_hi13(c1.y), f.b[gg][6], f.b[gg][7]);
        const float4 a = s0[gg], b = s1[gg];
        t0 += fmaf(a.x, dl[0] + dl[1], fmaf(a.z, dh[0] + dh[1], -fmaf(a.y, f.xs[gg][0], a.w * f.xs[gg][1])));
        t1 += fmaf(b.x, dl[2] + dl[3], fmaf(b.z, dh[2] + dh[3], -fmaf(b.y, f.xs[gg][0], b.w * f.xs[gg][1])));
    }
}

// Grid: one CTA per SM; block kStreamThreads.  Warp w decodes super-block
// w % kGuSbMax of the tile's gate rows (w < kGuSbMax) or up rows, as two
// 16-row MMA blocks.  Dynamic shared memory: the ring (ring stages of
// kGuTile gate rows then kGuTile up rows, pitch row_bytes), the scale table
// of one 16-row block of each half [2][16][H/64] float4 (each warp writes
// and reads its own rows and super-block, block by block), the per-warp
// partial sums [kMmaWarps][kGuTile][kMmaTokens].  Tiles in active-expert-
// major order.
__global__ void __launch_bounds__(kStreamThreads, 1)
moe_gate_up_stream_kernel(MoeDims d, QMatrix gate, QMatrix up, const float *__restrict__ x, uint32_t ldx,
                          const uint32_t *__restrict__ active, const uint32_t *__restrict__ offsets,
                          const uint32_t *__restrict__ pick_of_slot, uint32_t ring, float *__restrict__ act,
                          float *gate_dbg, float *up_dbg, ErrorWord err) {
    extern __shared__ __align__(128) uint8_t gsm[];
    __shared__ __align__(8) uint64_t full[kStreamRing];
    const uint32_t H = d.hidden, I = d.routed, rb = gate.row_bytes;
    const uint32_t SB = H / 256u, TR = 2u * kGuTile, tp = H / 64u;
    const uint32_t J = (I + kGuTile - 1u) / kGuTile;
    const StreamRing rg{full, gsm, TR * rb, ring};
    float4 *table = reinterpret_cast<float4 *>(gsm + (size_t)ring * rg.stage_bytes);
    float *red = reinterpret_cast<float *>(table + (size_t)2 * 16u * tp);
    ring_init(full, ring);
    pdl_wait();
    if (moe_err_raised(err)) return;
    uint32_t tb, te;
    tile_range((uint64_t)active[0] * J, tb, te);
    if (tb >= te) return;
    const uint32_t n_tiles = te - tb;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t sb = warp % kGuSbMax, half = warp / kGuSbMax;   // super-block; 0 gate rows, 1 up rows
    const bool worker = sb < SB;
    const uint32_t g = lane >> 2, q = lane & 3u;

    TileCursor pc;   // thread 0: the next tile to issue
    pc.start(tb, J);
    uint32_t issued = 0;
    auto issue = [&]() {
        const uint32_t e = active[1u + pc.a], r0 = pc.j * kGuTile, rows = min(kGuTile, I - r0);
        uint8_t *st = rg.stage(pc.slot);
        uint64_t *bar = rg.bar(pc.slot);
        const size_t off = ((size_t)e * I + r0) * rb;
        moe_expect(bar, 2u * rows * rb);
        moe_bulk(st, gate.data + off, rows * rb, bar);
        moe_bulk(st + (size_t)kGuTile * rb, up.data + off, rows * rb, bar);
        pc.next(J, ring);
        ++issued;
    };
    if (tid == 0)
        while (issued < n_tiles && issued < ring) issue();

    GuFrags f;
    float *pr = red + (size_t)warp * kGuTile * kMmaTokens;
    const float4 *tab = table + (size_t)half * 16u * tp;   // the warp's half of the 16-row table
    TileCursor c;
    c.start(tb, J);
    uint32_t cur = 0xFFFFFFFFu, s0 = 0, n = 0, loaded = 0xFFFFFFFFu;
    for (uint32_t k = 0; k < n_tiles; ++k, c.next(J, ring)) {
        const uint32_t r0 = c.j * kGuTile, rows = min(kGuTile, I - r0);
        if (c.a != cur) {
            const uint32_t e = active[1u + c.a];
            cur = c.a, s0 = offsets[e], n = offsets[e + 1u] - s0, loaded = 0xFFFFFFFFu;
        }
        const uint8_t *st = rg.stage(c.slot);
        const bool ok = moe_bar_wait(rg.bar(c.slot), c.phase);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                moe_raise(err, kErrTimeout | (1u << 8));
                rg.drain(c, issued - k, J);
            }
            return;
        }
        const uint8_t *blk = st + (size_t)half * kGuTile * rb;
        for (uint32_t g0 = 0; g0 < n; g0 += kMmaTokens) {
            const uint32_t nb = min(kMmaTokens, n - g0);
            if (worker) {
                if (loaded != g0) {
                    const uint32_t t = lane >> 3;   // this lane's token in the pass
                    gu_frags(t < nb ? x + (size_t)(pick_of_slot[s0 + g0 + t] / d.top_k) * ldx : nullptr, sb, lane,
                             f);
                    loaded = g0;
                }
                for (uint32_t b = 0; b < kGuTile / 16u; ++b) {   // the half's 16-row MMA blocks
                    {   // lanes 2r, 2r + 1: the scale entries of block row r's super-block sb
                        const uint32_t r = lane >> 1, hh = lane & 1u;
                        if (16u * b + r < rows) {
                            const uint4 hd =
                                *reinterpret_cast<const uint4 *>(blk + (size_t)(16u * b + r) * rb + sb * 144u);
                            float4 e0, e1;
                            q4k_header_entries(hd, hh, e0, e1);
                            float4 *tr = table + ((size_t)half * 16u + r) * tp + sb * 4u + 2u * hh;
                            tr[0] = e0;
                            tr[1] = e1;
                        }
                        __syncwarp();
                    }
                    float t0 = 0.0f, t1 = 0.0f;
                    gu_block(blk + (size_t)16u * b * rb, rb, tab, tp, sb, lane, f, t0, t1);
                    if (q < nb) {
                        pr[(16u * b + g) * kMmaTokens + q] = t0 * f.unscale;
                        pr[(16u * b + g + 8u) * kMmaTokens + q] = t1 * f.unscale;
                    }
                    __syncwarp();   // the table is rewritten by the next block
                }
            }
            __syncthreads();   // partial sums complete; the stage has been read
            const bool last = g0 + kMmaTokens >= n;
            if (last && tid == 0 && issued < n_tiles) issue();
            if (tid < kGuTile * nb) {   // one thread per (row, token): gate and up sums, SwiGLU
                const uint32_t i = tid % kGuTile, t = tid / kGuTile;
                if (i < rows) {
                    float sg = 0.0f, su = 0.0f;
                    for (uint32_t w = 0; w < SB; ++w) {
                        sg += red[((size_t)w * kGuTile + i) * kMmaTokens + t];
                        su += red[((size_t)(kGuSbMax + w) * kGuTile + i) * kMmaTokens + t];
                    }
                    const size_t oo = (size_t)(s0 + g0 + t) * I + r0 + i;
                    act[oo] = moe_swiglu(sg, su);
                    if (gate_dbg) {
                        gate_dbg[oo] = sg;
                        up_dbg[oo] = su;
                    }
                }
            }
            if (!last) __syncthreads();   // the partial sums are rewritten by the next pass
        }
        if (n == 0) {   // no rows to write (not produced by the dispatch): keep the ring going
            __syncthreads();
            if (tid == 0 && issued < n_tiles) issue();
        }
    }
}

// ---- planar Q8_0 down: row = I code bytes, then the I/32 fp16 block
// scales (pitch row_bytes).  A warp owns code blocks c0 .. c0 + nblk - 1 of
// every row; lane (g, q) reads bytes 8q .. 8q + 7 of each block.

// The fp16 pairs of sign-flipped code bytes (b0, b1) and (b2, b3) of word v:
// each byte c + 128 in the low mantissa byte of 1024: value 1152 + c.
__device__ __forceinline__ uint32_t q8_01(uint32_t v) { return __byte_perm(v, 0x64646464u, 0x4140u); }
__device__ __forceinline__ uint32_t q8_23(uint32_t v) { return __byte_perm(v, 0x64646464u, 0x4342u); }

struct DnFrags {
    uint32_t b[kDnMaxBpw][4];
    float xs[kDnMaxBpw];
    float unscale;
};

// arow: this lane's token's activation row (null past the pass's tokens).
__device__ __forceinline__ void dn_frags(const float *__restrict__ arow, uint32_t c0, uint32_t nblk, uint32_t lane,
                                         DnFrags &f) {
    const uint32_t g = lane >> 2, q = lane & 3u;
    const bool low = (g & 1u) != 0u;
    float v[kDnMaxBpw][8];
    float m = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < kDnMaxBpw; ++j) {
        float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
        if (arow && j < nblk) {
            const float *xr = arow + (c0 + j) * 32u + 8u * q;
            a = *reinterpret_cast<const float4 *>(xr);
            b = *reinterpret_cast<const float4 *>(xr + 4);
        }
        const float w8[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            v[j][i] = w8[i];
            m = fmaxf(m, fabsf(w8[i]));
        }
    }
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
    m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
    const int k = prescale_exp(m);
    const float sc = pow2i(k);
#pragma unroll
    for (uint32_t j = 0; j < kDnMaxBpw; ++j) {
#pragma unroll
        for (int i = 0; i < 4; ++i) f.b[j][i] = b_part(v[j][2 * i] * sc, v[j][2 * i + 1] * sc, low);
        float dx[4] = {0.f, 0.f, 0.f, 0.f};
        mma_f16(dx, kHOnes, kHOnes, kHOnes, kHOnes, f.b[j][0], f.b[j][1]);
        mma_f16(dx, kHOnes, kHOnes, kHOnes, kHOnes, f.b[j][2], f.b[j][3]);
        f.xs[j] = dx[0] + dx[1];
    }
    f.unscale = pow2i(-__shfl_sync(0xffffffffu, k, (int)(8u * q)));
}

// Partial sums over the warp's blocks of rows g, g + 8 of the 16-row block
// at `rows` (pitch rb), token q.  code: byte offset of the lane's first code
// (c0*32 + 8q); scale: byte offset of the first block's scale (I + 2*c0).
__device__ __forceinline__ void dn_block(const uint8_t *rows, uint32_t rb, uint32_t code, uint32_t scale,
                                         uint32_t nblk, uint32_t lane, const DnFrags &f, float &t0, float &t1) {
    const uint8_t *r0 = rows + (size_t)(lane >> 2) * rb, *r1 = r0 + (size_t)8 * rb;
#pragma unroll
    for (uint32_t j = 0; j < kDnMaxBpw; ++j) {
        if (j >= nblk) break;
        const uint2 a = *reinterpret_cast<const uint2 *>(r0 + code + 32u * j);
        const uint2 b = *reinterpret_cast<const uint2 *>(r1 + code + 32u * j);
        const uint32_t ax = a.x ^ 0x80808080u, ay = a.y ^ 0x80808080u, bx = b.x ^ 0x80808080u,
                       by = b.y ^ 0x80808080u;
        float dd[4] = {0.f, 0.f, 0.f, 0.f};
        mma_f16(dd, q8_01(ax), q8_01(bx), q8_23(ax), q8_23(bx), f.b[j][0], f.b[j][1]);
        mma_f16(dd, q8_01(ay), q8_01(by), q8_23(ay), q8_23(by), f.b[j][2], f.b[j][3]);
        const float d0 = __half2float(*reinterpret_cast<const __half *>(r0 + scale + 2u * j));
        const float d1 = __half2float(*reinterpret_cast<const __half *>(r1 + scale + 2u * j));
        t0 = fmaf(d0, (dd[0] + dd[1]) - 1152.0f * f.xs[j], t0);
        t1 = fmaf(d1, (dd[2] + dd[3]) - 1152.0f * f.xs[j], t1);
    }
}

// Grid: one CTA per SM; block kStreamThreads.  Dynamic shared memory: the
// ring (ring stages of kDnTile rows, pitch row_bytes), the per-warp partial
// sums [kMmaWarps][kDnTile][kMmaTokens].  Tiles in active-expert-major
// order; act [slots][I] by slot -> eout [slots][H].
__global__ void __launch_bounds__(kStreamThreads, 1)
moe_down_stream_kernel(MoeDims d, QMatrix down, const float *__restrict__ act, const uint32_t *__restrict__ active,
                       const uint32_t *__restrict__ offsets, uint32_t ring, float *__restrict__ eout, ErrorWord err) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ __align__(8) uint64_t full[kStreamRing];
    const uint32_t H = d.hidden, I = d.routed, rb = down.row_bytes;
    const uint32_t NB = I / 32u, bpw = (NB + kMmaWarps - 1u) / kMmaWarps;
    const uint32_t J = (H + kDnTile - 1u) / kDnTile;
    const StreamRing rg{full, dsm, kDnTile * rb, ring};
    float *red = reinterpret_cast<float *>(dsm + (size_t)ring * rg.stage_bytes);
    ring_init(full, ring);
    pdl_wait();
    if (moe_err_raised(err)) return;
    uint32_t tb, te;
    tile_range((uint64_t)active[0] * J, tb, te);
    if (tb >= te) return;
    const uint32_t n_tiles = te - tb;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t c0 = warp * bpw, nblk = c0 < NB ? min(bpw, NB - c0) : 0u;
    const uint32_t wk = (NB + bpw - 1u) / bpw;   // warps with blocks
    const bool worker = nblk > 0u;
    const uint32_t g = lane >> 2, q = lane & 3u;

    TileCursor pc;   // thread 0: the next tile to issue
    pc.start(tb, J);
    uint32_t issued = 0;
    auto issue = [&]() {
        const uint32_t e = active[1u + pc.a], r0 = pc.j * kDnTile, rows = min(kDnTile, H - r0);
        uint64_t *bar = rg.bar(pc.slot);
        moe_expect(bar, rows * rb);
        moe_bulk(rg.stage(pc.slot), down.data + ((size_t)e * H + r0) * rb, rows * rb, bar);
        pc.next(J, ring);
        ++issued;
    };
    if (tid == 0)
        while (issued < n_tiles && issued < ring) issue();

    DnFrags f;
    float *pr = red + (size_t)warp * kDnTile * kMmaTokens;
    TileCursor c;
    c.start(tb, J);
    uint32_t cur = 0xFFFFFFFFu, s0 = 0, n = 0, loaded = 0xFFFFFFFFu;
    for (uint32_t k = 0; k < n_tiles; ++k, c.next(J, ring)) {
        const uint32_t r0 = c.j * kDnTile, rows = min(kDnTile, H - r0);
        if (c.a != cur) {
            const uint32_t e = active[1u + c.a];
            cur = c.a, s0 = offsets[e], n = offsets[e + 1u] - s0, loaded = 0xFFFFFFFFu;
        }
        const uint8_t *st = rg.stage(c.slot);
        const bool ok = moe_bar_wait(rg.bar(c.slot), c.phase);
        if (__syncthreads_or(!ok)) {
            if (tid == 0) {
                moe_raise(err, kErrTimeout | (2u << 8));
                rg.drain(c, issued - k, J);
            }
            return;
        }
        for (uint32_t g0 = 0; g0 < n; g0 += kMmaTokens) {
            const uint32_t nb = min(kMmaTokens, n - g0);
            if (worker) {
                if (loaded != g0) {
                    const uint32_t t = lane >> 3;   // this lane's token in the pass
                    dn_frags(t < nb ? act + (size_t)(s0 + g0 + t) * I : nullptr, c0, nblk, lane, f);
                    loaded = g0;
                }
#pragma unroll
                for (uint32_t b = 0; b < kDnTile / 16u; ++b) {
                    float t0 = 0.0f, t1 = 0.0f;
                    dn_block(st + (size_t)b * 16u * rb, rb, c0 * 32u + 8u * q, I + 2u * c0, nblk, lane, f, t0, t1);
                    if (q < nb) {
                        pr[(b * 16u + g) * kMmaTokens + q] = t0 * f.unscale;
                        pr[(b * 16u + g + 8u) * kMmaTokens + q] = t1 * f.unscale;
                    }
                }
            }
            __syncthreads();   // partial sums complete; the stage has been read
            const bool last = g0 + kMmaTokens >= n;
            if (last && tid == 0 && issued < n_tiles) issue();
            for (uint32_t o = tid; o < kDnTile * nb; o += kStreamThreads) {   // one thread per (row, token)
                const uint32_t i = o % kDnTile, t = o / kDnTile;
                if (i < rows) {
                    float sum = 0.0f;
                    for (uint32_t w = 0; w < wk; ++w) sum += red[((size_t)w * kDnTile + i) * kMmaTokens + t];
                    eout[(size_t)(s0 + g0 + t) * H + r0 + i] = sum;
                }
            }
            if (!last) __syncthreads();   // the partial sums are rewritten by the next pass
        }
        if (n == 0) {
            __syncthreads();
            if (tid == 0 && issued < n_tiles) issue();
        }
    }
}

// ---------------------------------------------------------------- shared

// act[t][i] = swiglu(gu[t][i], gu[t][S + i])
__global__ void moe_swiglu_kernel(const float *__restrict__ gu, uint32_t S, uint32_t T, float *__restrict__ act,
                                  ErrorWord err) {
    pdl_wait();
    if (moe_err_raised(err)) return;
    const uint64_t n = (uint64_t)S * T;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
        const uint64_t t = i / S, c = i % S;
        act[i] = moe_swiglu(gu[t * 2 * S + c], gu[t * 2 * S + S + c]);
    }
}

// ---------------------------------------------------------------- combine

// One CTA per (token, 256 features): y = sum over the selected experts in
// ascending id of eout * weight (each product and sum rounded,
// src/kq_moe_qwen38.c:745-759), plus shared_out * sigmoid(shared gate logit)
// (:820-836).
__global__ void __launch_bounds__(kMoeThreads)
moe_combine_kernel(MoeDims d, const float *__restrict__ logits, uint32_t ldl, const uint32_t *__restrict__ sel_ids,
                   const float *__restrict__ sel_w, const uint32_t *__restrict__ slot,
                   const float *__restrict__ eout, const float *__restrict__ shared_out, float *__restrict__ y,
                   MoeDebug dbg, ErrorWord err) {
    __shared__ uint32_t order[kMoeMaxTopK];
    __shared__ float scale_s;
    __shared__ int bad;
    pdl_wait();
    if (moe_err_raised(err)) return;
    const uint32_t t = blockIdx.x, K = d.top_k, H = d.hidden;
    const int tid = threadIdx.x;
    if (tid == 0) {
        bad = 0;
        for (uint32_t p = 0; p < K; ++p) order[p] = p;
        for (uint32_t i = 1; i < K; ++i) {   // positions by ascending expert id
            const uint32_t v = order[i];
            uint32_t pos = i;
            while (pos > 0 && sel_ids[(size_t)t * K + order[pos - 1]] > sel_ids[(size_t)t * K + v]) {
                order[pos] = order[pos - 1];
                --pos;
            }
            order[pos] = v;
        }
        const float logit = logits[(size_t)t * ldl + d.experts];
        const float sc = moe_sigmoid(logit);
        if (!isfinite(logit) || !isfinite(sc)) bad = 1;
        scale_s = sc;
        if (dbg.scale && blockIdx.y == 0) {
            dbg.scale[2 * t] = logit;
            dbg.scale[2 * t + 1] = sc;
        }
    }
    __syncthreads();
    const float sc = scale_s;
    bool ok = bad == 0;
    for (uint32_t f = blockIdx.y * kMoeThreads + tid; f < H; f += kMoeThreads * gridDim.y) {
        float s = 0.0f;
        for (uint32_t q = 0; q < K; ++q) {
            const uint32_t p = order[q];
            const uint32_t sl = slot[(size_t)t * K + p];
            const float wo = __fmul_rn(eout[(size_t)sl * H + f], sel_w[(size_t)t * K + p]);
            s = __fadd_rn(s, wo);
            if (dbg.weighted) dbg.weighted[(size_t)sl * H + f] = wo;
        }
        const float gs = __fmul_rn(shared_out[(size_t)t * H + f], sc);
        const float out = __fadd_rn(s, gs);
        if (!isfinite(s) || !isfinite(gs) || !isfinite(out)) ok = false;
        y[(size_t)t * H + f] = out;
        if (dbg.routed_sum) {
            dbg.routed_sum[(size_t)t * H + f] = s;
            dbg.gated_shared[(size_t)t * H + f] = gs;
        }
    }
    if (!ok) moe_raise(err, kErrNonFinite);
}

// ---------------------------------------------------------------- host

size_t moe_workspace_bytes(const MoeDims &d, uint32_t T, bool debug) {
    const uint64_t E = d.experts, K = d.top_k, I = d.routed, S = d.shared, H = d.hidden;
    const uint64_t picks = (uint64_t)T * K;
    size_t b = 0;
    auto add = [&](uint64_t bytes) { b += (bytes + 255) & ~uint64_t(255); };
    add(T * (E + 1) * 4);   // logits
    add(T * E * 4);         // probabilities
    add(picks * 4);         // selected ids
    add(picks * 4);         // selected weights
    add(E * 4);             // counts
    add((E + 1) * 4);       // offsets
    add((E + 1) * 4);       // active experts
    add(picks * 4);         // rank
    add(picks * 4);         // slot
    add(picks * 4);         // pick of slot
    add(picks * I * 4);     // act
    add(picks * H * 4);     // eout
    add(T * 2 * S * 4);     // shared gate | up
    add(T * S * 4);         // shared act
    add(T * H * 4);         // shared out
    add(projection_workspace_floats(T, (uint32_t)(2 * S), (uint32_t)H) * 4);
    add(projection_workspace_floats(T, (uint32_t)H, (uint32_t)S) * 4);
    if (debug) {
        add(picks * I * 4 * 2);   // routed gate, up
        add(picks * H * 4);       // weighted outputs
        add(T * H * 4 * 2);       // routed sum, gated shared
        add(T * 2 * 4);           // shared logit, scale
    }
    return b;
}

void moe_carve(const MoeDims &d, uint32_t T, bool debug, void *ws, MoeBuffers &b) {
    const uint64_t E = d.experts, K = d.top_k, I = d.routed, S = d.shared, H = d.hidden;
    const uint64_t picks = (uint64_t)T * K;
    char *p = static_cast<char *>(ws);
    auto take = [&](uint64_t bytes) {
        char *r = p;
        p += (bytes + 255) & ~uint64_t(255);
        return r;
    };
    b.logits = reinterpret_cast<float *>(take(T * (E + 1) * 4));
    b.probs = reinterpret_cast<float *>(take(T * E * 4));
    b.sel_ids = reinterpret_cast<uint32_t *>(take(picks * 4));
    b.sel_w = reinterpret_cast<float *>(take(picks * 4));
    b.counts = reinterpret_cast<uint32_t *>(take(E * 4));
    b.offsets = reinterpret_cast<uint32_t *>(take((E + 1) * 4));
    b.active = reinterpret_cast<uint32_t *>(take((E + 1) * 4));
    b.rank = reinterpret_cast<uint32_t *>(take(picks * 4));
    b.slot = reinterpret_cast<uint32_t *>(take(picks * 4));
    b.pick_of_slot = reinterpret_cast<uint32_t *>(take(picks * 4));
    b.act = reinterpret_cast<float *>(take(picks * I * 4));
    b.eout = reinterpret_cast<float *>(take(picks * H * 4));
    b.shared_gu = reinterpret_cast<float *>(take(T * 2 * S * 4));
    b.shared_act = reinterpret_cast<float *>(take(T * S * 4));
    b.shared_out = reinterpret_cast<float *>(take(T * H * 4));
    b.proj_floats_gu = projection_workspace_floats(T, (uint32_t)(2 * S), (uint32_t)H);
    b.proj_gu = reinterpret_cast<float *>(take(b.proj_floats_gu * 4));
    b.proj_floats_down = projection_workspace_floats(T, (uint32_t)H, (uint32_t)S);
    b.proj_down = reinterpret_cast<float *>(take(b.proj_floats_down * 4));
    b.dbg = MoeDebug{};
    if (debug) {
        b.dbg.gate = reinterpret_cast<float *>(take(picks * I * 4 * 2));
        b.dbg.up = b.dbg.gate + picks * I;
        b.dbg.weighted = reinterpret_cast<float *>(take(picks * H * 4));
        b.dbg.routed_sum = reinterpret_cast<float *>(take(T * H * 4 * 2));
        b.dbg.gated_shared = b.dbg.routed_sum + (size_t)T * H;
        b.dbg.scale = reinterpret_cast<float *>(take(T * 2 * 4));
    }
}

void launch_moe_route(const MoeDims &d, const float *logits, uint32_t ldl, uint32_t T, MoeBuffers &b,
                      ErrorWord err, cudaStream_t stream) {
    const size_t smem = (size_t)d.experts * 4;
    static DeviceOnce attr;
    attr.run([] {
        cudaFuncSetAttribute(moe_route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)(kMoeMaxExperts * 4));
    });
    cudaMemsetAsync(b.counts, 0, (size_t)d.experts * 4, stream);
    launch_pdl(moe_route_kernel, T, kMoeThreads, smem, stream, d, logits, ldl, b.probs, b.sel_ids, b.sel_w,
               b.counts, b.rank, err);
    count_launch();
}

void launch_moe_dispatch(const MoeDims &d, uint32_t T, MoeBuffers &b, ErrorWord err, cudaStream_t stream) {
    static DeviceOnce attr;
    attr.run([] {
        cudaFuncSetAttribute(moe_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)((kMoeMaxExperts + 1) * 4));
    });
    launch_pdl(moe_dispatch_kernel, 1, kDispatchThreads, (size_t)(d.experts + 1) * 4, stream, d,
               (uint32_t)((uint64_t)T * d.top_k), b.sel_ids, b.counts, b.rank, b.offsets, b.active, b.slot,
               b.pick_of_slot, err);
    count_launch();
}

static bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0u; }

static int moe_sm_count() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

// Stages of a streamed kernel's ring that fit next to its fixed shared
// memory (0 when fewer than two fit).
static uint32_t stream_ring(size_t stage, size_t fixed) {
    if (fixed + 2 * stage > kStreamSmemLimit) return 0;
    return (uint32_t)std::min<size_t>(kStreamRing, (kStreamSmemLimit - fixed) / stage);
}

static size_t gate_up_fixed_bytes(const MoeDims &d) {
    return (size_t)2 * 16u * (d.hidden / 64u) * 16u + (size_t)kMmaWarps * kGuTile * kMmaTokens * 4u;
}

static size_t down_fixed_bytes() { return (size_t)kMmaWarps * kDnTile * kMmaTokens * 4u; }

// The streamed kernels' conditions: the types they decode (GGUF Q4_K rows,
// planar Q8_0 rows), 16-byte aligned rows and activations, the columns one
// CTA's warps cover, a ring of at least two stages.
static bool gate_up_stream_ok(const MoeDims &d, const QMatrix &g, const QMatrix &u, const float *x, uint32_t ldx) {
    return g.type == kTypeQ4_K && u.type == kTypeQ4_K && d.hidden % 256u == 0u && d.hidden / 256u <= kGuSbMax &&
           g.row_bytes == d.hidden / 256u * 144u && u.row_bytes == g.row_bytes && aligned16(g.data) &&
           aligned16(u.data) && aligned16(x) && ldx % 4u == 0u &&
           stream_ring((size_t)2 * kGuTile * g.row_bytes, gate_up_fixed_bytes(d)) >= 2u;
}

static bool down_stream_ok(const MoeDims &d, const QMatrix &m, const float *act) {
    return m.type == kTypeQ8_0 && m.layout == 1 && d.routed % 32u == 0u &&
           d.routed / 32u <= kMmaWarps * kDnMaxBpw && m.row_bytes % 16u == 0u &&
           m.row_bytes >= d.routed + d.routed / 16u && aligned16(m.data) && aligned16(act) &&
           stream_ring((size_t)kDnTile * m.row_bytes, down_fixed_bytes()) >= 2u;
}

void launch_moe_experts(const MoeDims &d, const MoeWeightsDev &w, const float *x, uint32_t ldx, uint32_t T,
                        MoeBuffers &b, ErrorWord err, cudaStream_t stream) {
    const uint32_t max_active = (uint32_t)std::min<uint64_t>(d.experts, (uint64_t)T * d.top_k);
    static DeviceOnce attr;
    static bool stream_attr_ok[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    attr.run([dev] {
        const cudaError_t e1 = cudaFuncSetAttribute(moe_gate_up_stream_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmemLimit);
        const cudaError_t e2 = cudaFuncSetAttribute(moe_down_stream_kernel,
                                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStreamSmemLimit);
        if (e1 != cudaSuccess || e2 != cudaSuccess)
            cudaGetLastError();   // the streamed kernels stay off on this device; nothing is left pending
        else if (dev >= 0 && dev < 64)
            stream_attr_ok[dev] = true;
    });
    const bool streamed = dev >= 0 && dev < 64 && stream_attr_ok[dev];
    const uint32_t sms = (uint32_t)moe_sm_count();
    {
        KernelTimer timer("moe_gate_up", stream);
        if (streamed && gate_up_stream_ok(d, w.gate, w.up, x, ldx)) {
            const size_t stage = (size_t)2 * kGuTile * w.gate.row_bytes, fixed = gate_up_fixed_bytes(d);
            const uint32_t ring = stream_ring(stage, fixed);
            const uint64_t tiles = (uint64_t)max_active * ((d.routed + kGuTile - 1) / kGuTile);
            const uint32_t grid = (uint32_t)std::min<uint64_t>(sms, tiles);
            launch_pdl(moe_gate_up_stream_kernel, grid, kStreamThreads, fixed + ring * stage, stream, d, w.gate,
                       w.up, x, ldx, b.active, b.offsets, b.pick_of_slot, ring, b.act, b.dbg.gate, b.dbg.up, err);
        } else {
            dim3 grid(max_active, (d.routed + kMoeRowsPerCta - 1) / kMoeRowsPerCta);
            launch_pdl(moe_gate_up_kernel, grid, kMoeThreads, 0, stream, d, w.gate, w.up, x, ldx, b.active,
                       b.offsets, b.pick_of_slot, b.act, b.dbg.gate, b.dbg.up, err);
        }
        count_launch();
    }
    {
        KernelTimer timer("moe_down", stream);
        if (streamed && down_stream_ok(d, w.down, b.act)) {
            const size_t stage = (size_t)kDnTile * w.down.row_bytes, fixed = down_fixed_bytes();
            const uint32_t ring = stream_ring(stage, fixed);
            const uint64_t tiles = (uint64_t)max_active * ((d.hidden + kDnTile - 1) / kDnTile);
            const uint32_t grid = (uint32_t)std::min<uint64_t>(sms, tiles);
            launch_pdl(moe_down_stream_kernel, grid, kStreamThreads, fixed + ring * stage, stream, d, w.down,
                       b.act, b.active, b.offsets, ring, b.eout, err);
        } else {
            dim3 grid(max_active, (d.hidden + kMoeRowsPerCta - 1) / kMoeRowsPerCta);
            launch_pdl(moe_down_kernel, grid, kMoeThreads, 0, stream, d, w.down, b.act, b.active, b.offsets, b.eout,
                       err);
        }
        count_launch();
    }
}

void launch_moe_swiglu(const float *gu, uint32_t S, uint32_t T, float *act, ErrorWord err, cudaStream_t stream) {
    const uint64_t n = (uint64_t)S * T;
    const uint32_t blocks = (uint32_t)std::min<uint64_t>((n + 255) / 256, 148u * 16u);
    launch_pdl(moe_swiglu_kernel, blocks, 256, 0, stream, gu, S, T, act, err);
    count_launch();
}

void launch_moe_combine(const MoeDims &d, uint32_t T, const MoeBuffers &b, float *y, ErrorWord err,
                        cudaStream_t stream) {
    const dim3 grid(T, (d.hidden + kMoeThreads - 1) / kMoeThreads);
    launch_pdl(moe_combine_kernel, grid, kMoeThreads, 0, stream, d, b.logits, d.experts + 1, b.sel_ids, b.sel_w, b.slot,
               b.eout, b.shared_out, y, b.dbg, err);
    count_launch();
}

void launch_moe(const MoeDims &d, const MoeWeightsDev &w, const float *x, uint32_t T, float *y, MoeBuffers &b,
                ErrorWord err, cudaStream_t stream) {
    const uint32_t E = d.experts, H = d.hidden, S = d.shared;
    {
        // router logits and the shared gate logit (row E), exact products
        KernelTimer timer("moe_router", stream);
        ProjSegments r{};
        r.count = 2;
        r.m[0] = w.router;
        r.out_offset[0] = 0;
        r.m[1] = w.shared_gate_weight;
        r.out_offset[1] = E;
        launch_projection_exact(r, x, H, b.logits, E + 1, T, err, stream);
    }
    launch_moe_route(d, b.logits, E + 1, T, b, err, stream);
    launch_moe_dispatch(d, T, b, err, stream);
    launch_moe_experts(d, w, x, H, T, b, err, stream);
    {
        KernelTimer timer("moe_shared", stream);
        ProjSegments s{};
        s.count = 2;
        s.m[0] = w.shared_gate;
        s.out_offset[0] = 0;
        s.m[1] = w.shared_up;
        s.out_offset[1] = S;
        launch_projection(s, x, H, b.shared_gu, 2 * S, T, err, stream, b.proj_gu, b.proj_floats_gu);
        launch_moe_swiglu(b.shared_gu, S, T, b.shared_act, err, stream);
        ProjSegments o{};
        o.count = 1;
        o.m[0] = w.shared_down;
        o.out_offset[0] = 0;
        launch_projection(o, b.shared_act, S, b.shared_out, H, T, err, stream, b.proj_down, b.proj_floats_down);
    }
    launch_moe_combine(d, T, b, y, err, stream);
}

}  // namespace kqb
