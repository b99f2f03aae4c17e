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
//   gate_up   one CTA per (active expert, 64 intermediate rows): gate and up
//             rows decoded once per group of up to 8 of the expert's tokens,
//             SwiGLU in the epilogue -> act[slot][I]
//   down      one CTA per (active expert, 64 hidden rows), four lanes per
//             row -> eout[slot][H]
//   combine   one CTA per token: the selected experts' weighted outputs
//             summed in ascending expert id (the reference's accumulation
//             order), plus the shared expert scaled by sigmoid(logit)
//
// Every pick's products are computed from its own token only, so the order
// of the picks inside an expert's group (which the atomics of the route
// kernel decide) does not change any value.
#include "kernels.hpp"
#include "quant.cuh"

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

// The reference's "worst" member of the selected set
// (src/kq_moe_qwen38.c:217-228): lowest probability, the lowest id among
// equal lowest probabilities.
__device__ __forceinline__ uint32_t worst_position(const float *p, const uint32_t *ids, uint32_t k) {
    uint32_t worst = 0;
    for (uint32_t pos = 1; pos < k; ++pos) {
        const uint32_t c = ids[pos], w = ids[worst];
        if (p[c] < p[w] || (p[c] == p[w] && c < w)) worst = pos;
    }
    return worst;
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
    if (tid == 0) {
        float s = 0.0f;
        for (uint32_t e = 0; e < E; ++e) s = __fadd_rn(s, sp[e]);
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
    if (tid == 0) {
        // top-k of src/kq_moe_qwen38.c:211-245; the worst member only
        // changes when the set does, so it is recomputed after a replacement
        for (uint32_t i = 0; i < K; ++i) ids[i] = i;
        uint32_t worst = worst_position(sp, ids, K);
        float wv = sp[ids[worst]];
        for (uint32_t i = K; i < E; ++i) {
            const float v = sp[i];
            if (v > wv) {
                ids[worst] = i;
                worst = worst_position(sp, ids, K);
                wv = sp[ids[worst]];
            }
        }
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

// ------------------------------------------------- staged (bulk-copy) paths
//
// Q4_K gate/up and planar Q8_0 down: a CTA copies its whole row block into
// shared memory with one bulk copy per row (HBM -> SMEM, mbarrier
// completion), then, per group of the expert's tokens, copies their
// activation rows into shared memory and decodes the block against them, so
// the block crosses HBM once whatever the token count.  Two (gate/up) or
// three (down) CTAs per SM keep the next blocks' copies in flight while one
// decodes.  Lane = sub * 8 + unit: the eight lanes of a shared-memory phase
// read the same activation words (a broadcast) and eight different rows,
// whose pitch is chosen so that they fall in distinct banks.  Codes become
// floats without a conversion instruction: a code byte placed in the
// mantissa of 2^23 (PRMT) minus 2^23 (one FADD) is the exact integer.

constexpr uint32_t kGuRows = 32;     // gate rows (and as many up rows) per CTA
constexpr uint32_t kGuGroup = 2;     // tokens per pass (activation rows staged)
constexpr uint32_t kDnRows = 64;     // down rows per CTA
constexpr uint32_t kDnGroup = 8;
constexpr uint32_t kMaxStageBytes = 112u * 1024u;
constexpr uint32_t kStageWaitPolls = 1u << 26;

__device__ __forceinline__ uint32_t moe_smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void moe_bulk(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(moe_smem_u32(dst)), "l"(src), "r"(bytes), "r"(moe_smem_u32(bar))
                 : "memory");
}

// Bounded wait for phase 0 of `bar`; false when it gave up.
__device__ __forceinline__ bool moe_bar_wait(uint64_t *bar) {
    const uint32_t a = moe_smem_u32(bar);
    for (uint32_t i = 0; i < kStageWaitPolls; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a)
            : "memory");
        if (done) return true;
    }
    return false;
}

// Byte k of `v` as the float value of that byte (0..255).
__device__ __forceinline__ float byte_float(uint32_t v, int k) {
    return __int_as_float(__byte_perm(v, 0x4B000000u, (uint32_t)k | 0x7540u)) - 8388608.0f;
}

// Copies `rows` rows of `row_bytes` from `src` (pitch row_bytes) to `dst`
// (pitch `dst_pitch`), and as many from `src2` to `dst2` when given, then
// waits for them; every thread returns the same verdict.
__device__ __forceinline__ bool stage_rows(uint8_t *dst, const uint8_t *src, uint32_t rows, uint32_t row_bytes,
                                           uint32_t dst_pitch, const uint8_t *src2, uint8_t *dst2, uint64_t *bar,
                                           int *ok, const ErrorWord &err) {
    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(moe_smem_u32(bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        const uint32_t total = rows * row_bytes * (src2 ? 2u : 1u);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(moe_smem_u32(bar)), "r"(total)
                     : "memory");
        for (uint32_t r = 0; r < rows; ++r) {
            moe_bulk(dst + (size_t)r * dst_pitch, src + (size_t)r * row_bytes, row_bytes, bar);
            if (src2) moe_bulk(dst2 + (size_t)r * dst_pitch, src2 + (size_t)r * row_bytes, row_bytes, bar);
        }
        *ok = 1;
        if (!moe_bar_wait(bar)) {
            moe_raise(err, kErrTimeout | (1u << 8));
            *ok = 0;
            moe_bar_wait(bar);   // let the copies in flight land before the CTA exits
        }
    }
    __syncthreads();
    return *ok != 0;
}

// `nb` activation rows (row ids rows_of(j), `cols` floats each) into
// shared memory xs[j][cols], all threads, 16-byte moves.
template <typename RowOf>
__device__ __forceinline__ void stage_acts(float *xs, const float *src, uint32_t ld, uint32_t cols, uint32_t nb,
                                           RowOf rows_of) {
    const uint32_t q = cols / 4u;
    for (uint32_t i = threadIdx.x; i < nb * q; i += blockDim.x) {
        const uint32_t j = i / q, c = i % q;
        reinterpret_cast<float4 *>(xs + (size_t)j * cols)[c] =
            reinterpret_cast<const float4 *>(src + (size_t)rows_of(j) * ld)[c];
    }
}

// 32 decoded Q4_K values of run c (multiple of 32) of a row in shared memory
// (144-byte super-blocks: fp16 d, fp16 dmin, 12 scale/min bytes, 128 code
// bytes), value = d*sc*q - dmin*m with one rounding per value.
__device__ __forceinline__ void q4k_run_smem(const uint8_t *row, uint32_t c, float (&w)[32]) {
    const uint8_t *sb = row + (c >> 8) * 144u;
    const uint32_t group = (c & 255u) >> 6, high = (c >> 5) & 1u;
    const uint4 hdr = *reinterpret_cast<const uint4 *>(sb);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(sb + 16u + group * 32u);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(sb + 32u + group * 32u);
    uint8_t h[16];
    bytes16(hdr, h);
    const float d = half_bits_to_float((uint32_t)h[0] | ((uint32_t)h[1] << 8));
    const float dmin = half_bits_to_float((uint32_t)h[2] | ((uint32_t)h[3] << 8));
    uint32_t sc, mn;
    q4k_scale_min(h + 4, (int)(2u * group + high), sc, mn);
    const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dmin, (float)mn);
    const uint32_t words[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t nib = (words[k] >> (4u * high)) & 0x0F0F0F0Fu;
#pragma unroll
        for (int b = 0; b < 4; ++b) w[4 * k + b] = fmaf(dl, byte_float(nib, b), -ml);
    }
}

// s += w . xs[0..32)
__device__ __forceinline__ float dot32_smem(const float (&w)[32], const float *xs, float s) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float4 v = reinterpret_cast<const float4 *>(xs)[i];
        s = fmaf(w[4 * i], v.x, s);
        s = fmaf(w[4 * i + 1], v.y, s);
        s = fmaf(w[4 * i + 2], v.z, s);
        s = fmaf(w[4 * i + 3], v.w, s);
    }
    return s;
}

// grid (max active experts, ceil(I / 32)), 256 threads.  Warp w owns local
// rows 4w..4w+3; lane = sub * 8 + unit with unit = row * 2 + {0 gate, 1 up}
// and the four subs splitting a row's 32-value runs.  Shared memory: gate
// rows, up rows (pitch rb + 16 keeps the eight units' rows in distinct
// banks), then kGuGroup activation rows.
__global__ void __launch_bounds__(kMoeThreads, 2)
moe_gate_up_staged_kernel(MoeDims d, QMatrix gate, QMatrix up, const float *__restrict__ x, uint32_t ldx,
                          const uint32_t *__restrict__ active, const uint32_t *__restrict__ offsets,
                          const uint32_t *__restrict__ pick_of_slot, float *__restrict__ act, float *gate_dbg,
                          float *up_dbg, ErrorWord err) {
    extern __shared__ __align__(128) uint8_t gsm[];
    __shared__ uint64_t bar;
    __shared__ int ok;
    pdl_wait();
    if (moe_err_raised(err) || blockIdx.x >= active[0]) return;
    const uint32_t e = active[1 + blockIdx.x];
    const uint32_t s0 = offsets[e], n = offsets[e + 1] - s0;
    const uint32_t I = d.routed, H = d.hidden, rb = gate.row_bytes, pitch = rb + 16u;
    const uint32_t r0 = blockIdx.y * kGuRows, rows = min(kGuRows, I - r0);
    uint8_t *gs = gsm, *us = gsm + (size_t)kGuRows * pitch;
    float *xs = reinterpret_cast<float *>(gsm + (size_t)2 * kGuRows * pitch);
    if (!stage_rows(gs, gate.data + ((size_t)e * I + r0) * rb, rows, rb, pitch, up.data + ((size_t)e * I + r0) * rb,
                    us, &bar, &ok, err))
        return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t unit = (uint32_t)lane & 7u, sub = (uint32_t)lane >> 3;
    const uint32_t lr = (uint32_t)warp * 4u + (unit >> 1);
    const bool is_up = (unit & 1u) != 0u, live = lr < rows;
    const uint8_t *row = (is_up ? us : gs) + (size_t)(live ? lr : 0u) * pitch;
    for (uint32_t g0 = 0; g0 < n; g0 += kGuGroup) {
        const uint32_t nb = min(kGuGroup, n - g0);
        __syncthreads();   // the previous group's activation rows are no longer read
        stage_acts(xs, x, ldx, H, nb, [&](uint32_t j) { return pick_of_slot[s0 + g0 + j] / d.top_k; });
        __syncthreads();
        float a0 = 0.0f, a1 = 0.0f;
        if (live) {
            for (uint32_t c = sub * 32u; c < H; c += 128u) {
                float w[32];
                q4k_run_smem(row, c, w);
                a0 = dot32_smem(w, xs + c, a0);
                if (nb > 1) a1 = dot32_smem(w, xs + H + c, a1);
            }
        }
        a0 += __shfl_xor_sync(0xffffffffu, a0, 8);
        a0 += __shfl_xor_sync(0xffffffffu, a0, 16);
        a1 += __shfl_xor_sync(0xffffffffu, a1, 8);
        a1 += __shfl_xor_sync(0xffffffffu, a1, 16);
        const float u0 = __shfl_down_sync(0xffffffffu, a0, 1), u1 = __shfl_down_sync(0xffffffffu, a1, 1);
        if (sub == 0 && !is_up && live) {
            const size_t o = (size_t)(s0 + g0) * I + r0 + lr;
            act[o] = moe_swiglu(a0, u0);
            if (gate_dbg) {
                gate_dbg[o] = a0;
                up_dbg[o] = u0;
            }
            if (nb > 1) {
                act[o + I] = moe_swiglu(a1, u1);
                if (gate_dbg) {
                    gate_dbg[o + I] = a1;
                    up_dbg[o + I] = u1;
                }
            }
        }
    }
}

// grid (max active experts, ceil(H / 64)), 256 threads.  Warp w owns local
// rows 8w..8w+7; lane = sub * 8 + row.  Planar Q8_0 rows: I code bytes,
// then the I/32 fp16 scales; shared memory: the rows (pitch rb), then
// kDnGroup activation rows.
__global__ void __launch_bounds__(kMoeThreads, 3)
moe_down_staged_kernel(MoeDims d, QMatrix down, const float *__restrict__ act, const uint32_t *__restrict__ active,
                       const uint32_t *__restrict__ offsets, float *__restrict__ eout, ErrorWord err) {
    extern __shared__ __align__(128) uint8_t dsm[];
    __shared__ uint64_t bar;
    __shared__ int ok;
    pdl_wait();
    if (moe_err_raised(err) || blockIdx.x >= active[0]) return;
    const uint32_t e = active[1 + blockIdx.x];
    const uint32_t s0 = offsets[e], n = offsets[e + 1] - s0;
    const uint32_t H = d.hidden, I = d.routed, rb = down.row_bytes;
    const uint32_t r0 = blockIdx.y * kDnRows, rows = min(kDnRows, H - r0);
    float *as = reinterpret_cast<float *>(dsm + (size_t)kDnRows * rb);
    if (!stage_rows(dsm, down.data + ((size_t)e * H + r0) * rb, rows, rb, rb, nullptr, nullptr, &bar, &ok, err))
        return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t lr = (uint32_t)warp * 8u + ((uint32_t)lane & 7u), sub = (uint32_t)lane >> 3;
    const bool live = lr < rows;
    const uint8_t *row = dsm + (size_t)(live ? lr : 0u) * rb;
    const uint16_t *scales = reinterpret_cast<const uint16_t *>(row + I);
    for (uint32_t g0 = 0; g0 < n; g0 += kDnGroup) {
        const uint32_t nb = min(kDnGroup, n - g0);
        __syncthreads();
        stage_acts(as, act + (size_t)(s0 + g0) * I, I, I, nb, [](uint32_t j) { return j; });
        __syncthreads();
        float acc[kDnGroup];
#pragma unroll
        for (int j = 0; j < (int)kDnGroup; ++j) acc[j] = 0.0f;
        if (live) {
            for (uint32_t c = sub * 32u; c < I; c += 128u) {
                const uint4 q0 = *reinterpret_cast<const uint4 *>(row + c);
                const uint4 q1 = *reinterpret_cast<const uint4 *>(row + c + 16u);
                const float dsc = half_bits_to_float(scales[c >> 5]);
                const uint32_t words[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u,
                                           q0.w ^ 0x80808080u, q1.x ^ 0x80808080u, q1.y ^ 0x80808080u,
                                           q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
                float w[32];
#pragma unroll
                for (int k = 0; k < 8; ++k)
#pragma unroll
                    for (int b = 0; b < 4; ++b) w[4 * k + b] = byte_float(words[k], b) - 128.0f;   // the int8 code
#pragma unroll
                for (int j = 0; j < (int)kDnGroup; ++j) {
                    if ((uint32_t)j >= nb) break;
                    acc[j] = fmaf(dsc, dot32_smem(w, as + (size_t)j * I + c, 0.0f), acc[j]);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < (int)kDnGroup; ++j) {
            if ((uint32_t)j >= nb) break;
            float v = acc[j];
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            if (sub == 0 && live) eout[(size_t)(s0 + g0 + j) * H + r0 + lr] = v;
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

// One CTA per token: y = sum over the selected experts in ascending id of
// eout * weight (each product and sum rounded, src/kq_moe_qwen38.c:745-759),
// plus shared_out * sigmoid(shared gate logit) (:820-836).
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
        if (dbg.scale) {
            dbg.scale[2 * t] = logit;
            dbg.scale[2 * t + 1] = sc;
        }
    }
    __syncthreads();
    const float sc = scale_s;
    bool ok = bad == 0;
    for (uint32_t f = tid; f < H; f += kMoeThreads) {
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

// The staged kernels' conditions: the types they decode, 16-byte aligned
// rows and float4-aligned activations, a row block within kMaxStageBytes.
static size_t gate_up_stage_bytes(const MoeDims &d, const QMatrix &g) {
    return (size_t)2 * kGuRows * (g.row_bytes + 16u) + (size_t)kGuGroup * d.hidden * 4u;
}

static size_t down_stage_bytes(const MoeDims &d, const QMatrix &m) {
    return (size_t)kDnRows * m.row_bytes + (size_t)kDnGroup * d.routed * 4u;
}

static bool gate_up_staged_ok(const MoeDims &d, const QMatrix &g, const QMatrix &u, const float *x, uint32_t ldx) {
    return g.type == kTypeQ4_K && u.type == kTypeQ4_K && g.row_bytes == u.row_bytes && g.row_bytes % 16u == 0u &&
           aligned16(g.data) && aligned16(u.data) && d.hidden % 256u == 0u && aligned16(x) && ldx % 4u == 0u &&
           gate_up_stage_bytes(d, g) <= kMaxStageBytes;
}

static bool down_staged_ok(const MoeDims &d, const QMatrix &m, const float *act) {
    return m.type == kTypeQ8_0 && m.layout == 1 && m.row_bytes % 16u == 0u && aligned16(m.data) &&
           d.routed % 32u == 0u && aligned16(act) && down_stage_bytes(d, m) <= kMaxStageBytes;
}

void launch_moe_experts(const MoeDims &d, const MoeWeightsDev &w, const float *x, uint32_t ldx, uint32_t T,
                        MoeBuffers &b, ErrorWord err, cudaStream_t stream) {
    const uint32_t max_active = (uint32_t)std::min<uint64_t>(d.experts, (uint64_t)T * d.top_k);
    static DeviceOnce attr;
    attr.run([] {
        cudaFuncSetAttribute(moe_gate_up_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kMaxStageBytes);
        cudaFuncSetAttribute(moe_down_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kMaxStageBytes);
    });
    {
        KernelTimer timer("moe_gate_up", stream);
        if (gate_up_staged_ok(d, w.gate, w.up, x, ldx)) {
            dim3 grid(max_active, (d.routed + kGuRows - 1) / kGuRows);
            launch_pdl(moe_gate_up_staged_kernel, grid, kMoeThreads, gate_up_stage_bytes(d, w.gate), stream,
                       d, w.gate, w.up, x, ldx, b.active, b.offsets, b.pick_of_slot, b.act, b.dbg.gate, b.dbg.up,
                       err);
        } else {
            dim3 grid(max_active, (d.routed + kMoeRowsPerCta - 1) / kMoeRowsPerCta);
            launch_pdl(moe_gate_up_kernel, grid, kMoeThreads, 0, stream, d, w.gate, w.up, x, ldx, b.active,
                       b.offsets, b.pick_of_slot, b.act, b.dbg.gate, b.dbg.up, err);
        }
        count_launch();
    }
    {
        KernelTimer timer("moe_down", stream);
        if (down_staged_ok(d, w.down, b.act)) {
            dim3 grid(max_active, (d.hidden + kDnRows - 1) / kDnRows);
            launch_pdl(moe_down_staged_kernel, grid, kMoeThreads, down_stage_bytes(d, w.down), stream, d,
                       w.down, b.act, b.active, b.offsets, b.eout, err);
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
    launch_pdl(moe_combine_kernel, T, kMoeThreads, 0, stream, d, b.logits, d.experts + 1, b.sel_ids, b.sel_w, b.slot,
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
