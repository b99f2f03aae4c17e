// Gated delta-net (GDN) kernels.
//
// Math follows the per-token loop of kq_gdn_execute_common
// (src/kq_gdn_qwen38.c:545-842 of Kestrel-Q):
//   conv + SiLU (:602-621), head split with consecutive key-head repeat
//   (:631-648), beta = sigmoid(b) and g = -exp(A_log) * softplus(a + dt_bias)
//   (:662-678), L2 norms with q scaled by 1/sqrt(dk) (:679-686), delta-rule
//   recurrence (:705-761) and gated RMSNorm with the norm weight applied
//   directly (:787-815).
//
// Work layout: items are (sequence b, token t) pairs, B sequences x T tokens
// per launch (decode: T = 1; prefill: B = 1).  The projections of all items
// are produced beforehand by the projection GEMM into `proj`
// ([B*T][ldp]: qkv | gate | beta | alpha).
#include "kernels.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>

namespace kqb {

__device__ __forceinline__ bool gdn_error_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}
__device__ __forceinline__ void gdn_raise(const ErrorWord &e, uint32_t code) {
    atomicCAS(e.word, 0ull, ((unsigned long long)code << 32) | e.call_id);
}

// Branch-stable sigmoid of kq_sigmoid_scalar (src/kq_numeric.c:628-638).
__device__ __forceinline__ float stable_sigmoid(float x) {
    if (x >= 0.0f) {
        float e = expf(-x);
        return 1.0f / (1.0f + e);
    }
    float e = expf(x);
    return e / (1.0f + e);
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) s += red[w];
    return s;
}

// ------------------------------------------------------------ conv + gates
//
// grid (Hk, B*T); 128 threads.  For key head kh it handles the q and k
// channels of kh and the v channels / gates of value heads
// kh*repeat .. kh*repeat+repeat-1.  Writes:
//   qk    [item][2][Hk][dk]  normalised (q additionally * 1/sqrt(dk))
//   v     [item][Vd]         SiLU(conv)
//   beta  [item][Hv]
//   decay [item][Hv]         exp(g)
// and, for the last token of each sequence, the new conv state.

constexpr int kConvThreads = 128;

__device__ __forceinline__ float conv_history(const GdnDims &d, const float *conv_in,
                                              const float *proj, uint32_t ldp,
                                              uint32_t seq_item0, int t, int j,
                                              uint32_t c) {
    // history slot j (0..K-1) after the shift for token t: x_{t-K+1+j}
    int src = t - (int)d.kernel + 1 + j;
    if (src >= 0) return proj[(size_t)(seq_item0 + src) * ldp + c];
    return conv_in[(size_t)c * d.kernel + (uint32_t)(t + 1 + j)];
}

// conv + SiLU of channel c for token t: taps in the reference's order
// (sum = sum + w_j * h_j, j = 0..K-1).  KT > 0 fixes the kernel size so that
// the K history loads and weight loads are all issued before the sum.
template <int KT>
__device__ __forceinline__ float conv_channel(const GdnDims &d, const GdnWeightsDev &w, const float *conv_in,
                                             float *conv_out, bool last, const float *proj, uint32_t ldp,
                                             uint32_t item0, int t, uint32_t c) {
    float s = 0.0f;
    if constexpr (KT > 0) {
        float hv[KT], wv[KT];
#pragma unroll
        for (int j = 0; j < KT; ++j) {
            hv[j] = conv_history(d, conv_in, proj, ldp, item0, t, j, c);
            wv[j] = w.conv[(size_t)c * KT + j];
        }
#pragma unroll
        for (int j = 0; j < KT; ++j) {
            s = __fadd_rn(s, __fmul_rn(wv[j], hv[j]));
            if (last) conv_out[(size_t)c * KT + j] = hv[j];
        }
    } else {
        for (uint32_t j = 0; j < d.kernel; ++j) {
            const float h = conv_history(d, conv_in, proj, ldp, item0, t, (int)j, c);
            s = __fadd_rn(s, __fmul_rn(w.conv[(size_t)c * d.kernel + j], h));
            if (last) conv_out[(size_t)c * d.kernel + j] = h;
        }
    }
    return s;
}

template <int KT>
__global__ void __launch_bounds__(kConvThreads)
gdn_conv_gates_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, uint32_t tokens,
                      const float *__restrict__ proj, uint32_t ldp,
                      float *__restrict__ qk, float *__restrict__ vout,
                      float *__restrict__ beta, float *__restrict__ decay,
                      float *__restrict__ logdecay, ErrorWord err) {
    pdl_wait();
    __shared__ float red[kConvThreads / 32];
    if (gdn_error_raised(err)) return;
    const uint32_t kh = blockIdx.x;
    const uint32_t item = blockIdx.y;
    const uint32_t b = item / tokens;
    const int t = (int)(item % tokens);
    const uint32_t item0 = b * tokens;
    const float *conv_in = p.conv_in[b];
    float *conv_out = p.conv_out[b];
    const bool last = (uint32_t)t == tokens - 1;
    const float *prow = proj + (size_t)item * ldp;
    bool bad = false;

    // q and k channels of key head kh: conv + SiLU, then L2 norm
    for (int which = 0; which < 2; ++which) {
        float val = 0.0f;
        const uint32_t i = threadIdx.x;
        if (i < d.key_dim) {
            uint32_t c = which * d.key_width + kh * d.key_dim + i;
            const float s = conv_channel<KT>(d, w, conv_in, conv_out, last, proj, ldp, item0, t, c);
            val = s * stable_sigmoid(s);
            bad |= !isfinite(val);
        }
        float sumsq = block_sum<kConvThreads>(i < d.key_dim ? val * val : 0.0f, red);
        float inv = 1.0f / sqrtf(sumsq + 1.0e-6f);
        if (i < d.key_dim) {
            float out = val * inv;
            if (which == 0) out = out * (1.0f / sqrtf((float)d.key_dim));
            qk[((size_t)item * 2 + which) * d.key_width + kh * d.key_dim + i] = out;
        }
    }
    // v channels of the value heads that share key head kh
    for (uint32_t r = 0; r < d.repeat; ++r) {
        uint32_t h = kh * d.repeat + r;
        for (uint32_t i = threadIdx.x; i < d.value_dim; i += blockDim.x) {
            uint32_t c = 2 * d.key_width + h * d.value_dim + i;
            const float s = conv_channel<KT>(d, w, conv_in, conv_out, last, proj, ldp, item0, t, c);
            float val = s * stable_sigmoid(s);
            bad |= !isfinite(val);
            vout[(size_t)item * d.value_width + h * d.value_dim + i] = val;
        }
        if (threadIdx.x == 0) {
            const float pb = prow[d.conv_channels + d.value_width + h];
            const float pa = prow[d.conv_channels + d.value_width + d.value_heads + h];
            float bt = stable_sigmoid(pb);
            float a = pa + w.dt_bias[h];
            float sp = a > 20.0f ? a : log1pf(expf(a));
            float g = -expf(w.a_log[h]) * sp;
            if (!isfinite(g) || g > 0.0f || !isfinite(bt)) {
                gdn_raise(err, kErrDecay);
            }
            beta[(size_t)item * d.value_heads + h] = bt;
            decay[(size_t)item * d.value_heads + h] = expf(g);
            if (logdecay) logdecay[(size_t)item * d.value_heads + h] = g;
        }
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

// Prefill with dk = dv = 128 and a 4-tap conv: one warp per (token, key
// head), 8 per CTA, REP value heads per key head.  Lane l owns channels
// 4l .. 4l+3 of the head's q, k and v blocks (16-byte loads and stores; the
// four history rows of a channel are re-read, mostly from L1/L2), and the
// L2 norms are warp reductions, so nothing waits at a CTA barrier.  Same
// arithmetic per value as gdn_conv_gates_kernel (taps in the reference's
// order).
template <int REP>
__global__ void __launch_bounds__(256)
gdn_conv_gates_warp_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, uint32_t tokens,
                           const float *__restrict__ proj, uint32_t ldp,
                           float *__restrict__ qk, float *__restrict__ vout,
                           float *__restrict__ beta, float *__restrict__ decay,
                           float *__restrict__ logdecay, ErrorWord err) {
    constexpr int K = 4, D = 128, NCH = 2 + REP;
    pdl_wait();
    if (gdn_error_raised(err)) return;
    const uint32_t pair = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (pair >= tokens * d.key_heads) return;
    const uint32_t t = pair / d.key_heads, kh = pair % d.key_heads;
    const int lane = threadIdx.x & 31;
    const float *conv_in = p.conv_in[0];
    float *conv_out = p.conv_out[0];
    const bool last = t == tokens - 1;
    float val[NCH][4];
    bool bad = false;
#pragma unroll
    for (int cc = 0; cc < NCH; ++cc) {
        const uint32_t c0 = (cc == 0 ? kh * D : cc == 1 ? d.key_width + kh * D
                                                      : 2 * d.key_width + (kh * REP + (cc - 2)) * D) + 4 * lane;
        float h[K][4];
#pragma unroll
        for (int j = 0; j < K; ++j) {
            const int src = (int)t - (K - 1) + j;
            if (src >= 0) {
                const float4 x = *reinterpret_cast<const float4 *>(proj + (size_t)src * ldp + c0);
                h[j][0] = x.x; h[j][1] = x.y; h[j][2] = x.z; h[j][3] = x.w;
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) h[j][e] = conv_in[(size_t)(c0 + e) * K + (t + 1 + j)];
            }
        }
        float wt[4][K];   // the four channels' taps: 16 consecutive weights
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float4 wq = *reinterpret_cast<const float4 *>(w.conv + (size_t)(c0 + e) * K);
            wt[e][0] = wq.x; wt[e][1] = wq.y; wt[e][2] = wq.z; wt[e][3] = wq.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            float sacc = 0.0f;
#pragma unroll
            for (int j = 0; j < K; ++j) sacc = __fadd_rn(sacc, __fmul_rn(wt[e][j], h[j][e]));
            val[cc][e] = sacc * stable_sigmoid(sacc);
            bad |= !isfinite(val[cc][e]);
        }
        if (last) {
#pragma unroll
            for (int e = 0; e < 4; ++e)
                *reinterpret_cast<float4 *>(conv_out + (size_t)(c0 + e) * K) = make_float4(h[0][e], h[1][e], h[2][e],
                                                                                           h[3][e]);
        }
    }
    float sq = 0.0f, sk = 0.0f;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        sq += val[0][e] * val[0][e];
        sk += val[1][e] * val[1][e];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        sq += __shfl_xor_sync(0xffffffffu, sq, o);
        sk += __shfl_xor_sync(0xffffffffu, sk, o);
    }
    const float iq = 1.0f / sqrtf(sq + 1.0e-6f), ik = 1.0f / sqrtf(sk + 1.0e-6f);
    const float qscale = 1.0f / sqrtf((float)d.key_dim);
    *reinterpret_cast<float4 *>(qk + ((size_t)t * 2 + 0) * d.key_width + kh * D + 4 * lane) =
        make_float4(val[0][0] * iq * qscale, val[0][1] * iq * qscale, val[0][2] * iq * qscale, val[0][3] * iq * qscale);
    *reinterpret_cast<float4 *>(qk + ((size_t)t * 2 + 1) * d.key_width + kh * D + 4 * lane) =
        make_float4(val[1][0] * ik, val[1][1] * ik, val[1][2] * ik, val[1][3] * ik);
#pragma unroll
    for (int r = 0; r < REP; ++r)
        *reinterpret_cast<float4 *>(vout + (size_t)t * d.value_width + (kh * REP + r) * D + 4 * lane) =
            make_float4(val[2 + r][0], val[2 + r][1], val[2 + r][2], val[2 + r][3]);
    if (lane < REP) {
        const float *prow = proj + (size_t)t * ldp;
        const uint32_t h = kh * REP + lane;
        const float pb = prow[d.conv_channels + d.value_width + h];
        const float pa = prow[d.conv_channels + d.value_width + d.value_heads + h];
        const float bt = stable_sigmoid(pb);
        const float a = pa + w.dt_bias[h];
        const float sp = a > 20.0f ? a : log1pf(expf(a));
        const float g = -expf(w.a_log[h]) * sp;
        if (!isfinite(g) || g > 0.0f || !isfinite(bt)) gdn_raise(err, kErrDecay);
        beta[(size_t)t * d.value_heads + h] = bt;
        decay[(size_t)t * d.value_heads + h] = expf(g);
        if (logdecay) logdecay[(size_t)t * d.value_heads + h] = g;
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) gdn_raise(err, kErrNonFinite);
}

// ------------------------------------------------------------ recurrence
//
// Fast path for dk = dv = 128: grid (Hv, B), 256 threads.  The head's
// 128 x 128 state (64 KB) is held in registers for all tokens of the launch:
// thread (warp w, lane l) owns columns 4l..4l+3 of rows w, w+8, ..., w+120.
// Per token: decay, read = S^T k, delta = (v - read) * beta, S += k delta^T,
// o = S^T q, then the gated RMSNorm of o.  The state is read from HBM once
// and written once per launch with 128-bit coalesced accesses.

constexpr int kRecThreads = 256;
constexpr int kDim = 128;
constexpr int kRows = kDim / (kRecThreads / 32);   // 16 rows per thread

__global__ void __launch_bounds__(kRecThreads, 2)
gdn_recurrence128_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, uint32_t tokens,
                         const float *__restrict__ qk, const float *__restrict__ vin,
                         const float *__restrict__ beta, const float *__restrict__ decay,
                         const float *__restrict__ proj, uint32_t ldp,
                         float *__restrict__ gated, ErrorWord err) {
    pdl_wait();
    __shared__ __align__(16) float ks[kDim];
    __shared__ __align__(16) float qs[kDim];
    __shared__ __align__(16) float part[kRecThreads / 32][kDim];
    __shared__ __align__(16) float delta[kDim];
    __shared__ float red[kRecThreads / 32];
    if (gdn_error_raised(err)) return;

    const uint32_t h = blockIdx.x;
    const uint32_t b = blockIdx.y;
    const uint32_t kh = h / d.repeat;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *sin_ = p.rec_in[b] + (size_t)h * kDim * kDim;
    float *sout = p.rec_out[b] + (size_t)h * kDim * kDim;

    float4 s[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j)
        s[j] = *reinterpret_cast<const float4 *>(sin_ + (size_t)(warp + 8 * j) * kDim + 4 * lane);

    bool bad = false;
    for (uint32_t t = 0; t < tokens; ++t) {
        const size_t item = (size_t)b * tokens + t;
        if (threadIdx.x < kDim) {
            qs[threadIdx.x] = qk[(item * 2 + 0) * d.key_width + kh * kDim + threadIdx.x];
            ks[threadIdx.x] = qk[(item * 2 + 1) * d.key_width + kh * kDim + threadIdx.x];
        }
        const float dec = decay[item * d.value_heads + h];
        const float bt = beta[item * d.value_heads + h];
        __syncthreads();
        // decay and read partials
        float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            s[j].x *= dec; s[j].y *= dec; s[j].z *= dec; s[j].w *= dec;
            float kv = ks[warp + 8 * j];
            r0 = fmaf(s[j].x, kv, r0);
            r1 = fmaf(s[j].y, kv, r1);
            r2 = fmaf(s[j].z, kv, r2);
            r3 = fmaf(s[j].w, kv, r3);
        }
        *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(r0, r1, r2, r3);
        __syncthreads();
        if (threadIdx.x < kDim) {
            float rd = 0.f;
#pragma unroll
            for (int wv = 0; wv < kRecThreads / 32; ++wv) rd += part[wv][threadIdx.x];
            float vv = vin[item * d.value_width + h * kDim + threadIdx.x];
            delta[threadIdx.x] = (vv - rd) * bt;
        }
        __syncthreads();
        // rank-1 update and output partials
        const float4 dl = *reinterpret_cast<const float4 *>(&delta[4 * lane]);
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            float kv = ks[warp + 8 * j];
            float qv = qs[warp + 8 * j];
            s[j].x = fmaf(kv, dl.x, s[j].x);
            s[j].y = fmaf(kv, dl.y, s[j].y);
            s[j].z = fmaf(kv, dl.z, s[j].z);
            s[j].w = fmaf(kv, dl.w, s[j].w);
            o0 = fmaf(s[j].x, qv, o0);
            o1 = fmaf(s[j].y, qv, o1);
            o2 = fmaf(s[j].z, qv, o2);
            o3 = fmaf(s[j].w, qv, o3);
        }
        *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(o0, o1, o2, o3);
        __syncthreads();
        // gated RMSNorm of o (threads 0..127 own one feature each)
        float o = 0.f;
        if (threadIdx.x < kDim) {
#pragma unroll
            for (int wv = 0; wv < kRecThreads / 32; ++wv) o += part[wv][threadIdx.x];
            bad |= !isfinite(o);
        }
        float sumsq = block_sum<kRecThreads>(threadIdx.x < kDim ? o * o : 0.f, red);
        if (threadIdx.x < kDim) {
            float mean = sumsq / (float)kDim;
            float inv = 1.0f / sqrtf(mean + d.eps);
            float z = proj[item * ldp + d.conv_channels + h * kDim + threadIdx.x];
            float g = (w.norm[threadIdx.x] * (o * inv)) * stable_sigmoid(z);
            bad |= !isfinite(g);
            gated[item * d.value_width + gated_head_pos(w, h) * kDim + threadIdx.x] = g;
        }
        // part/ks/qs are rewritten next token only after the barrier inside
        // block_sum's successor __syncthreads at the loop head
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        bad |= !isfinite(s[j].x) || !isfinite(s[j].y) || !isfinite(s[j].z) || !isfinite(s[j].w);
        *reinterpret_cast<float4 *>(sout + (size_t)(warp + 8 * j) * kDim + 4 * lane) = s[j];
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

// Decode (one token per sequence), dk = dv = 128, conv kernel 4: the conv /
// gate stage of gdn_conv_gates_kernel fused into the recurrence.  The CTA of
// (value head h, sequence b) computes q and k of key head h / repeat (both
// value heads of a key head compute them; the first writes their conv
// state), v of head h, beta and the decay, then runs the recurrence as
// gdn_recurrence128_kernel does.  Same arithmetic as the two kernels.
__global__ void __launch_bounds__(kRecThreads, 2)
gdn_decode_fused_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, const float *__restrict__ proj,
                        uint32_t ldp, float *__restrict__ gated, ErrorWord err) {
    pdl_wait();
    __shared__ __align__(16) float ks[kDim];
    __shared__ __align__(16) float qs[kDim];
    __shared__ __align__(16) float vs[kDim];
    __shared__ __align__(16) float part[kRecThreads / 32][kDim];
    __shared__ __align__(16) float delta[kDim];
    __shared__ float red[kRecThreads / 32];
    __shared__ float gates[2];   // beta, decay
    if (gdn_error_raised(err)) return;
    const uint32_t h = blockIdx.x;
    const uint32_t b = blockIdx.y;
    const uint32_t kh = h / d.repeat;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *sin_ = p.rec_in[b] + (size_t)h * kDim * kDim;
    float *sout = p.rec_out[b] + (size_t)h * kDim * kDim;
    const float *prow = proj + (size_t)b * ldp;
    const float *conv_in = p.conv_in[b];
    float *conv_out = p.conv_out[b];
    bool bad = false;

    // state loads first: they are independent of the prologue
    float4 s[kRows];
#pragma unroll
    for (int j = 0; j < kRows; ++j)
        s[j] = *reinterpret_cast<const float4 *>(sin_ + (size_t)(warp + 8 * j) * kDim + 4 * lane);

    // ---- prologue: threads 0..127 q (which 0) / 128..255 k (which 1)
    {
        const uint32_t which = threadIdx.x >> 7, i = threadIdx.x & (kDim - 1);
        const uint32_t c = which * d.key_width + kh * kDim + i;
        const bool writer = (h % d.repeat) == 0;
        const float sconv = conv_channel<4>(d, w, conv_in, conv_out, writer, prow, ldp, 0, 0, c);
        const float val = sconv * stable_sigmoid(sconv);
        bad |= !isfinite(val);
        // L2 norm of q and of k: two 128-thread halves
        float v2 = val * val;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v2 += __shfl_xor_sync(0xffffffffu, v2, o);
        if (lane == 0) red[warp] = v2;
        __syncthreads();
        const float sumsq = red[4 * which] + red[4 * which + 1] + red[4 * which + 2] + red[4 * which + 3];
        const float inv = 1.0f / sqrtf(sumsq + 1.0e-6f);
        float out = val * inv;
        if (which == 0) out = out * (1.0f / sqrtf((float)d.key_dim));
        (which == 0 ? qs : ks)[i] = out;
        // v of head h and the gates
        if (threadIdx.x < kDim) {
            const uint32_t cv = 2 * d.key_width + h * kDim + threadIdx.x;
            const float sv = conv_channel<4>(d, w, conv_in, conv_out, true, prow, ldp, 0, 0, cv);
            const float vv = sv * stable_sigmoid(sv);
            bad |= !isfinite(vv);
            vs[threadIdx.x] = vv;
        }
        if (threadIdx.x == 0) {
            const float pb = prow[d.conv_channels + d.value_width + h];
            const float pa = prow[d.conv_channels + d.value_width + d.value_heads + h];
            const float bt = stable_sigmoid(pb);
            const float a = pa + w.dt_bias[h];
            const float sp = a > 20.0f ? a : log1pf(expf(a));
            const float g = -expf(w.a_log[h]) * sp;
            if (!isfinite(g) || g > 0.0f || !isfinite(bt)) gdn_raise(err, kErrDecay);
            gates[0] = bt;
            gates[1] = expf(g);
        }
        __syncthreads();
    }
    // ---- recurrence (one token)
    {
        const float dec = gates[1];
        const float bt = gates[0];
        float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            s[j].x *= dec; s[j].y *= dec; s[j].z *= dec; s[j].w *= dec;
            float kv = ks[warp + 8 * j];
            r0 = fmaf(s[j].x, kv, r0);
            r1 = fmaf(s[j].y, kv, r1);
            r2 = fmaf(s[j].z, kv, r2);
            r3 = fmaf(s[j].w, kv, r3);
        }
        *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(r0, r1, r2, r3);
        __syncthreads();
        if (threadIdx.x < kDim) {
            float rd = 0.f;
#pragma unroll
            for (int wv = 0; wv < kRecThreads / 32; ++wv) rd += part[wv][threadIdx.x];
            delta[threadIdx.x] = (vs[threadIdx.x] - rd) * bt;
        }
        __syncthreads();
        const float4 dl = *reinterpret_cast<const float4 *>(&delta[4 * lane]);
        float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            float kv = ks[warp + 8 * j];
            float qv = qs[warp + 8 * j];
            s[j].x = fmaf(kv, dl.x, s[j].x);
            s[j].y = fmaf(kv, dl.y, s[j].y);
            s[j].z = fmaf(kv, dl.z, s[j].z);
            s[j].w = fmaf(kv, dl.w, s[j].w);
            o0 = fmaf(s[j].x, qv, o0);
            o1 = fmaf(s[j].y, qv, o1);
            o2 = fmaf(s[j].z, qv, o2);
            o3 = fmaf(s[j].w, qv, o3);
        }
        *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(o0, o1, o2, o3);
        __syncthreads();
        float o = 0.f;
        if (threadIdx.x < kDim) {
#pragma unroll
            for (int wv = 0; wv < kRecThreads / 32; ++wv) o += part[wv][threadIdx.x];
            bad |= !isfinite(o);
        }
        float sumsq = block_sum<kRecThreads>(threadIdx.x < kDim ? o * o : 0.f, red);
        if (threadIdx.x < kDim) {
            float mean = sumsq / (float)kDim;
            float inv = 1.0f / sqrtf(mean + d.eps);
            float z = prow[d.conv_channels + h * kDim + threadIdx.x];
            float g = (w.norm[threadIdx.x] * (o * inv)) * stable_sigmoid(z);
            bad |= !isfinite(g);
            gated[(size_t)b * d.value_width + gated_head_pos(w, h) * kDim + threadIdx.x] = g;
        }
    }
#pragma unroll
    for (int j = 0; j < kRows; ++j) {
        bad |= !isfinite(s[j].x) || !isfinite(s[j].y) || !isfinite(s[j].z) || !isfinite(s[j].w);
        *reinterpret_cast<float4 *>(sout + (size_t)(warp + 8 * j) * kDim + 4 * lane) = s[j];
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

// ------------------------------------------------------------ persistent decode
//
// The fused decode kernel above as a persistent loop: each CTA (two per SM)
// walks items (sequence b, value head h), item = n * gridDim.x + blockIdx.x,
// and while it computes item n the bulk-copy engine fetches item n+1's
// 64 KiB state and its conv / projection runs into shared memory, so the
// state stream never stops between items (the one-shot kernel leaves HBM
// idle while a CTA runs its prologue, recurrence and epilogue).  The state
// of item n goes back to HBM from registers.  Arithmetic identical to
// gdn_decode_fused_kernel.
//
// Shared memory: S (next state, 64 KiB) | IN[2] (per item: conv history of
// the q, k and v channels, 3 x 2 KiB, their conv taps, 3 x 2 KiB, and the
// projected q, k, v and gate rows, 4 x 512 B).  The norm weights stay in
// registers for the CTA's life.  Requires 16-byte aligned state, conv,
// conv-tap and projection rows (checked by the launcher).
constexpr uint32_t kPStateBytes = kDim * kDim * 4;
constexpr uint32_t kPConvRun = kDim * 4 * 4;           // 128 channels x 4 slots
constexpr uint32_t kPProjRun = kDim * 4;
constexpr uint32_t kPInBytes = 6 * kPConvRun + 4 * kPProjRun;
constexpr uint32_t kPSmem = kPStateBytes + 2 * kPInBytes + 128;
constexpr uint32_t kPWaitPolls = 1u << 26;

__device__ __forceinline__ uint32_t gdn_smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void gdn_bulk(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(gdn_smem_u32(dst)), "l"(src), "r"(bytes), "r"(gdn_smem_u32(bar))
                 : "memory");
}

// Bounded wait for phase `parity` of `bar` (one thread).
__device__ __forceinline__ bool gdn_bar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = gdn_smem_u32(bar);
    for (uint32_t i = 0; i < kPWaitPolls; ++i) {
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

__global__ void __launch_bounds__(kRecThreads, 2)
gdn_decode_persist_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, uint32_t batch, const float *__restrict__ proj,
                          uint32_t ldp, float *__restrict__ gated, ErrorWord err) {
    pdl_wait();
    extern __shared__ __align__(128) uint8_t psm[];
    __shared__ __align__(16) float ks[kDim];
    __shared__ __align__(16) float qs[kDim];
    __shared__ __align__(16) float vs[kDim];
    __shared__ __align__(16) float part[kRecThreads / 32][kDim];
    __shared__ __align__(16) float delta[kDim];
    __shared__ float red[kRecThreads / 32];
    __shared__ float gates[2];   // beta, decay
    __shared__ uint64_t bar;
    __shared__ uint32_t stop;
    if (gdn_error_raised(err)) return;
    float *S = reinterpret_cast<float *>((reinterpret_cast<uintptr_t>(psm) + 127) & ~uintptr_t(127));
    uint8_t *inbuf = reinterpret_cast<uint8_t *>(S) + kPStateBytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t items = batch * d.value_heads;
    bool bad = false;

    // item it: state, conv history and projected rows into IN[slot]
    auto fetch = [&](uint32_t it, uint32_t slot) {
        const uint32_t b = it / d.value_heads, h = it % d.value_heads, kh = h / d.repeat;
        uint8_t *in = inbuf + slot * kPInBytes;
        const float *prow = proj + (size_t)b * ldp;
        const float *conv_in = p.conv_in[b];
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                     ::"r"(gdn_smem_u32(&bar)), "r"(kPStateBytes + kPInBytes) : "memory");
        gdn_bulk(S, p.rec_in[b] + (size_t)h * kDim * kDim, kPStateBytes, &bar);
        gdn_bulk(in, conv_in + (size_t)(kh * kDim) * 4, kPConvRun, &bar);
        gdn_bulk(in + kPConvRun, conv_in + (size_t)(d.key_width + kh * kDim) * 4, kPConvRun, &bar);
        gdn_bulk(in + 2 * kPConvRun, conv_in + (size_t)(2 * d.key_width + h * kDim) * 4, kPConvRun, &bar);
        gdn_bulk(in + 3 * kPConvRun, w.conv + (size_t)(kh * kDim) * 4, kPConvRun, &bar);
        gdn_bulk(in + 4 * kPConvRun, w.conv + (size_t)(d.key_width + kh * kDim) * 4, kPConvRun, &bar);
        gdn_bulk(in + 5 * kPConvRun, w.conv + (size_t)(2 * d.key_width + h * kDim) * 4, kPConvRun, &bar);
        uint8_t *pr = in + 6 * kPConvRun;
        gdn_bulk(pr, prow + kh * kDim, kPProjRun, &bar);
        gdn_bulk(pr + kPProjRun, prow + d.key_width + kh * kDim, kPProjRun, &bar);
        gdn_bulk(pr + 2 * kPProjRun, prow + 2 * d.key_width + h * kDim, kPProjRun, &bar);
        gdn_bulk(pr + 3 * kPProjRun, prow + d.conv_channels + h * kDim, kPProjRun, &bar);
    };

    if (threadIdx.x == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(gdn_smem_u32(&bar)));
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        stop = 0u;
        if (blockIdx.x < items) fetch(blockIdx.x, 0);
    }
    __syncthreads();

    const float normw = threadIdx.x < kDim ? w.norm[threadIdx.x] : 0.0f;
    uint32_t n = 0;
    for (uint32_t it = blockIdx.x; it < items; it += gridDim.x, ++n) {
        const uint32_t b = it / d.value_heads, h = it % d.value_heads, kh = h / d.repeat;
        const uint32_t slot = n & 1u;
        // this item's inputs; the gate scalars by plain loads meanwhile
        const float *prow = proj + (size_t)b * ldp;
        float pb = 0.0f, pa = 0.0f, alog = 0.0f, dtb = 0.0f;
        if (threadIdx.x == 0) {
            pb = prow[d.conv_channels + d.value_width + h];
            pa = prow[d.conv_channels + d.value_width + d.value_heads + h];
            alog = w.a_log[h];
            dtb = w.dt_bias[h];
            if (!gdn_bar_wait(&bar, n & 1u)) {
                gdn_raise(err, kErrTimeout);
                stop = 1u;
            }
        }
        __syncthreads();
        if (stop) break;
        float4 s[kRows];
#pragma unroll
        for (int j = 0; j < kRows; ++j)
            s[j] = *reinterpret_cast<const float4 *>(S + (size_t)(warp + 8 * j) * kDim + 4 * lane);
        __syncthreads();   // S drained: the next item's state may land in it
        if (threadIdx.x == 0 && it + gridDim.x < items) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            fetch(it + gridDim.x, slot ^ 1u);
        }
        const uint8_t *in = inbuf + slot * kPInBytes;
        const float *cq = reinterpret_cast<const float *>(in);
        const float *ck = reinterpret_cast<const float *>(in + kPConvRun);
        const float *cv = reinterpret_cast<const float *>(in + 2 * kPConvRun);
        const float *tq = reinterpret_cast<const float *>(in + 3 * kPConvRun);   // conv taps
        const float *tk = reinterpret_cast<const float *>(in + 4 * kPConvRun);
        const float *tv = reinterpret_cast<const float *>(in + 5 * kPConvRun);
        const float *pq = reinterpret_cast<const float *>(in + 6 * kPConvRun);
        const float *pk = pq + kDim, *pv = pk + kDim, *pz = pv + kDim;
        float *conv_out = p.conv_out[b];
        float *sout = p.rec_out[b] + (size_t)h * kDim * kDim;

        // ---- conv + SiLU, L2 norms, gates (gdn_decode_fused_kernel's prologue)
        {
            const uint32_t which = threadIdx.x >> 7, i = threadIdx.x & (kDim - 1);
            const uint32_t c = which * d.key_width + kh * kDim + i;
            const float *hist = (which == 0 ? cq : ck) + 4 * i;
            const float hv[4] = {hist[1], hist[2], hist[3], (which == 0 ? pq : pk)[i]};
            const float *taps = (which == 0 ? tq : tk) + 4 * i;
            float sconv = 0.0f;
#pragma unroll
            for (int j = 0; j < 4; ++j) sconv = __fadd_rn(sconv, __fmul_rn(taps[j], hv[j]));
            if ((h % d.repeat) == 0) {
#pragma unroll
                for (int j = 0; j < 4; ++j) conv_out[(size_t)c * 4 + j] = hv[j];
            }
            const float val = sconv * stable_sigmoid(sconv);
            bad |= !isfinite(val);
            float v2 = val * val;
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v2 += __shfl_xor_sync(0xffffffffu, v2, o);
            if (lane == 0) red[warp] = v2;
            __syncthreads();
            const float sumsq = red[4 * which] + red[4 * which + 1] + red[4 * which + 2] + red[4 * which + 3];
            const float inv = 1.0f / sqrtf(sumsq + 1.0e-6f);
            float out = val * inv;
            if (which == 0) out = out * (1.0f / sqrtf((float)d.key_dim));
            (which == 0 ? qs : ks)[i] = out;
            if (threadIdx.x < kDim) {
                const uint32_t vc = 2 * d.key_width + h * kDim + threadIdx.x;
                const float *vh = cv + 4 * threadIdx.x;
                const float vhv[4] = {vh[1], vh[2], vh[3], pv[threadIdx.x]};
                const float *vt = tv + 4 * threadIdx.x;
                float sv = 0.0f;
#pragma unroll
                for (int j = 0; j < 4; ++j) sv = __fadd_rn(sv, __fmul_rn(vt[j], vhv[j]));
#pragma unroll
                for (int j = 0; j < 4; ++j) conv_out[(size_t)vc * 4 + j] = vhv[j];
                const float vv = sv * stable_sigmoid(sv);
                bad |= !isfinite(vv);
                vs[threadIdx.x] = vv;
            }
            if (threadIdx.x == 0) {
                const float bt = stable_sigmoid(pb);
                const float a = pa + dtb;
                const float sp = a > 20.0f ? a : log1pf(expf(a));
                const float g = -expf(alog) * sp;
                if (!isfinite(g) || g > 0.0f || !isfinite(bt)) gdn_raise(err, kErrDecay);
                gates[0] = bt;
                gates[1] = expf(g);
            }
            __syncthreads();
        }
        // ---- recurrence (one token)
        {
            const float dec = gates[1];
            const float bt = gates[0];
            float r0 = 0.f, r1 = 0.f, r2 = 0.f, r3 = 0.f;
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                s[j].x *= dec; s[j].y *= dec; s[j].z *= dec; s[j].w *= dec;
                const float kv = ks[warp + 8 * j];
                r0 = fmaf(s[j].x, kv, r0);
                r1 = fmaf(s[j].y, kv, r1);
                r2 = fmaf(s[j].z, kv, r2);
                r3 = fmaf(s[j].w, kv, r3);
            }
            *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(r0, r1, r2, r3);
            __syncthreads();
            if (threadIdx.x < kDim) {
                float rd = 0.f;
#pragma unroll
                for (int wv = 0; wv < kRecThreads / 32; ++wv) rd += part[wv][threadIdx.x];
                delta[threadIdx.x] = (vs[threadIdx.x] - rd) * bt;
            }
            __syncthreads();
            const float4 dl = *reinterpret_cast<const float4 *>(&delta[4 * lane]);
            float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
#pragma unroll
            for (int j = 0; j < kRows; ++j) {
                const float kv = ks[warp + 8 * j];
                const float qv = qs[warp + 8 * j];
                s[j].x = fmaf(kv, dl.x, s[j].x);
                s[j].y = fmaf(kv, dl.y, s[j].y);
                s[j].z = fmaf(kv, dl.z, s[j].z);
                s[j].w = fmaf(kv, dl.w, s[j].w);
                o0 = fmaf(s[j].x, qv, o0);
                o1 = fmaf(s[j].y, qv, o1);
                o2 = fmaf(s[j].z, qv, o2);
                o3 = fmaf(s[j].w, qv, o3);
            }
            *reinterpret_cast<float4 *>(&part[warp][4 * lane]) = make_float4(o0, o1, o2, o3);
            __syncthreads();
            float o = 0.f;
            if (threadIdx.x < kDim) {
#pragma unroll
                for (int wv = 0; wv < kRecThreads / 32; ++wv) o += part[wv][threadIdx.x];
                bad |= !isfinite(o);
            }
            const float sumsq = block_sum<kRecThreads>(threadIdx.x < kDim ? o * o : 0.f, red);
            if (threadIdx.x < kDim) {
                const float mean = sumsq / (float)kDim;
                const float inv = 1.0f / sqrtf(mean + d.eps);
                const float z = pz[threadIdx.x];
                const float g = (normw * (o * inv)) * stable_sigmoid(z);
                bad |= !isfinite(g);
                gated[(size_t)b * d.value_width + gated_head_pos(w, h) * kDim + threadIdx.x] = g;
            }
        }
#pragma unroll
        for (int j = 0; j < kRows; ++j) {
            bad |= !isfinite(s[j].x) || !isfinite(s[j].y) || !isfinite(s[j].z) || !isfinite(s[j].w);
            *reinterpret_cast<float4 *>(sout + (size_t)(warp + 8 * j) * kDim + 4 * lane) = s[j];
        }
        __syncthreads();   // ks / qs / vs / part / IN[slot] reads done before the next item overwrites them
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

// ------------------------------------------------------------ checkpoint path
//
// One token, grid (Hv), 128 threads, dynamic shared memory of 2 dk + 2 dv
// floats.  The arithmetic follows the reference's scalar loop step by step
// (src/kq_gdn_qwen38.c:602-815): products and sums separately rounded, the
// dot products, L2 sums and RMS sum taken sequentially by one thread, the
// recurrence one value feature per thread over the key features in order.
// Every intermediate the reference's observer sees is written out.
__global__ void __launch_bounds__(128)
gdn_debug_token_kernel(GdnDims d, GdnWeightsDev w, const float *__restrict__ conv_in, float *__restrict__ conv_out,
                       const float *__restrict__ rec_in, float *__restrict__ rec_out, const float *__restrict__ proj,
                       GdnDebugBufs o, ErrorWord err) {
    pdl_wait();
    extern __shared__ float dsm[];
    __shared__ float gates[2];   // beta, exp(g)
    __shared__ float inv[2];     // q / k inverse norms, then the RMS inverse
    if (gdn_error_raised(err)) return;
    const uint32_t dk = d.key_dim, dv = d.value_dim, K = d.kernel;
    float *sq = dsm, *sk = sq + dk, *sv = sk + dk, *sc = sv + dv;
    const uint32_t h = blockIdx.x, kh = h / d.repeat;
    const bool writer = (h % d.repeat) == 0;   // the key head's q / k channels are written once
    bool bad = false;
    // conv history shift (hist[j] = old hist[j + 1], hist[K-1] = projection),
    // taps dot, SiLU = x * sigmoid(x) (:602-621)
    auto conv = [&](uint32_t c, bool write) -> float {
        float s = 0.0f;
        for (uint32_t j = 0; j < K; ++j) {
            const float hv = j + 1 < K ? conv_in[(size_t)c * K + j + 1] : proj[c];
            s = __fadd_rn(s, __fmul_rn(w.conv[(size_t)c * K + j], hv));
            if (write) {
                conv_out[(size_t)c * K + j] = hv;
                o.conv_state[(size_t)c * K + j] = hv;
            }
        }
        return __fmul_rn(s, stable_sigmoid(s));
    };
    for (uint32_t i = threadIdx.x; i < dk; i += blockDim.x) {
        const uint32_t cq = kh * dk + i, ck = d.key_width + kh * dk + i;
        const float q = conv(cq, writer), k = conv(ck, writer);
        if (writer) {
            o.conv_out[cq] = q;
            o.conv_out[ck] = k;
        }
        o.q_raw[(size_t)h * dk + i] = q;
        o.k_raw[(size_t)h * dk + i] = k;
        sq[i] = q;
        sk[i] = k;
        bad |= !isfinite(q) || !isfinite(k);
    }
    for (uint32_t i = threadIdx.x; i < dv; i += blockDim.x) {
        const uint32_t cv = 2 * d.key_width + h * dv + i;
        const float v = conv(cv, true);
        o.conv_out[cv] = v;
        o.v[(size_t)h * dv + i] = v;
        sv[i] = v;
        bad |= !isfinite(v);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        // beta, log decay (:662-678), L2 sums (:338-360)
        const float pb = proj[d.conv_channels + d.value_width + h];
        const float pa = proj[d.conv_channels + d.value_width + d.value_heads + h];
        const float bt = stable_sigmoid(pb);
        const float a = __fadd_rn(pa, w.dt_bias[h]);
        const float sp = a > 20.0f ? a : log1pf(expf(a));
        const float g = __fmul_rn(-expf(w.a_log[h]), sp);
        if (!isfinite(a) || !isfinite(sp) || !isfinite(g) || g > 0.0f) gdn_raise(err, kErrDecay);
        o.log_decay[h] = g;
        o.beta[h] = bt;
        gates[0] = bt;
        gates[1] = expf(g);
        float s = 0.0f;
        for (uint32_t i = 0; i < dk; ++i) s = __fadd_rn(s, __fmul_rn(sq[i], sq[i]));
        inv[0] = 1.0f / sqrtf(__fadd_rn(s, 1.0e-6f));
        s = 0.0f;
        for (uint32_t i = 0; i < dk; ++i) s = __fadd_rn(s, __fmul_rn(sk[i], sk[i]));
        inv[1] = 1.0f / sqrtf(__fadd_rn(s, 1.0e-6f));
    }
    __syncthreads();
    const float qscale = 1.0f / sqrtf((float)dk);
    for (uint32_t i = threadIdx.x; i < dk; i += blockDim.x) {
        const float qn = __fmul_rn(__fmul_rn(sq[i], inv[0]), qscale);
        const float kn = __fmul_rn(sk[i], inv[1]);
        o.q_norm[(size_t)h * dk + i] = qn;
        o.k_norm[(size_t)h * dk + i] = kn;
        sq[i] = qn;
        sk[i] = kn;
    }
    __syncthreads();
    // delta rule (:705-761): S *= exp(g); read = S^T k; delta = (v - read) beta;
    // S += k delta^T; out = S^T q
    const float bt = gates[0], dec = gates[1];
    const float *S0 = rec_in + (size_t)h * dk * dv;
    float *S1 = rec_out + (size_t)h * dk * dv;
    for (uint32_t f = threadIdx.x; f < dv; f += blockDim.x) {
        float rd = 0.0f;
        for (uint32_t kf = 0; kf < dk; ++kf) {
            const float s = __fmul_rn(S0[(size_t)kf * dv + f], dec);
            S1[(size_t)kf * dv + f] = s;
            rd = __fadd_rn(rd, __fmul_rn(s, sk[kf]));
        }
        const float dl = __fmul_rn(__fsub_rn(sv[f], rd), bt);
        float co = 0.0f;
        for (uint32_t kf = 0; kf < dk; ++kf) {
            const float s = __fadd_rn(S1[(size_t)kf * dv + f], __fmul_rn(sk[kf], dl));
            S1[(size_t)kf * dv + f] = s;
            bad |= !isfinite(s);
            co = __fadd_rn(co, __fmul_rn(s, sq[kf]));
        }
        o.read[(size_t)h * dv + f] = rd;
        o.delta[(size_t)h * dv + f] = dl;
        o.core[(size_t)h * dv + f] = co;
        sc[f] = co;
        bad |= !isfinite(co);
    }
    __syncthreads();
    // gated RMSNorm, norm weight applied directly (:787-815)
    if (threadIdx.x == 0) {
        float s = 0.0f;
        for (uint32_t f = 0; f < dv; ++f) s = __fadd_rn(s, __fmul_rn(sc[f], sc[f]));
        inv[0] = 1.0f / sqrtf(__fadd_rn(s / (float)dv, d.eps));
    }
    __syncthreads();
    for (uint32_t f = threadIdx.x; f < dv; f += blockDim.x) {
        const float z = proj[d.conv_channels + h * dv + f];
        const float g = __fmul_rn(__fmul_rn(w.norm[f], __fmul_rn(sc[f], inv[0])), stable_sigmoid(z));
        o.gated[(size_t)h * dv + f] = g;
        o.gated_proj[(size_t)gated_head_pos(w, h) * dv + f] = g;
        bad |= !isfinite(g);
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

void launch_gdn_debug_token(const GdnDims &d, const GdnWeightsDev &w, const float *conv_in, float *conv_out,
                            const float *rec_in, float *rec_out, const float *proj, const GdnDebugBufs &b,
                            ErrorWord err, cudaStream_t stream) {
    const size_t smem = (size_t)(2 * d.key_dim + 2 * d.value_dim) * sizeof(float);
    launch_pdl(gdn_debug_token_kernel, dim3(d.value_heads), 128, smem, stream, d, w, conv_in, conv_out, rec_in,
               rec_out, proj, b, err);
    count_launch();
}

bool gdn_decode_fused_supported(const GdnDims &d) {
    return d.key_dim == kDim && d.value_dim == kDim && d.kernel == 4;
}

void launch_gdn_decode_fused(const GdnDims &d, const GdnWeightsDev &w, const GdnBatchPtrs &p, uint32_t batch,
                             const float *proj, uint32_t ldp, float *gated, ErrorWord err, cudaStream_t stream) {
    KernelTimer timer("gdn_recurrence", stream);
    // persistent form when every bulk-copy source is 16-byte aligned
    // (KQ_B200_GDN_PERSIST=0 selects the one-shot kernel: tuning and tests)
    const char *env = getenv("KQ_B200_GDN_PERSIST");
    bool persist = !(env && env[0] == '0') && (ldp % 4u) == 0u && (reinterpret_cast<uintptr_t>(proj) & 15u) == 0u &&
                   (reinterpret_cast<uintptr_t>(w.conv) & 15u) == 0u;
    for (uint32_t b = 0; b < batch && persist; ++b)
        persist = (reinterpret_cast<uintptr_t>(p.rec_in[b]) & 15u) == 0u &&
                  (reinterpret_cast<uintptr_t>(p.conv_in[b]) & 15u) == 0u;
    if (persist) {
        static DeviceOnce attr;
        static int per_sm[64];
        attr.run([] {
            int dev = 0;
            cudaGetDevice(&dev);
            cudaFuncSetAttribute(gdn_decode_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmem);
            int n = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, gdn_decode_persist_kernel, kRecThreads, kPSmem);
            per_sm[dev & 63] = n > 0 ? n : 1;
        });
        int dev = 0, sms = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        const uint32_t items = batch * d.value_heads;
        const uint32_t grid = std::min<uint32_t>(items, (uint32_t)(std::max(sms, 1) * per_sm[dev & 63]));
        launch_pdl(gdn_decode_persist_kernel, dim3(grid), kRecThreads, kPSmem, stream, d, w, p, batch, proj, ldp,
                   gated, err);
    } else {
        launch_pdl(gdn_decode_fused_kernel, dim3(d.value_heads, batch), kRecThreads, 0, stream, d, w, p, proj, ldp,
                   gated, err);
    }
    count_launch();
}

// Generic dims (any dk, dv <= 1024): one thread per value feature f, state
// streamed through global memory (rec_out doubles as the working copy).
__global__ void __launch_bounds__(128)
gdn_recurrence_generic_kernel(GdnDims d, GdnWeightsDev w, GdnBatchPtrs p, uint32_t tokens,
                              const float *__restrict__ qk, const float *__restrict__ vin,
                              const float *__restrict__ beta, const float *__restrict__ decay,
                              const float *__restrict__ proj, uint32_t ldp,
                              float *__restrict__ gated, ErrorWord err) {
    pdl_wait();
    __shared__ float red[4];
    if (gdn_error_raised(err)) return;
    const uint32_t h = blockIdx.x, b = blockIdx.y;
    const uint32_t kh = h / d.repeat;
    const uint32_t dk = d.key_dim, dv = d.value_dim;
    const float *sin_ = p.rec_in[b] + (size_t)h * dk * dv;
    float *S = p.rec_out[b] + (size_t)h * dk * dv;
    bool bad = false;
    for (uint32_t i = threadIdx.x; i < dk * dv; i += blockDim.x) S[i] = sin_[i];
    __syncthreads();
    for (uint32_t t = 0; t < tokens; ++t) {
        const size_t item = (size_t)b * tokens + t;
        const float *q = qk + (item * 2 + 0) * d.key_width + kh * dk;
        const float *k = qk + (item * 2 + 1) * d.key_width + kh * dk;
        const float dec = decay[item * d.value_heads + h];
        const float bt = beta[item * d.value_heads + h];
        float ssq_local = 0.f;
        float outs[8];
        int n = 0;
        for (uint32_t f = threadIdx.x; f < dv; f += blockDim.x, ++n) {
            float rd = 0.f;
            for (uint32_t kf = 0; kf < dk; ++kf) {
                float sv = S[kf * dv + f] * dec;
                S[kf * dv + f] = sv;
                rd = rd + sv * k[kf];
            }
            float dl = (vin[item * d.value_width + h * dv + f] - rd) * bt;
            float o = 0.f;
            for (uint32_t kf = 0; kf < dk; ++kf) {
                float sv = S[kf * dv + f] + k[kf] * dl;
                S[kf * dv + f] = sv;
                o = o + sv * q[kf];
                bad |= !isfinite(sv);
            }
            bad |= !isfinite(o);
            if (n < 8) outs[n] = o;
            ssq_local += o * o;
        }
        float sumsq = block_sum<128>(ssq_local, red);
        float mean = sumsq / (float)dv;
        float inv = 1.0f / sqrtf(mean + d.eps);
        n = 0;
        for (uint32_t f = threadIdx.x; f < dv && n < 8; f += blockDim.x, ++n) {
            float z = proj[item * ldp + d.conv_channels + h * dv + f];
            float g = (w.norm[f] * (outs[n] * inv)) * stable_sigmoid(z);
            bad |= !isfinite(g);
            gated[item * d.value_width + gated_head_pos(w, h) * dv + f] = g;
        }
        __syncthreads();
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) gdn_raise(err, kErrNonFinite);
}

void launch_gdn_conv_gates(const GdnDims &d, const GdnWeightsDev &w,
                           const GdnBatchPtrs &p, uint32_t batch,
                           uint32_t tokens, const float *proj, uint32_t ldp,
                           float *qk, float *v, float *beta, float *decay,
                           ErrorWord err, cudaStream_t stream, float *logdecay) {
    KernelTimer timer("gdn_conv", stream);
    const bool aligned = (ldp % 4u) == 0u && (reinterpret_cast<uintptr_t>(proj) & 15u) == 0u &&
                         (reinterpret_cast<uintptr_t>(w.conv) & 15u) == 0u;
    if (batch == 1 && tokens >= 64 && d.kernel == 4 && d.key_dim == 128 && d.value_dim == 128 && aligned &&
        (d.repeat == 1 || d.repeat == 2 || d.repeat == 4)) {
        const dim3 wgrid((tokens * d.key_heads + 7) / 8);
        if (d.repeat == 1)
            launch_pdl(gdn_conv_gates_warp_kernel<1>, wgrid, 256, 0, stream, d, w, p, tokens, proj, ldp, qk, v, beta,
                       decay, logdecay, err);
        else if (d.repeat == 2)
            launch_pdl(gdn_conv_gates_warp_kernel<2>, wgrid, 256, 0, stream, d, w, p, tokens, proj, ldp, qk, v, beta,
                       decay, logdecay, err);
        else
            launch_pdl(gdn_conv_gates_warp_kernel<4>, wgrid, 256, 0, stream, d, w, p, tokens, proj, ldp, qk, v, beta,
                       decay, logdecay, err);
        count_launch();
        return;
    }
    dim3 grid(d.key_heads, batch * tokens);
    if (d.kernel == 4)
        launch_pdl(gdn_conv_gates_kernel<4>, grid, kConvThreads, 0, stream, d, w, p, tokens, proj, ldp, qk, v,
                                                                   beta, decay, logdecay, err);
    else
        launch_pdl(gdn_conv_gates_kernel<0>, grid, kConvThreads, 0, stream, d, w, p, tokens, proj, ldp, qk, v,
                                                                   beta, decay, logdecay, err);
    count_launch();
}

void launch_gdn_recurrence(const GdnDims &d, const GdnWeightsDev &w,
                           const GdnBatchPtrs &p, uint32_t batch,
                           uint32_t tokens, const float *qk, const float *v,
                           const float *beta, const float *decay,
                           const float *proj, uint32_t ldp, float *gated,
                           ErrorWord err, cudaStream_t stream) {
    dim3 grid(d.value_heads, batch);
    KernelTimer timer("gdn_recurrence", stream);
    if (d.key_dim == kDim && d.value_dim == kDim) {
        launch_pdl(gdn_recurrence128_kernel, grid, kRecThreads, 0, stream, d, w, p, tokens, qk, v, beta,
                                                                  decay, proj, ldp, gated, err);
    } else {
        launch_pdl(gdn_recurrence_generic_kernel, grid, 128, 0, stream, d, w, p, tokens, qk, v, beta,
                                                               decay, proj, ldp, gated, err);
    }
    count_launch();
}

}  // namespace kqb
