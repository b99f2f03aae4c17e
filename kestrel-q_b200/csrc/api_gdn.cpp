// kq_gdn ABI on the B200: configs, device-resident states and execution.
//
// Replaces src/kq_gdn.c and the entry points of src/kq_gdn_qwen38.c of
// Kestrel-Q.  Validation order and status codes follow kq_gdn_validate_call
// (src/kq_gdn_qwen38.c:362-486); the transactional contract (state untouched
// on failure, :532-536,844-848) is kept with double-buffered device state
// that is only committed when the device reported no error.
#include <cfenv>
#include <cmath>
#include <algorithm>
#include <cstring>
#include <new>
#include <vector>

#include "kq_b200.h"
#include "kq_gdn.h"
#include "operators.hpp"
#include "provider.hpp"
#include "runtime.hpp"

using namespace kqb;

namespace {
constexpr uint32_t kGdnConfigMagic = 0x4b514743u;
constexpr uint32_t kGdnStateMagic = 0x4b514753u;
constexpr uint32_t kPrefillChunk = 8192;   // tokens per device pass
constexpr uint32_t kChunkedMinTokens = 32;  // prefill passes from this length use the chunked recurrence
}  // namespace

struct kq_gdn_config {
    uint32_t magic;
    uint32_t layer_id;
    kq_gdn_dimensions dims;
    uint32_t key_width, value_width, conv_channels, repeat;
    uint64_t recurrent_elements, conv_state_elements, token_scratch_bytes, scratch_bytes;
    kq_weight_provider *provider;
    QMatrix qkv, gate, beta, alpha, out;
    const float *a_log, *conv, *dt_bias, *norm;
    const int32_t *gated_head;   // output projection column heads (null: canonical)
    bool bound;
};

struct kq_gdn_state final : Rollbackable {
    uint32_t magic = 0;
    const kq_gdn_config *config = nullptr;
    int device = 0;
    float *conv[2] = {nullptr, nullptr};
    float *rec[2] = {nullptr, nullptr};
    int cur = 0, initialized = 0;
    int synced_cur = 0, synced_init = 0;
    std::vector<std::pair<uint32_t, int>> history;
    uint64_t owned_bytes = 0;

    void on_step(uint32_t id) override { history.push_back({id, cur}); }
    void on_error(uint32_t failing) override {
        int c = synced_cur, init = synced_init;
        for (auto &h : history)
            if (failing != 0 && h.first < failing) { c = h.second; init = 1; }
        cur = c;
        initialized = init;
        on_success();
    }
    void on_success() override {
        synced_cur = cur;
        synced_init = initialized;
        history.clear();
    }
};

static bool config_valid(const kq_gdn_config *c) { return c != nullptr && c->magic == kGdnConfigMagic; }
static bool state_valid(const kq_gdn_state *s) {
    return s != nullptr && s->magic == kGdnStateMagic && config_valid(s->config) && s->conv[0] && s->rec[0];
}

// Dimension checks and derived sizes of src/kq_gdn.c:124-229.
static kq_status validate_dims(const kq_gdn_dimensions *d, kq_gdn_config *c, kq_diagnostic *diag) {
    if (d->hidden_size == 0 || d->key_head_count == 0 || d->value_head_count == 0 ||
        d->key_head_dimension == 0 || d->value_head_dimension == 0 || d->conv_kernel_size != 4 ||
        d->value_head_count % d->key_head_count != 0 || !(d->rms_norm_epsilon > 0.0f) ||
        !std::isfinite(d->rms_norm_epsilon) ||
        (d->activation_dtype != KQ_GDN_ACTIVATION_F32 && d->activation_dtype != KQ_GDN_ACTIVATION_BF16))
        return fail(diag, KQ_STATUS_INCOMPATIBLE_GDN, "invalid GDN dimensions, head ratio, kernel, epsilon, or dtype");
    uint64_t key, value, conv, rec, conv_state;
    if (!mul_ok(d->key_head_count, d->key_head_dimension, &key) ||
        !mul_ok(d->value_head_count, d->value_head_dimension, &value) ||
        !add_ok(key, key, &conv) || !add_ok(conv, value, &conv) || key > UINT32_MAX ||
        value > UINT32_MAX || conv > UINT32_MAX)
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "GDN projection dimensions overflow");
    if (!mul_ok(d->value_head_count, d->key_head_dimension, &rec) ||
        !mul_ok(rec, d->value_head_dimension, &rec) || !mul_ok(conv, d->conv_kernel_size, &conv_state))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "GDN state dimensions overflow");
    // per-token F32 work space of the reference (same accounting)
    const uint64_t H = d->hidden_size, Hv = d->value_head_count, rk = (uint64_t)Hv * d->key_head_dimension;
    uint64_t tok = H + conv + value + Hv + Hv + conv + rk + rk + value + Hv + Hv + value + value + value +
                   value + H;
    uint64_t total = tok + rec + conv_state;
    if (total > (UINT64_MAX / 8))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "GDN total workspace byte count overflows size_t");
    // B200 kernel limits
    if (d->key_head_dimension > 128 || d->value_head_dimension > 1024)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_GDN,
                    "B200 GDN kernels support key heads up to 128 and value heads up to 1024 wide");
    c->key_width = (uint32_t)key;
    c->value_width = (uint32_t)value;
    c->conv_channels = (uint32_t)conv;
    c->repeat = d->value_head_count / d->key_head_count;
    c->recurrent_elements = rec;
    c->conv_state_elements = conv_state;
    c->token_scratch_bytes = tok * 4;
    c->scratch_bytes = total * 4;
    return KQ_STATUS_OK;
}

static GdnDims kernel_dims(const kq_gdn_config *c) {
    GdnDims g;
    g.hidden = c->dims.hidden_size;
    g.key_heads = c->dims.key_head_count;
    g.value_heads = c->dims.value_head_count;
    g.key_dim = c->dims.key_head_dimension;
    g.value_dim = c->dims.value_head_dimension;
    g.kernel = c->dims.conv_kernel_size;
    g.conv_channels = c->conv_channels;
    g.key_width = c->key_width;
    g.value_width = c->value_width;
    g.repeat = c->repeat;
    g.eps = c->dims.rms_norm_epsilon;
    return g;
}

struct GdnResolved {
    QMatrix qkv, gate, beta, alpha, out;
    GdnWeightsDev vec;
};

// Enqueues the operator for `batch` sequences x `tokens` tokens.  x / y are
// device arrays [batch*tokens][H]; mask (device, may be null) is [tokens]
// for batch == 1.  States flip optimistically and are registered for
// roll-back; the caller synchronises.
// `check_input`: the caller has not checked x for non-finite values; the
// in-projection (or a separate pass) does.
static kq_status gdn_enqueue(DeviceContext *c, const kq_gdn_config *cfg, const GdnResolved &w,
                             kq_gdn_state *const *states, uint32_t batch, uint32_t tokens,
                             const float *x, const uint8_t *mask, float *y, ErrorWord err,
                             kq_diagnostic *diag, bool check_input = false) {
    const GdnDims gd = kernel_dims(cfg);
    const uint32_t H = gd.hidden, C = gd.conv_channels, Vd = gd.value_width, Hv = gd.value_heads;
    const uint32_t ldp = C + Vd + 2 * Hv;
    const uint32_t chunk_tokens = batch == 1 ? std::min(tokens, kPrefillChunk) : 1u;
    const uint32_t group = batch == 1 ? 1u : std::min<uint32_t>(batch, kMaxBatch);
    const size_t items = (size_t)group * chunk_tokens;
    size_t need = Carve::round(items * ldp * 4) + Carve::round(items * 2 * gd.key_width * 4) +
                  Carve::round(items * Vd * 4) * 2 + Carve::round(items * Hv * 4) * 2 +
                  (mask ? Carve::round(items * H * 4) : 0) + 4096;
    // work space of the tensor-core projections (in-proj and out-proj)
    const size_t partial_floats = std::max(projection_workspace_floats((uint32_t)items, ldp, H),
                                           projection_workspace_floats((uint32_t)items, H, Vd));
    need += Carve::round(partial_floats * 4);
    // prefill of one sequence: chunked (WY-form) recurrence
    const bool chunked = batch == 1 && chunk_tokens >= kChunkedMinTokens && gdn_chunked_supported(gd);
    const size_t chunk_floats = chunked ? gdn_chunk_workspace_floats(gd, chunk_tokens) : 0;
    if (chunked) need += Carve::round(items * Hv * 4) + Carve::round(chunk_floats * 4);
    void *ws;
    kq_status st = c->workspace(need, &ws, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    float *proj = cv.take<float>(items * ldp);
    float *qk = cv.take<float>(items * 2 * gd.key_width);
    float *v = cv.take<float>(items * Vd);
    float *gated = cv.take<float>(items * Vd);
    float *beta = cv.take<float>(items * Hv);
    float *decay = cv.take<float>(items * Hv);
    float *xm = mask ? cv.take<float>(items * H) : nullptr;
    float *partial = partial_floats ? cv.take<float>(partial_floats) : nullptr;
    float *logdecay = chunked ? cv.take<float>(items * Hv) : nullptr;
    float *chunk_work = chunked ? cv.take<float>(chunk_floats) : nullptr;

    ProjSegments in{};
    in.count = 4;
    in.m[0] = w.qkv; in.out_offset[0] = 0;
    in.m[1] = w.gate; in.out_offset[1] = C;
    in.m[2] = w.beta; in.out_offset[2] = C + Vd;
    in.m[3] = w.alpha; in.out_offset[3] = C + Vd + Hv;
    ProjSegments out{};
    out.count = 1;
    out.m[0] = w.out;
    out.out_offset[0] = 0;

    for (uint32_t g0 = 0; g0 < batch; g0 += group) {
        const uint32_t gb = std::min(group, batch - g0);
        for (uint32_t t0 = 0; t0 < tokens; t0 += chunk_tokens) {
            const uint32_t tc = std::min(chunk_tokens, tokens - t0);
            const size_t row0 = (size_t)g0 * tokens + t0;   // batch==1 or tokens==1
            const float *xin = x + row0 * H;
            if (mask) {
                launch_mask_rows(xin, mask + t0, tc, H, xm, c->stream);
                xin = xm;
            }
            GdnBatchPtrs p;
            for (uint32_t b = 0; b < gb; ++b) {
                kq_gdn_state *s = states[g0 + b];
                p.conv_in[b] = s->conv[s->cur];
                p.conv_out[b] = s->conv[1 - s->cur];
                p.rec_in[b] = s->rec[s->cur];
                p.rec_out[b] = s->rec[1 - s->cur];
            }
            const uint32_t n_items = gb * tc;
            if (!launch_projection(in, xin, H, proj, ldp, n_items, err, c->stream, partial, partial_floats) &&
                check_input)
                launch_check_finite(xin, (uint64_t)n_items * H, err, c->stream);
            if (tc == 1 && gdn_decode_fused_supported(gd)) {
                launch_gdn_decode_fused(gd, w.vec, p, gb, proj, ldp, gated, err, c->stream);
            } else {
                launch_gdn_conv_gates(gd, w.vec, p, gb, tc, proj, ldp, qk, v, beta, decay, err, c->stream,
                                      logdecay);
                if (chunked && tc >= kChunkedMinTokens)
                    launch_gdn_chunked(gd, w.vec, p, tc, qk, v, beta, logdecay, proj, ldp, gated, chunk_work, err,
                                       c->stream);
                else
                    launch_gdn_recurrence(gd, w.vec, p, gb, tc, qk, v, beta, decay, proj, ldp, gated, err,
                                          c->stream);
            }
            if (!launch_projection(out, gated, Vd, y + row0 * H, H, n_items, err, c->stream, partial,
                                   partial_floats))
                launch_check_finite(y + row0 * H, (uint64_t)n_items * H, err, c->stream);
            for (uint32_t b = 0; b < gb; ++b) {
                kq_gdn_state *s = states[g0 + b];
                s->cur = 1 - s->cur;
                s->initialized = 1;
                s->on_step(err.call_id);
                c->dirty.insert(s);
            }
        }
    }
    KQB_CUDA(cudaGetLastError(), diag, "GDN launch");
    return KQ_STATUS_OK;
}

// Checkpoint path (an observer is attached): token by token, every
// intermediate the reference's observer sees (src/kq_gdn_qwen38.c:554-838,
// the 21 kinds of include/kq_gdn.h) computed on the device by the debug
// kernel, copied to the host and handed to the observer in the reference's
// order once the token has run without a device error.  The projections are
// the product's own.  The state keeps the call's contract: the caller's final
// synchronize commits it, or rolls the whole call back if a token failed (the
// observer has then seen the tokens before the failing one, as with the
// reference).
static kq_status gdn_debug_run(DeviceContext *c, const kq_gdn_config *cfg, const GdnResolved &w, kq_gdn_state *s,
                               uint32_t T, const float *x, const uint8_t *mask, float *y, ErrorWord err,
                               kq_gdn_checkpoint_observer observer, void *user, kq_diagnostic *diag) {
    const GdnDims gd = kernel_dims(cfg);
    const uint32_t H = gd.hidden, C = gd.conv_channels, Vd = gd.value_width, Hv = gd.value_heads;
    const uint32_t dk = gd.key_dim, dv = gd.value_dim, K = gd.kernel;
    const uint32_t ldp = C + Vd + 2 * Hv;
    const size_t rk = (size_t)Hv * dk, rec_n = cfg->recurrent_elements;
    const size_t need = Carve::round((size_t)H * 4) + Carve::round((size_t)ldp * 4) + Carve::round((size_t)C * 4) +
                        Carve::round((size_t)C * K * 4) + 4 * Carve::round(rk * 4) + 6 * Carve::round((size_t)Vd * 4) +
                        2 * Carve::round((size_t)Hv * 4) + 4096;
    void *ws;
    kq_status st = c->workspace(need, &ws, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    float *xm = cv.take<float>(H);
    float *proj = cv.take<float>(ldp);
    GdnDebugBufs b;
    b.conv_out = cv.take<float>(C);
    b.conv_state = cv.take<float>((size_t)C * K);
    b.q_raw = cv.take<float>(rk);
    b.k_raw = cv.take<float>(rk);
    b.q_norm = cv.take<float>(rk);
    b.k_norm = cv.take<float>(rk);
    b.v = cv.take<float>(Vd);
    b.read = cv.take<float>(Vd);
    b.delta = cv.take<float>(Vd);
    b.core = cv.take<float>(Vd);
    b.gated = cv.take<float>(Vd);
    b.gated_proj = w.vec.gated_head != nullptr ? cv.take<float>(Vd) : b.gated;
    b.log_decay = cv.take<float>(Hv);
    b.beta = cv.take<float>(Hv);
    ProjSegments in{};
    in.count = 4;
    in.m[0] = w.qkv; in.out_offset[0] = 0;
    in.m[1] = w.gate; in.out_offset[1] = C;
    in.m[2] = w.beta; in.out_offset[2] = C + Vd;
    in.m[3] = w.alpha; in.out_offset[3] = C + Vd + Hv;
    ProjSegments out{};
    out.count = 1;
    out.m[0] = w.out;
    out.out_offset[0] = 0;
    std::vector<float> hx(H), hp(ldp), hco(C), hcs((size_t)C * K), hqr(rk), hkr(rk), hqn(rk), hkn(rk), hv(Vd),
        hrd(Vd), hdl(Vd), hcr(Vd), hgt(Vd), hg(Hv), hb(Hv), hst(rec_n), hy(H);
    for (uint32_t t = 0; t < T; ++t) {
        const float *xt = x + (size_t)t * H;
        const float *xin = xt;
        if (mask) {
            launch_mask_rows(xt, mask + t, 1, H, xm, c->stream);
            xin = xm;
        }
        launch_projection(in, xin, H, proj, ldp, 1, err, c->stream);
        const int cur = s->cur;
        launch_gdn_debug_token(gd, w.vec, s->conv[cur], s->conv[1 - cur], s->rec[cur], s->rec[1 - cur], proj, b,
                               err, c->stream);
        float *yt = y + (size_t)t * H;
        if (!launch_projection(out, b.gated_proj, Vd, yt, H, 1, err, c->stream))
            launch_check_finite(yt, H, err, c->stream);
        s->cur = 1 - cur;
        s->initialized = 1;
        s->on_step(err.call_id);
        c->dirty.insert(s);
        KQB_CUDA(cudaGetLastError(), diag, "GDN checkpoint launch");
        KQB_CUDA(cudaStreamSynchronize(c->stream), diag, "GDN checkpoint sync");
        unsigned long long word = 0;
        KQB_CUDA(cudaMemcpy(&word, c->err_word, sizeof word, cudaMemcpyDeviceToHost), diag, "error word read");
        if (word != 0ull) return KQ_STATUS_OK;   // reported and rolled back by the caller's synchronize
        struct Copy { float *dst; const float *src; size_t n; } copies[] = {
            {hx.data(), xin, H}, {hp.data(), proj, ldp}, {hco.data(), b.conv_out, C},
            {hcs.data(), b.conv_state, (size_t)C * K}, {hqr.data(), b.q_raw, rk}, {hkr.data(), b.k_raw, rk},
            {hv.data(), b.v, Vd}, {hqn.data(), b.q_norm, rk}, {hkn.data(), b.k_norm, rk},
            {hg.data(), b.log_decay, Hv}, {hb.data(), b.beta, Hv}, {hrd.data(), b.read, Vd},
            {hdl.data(), b.delta, Vd}, {hcr.data(), b.core, Vd}, {hst.data(), s->rec[s->cur], rec_n},
            {hgt.data(), b.gated, Vd}, {hy.data(), yt, H}};
        for (const Copy &cp : copies)
            KQB_CUDA(cudaMemcpy(cp.dst, cp.src, cp.n * 4, cudaMemcpyDeviceToHost), diag, "checkpoint copy");
        auto emit = [&](kq_gdn_checkpoint_kind kind, uint32_t rank, uint64_t d0, uint64_t d1, uint64_t d2,
                        const float *v, uint64_t count) {
            kq_gdn_checkpoint cp;
            std::memset(&cp, 0, sizeof(cp));
            cp.kind = kind;
            cp.token_index = t;
            cp.rank = rank;
            cp.dimensions[0] = d0;
            cp.dimensions[1] = d1;
            cp.dimensions[2] = d2;
            cp.values = v;
            cp.value_count = count;
            observer(&cp, user);
        };
        emit(KQ_GDN_CHECKPOINT_MASKED_INPUT, 1, H, 0, 0, hx.data(), H);
        emit(KQ_GDN_CHECKPOINT_PROJECTED_QKV, 1, C, 0, 0, hp.data(), C);
        emit(KQ_GDN_CHECKPOINT_PROJECTED_GATE, 2, Hv, dv, 0, hp.data() + C, Vd);
        emit(KQ_GDN_CHECKPOINT_PROJECTED_BETA, 1, Hv, 0, 0, hp.data() + C + Vd, Hv);
        emit(KQ_GDN_CHECKPOINT_PROJECTED_ALPHA, 1, Hv, 0, 0, hp.data() + C + Vd + Hv, Hv);
        emit(KQ_GDN_CHECKPOINT_CONV_INPUT, 1, C, 0, 0, hp.data(), C);
        emit(KQ_GDN_CHECKPOINT_CONV_OUTPUT, 1, C, 0, 0, hco.data(), C);
        emit(KQ_GDN_CHECKPOINT_CONV_STATE, 2, C, K, 0, hcs.data(), (uint64_t)C * K);
        emit(KQ_GDN_CHECKPOINT_QUERY_BEFORE_NORM, 2, Hv, dk, 0, hqr.data(), rk);
        emit(KQ_GDN_CHECKPOINT_KEY_BEFORE_NORM, 2, Hv, dk, 0, hkr.data(), rk);
        emit(KQ_GDN_CHECKPOINT_VALUE, 2, Hv, dv, 0, hv.data(), Vd);
        emit(KQ_GDN_CHECKPOINT_NORMALIZED_SCALED_QUERY, 2, Hv, dk, 0, hqn.data(), rk);
        emit(KQ_GDN_CHECKPOINT_NORMALIZED_KEY, 2, Hv, dk, 0, hkn.data(), rk);
        emit(KQ_GDN_CHECKPOINT_LOG_DECAY, 1, Hv, 0, 0, hg.data(), Hv);
        emit(KQ_GDN_CHECKPOINT_BETA, 1, Hv, 0, 0, hb.data(), Hv);
        emit(KQ_GDN_CHECKPOINT_RECURRENT_READ, 2, Hv, dv, 0, hrd.data(), Vd);
        emit(KQ_GDN_CHECKPOINT_RECURRENT_DELTA, 2, Hv, dv, 0, hdl.data(), Vd);
        emit(KQ_GDN_CHECKPOINT_RECURRENT_OUTPUT, 2, Hv, dv, 0, hcr.data(), Vd);
        emit(KQ_GDN_CHECKPOINT_RECURRENT_STATE, 3, Hv, dk, dv, hst.data(), rec_n);
        emit(KQ_GDN_CHECKPOINT_GATED_NORM_OUTPUT, 2, Hv, dv, 0, hgt.data(), Vd);
        emit(KQ_GDN_CHECKPOINT_OPERATOR_OUTPUT, 1, H, 0, 0, hy.data(), H);
    }
    return KQ_STATUS_OK;
}

// Host/device staging + synchronous execution shared by the F32 and the
// provider entry points (`observer` non-null: the checkpoint path).
// F32 weight arrays (host: uploaded once and reused while their contents
// stay the same; device: used in place, checked on the device) as the
// operator's dense matrices.
static kq_status resolve_f32(DeviceContext *c, const kq_gdn_config *cfg, const kq_gdn_weights_f32 *wf, ErrorWord err,
                             GdnResolved *out, kq_diagnostic *diag) {
    const uint32_t H = cfg->dims.hidden_size;
    kq_status st = KQ_STATUS_OK;
    GdnResolved &w = *out;

    {
        const uint32_t Hh = H, C = cfg->conv_channels, Vd = cfg->value_width, Hv = cfg->dims.value_head_count;
        const float *ptrs[9] = {wf->a_log, wf->conv, wf->dt_bias, wf->alpha, wf->beta,
                                wf->qkv, wf->gate, wf->norm, wf->output};
        const uint64_t counts[9] = {wf->a_log_count, wf->conv_count, wf->dt_bias_count,
                                    wf->alpha_count, wf->beta_count, wf->qkv_count,
                                    wf->gate_count, wf->norm_count, wf->output_count};
        // host weights: uploaded once and reused while their contents stay
        // the same; device weights: used in place, checked on the device
        const float *dev[9];
        for (int i = 0; i < 9; ++i) {
            if (is_device_pointer(ptrs[i])) {
                dev[i] = ptrs[i];
                launch_check_finite(dev[i], counts[i], err, c->stream);
            } else {
                st = c->upload_cached(ptrs[i], counts[i], &dev[i], diag);
                if (st != KQ_STATUS_OK) return st;
            }
        }
        auto dense = [](const float *p, uint32_t rows, uint32_t cols) {
            QMatrix m{};
            m.data = reinterpret_cast<const uint8_t *>(p);
            m.type = 0;
            m.rows = rows;
            m.cols = cols;
            m.row_bytes = cols * 4;
            m.layout = 0;
            return m;
        };
        w.vec.a_log = dev[0];
        w.vec.conv = dev[1];
        w.vec.dt_bias = dev[2];
        w.alpha = dense(dev[3], Hv, Hh);
        w.beta = dense(dev[4], Hv, Hh);
        w.qkv = dense(dev[5], C, Hh);
        w.gate = dense(dev[6], Vd, Hh);
        w.vec.norm = dev[7];
        w.out = dense(dev[8], Hh, Vd);
    }
    return st;
}

static kq_status gdn_execute_sync(const kq_gdn_config *cfg, const GdnResolved *w_in,
                                  const kq_gdn_weights_f32 *wf, const float *hidden, uint64_t T,
                                  const uint8_t *mask, float *output, kq_gdn_state *state,
                                  kq_gdn_checkpoint_observer observer, void *user, kq_diagnostic *diag) {
    DeviceContext *c;
    kq_status st = context(&c, diag);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    const uint32_t H = cfg->dims.hidden_size;
    const uint64_t n = T * H;
    ErrorWord err = c->begin_call();

    // host inputs and the output go through the context's staging arena (no
    // allocation once it has grown to this call's size; the operator's own
    // work space is a separate arena)
    const bool x_host = !is_device_pointer(hidden);
    const bool m_host = mask != nullptr && !is_device_pointer(mask);
    void *stage;
    st = c->staging(Carve::round(n * 4) + (x_host ? Carve::round(n * 4) : 0) + (m_host ? Carve::round(T) : 0),
                    &stage, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve sc(stage);
    float *dy = sc.take<float>(n);
    const float *dx = hidden;
    if (x_host) {
        float *t = sc.take<float>(n);
        KQB_CUDA(cudaMemcpyAsync(t, hidden, n * 4, cudaMemcpyHostToDevice, c->stream), diag, "input copy");
        dx = t;
    }
    launch_check_finite(dx, n, err, c->stream);
    const uint8_t *dmask = mask;
    if (m_host) {
        uint8_t *t = sc.take<uint8_t>(T);
        KQB_CUDA(cudaMemcpyAsync(t, mask, T, cudaMemcpyHostToDevice, c->stream), diag, "mask copy");
        dmask = t;
    }

    GdnResolved w;
    if (w_in) {
        w = *w_in;
    } else {
        st = resolve_f32(c, cfg, wf, err, &w, diag);
        if (st != KQ_STATUS_OK) return st;
    }
    kq_gdn_state *states[1] = {state};
    st = observer != nullptr
             ? gdn_debug_run(c, cfg, w, state, (uint32_t)T, dx, dmask, dy, err, observer, user, diag)
             : gdn_enqueue(c, cfg, w, states, 1, (uint32_t)T, dx, dmask, dy, err, diag);
    if (st != KQ_STATUS_OK) {
        c->synchronize(nullptr);
        return st;
    }
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output, dy, n * 4,
                        is_device_pointer(output) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost),
             diag, "output copy");
    return KQ_STATUS_OK;
}

// kq_gdn_validate_call (src/kq_gdn_qwen38.c:362-486): everything that can be
// checked on the host before any device work.
static kq_status validate_call(const kq_gdn_config *config, const kq_gdn_weights_f32 *weights,
                               const float *hidden, uint64_t T, const uint8_t *mask, float *output,
                               uint64_t output_capacity, kq_gdn_state *state, void *scratch,
                               uint64_t scratch_bytes, bool provider_mode, kq_diagnostic *diag) {
    if (!config_valid(config) || (!provider_mode && weights == nullptr) || hidden == nullptr ||
        output == nullptr || !state_valid(state) || state->config != config || scratch == nullptr ||
        (state->initialized != 0 && state->initialized != 1))
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid compatible GDN call arguments are required");
    if (config->dims.activation_dtype != KQ_GDN_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_GDN,
                    "F32 scalar execution requires an F32 reference configuration");
    uint64_t n;
    if (T == 0 || !mul_ok(T, config->dims.hidden_size, &n) || n > (SIZE_MAX / 4) || T > UINT32_MAX)
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "GDN sequence element count is invalid or overflows");
    if (output_capacity < n) return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "GDN output capacity is too small");
    if (scratch_bytes < config->scratch_bytes || (reinterpret_cast<uintptr_t>(scratch) % alignof(float)) != 0)
        return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "GDN aligned scratch buffer is too small");
    if (mask != nullptr && !is_device_pointer(mask)) {
        for (uint64_t i = 0; i < T; ++i)
            if (mask[i] > 1) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "GDN padding mask must contain only zero or one");
    }
    if (!is_device_pointer(hidden)) {
        for (uint64_t i = 0; i < n; ++i)
            if (!std::isfinite(hidden[i])) return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "GDN hidden input must be finite");
    }
    if (!provider_mode) {
        const kq_gdn_weights_f32 *w = weights;
        const uint64_t Hv = config->dims.value_head_count, H = config->dims.hidden_size;
        const uint64_t want[9] = {Hv, (uint64_t)config->conv_channels * config->dims.conv_kernel_size, Hv,
                                  Hv * H, Hv * H, (uint64_t)config->conv_channels * H,
                                  (uint64_t)config->value_width * H, config->dims.value_head_dimension,
                                  H * config->value_width};
        const float *ptrs[9] = {w->a_log, w->conv, w->dt_bias, w->alpha, w->beta, w->qkv, w->gate, w->norm, w->output};
        const uint64_t have[9] = {w->a_log_count, w->conv_count, w->dt_bias_count, w->alpha_count,
                                  w->beta_count, w->qkv_count, w->gate_count, w->norm_count, w->output_count};
        // reference order: a_log, dt_bias, norm, conv, alpha, beta, qkv, gate, output
        const int order[9] = {0, 2, 7, 1, 3, 4, 5, 6, 8};
        for (int oi = 0; oi < 9; ++oi) {
            int i = order[oi];
            if (have[i] != want[i]) return fail(diag, KQ_STATUS_DIMENSION_MISMATCH, "GDN F32 weight count mismatch");
            if (ptrs[i] == nullptr) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "GDN F32 weights must be finite");
            if (!is_device_pointer(ptrs[i]))
                for (uint64_t k = 0; k < have[i]; ++k)
                    if (!std::isfinite(ptrs[i][k])) return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "GDN F32 weights must be finite");
        }
        const uint64_t out_bytes = output_capacity * 4, in_bytes = n * 4;
        for (int i = 0; i < 9; ++i) {
            if (ranges_overlap(ptrs[i], have[i] * 4, output, out_bytes) ||
                ranges_overlap(ptrs[i], have[i] * 4, scratch, scratch_bytes))
                return fail(diag, KQ_STATUS_ALIASING_VIOLATION, "GDN input, output, state, and scratch must not overlap");
        }
        (void)in_bytes;
    }
    const uint64_t in_bytes = n * 4, out_bytes = output_capacity * 4;
    if (ranges_overlap(hidden, in_bytes, output, out_bytes) || ranges_overlap(hidden, in_bytes, scratch, scratch_bytes) ||
        ranges_overlap(output, out_bytes, scratch, scratch_bytes))
        return fail(diag, KQ_STATUS_ALIASING_VIOLATION, "GDN input, output, state, and scratch must not overlap");
    for (int b = 0; b < 2; ++b) {
        if (ranges_overlap(state->conv[b], config->conv_state_elements * 4, hidden, in_bytes) ||
            ranges_overlap(state->conv[b], config->conv_state_elements * 4, output, out_bytes) ||
            ranges_overlap(state->rec[b], config->recurrent_elements * 4, hidden, in_bytes) ||
            ranges_overlap(state->rec[b], config->recurrent_elements * 4, output, out_bytes) ||
            ranges_overlap(state->rec[b], config->recurrent_elements * 4, scratch, scratch_bytes))
            return fail(diag, KQ_STATUS_ALIASING_VIOLATION, "GDN input, output, state, and scratch must not overlap");
    }
    if (std::fegetround() != FE_TONEAREST)
        return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "GDN scalar reference requires round-to-nearest");
    return KQ_STATUS_OK;
}

static bool resolve_bound(const kq_gdn_config *cfg, GdnResolved *w) {
    if (!cfg->bound) return false;
    w->qkv = cfg->qkv;
    w->gate = cfg->gate;
    w->beta = cfg->beta;
    w->alpha = cfg->alpha;
    w->out = cfg->out;
    w->vec.a_log = cfg->a_log;
    w->vec.conv = cfg->conv;
    w->vec.dt_bias = cfg->dt_bias;
    w->vec.norm = cfg->norm;
    w->vec.gated_head = cfg->gated_head;
    return true;
}

extern "C" {

kq_status kq_gdn_test_config_create(const kq_gdn_dimensions *dimensions, kq_gdn_config **out_config,
                                    kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (dimensions == nullptr || out_config == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "test GDN dimensions are required");
    *out_config = nullptr;
    auto *c = new (std::nothrow) kq_gdn_config();
    if (c == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate immutable GDN config");
    std::memset(c, 0, sizeof(*c));
    kq_status st = validate_dims(dimensions, c, diagnostic);
    if (st != KQ_STATUS_OK) {
        delete c;
        return st;
    }
    c->magic = kGdnConfigMagic;
    c->dims = *dimensions;
    *out_config = c;
    return KQ_STATUS_OK;
}

kq_status kq_gdn_config_create(const kq_model *, uint32_t, kq_gdn_config **out_config, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_config) *out_config = nullptr;
    return fail(diagnostic, KQ_STATUS_UNSUPPORTED_MODEL,
                "GGUF model configs are not supported by the B200 library; use kq_gdn_test_config_create");
}

kq_status kq_gdn_config_create_reference_f32(const kq_model *m, uint32_t l, kq_gdn_config **o, kq_diagnostic *d) {
    return kq_gdn_config_create(m, l, o, d);
}

void kq_gdn_config_close(kq_gdn_config *config) {
    if (config == nullptr) return;
    config->magic = 0;
    delete config;
}

uint32_t kq_gdn_config_layer_id(const kq_gdn_config *c) { return config_valid(c) ? c->layer_id : UINT32_MAX; }
uint32_t kq_gdn_config_hidden_size(const kq_gdn_config *c) { return config_valid(c) ? c->dims.hidden_size : 0; }
uint32_t kq_gdn_config_key_head_count(const kq_gdn_config *c) { return config_valid(c) ? c->dims.key_head_count : 0; }
uint32_t kq_gdn_config_value_head_count(const kq_gdn_config *c) { return config_valid(c) ? c->dims.value_head_count : 0; }
uint32_t kq_gdn_config_key_head_dimension(const kq_gdn_config *c) { return config_valid(c) ? c->dims.key_head_dimension : 0; }
uint32_t kq_gdn_config_value_head_dimension(const kq_gdn_config *c) { return config_valid(c) ? c->dims.value_head_dimension : 0; }
uint32_t kq_gdn_config_conv_channel_count(const kq_gdn_config *c) { return config_valid(c) ? c->conv_channels : 0; }
uint32_t kq_gdn_config_conv_kernel_size(const kq_gdn_config *c) { return config_valid(c) ? c->dims.conv_kernel_size : 0; }
kq_gdn_activation_dtype kq_gdn_config_activation_dtype(const kq_gdn_config *c) {
    return config_valid(c) ? c->dims.activation_dtype : KQ_GDN_ACTIVATION_F32;
}
uint64_t kq_gdn_config_owned_bytes(const kq_gdn_config *c) { return config_valid(c) ? sizeof(*c) : 0; }
uint64_t kq_gdn_config_recurrent_element_count(const kq_gdn_config *c) { return config_valid(c) ? c->recurrent_elements : 0; }
uint64_t kq_gdn_config_conv_state_element_count(const kq_gdn_config *c) { return config_valid(c) ? c->conv_state_elements : 0; }
uint64_t kq_gdn_config_scratch_bytes(const kq_gdn_config *c) { return config_valid(c) ? c->scratch_bytes : 0; }
uint64_t kq_gdn_config_token_scratch_bytes(const kq_gdn_config *c) { return config_valid(c) ? c->token_scratch_bytes : 0; }
uint64_t kq_gdn_config_dequant_scratch_bytes(const kq_gdn_config *c) { return config_valid(c) ? 256u * sizeof(float) : 0; }

kq_status kq_b200_gdn_config_bind(kq_gdn_config *config, kq_weight_provider *provider,
                                  const kq_b200_gdn_tensors *t, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || provider == nullptr || t == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, provider and tensors are required");
    const uint32_t H = config->dims.hidden_size, Hv = config->dims.value_head_count;
    struct M { const kq_semantic_tensor *s; uint32_t rows, cols; QMatrix *dst; } mats[5] = {
        {t->qkv, config->conv_channels, H, &config->qkv}, {t->gate, config->value_width, H, &config->gate},
        {t->beta, Hv, H, &config->beta}, {t->alpha, Hv, H, &config->alpha},
        {t->output, H, config->value_width, &config->out}};
    struct V { const kq_semantic_tensor *s; uint64_t count; const float **dst; } vecs[4] = {
        {t->a_log, Hv, &config->a_log}, {t->conv, config->conv_state_elements, &config->conv},
        {t->dt_bias, Hv, &config->dt_bias}, {t->norm, config->dims.value_head_dimension, &config->norm}};
    for (auto &m : mats) {
        ProviderTensor *p = provider_lookup(provider, m.s);
        if (p == nullptr || p->is_vector || p->parts[0] != nullptr)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "GDN provider matrix semantic is missing");
        if (p->m.rows != m.rows || p->m.cols != m.cols)
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_GDN, "GDN canonical tensor shape mismatch");
        // only the output projection may keep the model's tiled column
        // order, with one head position per value head of this config
        if (!p->col_heads.empty() &&
            (m.dst != &config->out || p->col_heads.size() != Hv ||
             p->head_width != config->dims.value_head_dimension))
            return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH,
                        "GDN tiled columns must belong to the output projection of this value-head geometry");
    }
    for (auto &v : vecs) {
        ProviderTensor *p = provider_lookup(provider, v.s);
        if (p == nullptr || !p->is_vector)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "GDN provider vector semantic is missing");
        if (p->vec_host.size() != v.count)
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_GDN, "GDN canonical tensor shape mismatch");
    }
    for (auto &m : mats) *m.dst = provider_lookup(provider, m.s)->m;
    for (auto &v : vecs) *v.dst = provider_lookup(provider, v.s)->vec_dev;
    config->gated_head = provider_lookup(provider, t->output)->col_heads_dev;
    config->provider = provider;
    config->bound = true;
    return KQ_STATUS_OK;
}

kq_status kq_gdn_state_create(const kq_gdn_config *config, kq_gdn_state **out_state, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || out_state == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid GDN config and state output are required");
    *out_state = nullptr;
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    auto *s = new (std::nothrow) kq_gdn_state();
    if (s == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate GDN stream state");
    s->device = c->device;
    const size_t cb = config->conv_state_elements * 4, rb = config->recurrent_elements * 4;
    for (int i = 0; i < 2; ++i) {
        if (cudaMalloc(&s->conv[i], cb) != cudaSuccess || cudaMalloc(&s->rec[i], rb) != cudaSuccess ||
            cudaMemsetAsync(s->conv[i], 0, cb, c->stream) != cudaSuccess ||
            cudaMemsetAsync(s->rec[i], 0, rb, c->stream) != cudaSuccess) {
            cudaGetLastError();
            for (int j = 0; j < 2; ++j) { cudaFree(s->conv[j]); cudaFree(s->rec[j]); }
            delete s;
            return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate GDN state arrays");
        }
    }
    s->magic = kGdnStateMagic;
    s->config = config;
    s->owned_bytes = sizeof(*s) + 2 * (cb + rb);
    *out_state = s;
    return KQ_STATUS_OK;
}

void kq_gdn_state_close(kq_gdn_state *state) {
    if (state == nullptr) return;
    DeviceContext *c = context_for(state->device);
    if (c) {
        std::lock_guard<std::recursive_mutex> lk(c->mu);
        cudaStreamSynchronize(c->stream);
        c->dirty.erase(state);
    }
    for (int j = 0; j < 2; ++j) { cudaFree(state->conv[j]); cudaFree(state->rec[j]); }
    state->magic = 0;
    delete state;
}

kq_status kq_gdn_state_reset(kq_gdn_state *state, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state)) return fail(diagnostic, KQ_STATUS_INVALID_GDN_STATE, "valid GDN state is required for reset");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    // on the library stream, so that later work on it sees the zeroed state
    KQB_CUDA(cudaMemsetAsync(state->conv[state->cur], 0, state->config->conv_state_elements * 4, c->stream),
             diagnostic, "reset");
    KQB_CUDA(cudaMemsetAsync(state->rec[state->cur], 0, state->config->recurrent_elements * 4, c->stream),
             diagnostic, "reset");
    state->initialized = 0;
    state->on_success();
    return KQ_STATUS_OK;
}

uint64_t kq_gdn_state_owned_bytes(const kq_gdn_state *s) { return state_valid(s) ? s->owned_bytes : 0; }

static uint16_t f32_to_bf16(float v) {
    uint32_t bits;
    std::memcpy(&bits, &v, 4);
    return (uint16_t)((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16);
}
static float bf16_to_f32(uint16_t h) {
    uint32_t bits = (uint32_t)h << 16;
    float v;
    std::memcpy(&v, &bits, 4);
    return v;
}

kq_status kq_gdn_state_export_f32(const kq_gdn_state *state, float *conv_state, uint64_t conv_capacity,
                                  float *recurrent_state, uint64_t recurrent_capacity, int *initialized,
                                  kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state) || conv_state == nullptr || recurrent_state == nullptr || initialized == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid GDN state and export buffers are required");
    const kq_gdn_config *cfg = state->config;
    if (conv_capacity < cfg->conv_state_elements || recurrent_capacity < cfg->recurrent_elements)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "GDN state export buffer is too small");
    if (ranges_overlap(conv_state, cfg->conv_state_elements * 4, recurrent_state, cfg->recurrent_elements * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "GDN state export buffers overlap");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    KQB_CUDA(copy_sync(conv_state, state->conv[state->cur], cfg->conv_state_elements * 4, cudaMemcpyDefault,
                       c->stream), diagnostic, "conv export");
    KQB_CUDA(copy_sync(recurrent_state, state->rec[state->cur], cfg->recurrent_elements * 4, cudaMemcpyDefault,
                       c->stream), diagnostic, "recurrent export");
    *initialized = state->initialized;
    return KQ_STATUS_OK;
}

kq_status kq_gdn_state_import_f32(kq_gdn_state *state, const float *conv_state, uint64_t conv_count,
                                  const float *recurrent_state, uint64_t recurrent_count, int initialized,
                                  kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state) || conv_state == nullptr || recurrent_state == nullptr ||
        (initialized != 0 && initialized != 1))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid GDN state import arguments are required");
    const kq_gdn_config *cfg = state->config;
    if (conv_count != cfg->conv_state_elements || recurrent_count != cfg->recurrent_elements)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN state import shape mismatch");
    if (initialized == 1 && cfg->dims.activation_dtype == KQ_GDN_ACTIVATION_F32 &&
        is_device_pointer(conv_state) && is_device_pointer(recurrent_state)) {
        // device-resident state: validate and copy on the device
        DeviceContext *c;
        kq_status st = context(&c, diagnostic);
        if (st != KQ_STATUS_OK) return st;
        std::lock_guard<std::recursive_mutex> lk(c->mu);
        c->synchronize(nullptr);
        ErrorWord err = c->begin_call();
        launch_check_finite(conv_state, conv_count, err, c->stream);
        launch_check_finite(recurrent_state, recurrent_count, err, c->stream);
        if (c->synchronize(nullptr) != KQ_STATUS_OK)
            return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "GDN imported state must be finite");
        // ordered on the library stream, and complete before the caller's
        // buffers may be reused
        KQB_CUDA(cudaMemcpyAsync(state->conv[state->cur], conv_state, conv_count * 4, cudaMemcpyDeviceToDevice,
                                 c->stream), diagnostic, "conv import");
        KQB_CUDA(cudaMemcpyAsync(state->rec[state->cur], recurrent_state, recurrent_count * 4,
                                 cudaMemcpyDeviceToDevice, c->stream), diagnostic, "rec import");
        KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "import");
        state->initialized = 1;
        state->on_success();
        return KQ_STATUS_OK;
    }
    std::vector<float> conv_h(conv_count), rec_h(recurrent_count);
    KQB_CUDA(cudaMemcpy(conv_h.data(), conv_state, conv_count * 4, cudaMemcpyDefault), diagnostic, "conv import");
    KQB_CUDA(cudaMemcpy(rec_h.data(), recurrent_state, recurrent_count * 4, cudaMemcpyDefault), diagnostic, "rec import");
    for (float v : conv_h) {
        if (!std::isfinite(v)) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "GDN convolution state must be finite");
        if (!initialized && v != 0.0f)
            return fail(diagnostic, KQ_STATUS_INVALID_GDN_STATE, "uninitialized GDN convolution state must be zero");
    }
    for (float v : rec_h) {
        if (!std::isfinite(v)) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "GDN recurrent state must be finite");
        if (!initialized && v != 0.0f)
            return fail(diagnostic, KQ_STATUS_INVALID_GDN_STATE, "uninitialized GDN recurrent state must be zero");
    }
    if (cfg->dims.activation_dtype == KQ_GDN_ACTIVATION_BF16)
        for (float &v : conv_h) v = bf16_to_f32(f32_to_bf16(v));
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    KQB_CUDA(copy_sync(state->conv[state->cur], conv_h.data(), conv_count * 4, cudaMemcpyHostToDevice, c->stream),
             diagnostic, "conv import");
    KQB_CUDA(copy_sync(state->rec[state->cur], rec_h.data(), recurrent_count * 4, cudaMemcpyHostToDevice,
                       c->stream), diagnostic, "rec import");
    state->initialized = initialized;
    state->on_success();
    return KQ_STATUS_OK;
}

kq_status kq_gdn_prefill_f32(const kq_gdn_config *config, const kq_gdn_weights_f32 *weights,
                             const float *hidden_states, uint64_t sequence_length, const uint8_t *padding_mask,
                             float *output, uint64_t output_capacity, kq_gdn_state *state, void *scratch,
                             uint64_t scratch_bytes, kq_gdn_checkpoint_observer observer, void *observer_user_data,
                             kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    kq_status st = validate_call(config, weights, hidden_states, sequence_length, padding_mask, output,
                                 output_capacity, state, scratch, scratch_bytes, false, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    return gdn_execute_sync(config, nullptr, weights, hidden_states, sequence_length, padding_mask, output,
                            state, observer, observer_user_data, diagnostic);
}

kq_status kq_gdn_decode_f32(const kq_gdn_config *config, const kq_gdn_weights_f32 *weights,
                            const float *hidden_token, float *output_token, uint64_t output_capacity,
                            kq_gdn_state *state, void *scratch, uint64_t scratch_bytes,
                            kq_gdn_checkpoint_observer observer, void *observer_user_data,
                            kq_diagnostic *diagnostic) {
    return kq_gdn_prefill_f32(config, weights, hidden_token, 1, nullptr, output_token, output_capacity, state,
                              scratch, scratch_bytes, observer, observer_user_data, diagnostic);
}

kq_status kq_gdn_execute_quantized(const kq_gdn_config *config, kq_weight_provider *provider,
                                   const float *hidden_states, uint64_t sequence_length,
                                   const uint8_t *padding_mask, float *output, uint64_t output_capacity,
                                   kq_gdn_state *state, void *scratch, uint64_t scratch_bytes,
                                   void *weight_scratch, uint64_t weight_scratch_bytes,
                                   kq_gdn_checkpoint_observer observer, void *observer_user_data,
                                   kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid compatible GDN call arguments are required");
    // provider weight scratch contract of src/kq_gdn_qwen38.c:876-884, sized
    // from this config instead of the target model's constants
    const uint64_t vec = (uint64_t)config->dims.value_head_count * 2 + config->conv_state_elements +
                         config->dims.value_head_dimension;
    const uint64_t need = (vec + config->conv_state_elements) * 4 + 65536;
    if (provider == nullptr || weight_scratch == nullptr || weight_scratch_bytes < need)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "GDN provider weight scratch is too small");
    kq_status st = validate_call(config, nullptr, hidden_states, sequence_length, padding_mask, output,
                                 output_capacity, state, scratch, scratch_bytes, true, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    GdnResolved w;
    if (!resolve_bound(config, &w) || config->provider != provider)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "GDN provider matrix semantic is missing");
    return gdn_execute_sync(config, &w, nullptr, hidden_states, sequence_length, padding_mask, output, state,
                            observer, observer_user_data, diagnostic);
}

kq_status kq_b200_gdn_decode_batch(const kq_gdn_config *config, kq_gdn_state *const *states, uint32_t batch,
                                   const float *hidden, float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || states == nullptr || batch == 0 || hidden == nullptr || output == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, states and device buffers are required");
    if (config->dims.activation_dtype != KQ_GDN_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_GDN, "batched decode requires an F32 configuration");
    GdnResolved w;
    if (!resolve_bound(config, &w))
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    for (uint32_t b = 0; b < batch; ++b) {
        if (!state_valid(states[b]) || states[b]->config != config)
            return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "every state must belong to the config");
        for (uint32_t o = 0; o < b; ++o)
            if (states[o] == states[b]) return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "states must be distinct");
    }
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    ErrorWord err = c->begin_call();
    return gdn_enqueue(c, config, w, states, batch, 1, hidden, nullptr, output, err, diagnostic,
                       /*check_input=*/true);
}

kq_status kq_b200_gdn_prefill_async(const kq_gdn_config *config, kq_gdn_state *state, const float *hidden,
                                    uint64_t T, float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || !state_valid(state) || state->config != config || hidden == nullptr ||
        output == nullptr || T == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, state and device buffers are required");
    if (T > UINT32_MAX || T * config->dims.hidden_size > SIZE_MAX / 4)
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "GDN sequence element count is invalid or overflows");
    if (config->dims.activation_dtype != KQ_GDN_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_GDN, "device prefill requires an F32 configuration");
    if (!is_device_pointer(hidden) || !is_device_pointer(output))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "device prefill takes device buffers");
    GdnResolved w;
    if (!resolve_bound(config, &w))
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    ErrorWord err = c->begin_call();
    kq_gdn_state *states[1] = {state};
    return gdn_enqueue(c, config, w, states, 1, (uint32_t)T, hidden, nullptr, output, err, diagnostic,
                       /*check_input=*/true);
}

const char *kq_gdn_checkpoint_kind_name(kq_gdn_checkpoint_kind kind) {
    static const char *names[] = {"MASKED_INPUT", "PROJECTED_QKV", "PROJECTED_GATE", "PROJECTED_BETA",
                                  "PROJECTED_ALPHA", "CONV_INPUT", "CONV_OUTPUT", "QUERY_BEFORE_NORM",
                                  "KEY_BEFORE_NORM", "VALUE", "NORMALIZED_SCALED_QUERY", "NORMALIZED_KEY",
                                  "LOG_DECAY", "BETA", "RECURRENT_READ", "RECURRENT_DELTA",
                                  "RECURRENT_OUTPUT", "RECURRENT_STATE", "CONV_STATE", "GATED_NORM_OUTPUT",
                                  "OPERATOR_OUTPUT"};
    if ((uint32_t)kind >= sizeof(names) / sizeof(names[0])) return "UNKNOWN";
    return names[(uint32_t)kind];
}

}  // extern "C"

// ---------------------------------------------------------------- layer bridge

namespace kqb {

kq_status gdn_layer_enqueue(DeviceContext *c, const kq_gdn_config *cfg, const kq_gdn_weights_f32 *wf,
                            kq_gdn_state *const *states, uint32_t batch, uint32_t tokens, const float *x,
                            const uint8_t *mask, float *y, ErrorWord err, kq_diagnostic *diag) {
    if (!config_valid(cfg) || states == nullptr || batch == 0 || tokens == 0 || (batch > 1 && tokens > 1))
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid compatible GDN call arguments are required");
    if (cfg->dims.activation_dtype != KQ_GDN_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_GDN, "F32 scalar execution requires an F32 reference configuration");
    for (uint32_t b = 0; b < batch; ++b)
        if (!state_valid(states[b]) || states[b]->config != cfg)
            return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "every state must belong to the config");
    GdnResolved w;
    if (wf != nullptr) {
        const uint64_t Hv = cfg->dims.value_head_count, H = cfg->dims.hidden_size;
        const uint64_t want[9] = {Hv, (uint64_t)cfg->conv_channels * cfg->dims.conv_kernel_size, Hv, Hv * H, Hv * H,
                                  (uint64_t)cfg->conv_channels * H, (uint64_t)cfg->value_width * H,
                                  cfg->dims.value_head_dimension, H * cfg->value_width};
        const float *ptrs[9] = {wf->a_log, wf->conv, wf->dt_bias, wf->alpha, wf->beta, wf->qkv, wf->gate, wf->norm,
                                wf->output};
        const uint64_t have[9] = {wf->a_log_count, wf->conv_count, wf->dt_bias_count, wf->alpha_count,
                                  wf->beta_count, wf->qkv_count, wf->gate_count, wf->norm_count, wf->output_count};
        for (int i = 0; i < 9; ++i) {
            if (have[i] != want[i]) return fail(diag, KQ_STATUS_DIMENSION_MISMATCH, "GDN F32 weight count mismatch");
            if (ptrs[i] == nullptr) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "GDN F32 weights must be finite");
        }
        kq_status st = resolve_f32(c, cfg, wf, err, &w, diag);
        if (st != KQ_STATUS_OK) return st;
    } else if (!resolve_bound(cfg, &w)) {
        return fail(diag, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "GDN provider matrix semantic is missing");
    }
    return gdn_enqueue(c, cfg, w, states, batch, tokens, x, mask, y, err, diag);
}

GdnSnapshot gdn_state_snapshot(const kq_gdn_state *s) { return GdnSnapshot{s->cur, s->initialized}; }

void gdn_state_restore(kq_gdn_state *s, const GdnSnapshot &snap) {
    s->cur = snap.cur;
    s->initialized = snap.initialized;
    s->on_success();
}

}  // namespace kqb
