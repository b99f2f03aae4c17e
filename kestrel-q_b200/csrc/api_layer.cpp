// kq_layer ABI on the B200: one decoder layer (gated residual, GDN or QSA
// mixer, gated residual, MoE) as one device call.
//
// Replaces src/kq_layer.c and src/kq_layer_qwen38.c of Kestrel-Q for the
// GDN and QSA families.  Argument checks and status codes follow
// kq_layer_execute (src/kq_layer.c:639-680), kq_layer_test_config_create
// (:220-262), kq_layer_state_create (:337-410) and the scratch formula of
// kq_layer_required_scratch_bytes (:529-566).  The sub-operators run through
// operators.hpp under the layer's single call id, so the device error word
// of any stage rolls every sub-state of the call back together.
#include <algorithm>
#include <cfenv>
#include <chrono>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "kq_b200.h"
#include "kq_layer.h"
#include "operators.hpp"
#include "provider.hpp"
#include "runtime.hpp"

using namespace kqb;

namespace {
constexpr uint32_t kLayerConfigMagic = 0x4b514c43u;
constexpr uint32_t kLayerStateMagic = 0x4b514c53u;
constexpr uint32_t kLayerSlice = 2048;                  // tokens per device pass without an observer
constexpr uint64_t kQuantizedWeightScratch = 1048576;   // src/kq_layer.c:24
}  // namespace

struct kq_layer_config {
    uint32_t magic;
    kq_layer_dimensions dims;
    kq_gdn_config *gdn;
    kq_qsa_config *qsa;
    kq_moe_config *moe;
    uint64_t gr_workspace_bytes;
    kq_weight_provider *provider;
    GrWeightsDev attn, mgr;   // bound provider tensors
    bool bound;
};

// The layer's own position follows its sub-state through the context's
// roll-back bookkeeping (advanced at enqueue time, restored when a call of
// the layer fails on the device).
struct kq_layer_state final : Rollbackable {
    uint32_t magic = 0;
    const kq_layer_config *config = nullptr;
    kq_gdn_state *gdn = nullptr;
    kq_qsa_state *qsa = nullptr;
    uint64_t qsa_capacity = 0;
    uint64_t position = 0;
    uint64_t owned_bytes = 0;
    // the state before the last committed synchronous call, for
    // kq_layer_state_rollback_last (one mixer pass only: a GDN state keeps
    // just the buffer that its last pass replaced)
    bool can_roll_back = false;
    uint64_t last_tokens = 0;
    GdnSnapshot gdn_before{0, 0};
    uint64_t qsa_before = 0;
    uint64_t synced_position = 0;
    std::vector<std::pair<uint32_t, uint64_t>> history;

    // called after `position` has advanced for call `id`
    void on_step(uint32_t id) override { history.push_back({id, position}); }
    void on_error(uint32_t failing) override {
        uint64_t pos = synced_position;
        for (auto &h : history)
            if (failing != 0 && h.first < failing) pos = h.second;
        position = pos;
        can_roll_back = false;
        on_success();
    }
    void on_success() override {
        synced_position = position;
        history.clear();
    }
};

static bool config_valid(const kq_layer_config *c) {
    return c != nullptr && c->magic == kLayerConfigMagic && c->moe != nullptr &&
           ((c->dims.family == KQ_LAYER_FAMILY_GDN && c->gdn != nullptr && c->qsa == nullptr) ||
            (c->dims.family == KQ_LAYER_FAMILY_QSA && c->qsa != nullptr && c->gdn == nullptr));
}

static bool state_valid(const kq_layer_state *s) {
    return s != nullptr && s->magic == kLayerStateMagic && config_valid(s->config) &&
           (s->gdn != nullptr || s->qsa != nullptr);
}

static GrDims gr_dims(const kq_layer_config *c) {
    return GrDims{c->dims.hidden_size, c->dims.branch_count, c->dims.gr_rank, c->dims.rms_epsilon};
}

static QMatrix dense(const float *p, uint32_t rows, uint32_t cols) {
    QMatrix m{};
    m.data = reinterpret_cast<const uint8_t *>(p);
    m.type = 0;
    m.rows = rows;
    m.cols = cols;
    m.row_bytes = cols * 4;
    m.layout = 0;
    return m;
}

// Gated-residual F32 arrays (host: through the upload cache; device: in
// place) with the shape checks of kq_layer_gr_validate
// (src/kq_layer_qwen38.c:9-35).
static kq_status gr_from_f32(DeviceContext *c, const kq_layer_config *cfg, const kq_layer_gr_weights_f32 &w,
                             GrWeightsDev *out, kq_diagnostic *diag) {
    const uint64_t W = (uint64_t)cfg->dims.hidden_size * cfg->dims.branch_count, R = cfg->dims.gr_rank,
                   B = cfg->dims.branch_count;
    if (w.norm == nullptr || w.down == nullptr || w.up == nullptr || w.inject == nullptr || w.norm_count != W ||
        w.down_count != R * W || w.up_count != W * R || w.inject_count != B * W)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_LAYER, "GR weights do not match branch/rank geometry");
    const float *src[4] = {w.norm, w.down, w.up, w.inject};
    const uint64_t cnt[4] = {W, R * W, W * R, B * W};
    const float *dev[4];
    for (int i = 0; i < 4; ++i) {
        if (is_device_pointer(src[i])) {
            dev[i] = src[i];
        } else {
            kq_status st = c->upload_cached(src[i], cnt[i], &dev[i], diag);
            if (st != KQ_STATUS_OK) return st;
        }
    }
    out->norm = dev[0];
    out->down = dense(dev[1], (uint32_t)R, (uint32_t)W);
    out->up = dense(dev[2], (uint32_t)W, (uint32_t)R);
    out->inject = dense(dev[3], (uint32_t)B, (uint32_t)W);
    return KQ_STATUS_OK;
}

namespace {

// Weights of one layer call: F32 arrays (kq_layer_*_f32) or the provider
// tensors bound to the config and its sub-configs.
struct LayerWeights {
    GrWeightsDev attn, mgr;
    const kq_gdn_weights_f32 *gdn = nullptr;
    const kq_qsa_weights_f32 *qsa = nullptr;
    const kq_moe_weights_f32 *moe = nullptr;
};

// Device buffers of one pass over n items (tokens of one sequence, or one
// token of each of n sequences).  With an observer both gated residuals
// keep their normalised branches and read gates.
struct LayerBufs {
    float *mixed, *awg, *block, *after, *moe_in, *mwg, *moe_out;
    GrBuffers gr_attn, gr_moe;
};

size_t layer_bytes(const kq_layer_config *cfg, uint32_t n, bool observed) {
    const uint64_t H = cfg->dims.hidden_size, B = cfg->dims.branch_count, W = H * B;
    const size_t gr = gr_workspace_bytes(gr_dims(cfg), n);
    return Carve::round(n * H * 4) * 4 + Carve::round(n * B * 4) * 2 + Carve::round(n * W * 4) +
           gr * (observed ? 2 : 1) + 256;
}

void layer_carve(const kq_layer_config *cfg, uint32_t n, bool observed, Carve &cv, LayerBufs &b) {
    const uint64_t H = cfg->dims.hidden_size, B = cfg->dims.branch_count, W = H * B;
    b.mixed = cv.take<float>(n * H);
    b.awg = cv.take<float>(n * B);
    b.block = cv.take<float>(n * H);
    b.after = cv.take<float>(n * W);
    b.moe_in = cv.take<float>(n * H);
    b.mwg = cv.take<float>(n * B);
    b.moe_out = cv.take<float>(n * H);
    const size_t gr = gr_workspace_bytes(gr_dims(cfg), n);
    gr_carve(gr_dims(cfg), n, cv.take<char>(gr), b.gr_attn);
    if (observed)
        gr_carve(gr_dims(cfg), n, cv.take<char>(gr), b.gr_moe);
    else
        b.gr_moe = b.gr_attn;
}

}  // namespace

// One pass of the layer over n items: x [n][B][H] -> y [n][B][H].  The
// mixer runs `batch` states x `tokens` tokens (n = batch * tokens).
static kq_status layer_pass(DeviceContext *c, const kq_layer_config *cfg, const LayerWeights &w,
                            kq_layer_state *const *states, uint32_t batch, uint32_t tokens, const float *x,
                            const uint8_t *mask, float *y, LayerBufs &b, ErrorWord err, kq_diagnostic *diag) {
    const GrDims gd = gr_dims(cfg);
    const uint32_t n = batch * tokens;
    launch_gr_read(gd, w.attn, x, n, b.mixed, b.awg, b.gr_attn, err, c->stream);
    kq_status st;
    if (cfg->gdn != nullptr) {
        std::vector<kq_gdn_state *> ss(batch);
        for (uint32_t i = 0; i < batch; ++i) ss[i] = states[i]->gdn;
        st = gdn_layer_enqueue(c, cfg->gdn, w.gdn, ss.data(), batch, tokens, b.mixed, mask, b.block, err, diag);
    } else {
        std::vector<kq_qsa_state *> ss(batch);
        for (uint32_t i = 0; i < batch; ++i) ss[i] = states[i]->qsa;
        st = qsa_layer_enqueue(c, cfg->qsa, w.qsa, ss.data(), batch, tokens, b.mixed, b.block, err, diag);
    }
    if (st != KQ_STATUS_OK) return st;
    launch_gr_write(gd, x, b.block, b.awg, n, b.after, err, c->stream);
    launch_gr_read(gd, w.mgr, b.after, n, b.moe_in, b.mwg, b.gr_moe, err, c->stream);
    st = moe_layer_enqueue(c, cfg->moe, w.moe, b.moe_in, n, b.moe_out, err, diag);
    if (st != KQ_STATUS_OK) return st;
    launch_gr_write(gd, b.after, b.moe_out, b.mwg, n, y, err, c->stream);
    KQB_CUDA(cudaGetLastError(), diag, "layer launch");
    return KQ_STATUS_OK;
}

// Copies one pass's values to the host and hands every checkpoint to the
// observer in the reference's order (src/kq_layer.c:683-814).
static kq_status emit_checkpoints(const kq_layer_config *cfg, uint32_t n, const float *x, const float *y,
                                  const LayerBufs &b, kq_layer_checkpoint_observer obs, void *user,
                                  kq_diagnostic *diag) {
    const uint64_t H = cfg->dims.hidden_size, B = cfg->dims.branch_count, W = H * B;
    auto get = [&](const float *src, uint64_t count, std::vector<float> &dst) -> kq_status {
        dst.resize(count);
        KQB_CUDA(cudaMemcpy(dst.data(), src, count * 4, cudaMemcpyDeviceToHost), diag, "checkpoint copy");
        return KQ_STATUS_OK;
    };
    std::vector<float> hx, hy, nm1, rg1, mixed, awg, block, after, nm2, rg2, moe_in, mwg, moe_out;
    struct F { const float *src; uint64_t count; std::vector<float> *dst; } fs[] = {
        {x, n * W, &hx}, {y, n * W, &hy}, {b.gr_attn.normalized, n * W, &nm1}, {b.gr_attn.read, n * W, &rg1},
        {b.mixed, n * H, &mixed}, {b.awg, n * B, &awg}, {b.block, n * H, &block}, {b.after, n * W, &after},
        {b.gr_moe.normalized, n * W, &nm2}, {b.gr_moe.read, n * W, &rg2}, {b.moe_in, n * H, &moe_in},
        {b.mwg, n * B, &mwg}, {b.moe_out, n * H, &moe_out}};
    for (const F &f : fs) {
        kq_status st = get(f.src, f.count, *f.dst);
        if (st != KQ_STATUS_OK) return st;
    }
    auto emit = [&](kq_layer_checkpoint_kind kind, uint64_t t, uint32_t rank, uint64_t d0, uint64_t d1,
                    const float *v, uint64_t count) {
        kq_layer_checkpoint cp;
        std::memset(&cp, 0, sizeof(cp));
        cp.kind = kind;
        cp.token_index = t;
        cp.rank = rank;
        cp.dimensions[0] = d0;
        cp.dimensions[1] = d1;
        cp.values = v;
        cp.value_count = count;
        obs(&cp, user);
    };
    for (uint64_t t = 0; t < n; ++t) emit(KQ_LAYER_CHECKPOINT_INPUT, t, 2, B, H, hx.data() + t * W, W);
    for (uint64_t t = 0; t < n; ++t) {
        emit(KQ_LAYER_CHECKPOINT_ATTN_GR_NORMALIZED, t, 2, B, H, nm1.data() + t * W, W);
        emit(KQ_LAYER_CHECKPOINT_ATTN_GR_READ_GATE, t, 2, B, H, rg1.data() + t * W, W);
        emit(KQ_LAYER_CHECKPOINT_MIXER_INPUT, t, 1, H, 0, mixed.data() + t * H, H);
    }
    for (uint64_t t = 0; t < n; ++t) {
        emit(KQ_LAYER_CHECKPOINT_MIXER_OUTPUT, t, 1, H, 0, block.data() + t * H, H);
        emit(KQ_LAYER_CHECKPOINT_ATTN_GR_WRITE_GATE, t, 1, B, 0, awg.data() + t * B, B);
        emit(KQ_LAYER_CHECKPOINT_AFTER_MIXER_RESIDUAL, t, 2, B, H, after.data() + t * W, W);
        emit(KQ_LAYER_CHECKPOINT_MOE_GR_NORMALIZED, t, 2, B, H, nm2.data() + t * W, W);
        emit(KQ_LAYER_CHECKPOINT_MOE_GR_READ_GATE, t, 2, B, H, rg2.data() + t * W, W);
        emit(KQ_LAYER_CHECKPOINT_MOE_INPUT, t, 1, H, 0, moe_in.data() + t * H, H);
    }
    for (uint64_t t = 0; t < n; ++t) {
        emit(KQ_LAYER_CHECKPOINT_MOE_OUTPUT, t, 1, H, 0, moe_out.data() + t * H, H);
        emit(KQ_LAYER_CHECKPOINT_MOE_GR_WRITE_GATE, t, 1, B, 0, mwg.data() + t * B, B);
        emit(KQ_LAYER_CHECKPOINT_OUTPUT, t, 2, B, H, hy.data() + t * W, W);
    }
    return KQ_STATUS_OK;
}

// Enqueues T tokens of one state (slices of kLayerSlice tokens, one slice
// with an observer) or one token of each of `batch` states, under one call;
// `y` is device.  Registers the states for roll-back.
static uint32_t pass_items(uint32_t batch, uint64_t T, bool observed) {
    if (batch > 1) return batch;
    return observed ? (uint32_t)T : (uint32_t)std::min<uint64_t>(T, kLayerSlice);
}

// The buffers come from `cv`, which the caller sized with
// layer_bytes(cfg, pass_items(...), observed) (the context's staging arena:
// the sub-operators use the separate work-space arena).
static kq_status layer_enqueue(DeviceContext *c, const kq_layer_config *cfg, const LayerWeights &w,
                               kq_layer_state *const *states, uint32_t batch, uint64_t T, const float *x,
                               const uint8_t *mask, float *y, ErrorWord err, bool observed, Carve &cv,
                               LayerBufs *kept, uint32_t *passes, kq_diagnostic *diag) {
    const uint64_t W = (uint64_t)cfg->dims.hidden_size * cfg->dims.branch_count;
    const uint32_t items = pass_items(batch, T, observed);
    const uint32_t slice = batch > 1 ? 1u : items;
    LayerBufs b;
    layer_carve(cfg, items, observed, cv, b);
    kq_status st;
    *passes = 0;
    for (uint64_t t0 = 0; t0 < T; t0 += slice) {
        const uint32_t n = (uint32_t)std::min<uint64_t>(slice, T - t0);
        st = layer_pass(c, cfg, w, states, batch, n, x + t0 * W, mask ? mask + t0 : nullptr, y + t0 * W, b, err,
                        diag);
        if (st != KQ_STATUS_OK) return st;
        ++*passes;
    }
    for (uint32_t i = 0; i < batch; ++i) {
        states[i]->position += T;
        states[i]->can_roll_back = false;
        states[i]->on_step(err.call_id);
        c->dirty.insert(states[i]);
    }
    if (kept) *kept = b;
    return KQ_STATUS_OK;
}

static kq_status required_scratch(const kq_layer_config *config, const kq_layer_state *state, uint64_t T,
                                  uint64_t *out, kq_diagnostic *diag);

// kq_layer_execute (src/kq_layer.c:639-827) for the GDN and QSA families:
// F32 weights (wf) or provider mode (provider), host or device buffers.
static kq_status layer_execute(const kq_layer_config *config, const kq_layer_weights_f32 *wf,
                               kq_weight_provider *provider, const float *input, uint64_t count, const uint8_t *mask,
                               float *output, uint64_t output_capacity, kq_layer_state *state, void *scratch,
                               uint64_t scratch_bytes, bool decode, kq_layer_checkpoint_observer obs, void *user,
                               kq_layer_metrics *metrics, kq_diagnostic *diag) {
    const auto t_start = std::chrono::steady_clock::now();
    if (!config_valid(config) || ((wf == nullptr) == (provider == nullptr)) || input == nullptr ||
        output == nullptr || !state_valid(state) || state->config != config || scratch == nullptr || count == 0 ||
        (decode && count != 1) || output == input || (void *)output == scratch || (const void *)input == scratch)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid compatible layer call arguments are required");
    const uint64_t H = config->dims.hidden_size, W = H * config->dims.branch_count;
    uint64_t total;
    if (!mul_ok(count, W, &total) || count > UINT32_MAX)
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer token/value count overflows");
    if (output_capacity < total) return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "layer output capacity is too small");
    uint64_t need;
    kq_status st = required_scratch(config, state, count, &need, diag);
    if (st != KQ_STATUS_OK) return st;
    if (provider != nullptr && !add_ok(need, kQuantizedWeightScratch, &need))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer scratch byte count overflows");
    if (scratch_bytes < need) return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "layer scratch is too small");
    if (wf != nullptr &&
        (wf->moe == nullptr || (config->gdn != nullptr && wf->gdn == nullptr) ||
         (config->qsa != nullptr && wf->qsa == nullptr)))
        return fail(diag, KQ_STATUS_INCOMPATIBLE_LAYER, "layer sub-operator weights are required");
    if (provider != nullptr && (!config->bound || config->provider != provider))
        return fail(diag, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "layer gated-residual tensors are not bound");
    const bool m_host = mask != nullptr && !is_device_pointer(mask);
    if (m_host)
        for (uint64_t i = 0; i < count; ++i)
            if (mask[i] > 1) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "padding mask must contain only zero or one");
    DeviceContext *c;
    st = context(&c, diag);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diag);   // settle earlier asynchronous work first
    if (st != KQ_STATUS_OK) return st;
    const bool x_host = !is_device_pointer(input);
    const bool observed = obs != nullptr;
    const uint32_t items = pass_items(1, count, observed);
    void *stage;
    st = c->staging(Carve::round(total * 4) * (x_host ? 2 : 1) + (m_host ? Carve::round(count) : 0) +
                        layer_bytes(config, items, observed),
                    &stage, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(stage);
    float *dy = cv.take<float>(total);
    const float *dx = input;
    if (x_host) {
        float *t = cv.take<float>(total);
        KQB_CUDA(cudaMemcpyAsync(t, input, total * 4, cudaMemcpyHostToDevice, c->stream), diag, "input copy");
        dx = t;
    }
    const uint8_t *dmask = mask;
    if (m_host) {
        uint8_t *t = cv.take<uint8_t>(count);
        KQB_CUDA(cudaMemcpyAsync(t, mask, count, cudaMemcpyHostToDevice, c->stream), diag, "mask copy");
        dmask = t;
    }
    ErrorWord err = c->begin_call();
    launch_check_finite(dx, total, err, c->stream);
    LayerWeights w;
    if (wf != nullptr) {
        st = gr_from_f32(c, config, wf->attention_gr, &w.attn, diag);
        if (st == KQ_STATUS_OK) st = gr_from_f32(c, config, wf->moe_gr, &w.mgr, diag);
        if (st != KQ_STATUS_OK) return st;
        w.gdn = wf->gdn;
        w.qsa = wf->qsa;
        w.moe = wf->moe;
    } else {
        w.attn = config->attn;
        w.mgr = config->mgr;
    }
    const GdnSnapshot gdn_before = state->gdn ? gdn_state_snapshot(state->gdn) : GdnSnapshot{0, 0};
    const uint64_t qsa_before = state->qsa ? qsa_state_committed_length(state->qsa) : 0;
    LayerBufs kept;
    uint32_t passes = 0;
    kq_layer_state *states[1] = {state};
    st = layer_enqueue(c, config, w, states, 1, count, dx, dmask, dy, err, observed, cv, &kept, &passes, diag);
    if (st != KQ_STATUS_OK) {
        c->synchronize(nullptr);
        return st;
    }
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output, dy, total * 4, is_device_pointer(output) ? cudaMemcpyDeviceToDevice
                                                                        : cudaMemcpyDeviceToHost),
             diag, "output copy");
    state->can_roll_back = passes == 1;
    state->last_tokens = count;
    state->gdn_before = gdn_before;
    state->qsa_before = qsa_before;
    if (observed) {
        st = emit_checkpoints(config, (uint32_t)count, dx, dy, kept, obs, user, diag);
        if (st != KQ_STATUS_OK) return st;
    }
    if (metrics != nullptr) {
        std::memset(metrics, 0, sizeof(*metrics));
        metrics->tokens_processed = count;
        metrics->scratch_bytes = need;
        metrics->gr_workspace_bytes = config->gr_workspace_bytes;
        metrics->transaction_staging_bytes = state->owned_bytes;
        metrics->qsa_selection_events = config->qsa != nullptr ? count : 0;
        metrics->elapsed_nanoseconds = (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
                                           std::chrono::steady_clock::now() - t_start)
                                           .count();
    }
    return KQ_STATUS_OK;
}

// src/kq_layer.c:529-566: the layer's own buffers plus the largest
// sub-operator scratch.
static kq_status required_scratch(const kq_layer_config *config, const kq_layer_state *state, uint64_t T,
                                  uint64_t *out, kq_diagnostic *diag) {
    if (!config_valid(config) || !state_valid(state) || state->config != config || T == 0 || out == nullptr)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid layer config, state and token count are required");
    const uint64_t H = config->dims.hidden_size, B = config->dims.branch_count, W = H * B;
    uint64_t floats, base, sub = 0, qsa = 0;
    if (!mul_ok(T, W * 3 + H * 4 + B * 2, &floats) || !add_ok(floats, W * 2 + config->dims.gr_rank, &floats) ||
        !mul_ok(floats, 4, &base))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer scratch byte count overflows");
    if (config->gdn != nullptr) sub = std::max<uint64_t>(sub, kq_gdn_config_scratch_bytes(config->gdn));
    if (config->qsa != nullptr) {
        kq_status st = kq_qsa_required_scratch_bytes(config->qsa, state->qsa, T, &qsa, diag);
        if (st != KQ_STATUS_OK) return st;
        sub = std::max(sub, qsa);
    }
    sub = std::max<uint64_t>(sub, kq_moe_config_scratch_bytes(config->moe));
    if (!add_ok(base, sub, out)) return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer scratch byte count overflows");
    return KQ_STATUS_OK;
}

extern "C" {

kq_status kq_layer_config_create(const kq_model *, uint32_t, kq_layer_config **out_config,
                                 kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_config) *out_config = nullptr;
    return fail(diagnostic, KQ_STATUS_UNSUPPORTED_MODEL,
                "GGUF model configs are not supported by the B200 library; use kq_layer_test_config_create");
}

kq_status kq_layer_config_create_reference_f32(const kq_model *model, uint32_t layer_id,
                                               kq_layer_config **out_config, kq_diagnostic *diagnostic) {
    return kq_layer_config_create(model, layer_id, out_config, diagnostic);
}

kq_status kq_layer_test_config_create(const kq_layer_dimensions *d, kq_gdn_config *gdn, kq_qsa_config *qsa,
                                      kq_moe_config *moe, kq_ple_config *ple, kq_ple_value_config *ple_value,
                                      kq_layer_config **out_config, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    // src/kq_layer.c:220-262
    if (d == nullptr || out_config == nullptr || moe == nullptr || d->hidden_size == 0 || d->branch_count == 0 ||
        d->gr_rank == 0 || !std::isfinite(d->rms_epsilon) || d->rms_epsilon <= 0.0f)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid layer dimensions and an MoE config are required");
    *out_config = nullptr;
    if (d->family == KQ_LAYER_FAMILY_PLE_GDN || ple != nullptr || ple_value != nullptr)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_LAYER,
                    "the PLE_GDN family needs the PLE operators, which the B200 library does not provide");
    auto *c = new (std::nothrow) kq_layer_config();
    if (c == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate layer config");
    std::memset(c, 0, sizeof(*c));
    c->magic = kLayerConfigMagic;
    c->dims = *d;
    c->gdn = gdn;
    c->qsa = qsa;
    c->moe = moe;
    c->gr_workspace_bytes = ((uint64_t)d->branch_count * d->hidden_size * 2 + d->hidden_size + d->gr_rank +
                             d->branch_count) * 4;
    if (!config_valid(c) || kq_moe_config_hidden_size(moe) != d->hidden_size ||
        (gdn != nullptr && kq_gdn_config_hidden_size(gdn) != d->hidden_size) ||
        (qsa != nullptr && kq_qsa_config_hidden_size(qsa) != d->hidden_size)) {
        delete c;
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_LAYER, "test layer subconfigs have incompatible geometry");
    }
    *out_config = c;
    return KQ_STATUS_OK;
}

void kq_layer_config_close(kq_layer_config *config) {
    if (config == nullptr || config->magic != kLayerConfigMagic) return;
    config->magic = 0;
    delete config;
}

uint32_t kq_layer_config_layer_id(const kq_layer_config *c) { return config_valid(c) ? c->dims.layer_id : UINT32_MAX; }
kq_layer_family kq_layer_config_family(const kq_layer_config *c) {
    return config_valid(c) ? c->dims.family : KQ_LAYER_FAMILY_INVALID;
}
uint32_t kq_layer_config_hidden_size(const kq_layer_config *c) { return config_valid(c) ? c->dims.hidden_size : 0; }
uint32_t kq_layer_config_branch_count(const kq_layer_config *c) { return config_valid(c) ? c->dims.branch_count : 0; }
uint32_t kq_layer_config_gr_rank(const kq_layer_config *c) { return config_valid(c) ? c->dims.gr_rank : 0; }
uint64_t kq_layer_config_owned_bytes(const kq_layer_config *c) {
    if (!config_valid(c)) return 0;
    return sizeof(*c) + kq_gdn_config_owned_bytes(c->gdn) + kq_qsa_config_owned_bytes(c->qsa) +
           kq_moe_config_owned_bytes(c->moe);
}
uint64_t kq_layer_config_gr_workspace_bytes(const kq_layer_config *c) {
    return config_valid(c) ? c->gr_workspace_bytes : 0;
}
uint64_t kq_layer_config_persistent_semantic_bytes(const kq_layer_config *c, uint64_t qsa_capacity) {
    if (!config_valid(c)) return 0;
    if (c->gdn != nullptr)   // F32 recurrent state and BF16 convolution history (src/kq_layer.c:306-318)
        return kq_gdn_config_recurrent_element_count(c->gdn) * 4 + kq_gdn_config_conv_state_element_count(c->gdn) * 2;
    uint64_t b;
    return mul_ok(kq_qsa_config_semantic_state_bytes_per_token(c->qsa), qsa_capacity, &b) ? b : 0;
}

kq_status kq_layer_state_create(const kq_layer_config *config, uint64_t qsa_capacity, kq_layer_state **out_state,
                                kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || out_state == nullptr || (config->qsa != nullptr && qsa_capacity == 0))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid layer config and QSA capacity are required");
    *out_state = nullptr;
    auto *s = new (std::nothrow) kq_layer_state();
    if (s == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate layer state");
    kq_status st = config->gdn != nullptr ? kq_gdn_state_create(config->gdn, &s->gdn, diagnostic)
                                          : kq_qsa_state_create(config->qsa, qsa_capacity, &s->qsa, diagnostic);
    if (st != KQ_STATUS_OK) {
        delete s;
        return st;
    }
    s->magic = kLayerStateMagic;
    s->config = config;
    s->qsa_capacity = qsa_capacity;
    s->owned_bytes = sizeof(*s) + (s->gdn ? kq_gdn_state_owned_bytes(s->gdn) : kq_qsa_state_owned_bytes(s->qsa));
    *out_state = s;
    return KQ_STATUS_OK;
}

void kq_layer_state_close(kq_layer_state *state) {
    if (state == nullptr || state->magic != kLayerStateMagic) return;
    if (DeviceContext *c = context_for(current_device())) {
        std::lock_guard<std::recursive_mutex> lk(c->mu);
        c->synchronize(nullptr);
        c->dirty.erase(state);
    }
    kq_gdn_state_close(state->gdn);
    kq_qsa_state_close(state->qsa);
    state->magic = 0;
    delete state;
}

kq_status kq_layer_state_reset(kq_layer_state *state, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state)) return fail(diagnostic, KQ_STATUS_INVALID_LAYER_STATE, "valid layer state is required");
    kq_status st = state->gdn ? kq_gdn_state_reset(state->gdn, diagnostic) : kq_qsa_state_reset(state->qsa, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    state->position = 0;
    state->can_roll_back = false;
    state->on_success();
    return KQ_STATUS_OK;
}

uint64_t kq_layer_state_owned_bytes(const kq_layer_state *s) { return state_valid(s) ? s->owned_bytes : 0; }
uint64_t kq_layer_state_position(const kq_layer_state *s) { return state_valid(s) ? s->position : 0; }

kq_status kq_layer_state_rollback_last(kq_layer_state *state, uint64_t token_count, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state))
        return fail(diagnostic, KQ_STATUS_INVALID_LAYER_STATE, "layer rollback has no matching commit");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (!state->can_roll_back || token_count == 0 || token_count != state->last_tokens ||
        state->position < token_count)
        return fail(diagnostic, KQ_STATUS_INVALID_LAYER_STATE, "layer rollback has no matching commit");
    if (state->gdn)
        gdn_state_restore(state->gdn, state->gdn_before);
    else
        qsa_state_truncate(state->qsa, state->qsa_before);
    state->position -= token_count;
    state->can_roll_back = false;
    state->on_success();
    return KQ_STATUS_OK;
}

kq_status kq_layer_required_scratch_bytes(const kq_layer_config *config, const kq_layer_state *state,
                                          uint64_t token_count, uint64_t *scratch_bytes, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    return required_scratch(config, state, token_count, scratch_bytes, diagnostic);
}

kq_status kq_layer_required_quantized_scratch_bytes(const kq_layer_config *config, const kq_layer_state *state,
                                                    uint64_t token_count, uint64_t *scratch_bytes,
                                                    kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (scratch_bytes == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "output is required");
    uint64_t base;
    kq_status st = required_scratch(config, state, token_count, &base, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (!add_ok(base, kQuantizedWeightScratch, scratch_bytes))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer scratch byte count overflows");
    return KQ_STATUS_OK;
}

kq_status kq_layer_prefill_f32(const kq_layer_config *c, const kq_layer_weights_f32 *w, const float *h,
                               const uint32_t *, uint64_t n, const uint8_t *mask, float *o, uint64_t cap,
                               kq_layer_state *s, void *scratch, uint64_t scratch_bytes,
                               kq_layer_checkpoint_observer observer, void *user, kq_layer_metrics *metrics,
                               kq_diagnostic *d) {
    kq_diagnostic_clear(d);
    if (w == nullptr) return fail(d, KQ_STATUS_INVALID_ARGUMENT, "valid compatible layer call arguments are required");
    return layer_execute(c, w, nullptr, h, n, mask, o, cap, s, scratch, scratch_bytes, false, observer, user, metrics,
                         d);
}

kq_status kq_layer_decode_f32(const kq_layer_config *c, const kq_layer_weights_f32 *w, const float *h, uint32_t,
                              float *o, uint64_t cap, kq_layer_state *s, void *scratch, uint64_t scratch_bytes,
                              kq_layer_checkpoint_observer observer, void *user, kq_layer_metrics *metrics,
                              kq_diagnostic *d) {
    kq_diagnostic_clear(d);
    if (w == nullptr) return fail(d, KQ_STATUS_INVALID_ARGUMENT, "valid compatible layer call arguments are required");
    return layer_execute(c, w, nullptr, h, 1, nullptr, o, cap, s, scratch, scratch_bytes, true, observer, user,
                         metrics, d);
}

kq_status kq_layer_prefill_quantized_f32(const kq_layer_config *c, kq_weight_provider *p, const float *h,
                                         const uint32_t *, uint64_t n, const uint8_t *mask, float *o, uint64_t cap,
                                         kq_layer_state *s, void *scratch, uint64_t scratch_bytes,
                                         kq_layer_checkpoint_observer observer, void *user,
                                         kq_layer_metrics *metrics, kq_diagnostic *d) {
    kq_diagnostic_clear(d);
    if (p == nullptr) return fail(d, KQ_STATUS_INVALID_ARGUMENT, "valid compatible layer call arguments are required");
    return layer_execute(c, nullptr, p, h, n, mask, o, cap, s, scratch, scratch_bytes, false, observer, user, metrics,
                         d);
}

kq_status kq_layer_decode_quantized_f32(const kq_layer_config *c, kq_weight_provider *p, const float *h, uint32_t,
                                        float *o, uint64_t cap, kq_layer_state *s, void *scratch,
                                        uint64_t scratch_bytes, kq_layer_checkpoint_observer observer, void *user,
                                        kq_layer_metrics *metrics, kq_diagnostic *d) {
    kq_diagnostic_clear(d);
    if (p == nullptr) return fail(d, KQ_STATUS_INVALID_ARGUMENT, "valid compatible layer call arguments are required");
    return layer_execute(c, nullptr, p, h, 1, nullptr, o, cap, s, scratch, scratch_bytes, true, observer, user,
                         metrics, d);
}

kq_status kq_b200_layer_config_bind(kq_layer_config *config, kq_weight_provider *provider,
                                    const kq_b200_layer_tensors *t, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || provider == nullptr || t == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, provider and tensors are required");
    const uint32_t H = config->dims.hidden_size, B = config->dims.branch_count, R = config->dims.gr_rank, W = H * B;
    struct Side {
        const kq_semantic_tensor *inject, *norm, *down, *up;
        GrWeightsDev *dst;
    } sides[2] = {{t->attention_inject, t->attention_norm, t->attention_down, t->attention_up, &config->attn},
                  {t->moe_inject, t->moe_norm, t->moe_down, t->moe_up, &config->mgr}};
    GrWeightsDev got[2];
    for (int i = 0; i < 2; ++i) {
        const Side &sd = sides[i];
        ProviderTensor *inj = provider_lookup(provider, sd.inject), *nm = provider_lookup(provider, sd.norm),
                       *dn = provider_lookup(provider, sd.down), *up = provider_lookup(provider, sd.up);
        if (inj == nullptr || nm == nullptr || dn == nullptr || up == nullptr || !nm->is_vector || inj->is_vector ||
            dn->is_vector || up->is_vector || inj->parts[0] || dn->parts[0] || up->parts[0] || inj->experts ||
            dn->experts || up->experts)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "required gated-residual tensor is missing");
        if (nm->vec_host.size() != W || inj->m.rows != B || inj->m.cols != W || dn->m.rows != R || dn->m.cols != W ||
            up->m.rows != W || up->m.cols != R)
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_LAYER, "GR weights do not match branch/rank geometry");
        got[i].norm = nm->vec_dev;
        got[i].inject = inj->m;
        got[i].down = dn->m;
        got[i].up = up->m;
    }
    config->attn = got[0];
    config->mgr = got[1];
    config->provider = provider;
    config->bound = true;
    return KQ_STATUS_OK;
}

// Device-buffer entry points: checks, then the layer under one call.
static kq_status layer_async(const kq_layer_config *config, kq_layer_state *const *states, uint32_t batch, uint64_t T,
                             const float *branches, float *output, kq_diagnostic *diagnostic) {
    if (!config_valid(config) || states == nullptr || batch == 0 || T == 0 || branches == nullptr ||
        output == nullptr || (batch > 1 && T > 1))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, states and device buffers are required");
    if (!config->bound)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    if (!is_device_pointer(branches) || !is_device_pointer(output))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "the layer's batched entry points take device buffers");
    const uint64_t W = (uint64_t)config->dims.hidden_size * config->dims.branch_count, n = batch * T;
    if (T > UINT32_MAX || n * W > SIZE_MAX / 4)
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "layer token/value count overflows");
    if (ranges_overlap(branches, n * W * 4, output, n * W * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "layer input and output must not overlap");
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
    void *stage;
    st = c->staging(layer_bytes(config, pass_items(batch, T, false), false), &stage, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(stage);
    ErrorWord err = c->begin_call();
    launch_check_finite(branches, n * W, err, c->stream);
    LayerWeights w;
    w.attn = config->attn;
    w.mgr = config->mgr;
    uint32_t passes = 0;
    return layer_enqueue(c, config, w, states, batch, T, branches, nullptr, output, err, false, cv, nullptr, &passes,
                         diagnostic);
}

kq_status kq_b200_layer_decode_batch(const kq_layer_config *config, kq_layer_state *const *states, uint32_t batch,
                                     const float *branches, float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    return layer_async(config, states, batch, 1, branches, output, diagnostic);
}

kq_status kq_b200_layer_prefill_async(const kq_layer_config *config, kq_layer_state *state, const float *branches,
                                      uint64_t T, float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    kq_layer_state *states[1] = {state};
    return layer_async(config, states, 1, T, branches, output, diagnostic);
}

const char *kq_layer_family_name(kq_layer_family f) {
    switch (f) {
    case KQ_LAYER_FAMILY_GDN: return "GDN";
    case KQ_LAYER_FAMILY_QSA: return "QSA";
    case KQ_LAYER_FAMILY_PLE_GDN: return "PLE_GDN";
    default: return "INVALID";
    }
}

const char *kq_layer_checkpoint_kind_name(kq_layer_checkpoint_kind k) {
    static const char *const names[] = {"INPUT", "PLE_OUTPUT", "PLE_ENHANCED_INPUT", "ATTN_GR_NORMALIZED",
                                        "ATTN_GR_READ_GATE", "MIXER_INPUT", "MIXER_OUTPUT", "ATTN_GR_WRITE_GATE",
                                        "AFTER_MIXER_RESIDUAL", "MOE_GR_NORMALIZED", "MOE_GR_READ_GATE",
                                        "MOE_INPUT", "MOE_OUTPUT", "MOE_GR_WRITE_GATE", "OUTPUT"};
    return (unsigned)k < sizeof(names) / sizeof(names[0]) ? names[k] : "UNKNOWN";
}

}  // extern "C"
