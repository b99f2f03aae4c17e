// kq_moe ABI on the B200: configs, provider binding and execution.
//
// Replaces src/kq_moe.c and the entry points of src/kq_moe_qwen38.c of
// Kestrel-Q.  Validation order and status codes follow
// kq_moe_execute_common (src/kq_moe_qwen38.c:604-660), kq_moe_route_f32
// (:276-376) and kq_moe_execute_routed_expert_f32 (:461-568); workspace
// sizes follow kq_moe_workspace_sizes (src/kq_moe.c:83-140) so that the
// caller-visible scratch contract is the reference's.  The device work runs
// in kernels_moe.cu.
#include <algorithm>
#include <cfenv>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "kq_b200.h"
#include "kq_moe.h"
#include "operators.hpp"
#include "provider.hpp"
#include "runtime.hpp"

using namespace kqb;

namespace {
constexpr uint32_t kMoeConfigMagic = 0x4b514d43u;
constexpr uint32_t kMoeChunk = 2048;   // tokens per device pass (bounds the expert work space)
}  // namespace

struct kq_moe_config {
    uint32_t magic;
    uint32_t layer_id;
    kq_moe_dimensions dims;
    uint64_t router_ws, top_k_ws, expert_ws, acc_ws, shared_ws, scratch_bytes;
    kq_weight_provider *provider;
    MoeWeightsDev w;
    bool bound;
};

static bool config_valid(const kq_moe_config *c) { return c != nullptr && c->magic == kMoeConfigMagic; }

static MoeDims dims_of(const kq_moe_config *c) {
    const kq_moe_dimensions &d = c->dims;
    return MoeDims{d.hidden_size, d.expert_count, d.top_k, d.routed_intermediate_size, d.shared_intermediate_size};
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

// Host or device F32 array -> device pointer (host arrays through the
// context's upload cache), checked for non-finite values on the device.
static kq_status device_weights(DeviceContext *c, const float *p, uint64_t count, ErrorWord err, const float **out,
                                kq_diagnostic *diag) {
    if (is_device_pointer(p)) {
        *out = p;
    } else {
        kq_status st = c->upload_cached(p, count, out, diag);
        if (st != KQ_STATUS_OK) return st;
    }
    launch_check_finite(*out, count, err, c->stream);
    return KQ_STATUS_OK;
}

static bool host_finite(const float *p, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        if (!std::isfinite(p[i])) return false;
    return true;
}

// Input and output of a synchronous call: device arrays in place, host
// arrays through the context's staging buffer.
struct SyncIo {
    const float *x = nullptr;
    float *y = nullptr;
};

static kq_status stage_io(DeviceContext *c, const float *hidden, uint64_t in_count, uint64_t out_count, SyncIo *io,
                          kq_diagnostic *diag) {
    void *stage;
    kq_status st = c->staging(Carve::round(in_count * 4) + Carve::round(out_count * 4), &stage, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(stage);
    if (is_device_pointer(hidden)) {
        io->x = hidden;
        cv.take<float>(in_count);
    } else {
        float *x = cv.take<float>(in_count);
        KQB_CUDA(cudaMemcpyAsync(x, hidden, in_count * 4, cudaMemcpyHostToDevice, c->stream), diag, "input copy");
        io->x = x;
    }
    io->y = cv.take<float>(out_count);
    return KQ_STATUS_OK;
}

// ------------------------------------------------------------ observers

namespace {

struct HostChunk {
    std::vector<float> logits, probs, sel_w, gate, up, act, eout, weighted, routed_sum, gated, scale, sgu, sact, sout,
        y;
    std::vector<uint32_t> sel_ids, slot;
};

template <typename T>
kq_status fetch(std::vector<T> &dst, const T *src, size_t n, kq_diagnostic *diag) {
    dst.resize(n);
    if (n == 0 || src == nullptr) return KQ_STATUS_OK;
    KQB_CUDA(cudaMemcpy(dst.data(), src, n * sizeof(T), cudaMemcpyDeviceToHost), diag, "checkpoint copy");
    return KQ_STATUS_OK;
}

// Copies one finished chunk's values to the host and hands them to the
// observers in the reference's order (src/kq_moe_qwen38.c:671-867).
kq_status emit_chunk(const MoeDims &d, uint64_t first_token, uint32_t T, const MoeBuffers &b, const float *y,
                     kq_moe_route_observer route_observer, kq_moe_checkpoint_observer observer, void *user,
                     kq_diagnostic *diag) {
    const size_t E = d.experts, K = d.top_k, I = d.routed, S = d.shared, H = d.hidden, picks = (size_t)T * K;
    HostChunk h;
    kq_status st;
#define KQB_FETCH(dst, src, n)                         \
    if ((st = fetch(dst, src, n, diag)) != KQ_STATUS_OK) return st
    KQB_FETCH(h.logits, b.logits, (size_t)T * (E + 1));
    KQB_FETCH(h.probs, b.probs, (size_t)T * E);
    KQB_FETCH(h.sel_ids, b.sel_ids, picks);
    KQB_FETCH(h.sel_w, b.sel_w, picks);
    if (observer != nullptr) {
        KQB_FETCH(h.slot, b.slot, picks);
        KQB_FETCH(h.gate, b.dbg.gate, picks * I);
        KQB_FETCH(h.up, b.dbg.up, picks * I);
        KQB_FETCH(h.act, b.act, picks * I);
        KQB_FETCH(h.eout, b.eout, picks * H);
        KQB_FETCH(h.weighted, b.dbg.weighted, picks * H);
        KQB_FETCH(h.routed_sum, b.dbg.routed_sum, (size_t)T * H);
        KQB_FETCH(h.gated, b.dbg.gated_shared, (size_t)T * H);
        KQB_FETCH(h.scale, b.dbg.scale, (size_t)T * 2);
        KQB_FETCH(h.sgu, b.shared_gu, (size_t)T * 2 * S);
        KQB_FETCH(h.sact, b.shared_act, (size_t)T * S);
        KQB_FETCH(h.sout, b.shared_out, (size_t)T * H);
        KQB_FETCH(h.y, y, (size_t)T * H);
    }
#undef KQB_FETCH
    std::vector<float> logits(E);
    for (uint32_t t = 0; t < T; ++t) {
        const uint64_t tok = first_token + t;
        std::memcpy(logits.data(), h.logits.data() + (size_t)t * (E + 1), E * 4);
        const float *probs = h.probs.data() + (size_t)t * E;
        const uint32_t *ids = h.sel_ids.data() + (size_t)t * K;
        const float *w = h.sel_w.data() + (size_t)t * K;
        if (route_observer != nullptr) {
            kq_moe_route r{};
            r.token_index = tok;
            r.router_logits = logits.data();
            r.router_probabilities = probs;
            r.expert_count = E;
            r.selected_expert_ids = ids;
            r.selected_weights = w;
            r.selected_count = (uint32_t)K;
            route_observer(&r, user);
        }
        if (observer == nullptr) continue;
        auto emit = [&](kq_moe_checkpoint_kind kind, uint32_t expert, uint32_t pos, const float *v, uint64_t n) {
            kq_moe_checkpoint cp;
            std::memset(&cp, 0, sizeof(cp));
            cp.kind = kind;
            cp.token_index = tok;
            cp.expert_id = expert;
            cp.top_k_position = pos;
            cp.rank = 1;
            cp.dimensions[0] = n;
            cp.values = v;
            cp.value_count = n;
            observer(&cp, user);
        };
        emit(KQ_MOE_CHECKPOINT_ROUTER_LOGITS, KQ_MOE_NO_EXPERT, UINT32_MAX, logits.data(), E);
        emit(KQ_MOE_CHECKPOINT_ROUTER_PROBABILITIES, KQ_MOE_NO_EXPERT, UINT32_MAX, probs, E);
        emit(KQ_MOE_CHECKPOINT_SELECTED_WEIGHTS, KQ_MOE_NO_EXPERT, UINT32_MAX, w, K);
        // the selected experts in ascending id (src/kq_moe_qwen38.c:695-760)
        std::vector<uint32_t> order(K);
        for (uint32_t p = 0; p < K; ++p) order[p] = p;
        std::sort(order.begin(), order.end(), [&](uint32_t a, uint32_t c) { return ids[a] < ids[c]; });
        for (uint32_t p : order) {
            const size_t sl = h.slot[(size_t)t * K + p];
            emit(KQ_MOE_CHECKPOINT_ROUTED_GATE, ids[p], p, h.gate.data() + sl * I, I);
            emit(KQ_MOE_CHECKPOINT_ROUTED_UP, ids[p], p, h.up.data() + sl * I, I);
            emit(KQ_MOE_CHECKPOINT_ROUTED_ACTIVATED, ids[p], p, h.act.data() + sl * I, I);
            emit(KQ_MOE_CHECKPOINT_ROUTED_EXPERT_OUTPUT, ids[p], p, h.eout.data() + sl * H, H);
            emit(KQ_MOE_CHECKPOINT_ROUTED_WEIGHTED_OUTPUT, ids[p], p, h.weighted.data() + sl * H, H);
        }
        emit(KQ_MOE_CHECKPOINT_ROUTED_WEIGHTED_SUM, KQ_MOE_NO_EXPERT, UINT32_MAX, h.routed_sum.data() + t * H, H);
        emit(KQ_MOE_CHECKPOINT_SHARED_GATE_PROJECTION, KQ_MOE_NO_EXPERT, UINT32_MAX, h.sgu.data() + t * 2 * S, S);
        emit(KQ_MOE_CHECKPOINT_SHARED_UP_PROJECTION, KQ_MOE_NO_EXPERT, UINT32_MAX, h.sgu.data() + t * 2 * S + S, S);
        emit(KQ_MOE_CHECKPOINT_SHARED_ACTIVATED, KQ_MOE_NO_EXPERT, UINT32_MAX, h.sact.data() + t * S, S);
        emit(KQ_MOE_CHECKPOINT_SHARED_OUTPUT, KQ_MOE_NO_EXPERT, UINT32_MAX, h.sout.data() + t * H, H);
        emit(KQ_MOE_CHECKPOINT_SHARED_SCALE_LOGIT, KQ_MOE_NO_EXPERT, UINT32_MAX, h.scale.data() + 2 * t, 1);
        emit(KQ_MOE_CHECKPOINT_SHARED_SCALE, KQ_MOE_NO_EXPERT, UINT32_MAX, h.scale.data() + 2 * t + 1, 1);
        emit(KQ_MOE_CHECKPOINT_GATED_SHARED_OUTPUT, KQ_MOE_NO_EXPERT, UINT32_MAX, h.gated.data() + t * H, H);
        emit(KQ_MOE_CHECKPOINT_OPERATOR_OUTPUT, KQ_MOE_NO_EXPERT, UINT32_MAX, h.y.data() + t * H, H);
    }
    return KQ_STATUS_OK;
}

}  // namespace

// Runs T tokens x -> y (device arrays) in chunks of kMoeChunk; with
// observers every chunk is synchronised and reported before the next runs.
static kq_status moe_run(DeviceContext *c, const kq_moe_config *cfg, const MoeWeightsDev &w, const float *x,
                         uint64_t T, float *y, ErrorWord err, kq_moe_route_observer route_observer,
                         kq_moe_checkpoint_observer observer, void *user, kq_diagnostic *diag) {
    const MoeDims d = dims_of(cfg);
    const bool observed = route_observer != nullptr || observer != nullptr;
    const uint32_t chunk = (uint32_t)std::min<uint64_t>(T, kMoeChunk);
    void *ws;
    kq_status st = c->workspace(moe_workspace_bytes(d, chunk, observer != nullptr), &ws, diag);
    if (st != KQ_STATUS_OK) return st;
    for (uint64_t t0 = 0; t0 < T; t0 += chunk) {
        const uint32_t n = (uint32_t)std::min<uint64_t>(chunk, T - t0);
        MoeBuffers b;
        moe_carve(d, n, observer != nullptr, ws, b);
        launch_moe(d, w, x + t0 * d.hidden, n, y + t0 * d.hidden, b, err, c->stream);
        KQB_CUDA(cudaGetLastError(), diag, "MoE launch");
        if (observed) {
            st = c->synchronize(diag);
            if (st != KQ_STATUS_OK) return st;
            st = emit_chunk(d, t0, n, b, y + t0 * d.hidden, route_observer, observer, user, diag);
            if (st != KQ_STATUS_OK) return st;
        }
    }
    return KQ_STATUS_OK;
}

// kq_moe_execute_common's checks (src/kq_moe_qwen38.c:619-660) up to the
// weights, which the caller checks.
static kq_status validate_call(const kq_moe_config *config, bool have_weights, const float *hidden, uint64_t T,
                               float *output, uint64_t output_capacity, void *scratch, uint64_t scratch_bytes,
                               kq_diagnostic *diag) {
    if (!config_valid(config) || !have_weights || hidden == nullptr || output == nullptr || scratch == nullptr)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "complete MoE execution arguments are required");
    const kq_moe_dimensions &d = config->dims;
    if (d.activation_dtype != KQ_MOE_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_MOE, "scalar execution requires an F32 MoE config");
    uint64_t n;
    if (T == 0 || !mul_ok(T, d.hidden_size, &n) || n > (UINT64_MAX / 4))
        return fail(diag, KQ_STATUS_LIMIT_EXCEEDED, "MoE token/value count is zero or overflows");
    if (output_capacity < n || scratch_bytes < config->scratch_bytes ||
        (reinterpret_cast<uintptr_t>(scratch) % alignof(float)) != 0)
        return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "MoE output or aligned scratch is too small");
    if (!is_device_pointer(hidden) && !host_finite(hidden, n))
        return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "MoE input must be finite");
    return KQ_STATUS_OK;
}

static kq_status check_overlaps(const float *hidden, float *output, uint64_t n, void *scratch, uint64_t scratch_bytes,
                                kq_diagnostic *diag) {
    if (ranges_overlap(hidden, n * 4, output, n * 4) || ranges_overlap(hidden, n * 4, scratch, scratch_bytes) ||
        ranges_overlap(output, n * 4, scratch, scratch_bytes))
        return fail(diag, KQ_STATUS_ALIASING_VIOLATION, "MoE input, output, and scratch must not overlap");
    return KQ_STATUS_OK;
}

static kq_status execute_sync(const kq_moe_config *config, const MoeWeightsDev *bound, const kq_moe_weights_f32 *wf,
                              const float *hidden, uint64_t T, float *output, kq_moe_route_observer route_observer,
                              kq_moe_checkpoint_observer observer, void *user, kq_diagnostic *diag) {
    if (std::fegetround() != FE_TONEAREST)
        return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "MoE scalar reference requires round-to-nearest");
    const kq_moe_dimensions &d = config->dims;
    const uint64_t n = T * d.hidden_size;
    DeviceContext *c;
    kq_status st = context(&c, diag);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diag);   // settle earlier asynchronous work first
    if (st != KQ_STATUS_OK) return st;
    SyncIo io;
    st = stage_io(c, hidden, n, n, &io, diag);
    if (st != KQ_STATUS_OK) return st;
    ErrorWord err = c->begin_call();
    launch_check_finite(io.x, n, err, c->stream);
    MoeWeightsDev w;
    if (bound) {
        w = *bound;
    } else {
        const uint32_t E = d.expert_count, H = d.hidden_size, I = d.routed_intermediate_size,
                       S = d.shared_intermediate_size;
        const float *p[8];
        const float *src[8] = {wf->router, wf->routed_gate, wf->routed_up, wf->routed_down,
                               wf->shared_gate, wf->shared_up, wf->shared_down, wf->shared_gate_weight};
        const uint64_t cnt[8] = {wf->router_count, wf->routed_gate_count, wf->routed_up_count,
                                 wf->routed_down_count, wf->shared_gate_count, wf->shared_up_count,
                                 wf->shared_down_count, wf->shared_gate_weight_count};
        for (int i = 0; i < 8; ++i) {
            st = device_weights(c, src[i], cnt[i], err, &p[i], diag);
            if (st != KQ_STATUS_OK) return st;
        }
        w.router = dense(p[0], E, H);
        w.gate = dense(p[1], E * I, H);
        w.up = dense(p[2], E * I, H);
        w.down = dense(p[3], E * H, I);
        w.shared_gate = dense(p[4], S, H);
        w.shared_up = dense(p[5], S, H);
        w.shared_down = dense(p[6], H, S);
        w.shared_gate_weight = dense(p[7], 1, H);
    }
    st = moe_run(c, config, w, io.x, T, io.y, err, route_observer, observer, user, diag);
    if (st != KQ_STATUS_OK) {
        c->synchronize(nullptr);
        return st;
    }
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output, io.y, n * 4, is_device_pointer(output) ? cudaMemcpyDeviceToDevice
                                                                         : cudaMemcpyDeviceToHost),
             diag, "output copy");
    return KQ_STATUS_OK;
}

extern "C" {

kq_status kq_moe_config_create(const kq_model *, uint32_t, kq_moe_config **out_config, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_config) *out_config = nullptr;
    return fail(diagnostic, KQ_STATUS_UNSUPPORTED_MODEL,
                "GGUF model configs are not supported by the B200 library; use kq_moe_test_config_create");
}

kq_status kq_moe_config_create_reference_f32(const kq_model *model, uint32_t layer_id, kq_moe_config **out_config,
                                             kq_diagnostic *diagnostic) {
    return kq_moe_config_create(model, layer_id, out_config, diagnostic);
}

kq_status kq_moe_test_config_create(const kq_moe_dimensions *d, kq_moe_config **out_config,
                                    kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (d == nullptr || out_config == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "test MoE dimensions are required");
    *out_config = nullptr;
    // src/kq_moe.c:83-140
    if (d->hidden_size == 0 || d->expert_count == 0 || d->top_k == 0 || d->top_k > d->expert_count ||
        d->routed_intermediate_size == 0 || d->shared_intermediate_size == 0 ||
        (d->activation_dtype != KQ_MOE_ACTIVATION_F32 && d->activation_dtype != KQ_MOE_ACTIVATION_BF16))
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "invalid MoE dimensions, top-k, or dtype");
    if (d->top_k > kMoeMaxTopK || d->expert_count > kMoeMaxExperts)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "the B200 MoE supports top_k <= 32 and 8192 experts");
    uint64_t router, top, expert, acc, shared, f, total = 0;
    const uint64_t H = d->hidden_size;
    if (!mul_ok(d->expert_count, 8, &router) || !mul_ok(d->top_k, 8, &top) ||
        !mul_ok(d->routed_intermediate_size, 3, &f) || !add_ok(f, H * 2, &f) || !mul_ok(f, 4, &expert) ||
        !mul_ok(H, 4, &acc) || !mul_ok(d->shared_intermediate_size, 3, &f) || !add_ok(f, H * 2, &f) ||
        !mul_ok(f, 4, &shared) || !add_ok(total, router, &total) || !add_ok(total, top, &total) ||
        !add_ok(total, expert, &total) || !add_ok(total, acc, &total) || !add_ok(total, shared, &total))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "MoE total workspace overflows");
    auto *c = new (std::nothrow) kq_moe_config();
    if (c == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate immutable MoE config");
    c->magic = kMoeConfigMagic;
    c->layer_id = KQ_MODEL_NO_LAYER;
    c->dims = *d;
    c->router_ws = router;
    c->top_k_ws = top;
    c->expert_ws = expert;
    c->acc_ws = acc;
    c->shared_ws = shared;
    c->scratch_bytes = total;
    *out_config = c;
    return KQ_STATUS_OK;
}

void kq_moe_config_close(kq_moe_config *config) {
    if (!config_valid(config)) return;
    config->magic = 0;
    delete config;
}

uint32_t kq_moe_config_layer_id(const kq_moe_config *c) { return config_valid(c) ? c->layer_id : UINT32_MAX; }
uint32_t kq_moe_config_hidden_size(const kq_moe_config *c) { return config_valid(c) ? c->dims.hidden_size : 0; }
uint32_t kq_moe_config_expert_count(const kq_moe_config *c) { return config_valid(c) ? c->dims.expert_count : 0; }
uint32_t kq_moe_config_top_k(const kq_moe_config *c) { return config_valid(c) ? c->dims.top_k : 0; }
uint32_t kq_moe_config_routed_intermediate_size(const kq_moe_config *c) {
    return config_valid(c) ? c->dims.routed_intermediate_size : 0;
}
uint32_t kq_moe_config_shared_intermediate_size(const kq_moe_config *c) {
    return config_valid(c) ? c->dims.shared_intermediate_size : 0;
}
kq_moe_activation_dtype kq_moe_config_activation_dtype(const kq_moe_config *c) {
    return config_valid(c) ? c->dims.activation_dtype : KQ_MOE_ACTIVATION_F32;
}
uint64_t kq_moe_config_owned_bytes(const kq_moe_config *c) { return config_valid(c) ? sizeof(*c) : 0; }
uint64_t kq_moe_config_router_workspace_bytes(const kq_moe_config *c) { return config_valid(c) ? c->router_ws : 0; }
uint64_t kq_moe_config_top_k_workspace_bytes(const kq_moe_config *c) { return config_valid(c) ? c->top_k_ws : 0; }
uint64_t kq_moe_config_one_expert_workspace_bytes(const kq_moe_config *c) {
    return config_valid(c) ? c->expert_ws : 0;
}
uint64_t kq_moe_config_routed_accumulation_workspace_bytes(const kq_moe_config *c) {
    return config_valid(c) ? c->acc_ws : 0;
}
uint64_t kq_moe_config_shared_workspace_bytes(const kq_moe_config *c) { return config_valid(c) ? c->shared_ws : 0; }
uint64_t kq_moe_config_scratch_bytes(const kq_moe_config *c) { return config_valid(c) ? c->scratch_bytes : 0; }

kq_status kq_moe_route_f32(const kq_moe_config *config, const float *router_weight, uint64_t router_weight_count,
                           const float *hidden_token, float *router_logits, uint64_t router_logits_capacity,
                           float *router_probabilities, uint64_t router_probabilities_capacity,
                           uint32_t *selected_expert_ids, uint64_t selected_ids_capacity, float *selected_weights,
                           uint64_t selected_weights_capacity, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || router_weight == nullptr || hidden_token == nullptr || router_logits == nullptr ||
        router_probabilities == nullptr || selected_expert_ids == nullptr || selected_weights == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "complete MoE route arguments are required");
    const kq_moe_dimensions &d = config->dims;
    if (d.activation_dtype != KQ_MOE_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "scalar routing requires an F32 MoE reference config");
    const uint64_t E = d.expert_count, H = d.hidden_size, K = d.top_k;
    if (router_weight_count != E * H)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "MoE router weight shape mismatch");
    if (router_logits_capacity < E || router_probabilities_capacity < E || selected_ids_capacity < K ||
        selected_weights_capacity < K)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "MoE route output capacity is too small");
    struct R { const void *p; uint64_t n; } r[6] = {{router_weight, E * H * 4}, {hidden_token, H * 4},
                                                    {router_logits, E * 4}, {router_probabilities, E * 4},
                                                    {selected_expert_ids, K * 4}, {selected_weights, K * 4}};
    for (int i = 0; i < 6; ++i)
        for (int j = i + 1; j < 6; ++j)
            if (ranges_overlap(r[i].p, r[i].n, r[j].p, r[j].n))
                return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "MoE route inputs and outputs must not overlap");
    if ((!is_device_pointer(router_weight) && !host_finite(router_weight, E * H)) ||
        (!is_device_pointer(hidden_token) && !host_finite(hidden_token, H)))
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "MoE router weights and input must be finite");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    SyncIo io;
    st = stage_io(c, hidden_token, H, 1, &io, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    ErrorWord err = c->begin_call();
    launch_check_finite(io.x, H, err, c->stream);
    const float *wr;
    st = device_weights(c, router_weight, E * H, err, &wr, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    const MoeDims md = dims_of(config);
    void *ws;
    st = c->workspace(moe_workspace_bytes(md, 1, false), &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    MoeBuffers b;
    moe_carve(md, 1, false, ws, b);
    ProjSegments seg{};
    seg.count = 1;
    seg.m[0] = dense(wr, (uint32_t)E, (uint32_t)H);
    launch_projection_exact(seg, io.x, (uint32_t)H, b.logits, (uint32_t)E, 1, err, c->stream);
    launch_moe_route(md, b.logits, (uint32_t)E, 1, b, err, c->stream);
    KQB_CUDA(cudaGetLastError(), diagnostic, "MoE route launch");
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(router_logits, b.logits, E * 4, cudaMemcpyDefault), diagnostic, "route copy");
    KQB_CUDA(cudaMemcpy(router_probabilities, b.probs, E * 4, cudaMemcpyDefault), diagnostic, "route copy");
    KQB_CUDA(cudaMemcpy(selected_expert_ids, b.sel_ids, K * 4, cudaMemcpyDefault), diagnostic, "route copy");
    KQB_CUDA(cudaMemcpy(selected_weights, b.sel_w, K * 4, cudaMemcpyDefault), diagnostic, "route copy");
    return KQ_STATUS_OK;
}

kq_status kq_moe_execute_routed_expert_f32(const kq_moe_config *config,
                                           const kq_moe_routed_expert_weights_f32 *weights, uint32_t expert_id,
                                           const float *hidden_token, float *output_token, uint64_t output_capacity,
                                           void *scratch, uint64_t scratch_bytes, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || weights == nullptr || hidden_token == nullptr || output_token == nullptr ||
        scratch == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "complete routed-expert arguments are required");
    const kq_moe_dimensions &d = config->dims;
    if (d.activation_dtype != KQ_MOE_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "scalar expert execution requires F32 config");
    if (expert_id >= d.expert_count)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "routed expert ID is out of range");
    if (output_capacity < d.hidden_size || scratch_bytes < config->expert_ws ||
        (reinterpret_cast<uintptr_t>(scratch) % alignof(float)) != 0)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "routed expert output or scratch is too small");
    const uint64_t H = d.hidden_size, I = d.routed_intermediate_size, member = I * H;
    if (weights->gate == nullptr || weights->gate_count != member)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "MoE routed member gate shape/data mismatch");
    if (weights->up == nullptr || weights->up_count != member)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "MoE routed member up shape/data mismatch");
    if (weights->down == nullptr || weights->down_count != member)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "MoE routed member down shape/data mismatch");
    if (!is_device_pointer(hidden_token) && !host_finite(hidden_token, H))
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "MoE expert input must be finite");
    if (ranges_overlap(hidden_token, H * 4, output_token, H * 4) ||
        ranges_overlap(hidden_token, H * 4, scratch, scratch_bytes) ||
        ranges_overlap(output_token, H * 4, scratch, scratch_bytes))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "routed expert buffers must not overlap");
    const float *wp[3] = {weights->gate, weights->up, weights->down};
    for (const float *p : wp)
        if (ranges_overlap(p, member * 4, output_token, H * 4) || ranges_overlap(p, member * 4, scratch, scratch_bytes))
            return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION,
                        "MoE weights must not overlap writable expert buffers");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    SyncIo io;
    st = stage_io(c, hidden_token, H, H, &io, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    ErrorWord err = c->begin_call();
    launch_check_finite(io.x, H, err, c->stream);
    const float *dev[3];
    for (int i = 0; i < 3; ++i) {
        st = device_weights(c, wp[i], member, err, &dev[i], diagnostic);
        if (st != KQ_STATUS_OK) return st;
    }
    // one expert, one token: the grouped kernels over a one-expert stack
    const MoeDims md{(uint32_t)H, 1, 1, (uint32_t)I, d.shared_intermediate_size};
    MoeWeightsDev w{};
    w.gate = dense(dev[0], (uint32_t)I, (uint32_t)H);
    w.up = dense(dev[1], (uint32_t)I, (uint32_t)H);
    w.down = dense(dev[2], (uint32_t)H, (uint32_t)I);
    void *ws;
    st = c->workspace(moe_workspace_bytes(md, 1, false), &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    MoeBuffers b;
    moe_carve(md, 1, false, ws, b);
    static const uint32_t offsets[2] = {0, 1}, active[2] = {1, 0}, pick[1] = {0};
    KQB_CUDA(cudaMemcpyAsync(b.offsets, offsets, sizeof offsets, cudaMemcpyHostToDevice, c->stream), diagnostic,
             "dispatch copy");
    KQB_CUDA(cudaMemcpyAsync(b.active, active, sizeof active, cudaMemcpyHostToDevice, c->stream), diagnostic,
             "dispatch copy");
    KQB_CUDA(cudaMemcpyAsync(b.pick_of_slot, pick, sizeof pick, cudaMemcpyHostToDevice, c->stream), diagnostic,
             "dispatch copy");
    launch_moe_experts(md, w, io.x, (uint32_t)H, 1, b, err, c->stream);
    launch_check_finite(b.eout, H, err, c->stream);
    KQB_CUDA(cudaGetLastError(), diagnostic, "MoE expert launch");
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output_token, b.eout, H * 4, cudaMemcpyDefault), diagnostic, "expert output copy");
    return KQ_STATUS_OK;
}

kq_status kq_moe_execute_f32(const kq_moe_config *config, const kq_moe_weights_f32 *weights,
                             const float *hidden_states, uint64_t token_count, float *output, uint64_t output_capacity,
                             void *scratch, uint64_t scratch_bytes, kq_moe_route_observer route_observer,
                             kq_moe_checkpoint_observer checkpoint_observer, void *observer_user_data,
                             kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    kq_status st = validate_call(config, weights != nullptr, hidden_states, token_count, output, output_capacity,
                                 scratch, scratch_bytes, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    // src/kq_moe_qwen38.c:82-126: shapes, then the overlap rules
    const kq_moe_dimensions &d = config->dims;
    const uint64_t E = d.expert_count, H = d.hidden_size, I = d.routed_intermediate_size,
                   S = d.shared_intermediate_size;
    struct Wt { const float *p; uint64_t count, want; const char *msg; } wt[8] = {
        {weights->router, weights->router_count, E * H, "MoE router shape/data mismatch"},
        {weights->routed_gate, weights->routed_gate_count, E * I * H, "MoE routed gate shape/data mismatch"},
        {weights->routed_up, weights->routed_up_count, E * I * H, "MoE routed up shape/data mismatch"},
        {weights->routed_down, weights->routed_down_count, E * I * H, "MoE routed down shape/data mismatch"},
        {weights->shared_gate, weights->shared_gate_count, S * H, "MoE shared gate shape/data mismatch"},
        {weights->shared_up, weights->shared_up_count, S * H, "MoE shared up shape/data mismatch"},
        {weights->shared_down, weights->shared_down_count, S * H, "MoE shared down shape/data mismatch"},
        {weights->shared_gate_weight, weights->shared_gate_weight_count, H,
         "MoE shared scale gate shape/data mismatch"}};
    for (const Wt &w : wt) {
        if (w.count != w.want) return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, w.msg);
        if (w.p == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, w.msg);
    }
    const uint64_t n = token_count * H;
    st = check_overlaps(hidden_states, output, n, scratch, scratch_bytes, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    for (const Wt &w : wt)
        if (ranges_overlap(w.p, w.count * 4, output, n * 4) || ranges_overlap(w.p, w.count * 4, scratch, scratch_bytes))
            return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION,
                        "MoE weights must not overlap writable execution buffers");
    return execute_sync(config, nullptr, weights, hidden_states, token_count, output, route_observer,
                        checkpoint_observer, observer_user_data, diagnostic);
}

kq_status kq_moe_execute_quantized(const kq_moe_config *config, kq_weight_provider *provider,
                                   const float *hidden_states, uint64_t token_count, float *output,
                                   uint64_t output_capacity, void *scratch, uint64_t scratch_bytes,
                                   void *weight_scratch, uint64_t weight_scratch_bytes,
                                   kq_moe_route_observer route_observer, kq_moe_checkpoint_observer checkpoint_observer,
                                   void *observer_user_data, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    // src/kq_moe_qwen38.c:882-899
    if (provider == nullptr || weight_scratch == nullptr || weight_scratch_bytes < 65536)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "MoE provider weight scratch is too small");
    kq_status st = validate_call(config, true, hidden_states, token_count, output, output_capacity, scratch,
                                 scratch_bytes, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (!config->bound || config->provider != provider)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "MoE provider weights are not bound to the config");
    st = check_overlaps(hidden_states, output, token_count * config->dims.hidden_size, scratch, scratch_bytes,
                        diagnostic);
    if (st != KQ_STATUS_OK) return st;
    return execute_sync(config, &config->w, nullptr, hidden_states, token_count, output, route_observer,
                        checkpoint_observer, observer_user_data, diagnostic);
}

kq_status kq_b200_moe_config_bind(kq_moe_config *config, kq_weight_provider *provider,
                                  const kq_b200_moe_tensors *t, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || provider == nullptr || t == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, provider and tensors are required");
    const kq_moe_dimensions &d = config->dims;
    const uint32_t E = d.expert_count, H = d.hidden_size, I = d.routed_intermediate_size,
                   S = d.shared_intermediate_size;
    // (semantic, part, experts, rows per expert, columns, destination)
    struct M {
        const kq_semantic_tensor *s;
        kq_binding_part_role part;
        uint32_t experts, rows, cols;
        QMatrix *dst;
    } mats[8] = {{t->router, KQ_BINDING_PART_WHOLE, 0, E, H, &config->w.router},
                 {t->routed_down, KQ_BINDING_PART_WHOLE, E, H, I, &config->w.down},
                 {t->routed_gate_up, KQ_BINDING_PART_GATE, E, I, H, &config->w.gate},
                 {t->routed_gate_up, KQ_BINDING_PART_UP, E, I, H, &config->w.up},
                 {t->shared_down, KQ_BINDING_PART_WHOLE, 0, H, S, &config->w.shared_down},
                 {t->shared_gate, KQ_BINDING_PART_WHOLE, 0, S, H, &config->w.shared_gate},
                 {t->shared_up, KQ_BINDING_PART_WHOLE, 0, S, H, &config->w.shared_up},
                 {t->shared_gate_weight, KQ_BINDING_PART_WHOLE, 0, 1, H, &config->w.shared_gate_weight}};
    for (const M &m : mats) {
        ProviderTensor *p = provider_part(provider, m.s, m.part);
        if (p == nullptr || p->is_vector)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "required MoE semantic tensor is missing");
        if (p->experts != m.experts || (m.experts ? p->expert_rows : p->m.rows) != m.rows || p->m.cols != m.cols ||
            !p->col_heads.empty())
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "MoE tensor shape mismatch");
    }
    for (const M &m : mats) *m.dst = provider_part(provider, m.s, m.part)->m;
    config->provider = provider;
    config->bound = true;
    return KQ_STATUS_OK;
}

kq_status kq_b200_moe_execute_async(const kq_moe_config *config, const float *hidden, uint64_t tokens, float *output,
                                    kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || hidden == nullptr || output == nullptr || tokens == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config and device buffers are required");
    if (config->dims.activation_dtype != KQ_MOE_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_MOE, "execution requires an F32 MoE config");
    if (!config->bound)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    if (!is_device_pointer(hidden) || !is_device_pointer(output))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "asynchronous MoE takes device buffers");
    const uint64_t n = tokens * config->dims.hidden_size;
    if (ranges_overlap(hidden, n * 4, output, n * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "MoE input and output must not overlap");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    ErrorWord err = c->begin_call();
    launch_check_finite(hidden, n, err, c->stream);
    st = moe_run(c, config, config->w, hidden, tokens, output, err, nullptr, nullptr, nullptr, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaGetLastError(), diagnostic, "MoE launch");
    return KQ_STATUS_OK;
}

const char *kq_moe_checkpoint_kind_name(kq_moe_checkpoint_kind kind) {
    static const char *const names[] = {"ROUTER_LOGITS", "ROUTER_PROBABILITIES", "SELECTED_WEIGHTS",
                                        "ROUTED_GATE", "ROUTED_UP", "ROUTED_ACTIVATED",
                                        "ROUTED_EXPERT_OUTPUT", "ROUTED_WEIGHTED_OUTPUT", "ROUTED_WEIGHTED_SUM",
                                        "SHARED_GATE_PROJECTION", "SHARED_UP_PROJECTION", "SHARED_ACTIVATED",
                                        "SHARED_OUTPUT", "SHARED_SCALE_LOGIT", "SHARED_SCALE",
                                        "GATED_SHARED_OUTPUT", "OPERATOR_OUTPUT"};
    return (uint32_t)kind < sizeof(names) / sizeof(names[0]) ? names[(uint32_t)kind] : "INVALID";
}

}  // extern "C"

// ---------------------------------------------------------------- layer bridge

namespace kqb {

kq_status moe_layer_enqueue(DeviceContext *c, const kq_moe_config *cfg, const kq_moe_weights_f32 *wf, const float *x,
                            uint64_t tokens, float *y, ErrorWord err, kq_diagnostic *diag) {
    if (!config_valid(cfg) || tokens == 0)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "complete MoE execution arguments are required");
    const kq_moe_dimensions &d = cfg->dims;
    if (d.activation_dtype != KQ_MOE_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_MOE, "scalar execution requires an F32 MoE config");
    MoeWeightsDev w;
    if (wf != nullptr) {
        const uint64_t E = d.expert_count, H = d.hidden_size, I = d.routed_intermediate_size,
                       S = d.shared_intermediate_size;
        const float *src[8] = {wf->router, wf->routed_gate, wf->routed_up, wf->routed_down,
                               wf->shared_gate, wf->shared_up, wf->shared_down, wf->shared_gate_weight};
        const uint64_t cnt[8] = {wf->router_count, wf->routed_gate_count, wf->routed_up_count,
                                 wf->routed_down_count, wf->shared_gate_count, wf->shared_up_count,
                                 wf->shared_down_count, wf->shared_gate_weight_count};
        const uint64_t want[8] = {E * H, E * I * H, E * I * H, E * I * H, S * H, S * H, S * H, H};
        const float *p[8];
        for (int i = 0; i < 8; ++i) {
            if (cnt[i] != want[i]) return fail(diag, KQ_STATUS_DIMENSION_MISMATCH, "MoE weight shape/data mismatch");
            if (src[i] == nullptr) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "MoE weight shape/data mismatch");
            kq_status st = device_weights(c, src[i], cnt[i], err, &p[i], diag);
            if (st != KQ_STATUS_OK) return st;
        }
        w.router = dense(p[0], (uint32_t)E, (uint32_t)H);
        w.gate = dense(p[1], (uint32_t)(E * I), (uint32_t)H);
        w.up = dense(p[2], (uint32_t)(E * I), (uint32_t)H);
        w.down = dense(p[3], (uint32_t)(E * H), (uint32_t)I);
        w.shared_gate = dense(p[4], (uint32_t)S, (uint32_t)H);
        w.shared_up = dense(p[5], (uint32_t)S, (uint32_t)H);
        w.shared_down = dense(p[6], (uint32_t)H, (uint32_t)S);
        w.shared_gate_weight = dense(p[7], 1, (uint32_t)H);
    } else {
        if (!cfg->bound)
            return fail(diag, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "MoE provider weights are not bound to the config");
        w = cfg->w;
    }
    return moe_run(c, cfg, w, x, tokens, y, err, nullptr, nullptr, nullptr, diag);
}

}  // namespace kqb
