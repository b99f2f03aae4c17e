// kq_qsa ABI on the B200: configs, device-resident KV / index-key caches and
// execution.
//
// Replaces src/kq_qsa.c and the entry points of src/kq_qsa_qwen38.c of
// Kestrel-Q.  Validation order and status codes follow kq_qsa_validate_call
// (src/kq_qsa_qwen38.c:394-489).  New rows are appended beyond the committed
// length and the length is advanced only after the device reported success,
// so a failed call leaves the state and the output untouched (:818-827).
#include <algorithm>
#include <cfenv>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "kq_b200.h"
#include "kq_qsa.h"
#include "operators.hpp"
#include "provider.hpp"
#include "runtime.hpp"

using namespace kqb;

namespace {
constexpr uint32_t kQsaConfigMagic = 0x4b515143u;
constexpr uint32_t kQsaStateMagic = 0x4b515153u;
}  // namespace

struct kq_qsa_config {
    uint32_t magic;
    uint32_t layer_id;
    kq_qsa_dimensions dims;
    uint32_t repeat, block_topk, sel_capacity;
    uint64_t kv_per_token, raw_per_token, bytes_per_token;
    // RoPE table (device), grown to the largest state capacity
    mutable float *rope_cos;
    mutable float *rope_sin;
    mutable uint32_t rope_positions;
    kq_weight_provider *provider;
    QMatrix q, k, v, o, iq, ik;
    const float *q_norm, *k_norm, *iq_norm, *ik_norm;
    bool bound;
};

struct kq_qsa_state final : Rollbackable {
    uint32_t magic = 0;
    const kq_qsa_config *config = nullptr;
    int device = 0;
    uint64_t capacity = 0, length = 0;
    float *key = nullptr, *value = nullptr, *raw = nullptr, *block_keys = nullptr;
    // bf16 hi / lo copies of the K / V rows for the tensor-core attention
    // (null when it does not cover the geometry)
    uint16_t *key_split = nullptr, *value_split = nullptr;
    uint64_t owned_bytes = 0;
    uint64_t synced_length = 0;
    std::vector<std::pair<uint32_t, uint64_t>> history;
    // complete blocks whose normalised, rotated key is cached, and the
    // index-key norm weights that cache was built with
    uint64_t bk_valid = 0;
    std::vector<float> bk_norm;

    void on_step(uint32_t id) override { history.push_back({id, length}); }
    void on_error(uint32_t failing) override {
        uint64_t len = synced_length;
        for (auto &h : history)
            if (failing != 0 && h.first < failing) len = h.second;
        length = len;
        bk_valid = std::min<uint64_t>(bk_valid, len / config->dims.block_size);
        on_success();
    }
    void on_success() override {
        synced_length = length;
        history.clear();
    }
};

static bool config_valid(const kq_qsa_config *c) { return c != nullptr && c->magic == kQsaConfigMagic; }
static bool state_valid(const kq_qsa_state *s) {
    return s != nullptr && s->magic == kQsaStateMagic && config_valid(s->config) && s->key && s->value &&
           s->raw && s->length <= s->capacity;
}

// src/kq_qsa.c:95-152
static kq_status validate_dims(const kq_qsa_dimensions *d, kq_qsa_config *c, kq_diagnostic *diag) {
    if (d->hidden_size == 0 || d->query_head_count == 0 || d->key_value_head_count == 0 ||
        d->head_dimension == 0 || d->query_head_count % d->key_value_head_count != 0 ||
        d->index_query_head_count == 0 || d->index_head_dimension == 0 || d->block_size == 0 ||
        d->token_budget == 0 || d->token_budget % d->block_size != 0 || d->max_context == 0 ||
        d->rotary_dimension == 0 || (d->rotary_dimension & 1u) != 0 ||
        d->rotary_dimension > d->head_dimension || d->rotary_dimension > d->index_head_dimension ||
        !(d->rms_norm_epsilon > 0.0f) || !std::isfinite(d->rms_norm_epsilon) || !(d->rope_theta > 1.0f) ||
        !std::isfinite(d->rope_theta) ||
        (d->activation_dtype != KQ_QSA_ACTIVATION_F32 && d->activation_dtype != KQ_QSA_ACTIVATION_BF16))
        return fail(diag, KQ_STATUS_INCOMPATIBLE_QSA,
                    "invalid QSA dimensions, block geometry, RoPE, epsilon, or dtype");
    uint64_t kv, total;
    if (!mul_ok(d->key_value_head_count, d->head_dimension, &kv) || !add_ok(kv, kv, &total) ||
        !add_ok(total, d->index_head_dimension, &total))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "QSA state geometry overflows");
    uint64_t eb = d->activation_dtype == KQ_QSA_ACTIVATION_BF16 ? 2 : 4;
    if (!mul_ok(total, eb, &c->bytes_per_token))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "QSA state byte count overflows");
    if (d->token_budget > UINT32_MAX - (d->block_size - 1))
        return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "QSA selected-token capacity overflows");
    c->repeat = d->query_head_count / d->key_value_head_count;
    c->block_topk = d->token_budget / d->block_size;
    c->sel_capacity = d->token_budget + d->block_size - 1;
    c->kv_per_token = kv;
    c->raw_per_token = d->index_head_dimension;
    // B200 kernel limits
    const uint32_t hd = d->head_dimension;
    if (c->block_topk > 1024 || c->repeat > 8 || !(hd <= 32 || hd == 64 || hd == 128 || hd == 256))
        return fail(diag, KQ_STATUS_INCOMPATIBLE_QSA,
                    "B200 QSA kernels support up to 1024 selected blocks, 8 query heads per KV head "
                    "and head dimensions <= 32, 64, 128 or 256");
    return KQ_STATUS_OK;
}

// RoPE cos/sin table with the reference's expression (src/kq_qsa_qwen38.c:265-270)
// evaluated by the host libm, so device rotations use the very same factors.
static kq_status ensure_rope(const kq_qsa_config *c, uint64_t positions, kq_diagnostic *diag) {
    if (positions <= c->rope_positions) return KQ_STATUS_OK;
    const uint32_t rot = c->dims.rotary_dimension, half = rot / 2;
    std::vector<float> freq(half);
    for (uint32_t i = 0; i < half; ++i) {
        float e = (2.0f * (float)i) / (float)rot;
        freq[i] = 1.0f / powf(c->dims.rope_theta, e);
    }
    std::vector<float> cs((size_t)positions * half), sn((size_t)positions * half);
    for (uint64_t p = 0; p < positions; ++p)
        for (uint32_t i = 0; i < half; ++i) {
            float ang = (float)p * freq[i];
            cs[p * half + i] = cosf(ang);
            sn[p * half + i] = sinf(ang);
        }
    float *dc = nullptr, *ds = nullptr;
    KQB_CUDA(cudaMalloc(&dc, cs.size() * 4), diag, "rope table");
    if (cudaMalloc(&ds, sn.size() * 4) != cudaSuccess) {
        cudaFree(dc);
        return fail(diag, KQ_STATUS_OUT_OF_MEMORY, "rope table");
    }
    cudaMemcpy(dc, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(ds, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    cudaDeviceSynchronize();
    if (c->rope_cos) cudaFree(c->rope_cos);
    if (c->rope_sin) cudaFree(c->rope_sin);
    c->rope_cos = dc;
    c->rope_sin = ds;
    c->rope_positions = (uint32_t)positions;
    return KQ_STATUS_OK;
}

static QsaDims kernel_dims(const kq_qsa_config *c) {
    QsaDims d;
    d.hidden = c->dims.hidden_size;
    d.q_heads = c->dims.query_head_count;
    d.kv_heads = c->dims.key_value_head_count;
    d.head_dim = c->dims.head_dimension;
    d.index_heads = c->dims.index_query_head_count;
    d.index_dim = c->dims.index_head_dimension;
    d.block = c->dims.block_size;
    d.budget = c->dims.token_budget;
    d.topk = c->block_topk;
    d.rotary = c->dims.rotary_dimension;
    d.repeat = c->repeat;
    d.sel_capacity = c->sel_capacity;
    d.eps = c->dims.rms_norm_epsilon;
    d.inv_sqrt_head = 1.0f / sqrtf((float)c->dims.head_dimension);
    d.sqrt_index_dim = sqrtf((float)c->dims.index_head_dimension);
    d.sqrt_head_dim = sqrtf((float)c->dims.head_dimension);
    return d;
}

struct QsaResolved {
    QMatrix q, k, v, o, iq, ik;
    const float *q_norm, *k_norm, *iq_norm, *ik_norm;
};

struct SelectionCopy {
    std::vector<float> scores;
    std::vector<uint32_t> selected;
    uint32_t count = 0;
};

// Device arrays of one token's checkpoint data, filled by qsa_enqueue on the
// per-token path when the checkpoint observer is attached.
struct QsaDebugOut {
    const float *q = nullptr, *iq = nullptr, *gated = nullptr;
    float *logits = nullptr, *probs = nullptr, *context = nullptr;
};

// Token sharding of the indexer in a tensor-parallel prefill: this rank
// scores and selects only the 64-token chunks c with c % world == rank, and
// `exchange` completes the selection rows of every chunk (a sum over ranks
// of buffers that are zero outside each rank's chunks).
// Tokens per launch sequence of a one-sequence prefill (uniform batches).
constexpr uint32_t kPrefillEntries = 1024;

// With `parts` > 1 the attention is split by token as well: this rank's
// config holds every query head of one key/value head, and it runs the
// attention, gate and out-projection only for token part `part` of `parts`
// (contiguous, in whole launch groups), writing zero output rows elsewhere.
struct TokenShard {
    uint32_t rank = 0, world = 1;
    kq_b200_exchange_fn exchange = nullptr;
    void *user = nullptr;
    uint32_t part = 0, parts = 1;
};

// Enqueues the operator for `batch` sequences x `tokens` tokens (batch == 1
// or tokens == 1).  x / y are device [batch*tokens][H].  When `selection` is
// non-null (batch == 1) the stream is synchronised after every token and the
// selection of each token is copied out.
// `check_input`: the caller has not checked x for non-finite values; the
// main projection (or a separate pass) does.
static kq_status qsa_enqueue(DeviceContext *c, const kq_qsa_config *cfg, const QsaResolved &w,
                             kq_qsa_state *const *states, uint32_t batch, uint32_t tokens, const float *x,
                             float *y, ErrorWord err, std::vector<SelectionCopy> *selection,
                             kq_diagnostic *diag, bool check_input = false, const TokenShard *shard = nullptr,
                             QsaDebugOut *debug = nullptr) {
    const QsaDims d = kernel_dims(cfg);
    const uint32_t H = d.hidden, hd = d.head_dim;
    const uint32_t qw = d.q_heads * hd, kvw = d.kv_heads * hd;
    const uint32_t ldp = 2 * qw + 2 * kvw;
    const uint32_t ldi = d.index_heads * d.index_dim + d.index_dim;
    const size_t items = (size_t)batch * tokens;
    // A prefill of one sequence without a selection observer runs `unit`
    // tokens per launch sequence, as entries of a uniform batch over the same
    // cache (entry i at position L + t0 + i).
    const bool chunked = batch == 1 && tokens > 1 && selection == nullptr && debug == nullptr;
    // two passes (index / attention) around the selection exchange
    const bool sharded = chunked && shard != nullptr && shard->world > 1;
    // sharded: the index work (index queries, scores, top-k) is owned in
    // groups of `group` 64-token chunks, group u on rank u % world
    // (interleaved: later chunks score more blocks); one launch sequence per
    // group
    const uint32_t nchunks = (tokens + 63) / 64;
    const uint32_t group = sharded ? std::max<uint32_t>(1, std::min<uint32_t>(8, nchunks / (4 * shard->world))) : 1u;
    const uint32_t unit = sharded ? group * 64u : kPrefillEntries;
    auto owned = [&](uint32_t t0) { return !sharded || (t0 / unit) % shard->world == shard->rank; };
    // the rank's token range for attention: launch groups [u0, u1)
    const uint32_t parts = sharded ? shard->parts : 1u, part = sharded ? shard->part : 0u;
    const uint32_t ngroups = (tokens + unit - 1) / unit;
    const uint32_t tb = std::min<uint32_t>(tokens, (uint32_t)((uint64_t)ngroups * part / parts) * unit);
    const uint32_t te = std::min<uint32_t>(tokens, (uint32_t)((uint64_t)ngroups * (part + 1) / parts) * unit);
    auto attends = [&](uint32_t t0) { return t0 >= tb && t0 < te; };
    const uint32_t entries = chunked ? std::min<uint32_t>(tokens, unit) : batch;
    uint32_t max_blocks = 1;
    for (uint32_t b = 0; b < batch; ++b)
        max_blocks = std::max<uint32_t>(max_blocks, (uint32_t)((states[b]->length + tokens) / d.block));
    // about 16 tiles of 16 selected tokens per split, and at least two waves
    // of CTAs over the 148 SMs for small batches
    const uint32_t tiles = (d.sel_capacity + 15) / 16;
    const uint32_t per_seq = entries * d.kv_heads;
    // (the head-blocked attention kernel takes at most 32 tiles per split)
    // about 16 tiles of 16 selected tokens per split for decode batches, 32
    // (the kernel's limit) for prefill batches, which have CTAs to spare
    const uint32_t tiles_per_split = chunked ? 32u : 16u;
    uint32_t splits = std::max<uint32_t>((tiles + tiles_per_split - 1) / tiles_per_split,
                                         (3 * 148 + per_seq - 1) / per_seq);
    splits = std::max<uint32_t>(1, std::min<uint32_t>(splits, tiles));
    const size_t need = Carve::round(items * ldp * 4) + Carve::round(items * ldi * 4) +
                        Carve::round(items * qw * 4) + Carve::round((size_t)entries * qw * 4) +
                        Carve::round((size_t)entries * d.index_heads * d.index_dim * 4) +
                        Carve::round((size_t)entries * max_blocks * 4) +
                        Carve::round((size_t)entries * d.topk * 4) + Carve::round((size_t)entries * 4) +
                        Carve::round((size_t)entries * d.q_heads * splits * hd * 4) +
                        Carve::round((size_t)entries * d.q_heads * splits * 2 * 4) + 8192 +
                        (sharded ? Carve::round(items * (d.topk + 1) * 4) + Carve::round(items * qw * 4) : 0) +
                        (debug ? 2 * Carve::round((size_t)d.q_heads * d.sel_capacity * 4) + Carve::round(qw * 4) : 0);
    const size_t partial_floats = std::max(projection_workspace_floats((uint32_t)items, ldp, H),
                                           projection_workspace_floats((uint32_t)items, H, qw));
    void *ws;
    kq_status st = c->workspace(need + Carve::round(partial_floats * 4), &ws, diag);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    float *proj = cv.take<float>(items * ldp);
    float *iproj = cv.take<float>(items * ldi);
    float *gated = cv.take<float>(items * qw);
    float *qv = cv.take<float>((size_t)entries * qw);
    float *iqv = cv.take<float>((size_t)entries * d.index_heads * d.index_dim);
    float *scores = cv.take<float>((size_t)entries * max_blocks);
    uint32_t *sel = cv.take<uint32_t>((size_t)entries * d.topk);
    uint32_t *sel_count = cv.take<uint32_t>(entries);
    float *part_o = cv.take<float>((size_t)entries * d.q_heads * splits * hd);
    float *part_ml = cv.take<float>((size_t)entries * d.q_heads * splits * 2);
    float *partial = partial_floats ? cv.take<float>(partial_floats) : nullptr;
    // sharded: every token's selection ([T][topk] then [T] counts) and query
    uint32_t *sel_all = sharded ? cv.take<uint32_t>(items * (d.topk + 1)) : nullptr;
    float *q_all = sharded ? cv.take<float>(items * qw) : nullptr;
    if (debug) {
        debug->logits = cv.take<float>((size_t)d.q_heads * d.sel_capacity);
        debug->probs = cv.take<float>((size_t)d.q_heads * d.sel_capacity);
        debug->context = cv.take<float>(qw);
        debug->q = qv;
        debug->iq = iqv;
        debug->gated = gated;
    }

    ProjSegments main{};
    main.count = 3;
    main.m[0] = w.q; main.out_offset[0] = 0;
    main.m[1] = w.k; main.out_offset[1] = 2 * qw;
    main.m[2] = w.v; main.out_offset[2] = 2 * qw + kvw;
    ProjSegments index{};
    index.count = 2;
    index.m[0] = w.iq; index.out_offset[0] = 0;
    index.m[1] = w.ik; index.out_offset[1] = d.index_heads * d.index_dim;
    ProjSegments out{};
    out.count = 1;
    out.m[0] = w.o;
    out.out_offset[0] = 0;

    QsaWeightsDev wd;
    wd.q_norm = w.q_norm;
    wd.k_norm = w.k_norm;
    wd.iq_norm = w.iq_norm;
    wd.ik_norm = w.ik_norm;
    wd.rope_cos = cfg->rope_cos;
    wd.rope_sin = cfg->rope_sin;
    wd.rope_positions = cfg->rope_positions;

    for (uint32_t g0 = 0; g0 < batch; g0 += kMaxBatch) {
        const uint32_t gb = std::min<uint32_t>(kMaxBatch, batch - g0);
        const size_t row0 = (size_t)g0 * tokens;
        const size_t n_items = (size_t)gb * tokens;
        if (parts == 1) {
            if (!launch_projection(main, x + row0 * H, H, proj, ldp, (uint32_t)n_items, err, c->stream, partial,
                                   partial_floats) &&
                check_input)
                launch_check_finite(x + row0 * H, n_items * H, err, c->stream);
        } else {
            // keys and values of every token, queries / gates of this rank's tokens
            ProjSegments kv{};
            kv.count = 2;
            kv.m[0] = w.k; kv.out_offset[0] = 2 * qw;
            kv.m[1] = w.v; kv.out_offset[1] = 2 * qw + kvw;
            if (!launch_projection(kv, x, H, proj, ldp, tokens, err, c->stream, partial, partial_floats) &&
                check_input)
                launch_check_finite(x, (uint64_t)tokens * H, err, c->stream);
            ProjSegments qg{};
            qg.count = 1;
            qg.m[0] = w.q; qg.out_offset[0] = 0;
            if (te > tb)
                launch_projection(qg, x + (size_t)tb * H, H, proj + (size_t)tb * ldp, ldp, te - tb, err, c->stream,
                                  partial, partial_floats);
        }
        // sharded: raw index keys for every token, index queries only for
        // this rank's groups
        if (!sharded) {
            launch_projection_exact(index, x + row0 * H, H, iproj, ldi, (uint32_t)n_items, err, c->stream);
        } else {
            ProjSegments raw_key{};
            raw_key.count = 1;
            raw_key.m[0] = w.ik;
            raw_key.out_offset[0] = d.index_heads * d.index_dim;
            launch_projection_exact(raw_key, x, H, iproj, ldi, tokens, err, c->stream);
            ProjSegments queries{};
            queries.count = 1;
            queries.m[0] = w.iq;
            queries.out_offset[0] = 0;
            for (uint32_t t0 = 0; t0 < tokens; t0 += unit) {
                if (!owned(t0)) continue;
                const uint32_t n = std::min<uint32_t>(unit, tokens - t0);
                launch_projection_exact(queries, x + (size_t)t0 * H, H, iproj + (size_t)t0 * ldi, ldi, n, err,
                                        c->stream);
            }
        }
        for (uint32_t b = 0; b < gb; ++b) {
            kq_qsa_state *s = states[g0 + b];
            const uint64_t complete = s->length / d.block;
            if (s->bk_valid < complete) {
                QsaSeq sq{s->key, s->value, s->raw, s->block_keys, (uint32_t)s->length, (uint32_t)s->capacity};
                launch_qsa_block_keys(d, wd, sq, (uint32_t)s->bk_valid, (uint32_t)complete, err, c->stream);
            }
        }
        if (chunked) {
            kq_qsa_state *s = states[0];
            const QsaSeq seq{s->key,    s->value,       s->raw,         s->block_keys, (uint32_t)s->length,
                             (uint32_t)s->capacity, s->key_split, s->value_split};
            auto uniform_batch = [&](uint32_t t0) {
                QsaBatch qb;
                qb.s[0] = seq;
                qb.s[0].length = (uint32_t)s->length + t0;
                qb.uniform = 1;
                return qb;
            };
            uint32_t *cnt_all = sharded ? sel_all + (size_t)tokens * d.topk : nullptr;
            if (sharded)
                KQB_CUDA(cudaMemsetAsync(sel_all, 0, (size_t)tokens * (d.topk + 1) * 4, c->stream), diag, "selection");
            // pass 1 (the only pass without sharding): cache rows, queries and
            // block keys of every group; scores and top-k of the owned ones
            for (uint32_t t0 = 0; t0 < tokens; t0 += unit) {
                const uint32_t n = std::min<uint32_t>(unit, tokens - t0);
                const uint32_t pos0 = (uint32_t)s->length + t0;
                const QsaBatch qb = uniform_batch(t0);
                const float *pt = proj + (size_t)t0 * ldp;
                float *qdst = sharded ? q_all + (size_t)t0 * qw : qv;
                launch_qsa_prepare(d, wd, qb, n, pt, ldp, iproj + (size_t)t0 * ldi, ldi, qdst, iqv, false, owned(t0),
                                   attends(t0), err, c->stream);
                // keys of the blocks this group completes, once all their raw rows are written
                launch_qsa_block_keys(d, wd, seq, pos0 / d.block, (pos0 + n) / d.block, err, c->stream);
                if (!owned(t0)) continue;
                const uint32_t nb_max = std::max<uint32_t>(1, (pos0 + n) / d.block);
                uint32_t *sdst = sharded ? sel_all + (size_t)t0 * d.topk : sel;
                uint32_t *cdst = sharded ? cnt_all + t0 : sel_count;
                launch_qsa_score(d, qb, n, iqv, scores, max_blocks, nb_max, true, err, c->stream);
                launch_qsa_select(d, qb, n, scores, max_blocks, sdst, cdst, false, err, c->stream);
                if (sharded) continue;
                launch_qsa_attend(d, qb, n, qv, sel, sel_count, part_o, part_ml, splits, err, c->stream);
                launch_qsa_combine(d, n, part_o, part_ml, splits, pt, ldp, gated + (size_t)t0 * qw, err, c->stream);
            }
            if (sharded) {
                KQB_CUDA(cudaGetLastError(), diag, "QSA index pass");
                if (shard->exchange(sel_all, (uint64_t)tokens * (d.topk + 1), c->stream, shard->user) != 0)
                    return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "QSA selection exchange failed");
                // pass 2: attention of this rank's groups with the exchanged selections
                for (uint32_t t0 = tb; t0 < te; t0 += unit) {
                    const uint32_t n = std::min<uint32_t>(unit, tokens - t0);
                    const QsaBatch qb = uniform_batch(t0);
                    launch_qsa_attend(d, qb, n, q_all + (size_t)t0 * qw, sel_all + (size_t)t0 * d.topk,
                                      cnt_all + t0, part_o, part_ml, splits, err, c->stream);
                    launch_qsa_combine(d, n, part_o, part_ml, splits, proj + (size_t)t0 * ldp, ldp,
                                       gated + (size_t)t0 * qw, err, c->stream);
                }
            }
        }
        for (uint32_t t = 0; !chunked && t < tokens; ++t) {
            QsaBatch qb;
            uint32_t nb_max = 1;
            for (uint32_t b = 0; b < gb; ++b) {
                kq_qsa_state *s = states[g0 + b];
                qb.s[b].key = s->key;
                qb.s[b].value = s->value;
                qb.s[b].key_split = s->key_split;
                qb.s[b].value_split = s->value_split;
                qb.s[b].raw = s->raw;
                qb.s[b].block_keys = s->block_keys;
                qb.s[b].length = (uint32_t)(s->length + t);
                qb.s[b].capacity = (uint32_t)s->capacity;
                nb_max = std::max<uint32_t>(nb_max, (qb.s[b].length + 1) / d.block);
            }
            const float *pt = proj + (size_t)t * ldp;      // batch==1: token rows; tokens==1: t==0
            const float *it = iproj + (size_t)t * ldi;
            launch_qsa_prepare(d, wd, qb, gb, pt, ldp * tokens, it, ldi * tokens, qv, iqv, true, true, true, err,
                               c->stream);
            launch_qsa_score(d, qb, gb, iqv, scores, max_blocks, nb_max, false, err, c->stream);
            launch_qsa_select(d, qb, gb, scores, max_blocks, sel, sel_count, selection != nullptr || debug != nullptr,
                              err, c->stream);
            launch_qsa_attend(d, qb, gb, qv, sel, sel_count, part_o, part_ml, splits, err, c->stream);
            launch_qsa_combine(d, gb, part_o, part_ml, splits, pt, ldp * tokens, gated + (size_t)t * qw, err,
                               c->stream);
            if (debug)
                launch_qsa_debug_attention(d, qb, qv, sel, sel_count, debug->logits, debug->probs, debug->context,
                                           err, c->stream);
            if (selection != nullptr) {
                KQB_CUDA(cudaStreamSynchronize(c->stream), diag, "selection sync");
                SelectionCopy sc;
                const uint32_t nb = (qb.s[0].length + 1) / d.block;
                sc.scores.resize(nb);
                sc.selected.resize(d.topk);
                if (nb)
                    KQB_CUDA(cudaMemcpy(sc.scores.data(), scores, nb * 4, cudaMemcpyDeviceToHost), diag, "scores");
                KQB_CUDA(cudaMemcpy(sc.selected.data(), sel, d.topk * 4, cudaMemcpyDeviceToHost), diag, "sel");
                KQB_CUDA(cudaMemcpy(&sc.count, sel_count, 4, cudaMemcpyDeviceToHost), diag, "count");
                selection->push_back(std::move(sc));
            }
        }
        if (parts == 1) {
            if (!launch_projection(out, gated, qw, y + row0 * H, H, (uint32_t)n_items, err, c->stream, partial,
                                   partial_floats))
                launch_check_finite(y + row0 * H, n_items * H, err, c->stream);
        } else {
            // this rank's rows; zeros elsewhere (other ranks add theirs)
            if (tb > 0) KQB_CUDA(cudaMemsetAsync(y, 0, (size_t)tb * H * 4, c->stream), diag, "output rows");
            if (te < tokens)
                KQB_CUDA(cudaMemsetAsync(y + (size_t)te * H, 0, (size_t)(tokens - te) * H * 4, c->stream), diag,
                         "output rows");
            if (te > tb &&
                !launch_projection(out, gated + (size_t)tb * qw, qw, y + (size_t)tb * H, H, te - tb, err, c->stream,
                                   partial, partial_floats))
                launch_check_finite(y + (size_t)tb * H, (uint64_t)(te - tb) * H, err, c->stream);
        }
        for (uint32_t b = 0; b < gb; ++b) {
            kq_qsa_state *s = states[g0 + b];
            s->length += tokens;
            s->bk_valid = s->length / d.block;
            s->on_step(err.call_id);
            c->dirty.insert(s);
        }
    }
    KQB_CUDA(cudaGetLastError(), diag, "QSA launch");
    return KQ_STATUS_OK;
}

// src/kq_qsa.c:622-687 (same accounting, so callers size scratch identically)
static kq_status scratch_bytes_for(const kq_qsa_config *config, const kq_qsa_state *state, uint64_t T,
                                   uint64_t *out, kq_diagnostic *diag) {
    uint64_t qw, iqw, sel;
    if (!config_valid(config) || !state_valid(state) || state->config != config || T == 0 || out == nullptr ||
        !mul_ok(config->dims.query_head_count, config->dims.head_dimension, &qw) ||
        !mul_ok(config->dims.index_query_head_count, config->dims.index_head_dimension, &iqw) ||
        !add_ok(state->length, T, &sel) || sel > state->capacity)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid QSA state, sequence, and scratch output are required");
    const uint64_t kvw = config->kv_per_token, raw = config->raw_per_token;
    const uint64_t blocks = state->capacity / config->dims.block_size;
    const uint64_t selected = config->sel_capacity;
    uint64_t total = 0, tmp;
    uint64_t state_width = kvw + kvw + raw;
    auto acc = [&](uint64_t v) { return add_ok(total, v, &total); };
    bool ok = mul_ok(T, state_width, &tmp) && acc(tmp) && mul_ok(T, config->dims.hidden_size, &tmp) && acc(tmp) &&
              acc(qw + qw) && acc(qw) && acc(kvw) && acc(kvw) && acc(iqw) && acc(raw) &&
              mul_ok(blocks, raw, &tmp) && acc(tmp) && acc(blocks) && acc(blocks) && acc(config->block_topk) &&
              acc(selected) && mul_ok(config->dims.query_head_count, selected, &tmp) && acc(tmp) && acc(tmp) &&
              acc(qw) && acc(qw) && acc(config->dims.hidden_size) && mul_ok(total, 4, out);
    if (!ok) return fail(diag, KQ_STATUS_ARITHMETIC_OVERFLOW, "QSA scratch byte count overflows");
    return KQ_STATUS_OK;
}

static kq_status validate_call(const kq_qsa_config *config, const kq_qsa_weights_f32 *weights, const float *hidden,
                               uint64_t T, float *output, uint64_t output_capacity, kq_qsa_state *state,
                               void *scratch, uint64_t scratch_bytes, bool provider_mode, kq_diagnostic *diag) {
    if (!config_valid(config) || (!provider_mode && weights == nullptr) || hidden == nullptr ||
        output == nullptr || !state_valid(state) || state->config != config || scratch == nullptr)
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid compatible QSA call arguments are required");
    if (config->dims.activation_dtype != KQ_QSA_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_QSA, "scalar execution requires an F32 QSA reference config");
    uint64_t total, n;
    if (T == 0 || !add_ok(state->length, T, &total) || total > state->capacity ||
        !mul_ok(T, config->dims.hidden_size, &n) || n > SIZE_MAX / 4)
        return fail(diag, KQ_STATUS_LIMIT_EXCEEDED, "QSA sequence exceeds bounded state capacity or overflows");
    if (output_capacity < n) return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "QSA output capacity is too small");
    uint64_t need;
    kq_status st = scratch_bytes_for(config, state, T, &need, diag);
    if (st != KQ_STATUS_OK) return st;
    if (scratch_bytes < need || reinterpret_cast<uintptr_t>(scratch) % alignof(float) != 0)
        return fail(diag, KQ_STATUS_BUFFER_TOO_SMALL, "QSA aligned scratch buffer is too small");
    if (!is_device_pointer(hidden))
        for (uint64_t i = 0; i < n; ++i)
            if (!std::isfinite(hidden[i])) return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "QSA input must be finite");
    if (!provider_mode) {
        const kq_qsa_dimensions &d = config->dims;
        const uint64_t qw = (uint64_t)d.query_head_count * d.head_dimension, H = d.hidden_size;
        struct W { const float *p; uint64_t have, want; const char *msg; } ws[10] = {
            {weights->query, weights->query_count, 2 * qw * H, "QSA query projection shape/data mismatch"},
            {weights->key, weights->key_count, config->kv_per_token * H, "QSA key projection shape/data mismatch"},
            {weights->value, weights->value_count, config->kv_per_token * H, "QSA value projection shape/data mismatch"},
            {weights->output, weights->output_count, H * qw, "QSA output projection shape/data mismatch"},
            {weights->query_norm, weights->query_norm_count, d.head_dimension, "QSA query norm shape/data mismatch"},
            {weights->key_norm, weights->key_norm_count, d.head_dimension, "QSA key norm shape/data mismatch"},
            {weights->index_query, weights->index_query_count, (uint64_t)d.index_query_head_count * d.index_head_dimension * H,
             "QSA index query projection shape/data mismatch"},
            {weights->index_key, weights->index_key_count, (uint64_t)d.index_head_dimension * H,
             "QSA index key projection shape/data mismatch"},
            {weights->index_query_norm, weights->index_query_norm_count, d.index_head_dimension,
             "QSA index query norm shape/data mismatch"},
            {weights->index_key_norm, weights->index_key_norm_count, d.index_head_dimension,
             "QSA index key norm shape/data mismatch"}};
        for (auto &w : ws) {
            if (w.have != w.want) return fail(diag, KQ_STATUS_DIMENSION_MISMATCH, w.msg);
            if (w.p == nullptr) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, w.msg);
            if (!is_device_pointer(w.p))
                for (uint64_t i = 0; i < w.have; ++i)
                    if (!std::isfinite(w.p[i])) return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, w.msg);
        }
    }
    const uint64_t hb = n * 4, ob = output_capacity * 4;
    const uint64_t kvb = state->capacity * config->kv_per_token * 4, rb = state->capacity * config->raw_per_token * 4;
    if (ranges_overlap(hidden, hb, output, ob) || ranges_overlap(hidden, hb, scratch, scratch_bytes) ||
        ranges_overlap(output, ob, scratch, scratch_bytes) || ranges_overlap(state->key, kvb, scratch, scratch_bytes) ||
        ranges_overlap(state->value, kvb, scratch, scratch_bytes) ||
        ranges_overlap(state->raw, rb, scratch, scratch_bytes) || ranges_overlap(state->key, kvb, output, ob) ||
        ranges_overlap(state->value, kvb, output, ob))
        return fail(diag, KQ_STATUS_ALIASING_VIOLATION, "QSA input, output, state, and scratch must not overlap");
    if (std::fegetround() != FE_TONEAREST)
        return fail(diag, KQ_STATUS_NUMERIC_DOMAIN, "QSA scalar reference requires round-to-nearest");
    return KQ_STATUS_OK;
}

static void emit_selections(const kq_qsa_config *cfg, uint64_t L0, const std::vector<SelectionCopy> &sels,
                            kq_qsa_selection_observer obs, void *user, uint64_t token0 = 0) {
    const uint32_t blk = cfg->dims.block_size;
    for (size_t t = 0; t < sels.size(); ++t) {
        const SelectionCopy &s = sels[t];
        const uint64_t pos = L0 + t;
        const uint64_t nb = (pos + 1) / blk, tail = (pos + 1) % blk;
        std::vector<uint32_t> ids(nb), toks;
        for (uint64_t i = 0; i < nb; ++i) ids[i] = (uint32_t)i;
        for (uint32_t i = 0; i < s.count; ++i)
            for (uint32_t o = 0; o < blk; ++o) toks.push_back(s.selected[i] * blk + o);
        for (uint64_t i = 0; i < tail; ++i) toks.push_back((uint32_t)(nb * blk + i));
        kq_qsa_selection sel;
        std::memset(&sel, 0, sizeof(sel));
        sel.token_index = token0 + t;
        sel.absolute_position = pos;
        sel.candidate_block_ids = ids.data();
        sel.candidate_scores = s.scores.data();
        sel.candidate_count = nb;
        sel.selected_block_ids = s.selected.data();
        sel.selected_block_count = s.count;
        sel.selected_token_positions = toks.data();
        sel.selected_token_count = toks.size();
        sel.tail_count = tail;
        obs(&sel, user);
    }
}

// Checkpoint path (a checkpoint observer is attached): one token per launch
// sequence through the product kernels, with the selection in the reference's
// rank order and the attention's logits, probabilities and ungated context
// from the debug kernel; after each token the 12 checkpoints of
// include/kq_qsa.h are copied to the host and handed to the observer in the
// reference's order (src/kq_qsa_qwen38.c:687-815), after the token's
// selection observer call.  A device error stops the emission; the caller's
// final synchronize rolls the whole call back.
static kq_status qsa_debug_run(DeviceContext *c, const kq_qsa_config *cfg, const QsaResolved &w, kq_qsa_state *s,
                               uint32_t T, const float *x, float *y, ErrorWord err,
                               kq_qsa_selection_observer sel_obs, kq_qsa_checkpoint_observer ck_obs, void *user,
                               kq_diagnostic *diag) {
    const QsaDims d = kernel_dims(cfg);
    const uint32_t H = d.hidden, hd = d.head_dim, qw = d.q_heads * hd, kvw = d.kv_heads * hd;
    const uint32_t di = d.index_dim, iqw = d.index_heads * di;
    const uint32_t ld = block_key_ld((uint32_t)s->capacity, d.block);
    std::vector<float> hiq(iqw), hraw(di), hq(qw), hk(kvw), hv(kvw), hctx(qw), hgt(qw), hy(H), hbk, hbkt,
        hlg, hpr;
    for (uint32_t t = 0; t < T; ++t) {
        const uint64_t pos = s->length;
        std::vector<SelectionCopy> sels;
        QsaDebugOut dbg;
        kq_qsa_state *states[1] = {s};
        kq_status st = qsa_enqueue(c, cfg, w, states, 1, 1, x + (size_t)t * H, y + (size_t)t * H, err, &sels, diag,
                                   false, nullptr, &dbg);
        if (st != KQ_STATUS_OK) return st;
        KQB_CUDA(cudaStreamSynchronize(c->stream), diag, "QSA checkpoint sync");
        unsigned long long word = 0;
        KQB_CUDA(cudaMemcpy(&word, c->err_word, sizeof word, cudaMemcpyDeviceToHost), diag, "error word read");
        if (word != 0ull) return KQ_STATUS_OK;   // reported and rolled back by the caller's synchronize
        const uint64_t nb = (pos + 1) / d.block, tail = (pos + 1) % d.block;
        const uint64_t ntok = (uint64_t)sels[0].count * d.block + tail;
        hbk.resize(nb * di);
        hbkt.resize(nb * di);
        hlg.resize((size_t)d.q_heads * ntok);
        hpr.resize((size_t)d.q_heads * ntok);
        struct Copy { float *dst; const float *src; size_t n; } copies[] = {
            {hiq.data(), dbg.iq, iqw}, {hraw.data(), s->raw + pos * di, di}, {hq.data(), dbg.q, qw},
            {hk.data(), s->key + pos * kvw, kvw}, {hv.data(), s->value + pos * kvw, kvw},
            {hlg.data(), dbg.logits, hlg.size()}, {hpr.data(), dbg.probs, hpr.size()},
            {hctx.data(), dbg.context, qw}, {hgt.data(), dbg.gated, qw}, {hy.data(), y + (size_t)t * H, H}};
        for (const Copy &cp : copies)
            if (cp.n) KQB_CUDA(cudaMemcpy(cp.dst, cp.src, cp.n * 4, cudaMemcpyDeviceToHost), diag, "checkpoint copy");
        if (nb) {
            // the cached block keys are feature-major [di][ld]: rows of nb, then transposed
            KQB_CUDA(cudaMemcpy2D(hbkt.data(), nb * 4, s->block_keys, (size_t)ld * 4, nb * 4, di,
                                  cudaMemcpyDeviceToHost), diag, "block key copy");
            for (uint64_t b = 0; b < nb; ++b)
                for (uint32_t f = 0; f < di; ++f) hbk[b * di + f] = hbkt[(size_t)f * nb + b];
        }
        if (sel_obs) emit_selections(cfg, pos, sels, sel_obs, user, t);
        auto emit = [&](kq_qsa_checkpoint_kind kind, uint32_t rank, uint64_t d0, uint64_t d1, const float *v,
                        uint64_t count) {
            kq_qsa_checkpoint cp;
            std::memset(&cp, 0, sizeof(cp));
            cp.kind = kind;
            cp.token_index = t;
            cp.rank = rank;
            cp.dimensions[0] = d0;
            cp.dimensions[1] = d1;
            cp.values = v;
            cp.value_count = count;
            ck_obs(&cp, user);
        };
        emit(KQ_QSA_CHECKPOINT_INDEX_QUERY, 2, d.index_heads, di, hiq.data(), iqw);
        emit(KQ_QSA_CHECKPOINT_RAW_INDEX_KEY, 1, di, 0, hraw.data(), di);
        emit(KQ_QSA_CHECKPOINT_BLOCK_KEYS, 2, nb, di, hbk.data(), nb * di);
        emit(KQ_QSA_CHECKPOINT_CANDIDATE_SCORES, 1, nb, 0, sels[0].scores.data(), nb);
        emit(KQ_QSA_CHECKPOINT_QUERY, 2, d.q_heads, hd, hq.data(), qw);
        emit(KQ_QSA_CHECKPOINT_KEY, 2, d.kv_heads, hd, hk.data(), kvw);
        emit(KQ_QSA_CHECKPOINT_VALUE, 2, d.kv_heads, hd, hv.data(), kvw);
        emit(KQ_QSA_CHECKPOINT_ATTENTION_LOGITS, 2, d.q_heads, ntok, hlg.data(), hlg.size());
        emit(KQ_QSA_CHECKPOINT_ATTENTION_PROBABILITIES, 2, d.q_heads, ntok, hpr.data(), hpr.size());
        emit(KQ_QSA_CHECKPOINT_HEAD_CONTEXT, 2, d.q_heads, hd, hctx.data(), qw);
        emit(KQ_QSA_CHECKPOINT_GATED_CONTEXT, 2, d.q_heads, hd, hgt.data(), qw);
        emit(KQ_QSA_CHECKPOINT_OPERATOR_OUTPUT, 1, H, 0, hy.data(), H);
    }
    return KQ_STATUS_OK;
}

// F32 weight arrays (host: uploaded once and reused while their contents
// stay the same; device: used in place, checked on the device) as the
// operator's dense matrices.
static kq_status resolve_f32(DeviceContext *c, const kq_qsa_config *cfg, const kq_qsa_weights_f32 *wf, ErrorWord err,
                             QsaResolved *out, kq_diagnostic *diag) {
    const uint32_t H = cfg->dims.hidden_size;
    kq_status st = KQ_STATUS_OK;
    QsaResolved &w = *out;
    {
        const kq_qsa_dimensions &d = cfg->dims;
        const uint32_t qw = d.query_head_count * d.head_dimension, kvw = (uint32_t)cfg->kv_per_token;
        const float *ptrs[10] = {wf->query, wf->key, wf->value, wf->output, wf->query_norm, wf->key_norm,
                                 wf->index_query, wf->index_key, wf->index_query_norm, wf->index_key_norm};
        const uint64_t counts[10] = {wf->query_count, wf->key_count, wf->value_count, wf->output_count,
                                     wf->query_norm_count, wf->key_norm_count, wf->index_query_count,
                                     wf->index_key_count, wf->index_query_norm_count, wf->index_key_norm_count};
        // host weights: uploaded once and reused while their contents stay
        // the same; device weights: used in place, checked on the device
        const float *dev[10];
        for (int i = 0; i < 10; ++i) {
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
        w.q = dense(dev[0], 2 * qw, H);
        w.k = dense(dev[1], kvw, H);
        w.v = dense(dev[2], kvw, H);
        w.o = dense(dev[3], H, qw);
        w.q_norm = dev[4];
        w.k_norm = dev[5];
        w.iq = dense(dev[6], d.index_query_head_count * d.index_head_dimension, H);
        w.ik = dense(dev[7], d.index_head_dimension, H);
        w.iq_norm = dev[8];
        w.ik_norm = dev[9];
        }
    return st;
}

// The state's cached block keys were built with one index-key norm; another
// norm invalidates them.
static kq_status sync_block_key_norm(const kq_qsa_config *cfg, const QsaResolved &w, kq_qsa_state *state,
                                     kq_diagnostic *diag) {
    std::vector<float> norm(cfg->dims.index_head_dimension);
    KQB_CUDA(cudaMemcpy(norm.data(), w.ik_norm, norm.size() * 4, cudaMemcpyDefault), diag, "norm read");
    if (norm != state->bk_norm) {
        state->bk_norm = norm;
        state->bk_valid = 0;
    }
    return KQ_STATUS_OK;
}

static kq_status qsa_execute_sync(const kq_qsa_config *cfg, const QsaResolved *w_in, const kq_qsa_weights_f32 *wf,
                                  const float *hidden, uint64_t T, float *output, kq_qsa_state *state,
                                  kq_qsa_selection_observer sel_obs, kq_qsa_checkpoint_observer ck_obs, void *user,
                                  kq_diagnostic *diag) {
    DeviceContext *c;
    kq_status st = context(&c, diag);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    const uint32_t H = cfg->dims.hidden_size;
    const uint64_t n = T * H;
    ErrorWord err = c->begin_call();
    // host input and the output go through the context's staging arena (no
    // allocation once it has grown to this call's size)
    const bool x_host = !is_device_pointer(hidden);
    void *stage;
    st = c->staging(Carve::round(n * 4) + (x_host ? Carve::round(n * 4) : 0), &stage, diag);
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

    QsaResolved w;
    if (w_in) {
        w = *w_in;
    } else {
        st = resolve_f32(c, cfg, wf, err, &w, diag);
        if (st != KQ_STATUS_OK) return st;
    }
    st = sync_block_key_norm(cfg, w, state, diag);
    if (st != KQ_STATUS_OK) return st;
    const uint64_t L0 = state->length;
    std::vector<SelectionCopy> sels;
    kq_qsa_state *states[1] = {state};
    st = ck_obs != nullptr
             ? qsa_debug_run(c, cfg, w, state, (uint32_t)T, dx, dy, err, sel_obs, ck_obs, user, diag)
             : qsa_enqueue(c, cfg, w, states, 1, (uint32_t)T, dx, dy, err, sel_obs ? &sels : nullptr, diag);
    if (st != KQ_STATUS_OK) {
        c->synchronize(nullptr);
        return st;
    }
    st = c->synchronize(diag);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output, dy, n * 4,
                        is_device_pointer(output) ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost),
             diag, "output copy");
    if (sel_obs && ck_obs == nullptr) emit_selections(cfg, L0, sels, sel_obs, user);
    return KQ_STATUS_OK;
}

extern "C" {

kq_status kq_qsa_test_config_create(const kq_qsa_dimensions *dimensions, kq_qsa_config **out_config,
                                    kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (dimensions == nullptr || out_config == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "test QSA dimensions are required");
    *out_config = nullptr;
    auto *c = new (std::nothrow) kq_qsa_config();
    if (c == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate QSA config");
    std::memset(c, 0, sizeof(*c));
    kq_status st = validate_dims(dimensions, c, diagnostic);
    if (st != KQ_STATUS_OK) {
        delete c;
        return st;
    }
    c->magic = kQsaConfigMagic;
    c->dims = *dimensions;
    *out_config = c;
    return KQ_STATUS_OK;
}

kq_status kq_qsa_config_create(const kq_model *, uint32_t, kq_qsa_config **out_config, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_config) *out_config = nullptr;
    return fail(diagnostic, KQ_STATUS_UNSUPPORTED_MODEL,
                "GGUF model configs are not supported by the B200 library; use kq_qsa_test_config_create");
}

kq_status kq_qsa_config_create_reference_f32(const kq_model *m, uint32_t l, kq_qsa_config **o, kq_diagnostic *d) {
    return kq_qsa_config_create(m, l, o, d);
}

void kq_qsa_config_close(kq_qsa_config *config) {
    if (config == nullptr) return;
    cudaDeviceSynchronize();
    if (config->rope_cos) cudaFree(config->rope_cos);
    if (config->rope_sin) cudaFree(config->rope_sin);
    config->magic = 0;
    delete config;
}

uint32_t kq_qsa_config_layer_id(const kq_qsa_config *c) { return config_valid(c) ? c->layer_id : UINT32_MAX; }
uint32_t kq_qsa_config_hidden_size(const kq_qsa_config *c) { return config_valid(c) ? c->dims.hidden_size : 0; }
uint32_t kq_qsa_config_query_head_count(const kq_qsa_config *c) { return config_valid(c) ? c->dims.query_head_count : 0; }
uint32_t kq_qsa_config_key_value_head_count(const kq_qsa_config *c) { return config_valid(c) ? c->dims.key_value_head_count : 0; }
uint32_t kq_qsa_config_head_dimension(const kq_qsa_config *c) { return config_valid(c) ? c->dims.head_dimension : 0; }
uint32_t kq_qsa_config_index_query_head_count(const kq_qsa_config *c) { return config_valid(c) ? c->dims.index_query_head_count : 0; }
uint32_t kq_qsa_config_index_head_dimension(const kq_qsa_config *c) { return config_valid(c) ? c->dims.index_head_dimension : 0; }
uint32_t kq_qsa_config_block_size(const kq_qsa_config *c) { return config_valid(c) ? c->dims.block_size : 0; }
uint32_t kq_qsa_config_block_selection_limit(const kq_qsa_config *c) { return config_valid(c) ? c->block_topk : 0; }
uint32_t kq_qsa_config_context_limit(const kq_qsa_config *c) { return config_valid(c) ? c->dims.max_context : 0; }
kq_qsa_activation_dtype kq_qsa_config_activation_dtype(const kq_qsa_config *c) {
    return config_valid(c) ? c->dims.activation_dtype : KQ_QSA_ACTIVATION_F32;
}
uint64_t kq_qsa_config_owned_bytes(const kq_qsa_config *c) { return config_valid(c) ? sizeof(*c) : 0; }
uint64_t kq_qsa_config_semantic_state_bytes_per_token(const kq_qsa_config *c) {
    return config_valid(c) ? c->bytes_per_token : 0;
}

kq_status kq_b200_qsa_config_bind(kq_qsa_config *config, kq_weight_provider *provider,
                                  const kq_b200_qsa_tensors *t, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || provider == nullptr || t == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, provider and tensors are required");
    const kq_qsa_dimensions &d = config->dims;
    const uint32_t H = d.hidden_size, qw = d.query_head_count * d.head_dimension, kvw = (uint32_t)config->kv_per_token;
    // the index projections may be one split semantic (INDEX_QUERY and
    // INDEX_KEY parts, src/kq_qsa.c:184-201) or two whole ones
    struct M { const kq_semantic_tensor *s; uint32_t rows, cols; QMatrix *dst; kq_binding_part_role part; } mats[6] = {
        {t->query, 2 * qw, H, &config->q, KQ_BINDING_PART_WHOLE},
        {t->key, kvw, H, &config->k, KQ_BINDING_PART_WHOLE},
        {t->value, kvw, H, &config->v, KQ_BINDING_PART_WHOLE},
        {t->output, H, qw, &config->o, KQ_BINDING_PART_WHOLE},
        {t->index_query, d.index_query_head_count * d.index_head_dimension, H, &config->iq,
         KQ_BINDING_PART_INDEX_QUERY},
        {t->index_key, d.index_head_dimension, H, &config->ik, KQ_BINDING_PART_INDEX_KEY}};
    auto matrix = [&](const M &m) -> ProviderTensor * {
        ProviderTensor *p = provider_lookup(provider, m.s);
        if (p != nullptr && p->parts[0] != nullptr) return provider_part(provider, m.s, m.part);
        return p;
    };
    struct V { const kq_semantic_tensor *s; uint64_t count; const float **dst; } vecs[4] = {
        {t->query_norm, d.head_dimension, &config->q_norm}, {t->key_norm, d.head_dimension, &config->k_norm},
        {t->index_query_norm, d.index_head_dimension, &config->iq_norm},
        {t->index_key_norm, d.index_head_dimension, &config->ik_norm}};
    for (auto &m : mats) {
        ProviderTensor *p = matrix(m);
        if (p == nullptr || p->is_vector)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "required QSA semantic tensor is missing");
        if (!p->col_heads.empty())
            return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH, "QSA tensors keep canonical columns");
        if (p->m.rows != m.rows || p->m.cols != m.cols)
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_QSA, "QSA canonical tensor shape mismatch");
    }
    for (auto &v : vecs) {
        ProviderTensor *p = provider_lookup(provider, v.s);
        if (p == nullptr || !p->is_vector)
            return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "required QSA semantic tensor is missing");
        if (p->vec_host.size() != v.count)
            return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_QSA, "QSA canonical tensor shape mismatch");
    }
    for (auto &m : mats) *m.dst = matrix(m)->m;
    for (auto &v : vecs) *v.dst = provider_lookup(provider, v.s)->vec_dev;
    config->provider = provider;
    config->bound = true;
    return KQ_STATUS_OK;
}

kq_status kq_qsa_state_create(const kq_qsa_config *config, uint64_t token_capacity, kq_qsa_state **out_state,
                              kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_state == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "QSA state output is required");
    *out_state = nullptr;
    if (!config_valid(config) || token_capacity == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid QSA config and bounded positive capacity are required");
    if (token_capacity > config->dims.max_context)
        return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, "QSA state capacity exceeds the context limit");
    if (token_capacity > UINT32_MAX / 2)
        return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, "QSA state capacity exceeds the device index range");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = ensure_rope(config, token_capacity, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    auto *s = new (std::nothrow) kq_qsa_state();
    if (s == nullptr) return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate QSA state object");
    s->device = c->device;
    const size_t kvb = token_capacity * config->kv_per_token * 4, rb = token_capacity * config->raw_per_token * 4;
    const size_t bkb = std::max<uint64_t>(4, block_key_ld((uint32_t)token_capacity, config->dims.block_size)) *
                       config->raw_per_token * 4;
    if (cudaMalloc(&s->key, kvb) != cudaSuccess || cudaMalloc(&s->value, kvb) != cudaSuccess ||
        cudaMalloc(&s->raw, rb) != cudaSuccess || cudaMalloc(&s->block_keys, bkb) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(s->key); cudaFree(s->value); cudaFree(s->raw); cudaFree(s->block_keys);
        delete s;
        return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate bounded QSA cache buffers");
    }
    size_t split_bytes = 0;
    if (qsa_split_cache_used(kernel_dims(config))) {
        // hi + lo bf16 (1040-byte rows of 256 features)
        split_bytes = token_capacity * config->dims.key_value_head_count * kQsaSplitRow * 2;
        if (cudaMalloc(&s->key_split, split_bytes) != cudaSuccess ||
            cudaMalloc(&s->value_split, split_bytes) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(s->key); cudaFree(s->value); cudaFree(s->raw); cudaFree(s->block_keys);
            cudaFree(s->key_split); cudaFree(s->value_split);
            delete s;
            return fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY, "could not allocate bounded QSA cache buffers");
        }
        cudaMemsetAsync(s->key_split, 0, split_bytes, c->stream);
        cudaMemsetAsync(s->value_split, 0, split_bytes, c->stream);
    }
    cudaMemsetAsync(s->key, 0, kvb, c->stream);
    cudaMemsetAsync(s->value, 0, kvb, c->stream);
    cudaMemsetAsync(s->raw, 0, rb, c->stream);
    cudaMemsetAsync(s->block_keys, 0, bkb, c->stream);
    s->magic = kQsaStateMagic;
    s->config = config;
    s->capacity = token_capacity;
    s->owned_bytes = sizeof(*s) + 2 * kvb + rb + bkb + 2 * split_bytes;
    *out_state = s;
    return KQ_STATUS_OK;
}

void kq_qsa_state_close(kq_qsa_state *state) {
    if (state == nullptr) return;
    DeviceContext *c = context_for(state->device);
    if (c) {
        std::lock_guard<std::recursive_mutex> lk(c->mu);
        cudaStreamSynchronize(c->stream);
        c->dirty.erase(state);
    }
    cudaFree(state->key); cudaFree(state->value); cudaFree(state->raw); cudaFree(state->block_keys);
    cudaFree(state->key_split); cudaFree(state->value_split);
    state->magic = 0;
    delete state;
}

kq_status kq_qsa_state_reset(kq_qsa_state *state, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!state_valid(state)) return fail(diagnostic, KQ_STATUS_INVALID_QSA_STATE, "valid QSA state is required for reset");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    state->length = 0;
    state->bk_valid = 0;
    state->on_success();
    return KQ_STATUS_OK;
}

uint64_t kq_qsa_state_length(const kq_qsa_state *s) { return state_valid(s) ? s->length : 0; }
uint64_t kq_qsa_state_capacity(const kq_qsa_state *s) { return state_valid(s) ? s->capacity : 0; }
uint64_t kq_qsa_state_owned_bytes(const kq_qsa_state *s) { return state_valid(s) ? s->owned_bytes : 0; }

kq_status kq_qsa_state_export_f32(const kq_qsa_state *state, float *key_cache, uint64_t key_capacity,
                                  float *value_cache, uint64_t value_capacity, float *raw_cache,
                                  uint64_t raw_capacity, uint64_t *length, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    uint64_t kv_count, raw_count;
    if (!state_valid(state) || key_cache == nullptr || value_cache == nullptr || raw_cache == nullptr ||
        length == nullptr || !mul_ok(state->length, state->config->kv_per_token, &kv_count) ||
        !mul_ok(state->length, state->config->raw_per_token, &raw_count))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid QSA state and export buffers are required");
    if (key_capacity < kv_count || value_capacity < kv_count || raw_capacity < raw_count)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "QSA state export capacity is too small");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    if (kv_count) {
        KQB_CUDA(copy_sync(key_cache, state->key, kv_count * 4, cudaMemcpyDefault, c->stream), diagnostic,
                 "key export");
        KQB_CUDA(copy_sync(value_cache, state->value, kv_count * 4, cudaMemcpyDefault, c->stream), diagnostic,
                 "value export");
        KQB_CUDA(copy_sync(raw_cache, state->raw, raw_count * 4, cudaMemcpyDefault, c->stream), diagnostic,
                 "raw export");
    }
    *length = state->length;
    return KQ_STATUS_OK;
}

// The hi / lo copies of imported K / V rows (the appends of later calls
// write their own).
static void split_imported_rows(kq_qsa_state *s, uint64_t length, cudaStream_t stream) {
    if (s->key_split == nullptr || length == 0) return;
    const uint32_t kvh = s->config->dims.key_value_head_count;
    launch_qsa_split_rows(s->key, s->key_split, length, kvh, s->capacity, stream);
    launch_qsa_split_rows(s->value, s->value_split, length, kvh, s->capacity, stream);
}

kq_status kq_qsa_state_import_f32(kq_qsa_state *state, const float *key_cache, uint64_t key_count,
                                  const float *value_cache, uint64_t value_count, const float *raw_cache,
                                  uint64_t raw_count, uint64_t length, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    uint64_t ekv, eraw;
    if (!state_valid(state) || key_cache == nullptr || value_cache == nullptr || raw_cache == nullptr ||
        length > state->capacity || !mul_ok(length, state->config->kv_per_token, &ekv) ||
        !mul_ok(length, state->config->raw_per_token, &eraw))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid bounded QSA import arguments are required");
    if (key_count != ekv || value_count != ekv || raw_count != eraw)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "QSA imported cache shape does not match length");
    if (state->config->dims.activation_dtype == KQ_QSA_ACTIVATION_F32 && ekv &&
        is_device_pointer(key_cache) && is_device_pointer(value_cache) && is_device_pointer(raw_cache)) {
        // device-resident caches: validate and copy on the device
        DeviceContext *c;
        kq_status st = context(&c, diagnostic);
        if (st != KQ_STATUS_OK) return st;
        std::lock_guard<std::recursive_mutex> lk(c->mu);
        c->synchronize(nullptr);
        ErrorWord err = c->begin_call();
        launch_check_finite(key_cache, ekv, err, c->stream);
        launch_check_finite(value_cache, ekv, err, c->stream);
        launch_check_finite(raw_cache, eraw, err, c->stream);
        if (c->synchronize(nullptr) != KQ_STATUS_OK)
            return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "QSA imported K/V state must be finite");
        // ordered on the library stream, and complete before the caller's
        // buffers may be reused
        KQB_CUDA(cudaMemcpyAsync(state->key, key_cache, ekv * 4, cudaMemcpyDeviceToDevice, c->stream), diagnostic,
                 "import");
        KQB_CUDA(cudaMemcpyAsync(state->value, value_cache, ekv * 4, cudaMemcpyDeviceToDevice, c->stream),
                 diagnostic, "import");
        KQB_CUDA(cudaMemcpyAsync(state->raw, raw_cache, eraw * 4, cudaMemcpyDeviceToDevice, c->stream), diagnostic,
                 "import");
        split_imported_rows(state, length, c->stream);
        KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "import");
        state->bk_valid = 0;
        state->length = length;
        state->on_success();
        return KQ_STATUS_OK;
    }
    std::vector<float> kh(ekv), vh(ekv), rh(eraw);
    if (ekv) {
        KQB_CUDA(cudaMemcpy(kh.data(), key_cache, ekv * 4, cudaMemcpyDefault), diagnostic, "import");
        KQB_CUDA(cudaMemcpy(vh.data(), value_cache, ekv * 4, cudaMemcpyDefault), diagnostic, "import");
    }
    if (eraw) KQB_CUDA(cudaMemcpy(rh.data(), raw_cache, eraw * 4, cudaMemcpyDefault), diagnostic, "import");
    for (uint64_t i = 0; i < ekv; ++i)
        if (!std::isfinite(kh[i]) || !std::isfinite(vh[i]))
            return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "QSA imported K/V state must be finite");
    for (uint64_t i = 0; i < eraw; ++i)
        if (!std::isfinite(rh[i])) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "QSA imported index state must be finite");
    if (state->config->dims.activation_dtype == KQ_QSA_ACTIVATION_BF16) {
        auto round = [](float v) {
            uint32_t bits;
            std::memcpy(&bits, &v, 4);
            bits = ((bits + 0x7fffu + ((bits >> 16) & 1u)) >> 16) << 16;
            std::memcpy(&v, &bits, 4);
            return v;
        };
        for (auto &v : kh) v = round(v);
        for (auto &v : vh) v = round(v);
        for (auto &v : rh) v = round(v);
    }
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    c->synchronize(nullptr);
    if (ekv) {
        KQB_CUDA(copy_sync(state->key, kh.data(), ekv * 4, cudaMemcpyHostToDevice, c->stream), diagnostic, "import");
        KQB_CUDA(copy_sync(state->value, vh.data(), ekv * 4, cudaMemcpyHostToDevice, c->stream), diagnostic,
                 "import");
        KQB_CUDA(copy_sync(state->raw, rh.data(), eraw * 4, cudaMemcpyHostToDevice, c->stream), diagnostic,
                 "import");
        split_imported_rows(state, length, c->stream);
        KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "import");
    }
    // cached block keys are rebuilt from the imported raw keys by the next
    // call, which knows the index-key norm weights
    state->bk_valid = 0;
    state->length = length;
    state->on_success();
    return KQ_STATUS_OK;
}

kq_status kq_qsa_required_scratch_bytes(const kq_qsa_config *config, const kq_qsa_state *state,
                                        uint64_t sequence_length, uint64_t *scratch_bytes, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    return scratch_bytes_for(config, state, sequence_length, scratch_bytes, diagnostic);
}

// Stable top-k (src/kq_qsa_qwen38.c:361-392); host-side selection helper of
// the ABI, same insertion semantics.
kq_status kq_qsa_select_blocks_f32(const float *scores, uint64_t count, uint64_t limit, uint32_t *selected,
                                   uint64_t capacity, uint64_t *selected_count, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    uint64_t required = count < limit ? count : limit;
    if (selected_count == nullptr || limit == 0 || count > UINT32_MAX || (count != 0 && scores == nullptr) ||
        (required != 0 && selected == nullptr))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid bounded QSA selection arguments are required");
    *selected_count = 0;
    if (capacity < required) return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "QSA selected-block output is too small");
    for (uint64_t i = 0; i < count; ++i)
        if (!std::isfinite(scores[i])) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "QSA candidate scores must be finite");
    // order by (score desc, id asc) and keep the first `required`
    std::vector<uint32_t> ids(count);
    for (uint64_t i = 0; i < count; ++i) ids[i] = (uint32_t)i;
    std::stable_sort(ids.begin(), ids.end(), [&](uint32_t a, uint32_t b) { return scores[a] > scores[b]; });
    for (uint64_t i = 0; i < required; ++i) selected[i] = ids[i];
    *selected_count = required;
    return KQ_STATUS_OK;
}

kq_status kq_qsa_prefill_f32(const kq_qsa_config *config, const kq_qsa_weights_f32 *weights,
                             const float *hidden_states, uint64_t sequence_length, float *output,
                             uint64_t output_capacity, kq_qsa_state *state, void *scratch, uint64_t scratch_bytes,
                             kq_qsa_selection_observer selection_observer,
                             kq_qsa_checkpoint_observer checkpoint_observer, void *observer_user_data,
                             kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    kq_status st = validate_call(config, weights, hidden_states, sequence_length, output, output_capacity, state,
                                 scratch, scratch_bytes, false, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    return qsa_execute_sync(config, nullptr, weights, hidden_states, sequence_length, output, state,
                            selection_observer, checkpoint_observer, observer_user_data, diagnostic);
}

kq_status kq_qsa_decode_f32(const kq_qsa_config *config, const kq_qsa_weights_f32 *weights,
                            const float *hidden_token, float *output_token, uint64_t output_capacity,
                            kq_qsa_state *state, void *scratch, uint64_t scratch_bytes,
                            kq_qsa_selection_observer selection_observer,
                            kq_qsa_checkpoint_observer checkpoint_observer, void *observer_user_data,
                            kq_diagnostic *diagnostic) {
    return kq_qsa_prefill_f32(config, weights, hidden_token, 1, output_token, output_capacity, state, scratch,
                              scratch_bytes, selection_observer, checkpoint_observer, observer_user_data,
                              diagnostic);
}

kq_status kq_qsa_execute_quantized(const kq_qsa_config *config, kq_weight_provider *provider,
                                   const float *hidden_states, uint64_t sequence_length, float *output,
                                   uint64_t output_capacity, kq_qsa_state *state, void *scratch,
                                   uint64_t scratch_bytes, void *weight_scratch, uint64_t weight_scratch_bytes,
                                   kq_qsa_selection_observer selection_observer,
                                   kq_qsa_checkpoint_observer checkpoint_observer, void *observer_user_data,
                                   kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid compatible QSA call arguments are required");
    const uint64_t vec = 2ull * config->dims.head_dimension + 2ull * config->dims.index_head_dimension;
    const uint64_t need = vec * 4 + (uint64_t)config->dims.head_dimension * 4 + 65536;
    if (provider == nullptr || weight_scratch == nullptr || weight_scratch_bytes < need)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "QSA provider weight scratch is too small");
    kq_status st = validate_call(config, nullptr, hidden_states, sequence_length, output, output_capacity, state,
                                 scratch, scratch_bytes, true, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (!config->bound || config->provider != provider)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "required QSA semantic tensor is missing");
    QsaResolved w{config->q, config->k, config->v, config->o, config->iq, config->ik,
                  config->q_norm, config->k_norm, config->iq_norm, config->ik_norm};
    return qsa_execute_sync(config, &w, nullptr, hidden_states, sequence_length, output, state, selection_observer,
                            checkpoint_observer, observer_user_data, diagnostic);
}

kq_status kq_b200_qsa_decode_batch(const kq_qsa_config *config, kq_qsa_state *const *states, uint32_t batch,
                                   const float *hidden, float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (!config_valid(config) || states == nullptr || batch == 0 || hidden == nullptr || output == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, states and device buffers are required");
    if (config->dims.activation_dtype != KQ_QSA_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_QSA, "batched decode requires an F32 configuration");
    if (!config->bound)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    for (uint32_t b = 0; b < batch; ++b) {
        if (!state_valid(states[b]) || states[b]->config != config)
            return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "every state must belong to the config");
        if (states[b]->length + 1 > states[b]->capacity)
            return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, "QSA sequence exceeds bounded state capacity");
        for (uint32_t o = 0; o < b; ++o)
            if (states[o] == states[b]) return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "states must be distinct");
    }
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    QsaResolved w{config->q, config->k, config->v, config->o, config->iq, config->ik,
                  config->q_norm, config->k_norm, config->iq_norm, config->ik_norm};
    ErrorWord err = c->begin_call();
    return qsa_enqueue(c, config, w, states, batch, 1, hidden, output, err, nullptr, diagnostic,
                       /*check_input=*/true);
}

kq_status kq_b200_qsa_prefill_async(const kq_qsa_config *config, kq_qsa_state *state, const float *hidden,
                                    uint64_t T, float *output, kq_diagnostic *diagnostic) {
    return kq_b200_qsa_prefill_sharded_async(config, state, hidden, T, output, 0, 1, nullptr, nullptr, diagnostic);
}

kq_status kq_b200_qsa_prefill_sharded_async(const kq_qsa_config *config, kq_qsa_state *state, const float *hidden,
                                            uint64_t T, float *output, uint32_t rank, uint32_t world,
                                            kq_b200_exchange_fn exchange, void *user, kq_diagnostic *diagnostic) {
    return kq_b200_qsa_prefill_split_async(config, state, hidden, T, output, rank, world, 0, 1, exchange, user,
                                           diagnostic);
}

kq_status kq_b200_qsa_prefill_split_async(const kq_qsa_config *config, kq_qsa_state *state, const float *hidden,
                                          uint64_t T, float *output, uint32_t rank, uint32_t world,
                                          uint32_t token_part, uint32_t token_parts, kq_b200_exchange_fn exchange,
                                          void *user, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (world == 0 || rank >= world || (world > 1 && exchange == nullptr))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "rank < world and an exchange function are required");
    if (token_parts == 0 || token_part >= token_parts || (token_parts > 1 && world == 1))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "token_part < token_parts (split only across ranks)");
    if (!config_valid(config) || !state_valid(state) || state->config != config || hidden == nullptr ||
        output == nullptr || T == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid config, state and device buffers are required");
    if (config->dims.activation_dtype != KQ_QSA_ACTIVATION_F32)
        return fail(diagnostic, KQ_STATUS_INCOMPATIBLE_QSA, "device prefill requires an F32 configuration");
    if (!config->bound)
        return fail(diagnostic, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "config has no bound provider weights");
    uint64_t total;
    if (!add_ok(state->length, T, &total) || total > state->capacity || T > UINT32_MAX)
        return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, "QSA sequence exceeds bounded state capacity");
    if (!is_device_pointer(hidden) || !is_device_pointer(output))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "device prefill takes device buffers");
    DeviceContext *c;
    kq_status st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    QsaResolved w{config->q, config->k, config->v, config->o, config->iq, config->ik,
                  config->q_norm, config->k_norm, config->iq_norm, config->ik_norm};
    ErrorWord err = c->begin_call();
    kq_qsa_state *states[1] = {state};
    TokenShard shard;
    shard.rank = rank;
    shard.world = world;
    shard.exchange = exchange;
    shard.user = user;
    shard.part = token_part;
    shard.parts = token_parts;
    return qsa_enqueue(c, config, w, states, 1, (uint32_t)T, hidden, output, err, nullptr, diagnostic,
                       /*check_input=*/true, &shard);
}

const char *kq_qsa_checkpoint_kind_name(kq_qsa_checkpoint_kind kind) {
    static const char *names[] = {"INDEX_QUERY", "RAW_INDEX_KEY", "BLOCK_KEYS", "CANDIDATE_SCORES", "QUERY", "KEY",
                                  "VALUE", "ATTENTION_LOGITS", "ATTENTION_PROBABILITIES", "HEAD_CONTEXT",
                                  "GATED_CONTEXT", "OPERATOR_OUTPUT"};
    if ((uint32_t)kind >= sizeof(names) / sizeof(names[0])) return "UNKNOWN";
    return names[(uint32_t)kind];
}

}  // extern "C"

// ---------------------------------------------------------------- layer bridge

namespace kqb {

kq_status qsa_layer_enqueue(DeviceContext *c, const kq_qsa_config *cfg, const kq_qsa_weights_f32 *wf,
                            kq_qsa_state *const *states, uint32_t batch, uint32_t tokens, const float *x, float *y,
                            ErrorWord err, kq_diagnostic *diag) {
    if (!config_valid(cfg) || states == nullptr || batch == 0 || tokens == 0 || (batch > 1 && tokens > 1))
        return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "valid compatible QSA call arguments are required");
    if (cfg->dims.activation_dtype != KQ_QSA_ACTIVATION_F32)
        return fail(diag, KQ_STATUS_INCOMPATIBLE_QSA, "scalar execution requires an F32 QSA reference config");
    for (uint32_t b = 0; b < batch; ++b) {
        if (!state_valid(states[b]) || states[b]->config != cfg)
            return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "every state must belong to the config");
        if (states[b]->length + tokens > states[b]->capacity)
            return fail(diag, KQ_STATUS_LIMIT_EXCEEDED, "QSA sequence exceeds bounded state capacity or overflows");
    }
    QsaResolved w;
    if (wf != nullptr) {
        const kq_qsa_dimensions &d = cfg->dims;
        const uint64_t qw = (uint64_t)d.query_head_count * d.head_dimension, H = d.hidden_size;
        const float *ptrs[10] = {wf->query, wf->key, wf->value, wf->output, wf->query_norm, wf->key_norm,
                                 wf->index_query, wf->index_key, wf->index_query_norm, wf->index_key_norm};
        const uint64_t have[10] = {wf->query_count, wf->key_count, wf->value_count, wf->output_count,
                                   wf->query_norm_count, wf->key_norm_count, wf->index_query_count,
                                   wf->index_key_count, wf->index_query_norm_count, wf->index_key_norm_count};
        const uint64_t want[10] = {2 * qw * H, cfg->kv_per_token * H, cfg->kv_per_token * H, H * qw,
                                   d.head_dimension, d.head_dimension,
                                   (uint64_t)d.index_query_head_count * d.index_head_dimension * H,
                                   (uint64_t)d.index_head_dimension * H, d.index_head_dimension, d.index_head_dimension};
        for (int i = 0; i < 10; ++i) {
            if (have[i] != want[i]) return fail(diag, KQ_STATUS_DIMENSION_MISMATCH, "QSA F32 weight shape mismatch");
            if (ptrs[i] == nullptr) return fail(diag, KQ_STATUS_INVALID_ARGUMENT, "QSA F32 weights are required");
        }
        kq_status st = resolve_f32(c, cfg, wf, err, &w, diag);
        if (st != KQ_STATUS_OK) return st;
        for (uint32_t b = 0; b < batch; ++b) {
            st = sync_block_key_norm(cfg, w, states[b], diag);
            if (st != KQ_STATUS_OK) return st;
        }
    } else {
        if (!cfg->bound)
            return fail(diag, KQ_STATUS_SEMANTIC_MAPPING_FAILED, "QSA provider matrix semantic is missing");
        w = QsaResolved{cfg->q, cfg->k, cfg->v, cfg->o, cfg->iq, cfg->ik, cfg->q_norm, cfg->k_norm, cfg->iq_norm,
                        cfg->ik_norm};
    }
    return qsa_enqueue(c, cfg, w, states, batch, tokens, x, y, err, nullptr, diag);
}

uint64_t qsa_state_committed_length(const kq_qsa_state *s) { return s->length; }

void qsa_state_truncate(kq_qsa_state *s, uint64_t length) {
    if (length < s->length) {
        s->length = length;
        s->bk_valid = std::min<uint64_t>(s->bk_valid, length / s->config->dims.block_size);
    }
    s->on_success();
}

}  // namespace kqb
