/*
 * kq_oracle — CPU restatement of Kestrel-Q's GDN / QSA / MoE / GGUF-dequant hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This code is the checker for the B200 kernels: it
 * is loaded by tests/, by __graft_entry__.smoke() and by bench.py's
 * cpu_baseline leg, never by the product library.  Every function restates the
 * reference's scalar C with the same operation order (compiled with
 * -fno-fast-math -ffp-contract=off) so that its results are bit-identical to
 * the reference's own operators; tests/test_oracle_pin.py checks that against
 * the reference compiled from source (oracle/_ref) and against the reference's
 * golden vectors (tests/golden/).
 *
 * Q6_K is absent from the reference (src/kq_gguf.c:57-65 of Kestrel-Q); its
 * decoder here is restated from the public GGUF block format and is the only
 * part whose parity is pinned by this restatement alone.
 */
#ifndef KQ_ORACLE_H
#define KQ_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    KQO_OK = 0,
    KQO_INVALID_ARGUMENT = 1,
    KQO_NUMERIC_DOMAIN = 2,
    KQO_UNSUPPORTED_TYPE = 3,
    KQO_LIMIT_EXCEEDED = 4
};

/* GGUF type ids (src/kq_gguf.c:57-65 of Kestrel-Q, plus Q6_K = 14). */
enum {
    KQO_TYPE_F32 = 0,
    KQO_TYPE_Q8_0 = 8,
    KQO_TYPE_Q4_K = 12,
    KQO_TYPE_Q6_K = 14,
    KQO_TYPE_BF16 = 30
};

int kqo_block_geometry(uint32_t type_id, uint64_t *block_elements,
                       uint64_t *bytes_per_block);
int kqo_dequantize(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                   float *output, uint64_t output_capacity);
int kqo_row_dot(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                const float *activation, uint64_t count, float *output);
/* rows x cols matrix of packed rows; y[b*rows + r] for each of `batch` inputs. */
int kqo_matvec(uint32_t type_id, const void *packed, uint64_t rows,
               uint64_t cols, const float *x, uint64_t batch, float *y);

typedef struct kqo_gdn_dims {
    uint32_t hidden_size;
    uint32_t key_heads;
    uint32_t value_heads;
    uint32_t key_dim;
    uint32_t value_dim;
    uint32_t conv_kernel;
    float rms_norm_epsilon;
} kqo_gdn_dims;

typedef struct kqo_gdn_weights {
    const float *a_log;    /* [Hv] */
    const float *conv;     /* [C][K] */
    const float *dt_bias;  /* [Hv] */
    const float *alpha;    /* [Hv][H] */
    const float *beta;     /* [Hv][H] */
    const float *qkv;      /* [C][H] */
    const float *gate;     /* [Hv*dv][H] */
    const float *norm;     /* [dv] */
    const float *output;   /* [H][Hv*dv] */
} kqo_gdn_weights;

/* Checkpoint callback of the observed runs: `kind` is the operator's
 * checkpoint enumerator (kq_gdn_checkpoint_kind / kq_qsa_checkpoint_kind of
 * the reference headers), emitted in the reference's order with its rank and
 * dimensions (src/kq_gdn_qwen38.c:248-271, src/kq_qsa_qwen38.c:309-330). */
typedef void (*kqo_checkpoint_fn)(uint32_t kind, uint64_t token, uint32_t rank, const uint64_t *dims,
                                  const float *values, uint64_t count, void *user);

/* Runs T tokens; conv_state [C*K] and recurrent_state [Hv*dk*dv] are updated
 * in place only on success (the reference's transactional contract). */
int kqo_gdn_run(const kqo_gdn_dims *dims, const kqo_gdn_weights *weights,
                const float *hidden, uint64_t tokens, const uint8_t *mask,
                float *output, float *conv_state, float *recurrent_state);
/* kqo_gdn_run with the reference's 21 checkpoints per token sent to `cb`. */
int kqo_gdn_run_observed(const kqo_gdn_dims *dims, const kqo_gdn_weights *weights,
                         const float *hidden, uint64_t tokens, const uint8_t *mask,
                         float *output, float *conv_state, float *recurrent_state,
                         kqo_checkpoint_fn cb, void *user);

typedef struct kqo_qsa_dims {
    uint32_t hidden_size;
    uint32_t query_heads;
    uint32_t kv_heads;
    uint32_t head_dim;
    uint32_t index_heads;
    uint32_t index_dim;
    uint32_t block_size;
    uint32_t token_budget;
    uint32_t rotary_dim;
    float rms_norm_epsilon;
    float rope_theta;
} kqo_qsa_dims;

typedef struct kqo_qsa_weights {
    const float *query;       /* [Hq][2][d] rows x H (q, gate interleaved) */
    const float *key;         /* [Hkv*d][H] */
    const float *value;       /* [Hkv*d][H] */
    const float *output;      /* [H][Hq*d] */
    const float *query_norm;  /* [d] (1+w form) */
    const float *key_norm;    /* [d] */
    const float *index_query; /* [Hi*di][H] */
    const float *index_key;   /* [di][H] */
    const float *index_query_norm; /* [di] */
    const float *index_key_norm;   /* [di] */
} kqo_qsa_weights;

/* Caches are [capacity][Hkv*d] (K, V) and [capacity][di] (raw index keys);
 * *length is advanced only on success.  Optional per-token selection outputs:
 * selected_ids [T][budget/block], selected_counts [T], scores
 * [T][capacity/block] (candidate scores of the complete blocks). */
int kqo_qsa_run(const kqo_qsa_dims *dims, const kqo_qsa_weights *weights,
                const float *hidden, uint64_t tokens, float *output,
                float *key_cache, float *value_cache, float *raw_cache,
                uint64_t capacity, uint64_t *length,
                uint32_t *selected_ids, uint32_t *selected_counts,
                float *scores);
/* kqo_qsa_run with the reference's 12 checkpoints per token sent to `cb`. */
int kqo_qsa_run_observed(const kqo_qsa_dims *dims, const kqo_qsa_weights *weights,
                         const float *hidden, uint64_t tokens, float *output,
                         float *key_cache, float *value_cache, float *raw_cache,
                         uint64_t capacity, uint64_t *length,
                         uint32_t *selected_ids, uint32_t *selected_counts,
                         float *scores, kqo_checkpoint_fn cb, void *user);

typedef struct kqo_moe_dims {
    uint32_t hidden_size;
    uint32_t expert_count;
    uint32_t top_k;
    uint32_t routed_intermediate_size;
    uint32_t shared_intermediate_size;
} kqo_moe_dims;

typedef struct kqo_moe_weights {
    const float *router;             /* [E][H] */
    const float *routed_gate;        /* [E][I][H] */
    const float *routed_up;          /* [E][I][H] */
    const float *routed_down;        /* [E][H][I] */
    const float *shared_gate;        /* [S][H] */
    const float *shared_up;          /* [S][H] */
    const float *shared_down;        /* [H][S] */
    const float *shared_gate_weight; /* [H] */
} kqo_moe_weights;

/* MoE checkpoint callback: kind is kq_moe_checkpoint_kind (include/kq_moe.h
 * of the reference); expert and position are UINT32_MAX for token-level
 * checkpoints. */
typedef void (*kqo_moe_checkpoint_fn)(uint32_t kind, uint64_t token, uint32_t expert, uint32_t position,
                                      uint32_t rank, const uint64_t *dims, const float *values, uint64_t count,
                                      void *user);

/* T tokens through router, top-k experts and the gated shared expert
 * (src/kq_moe_qwen38.c:604-867).  Optional per-token route outputs:
 * logits [T][E], probabilities [T][E], selected ids [T][K] (top-k order) and
 * renormalised weights [T][K]. */
int kqo_moe_run(const kqo_moe_dims *dims, const kqo_moe_weights *weights, const float *hidden,
                uint64_t tokens, float *output, float *logits, float *probabilities, uint32_t *selected_ids,
                float *selected_weights);
int kqo_moe_run_observed(const kqo_moe_dims *dims, const kqo_moe_weights *weights, const float *hidden,
                         uint64_t tokens, float *output, float *logits, float *probabilities,
                         uint32_t *selected_ids, float *selected_weights, kqo_moe_checkpoint_fn cb, void *user);

typedef struct kqo_layer_dims {
    uint32_t hidden_size;
    uint32_t branch_count;
    uint32_t gr_rank;
    float rms_epsilon;
    uint32_t family;   /* 1 GDN, 2 QSA (kq_layer_family) */
} kqo_layer_dims;

typedef struct kqo_gr_weights {
    const float *norm;    /* [B*H] (1 + w form) */
    const float *down;    /* [R][B*H] */
    const float *up;      /* [B*H][R] */
    const float *inject;  /* [B][B*H] */
} kqo_gr_weights;

/* One decoder layer (gated residual, GDN or QSA mixer, gated residual, MoE)
 * over T tokens of [B][H] branches: src/kq_layer.c:639-827 without PLE.
 * Pass the GDN arguments (and NULL QSA ones) for family 1, the QSA ones for
 * family 2; state arrays and *length change only on success. */
int kqo_layer_run_observed(const kqo_layer_dims *dims, const kqo_gr_weights *attn_gr, const kqo_gr_weights *moe_gr,
                           const kqo_gdn_dims *gdn_dims, const kqo_gdn_weights *gdn_weights, float *conv_state,
                           float *recurrent_state, const kqo_qsa_dims *qsa_dims, const kqo_qsa_weights *qsa_weights,
                           float *key_cache, float *value_cache, float *raw_cache, uint64_t capacity,
                           uint64_t *length, const kqo_moe_dims *moe_dims, const kqo_moe_weights *moe_weights,
                           const float *input, uint64_t tokens, const uint8_t *mask, float *output,
                           kqo_checkpoint_fn cb, void *user);

/* Stable top-k by (score desc, id asc): src/kq_qsa_qwen38.c:328-359. */
uint64_t kqo_select_blocks(const float *scores, uint64_t count, uint64_t limit,
                           uint32_t *selected);

#ifdef __cplusplus
}
#endif

#endif
