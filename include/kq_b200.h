/*
 * kq_b200 — B200-specific additions to the Kestrel-Q operator ABI.
 *
 * Three groups of entry points:
 *
 *  1. Reference internals that the reference's layer code calls and that a
 *     drop-in therefore has to export (declared in Kestrel-Q's
 *     src/kq_gdn_internal.h and src/kq_qsa_internal.h):
 *       kq_gdn_test_config_create   src/kq_gdn_internal.h:61-64
 *       kq_gdn_execute_quantized    src/kq_gdn_internal.h:81-96
 *       kq_qsa_test_config_create   src/kq_qsa_internal.h:65-68
 *       kq_qsa_execute_quantized    src/kq_qsa_internal.h:94-102
 *       kq_moe_test_config_create   src/kq_moe_internal.h:45-48
 *       kq_moe_execute_quantized    src/kq_moe_internal.h:52-60
 *       kq_layer_test_config_create src/kq_layer_internal.h:73-77
 *       kq_layer_state_rollback_last src/kq_layer_internal.h:64-66
 *     The dimension records keep the reference's field order and types
 *     (src/kq_gdn_internal.h:11-20, src/kq_qsa_internal.h:11-25,
 *     src/kq_moe_internal.h:10-17, src/kq_layer_internal.h:9-16).
 *
 *  2. The device weight provider that stands in for the GGUF-backed one
 *     (src/kq_weight_provider.c:378-509): quantized GGUF blocks are uploaded
 *     once to HBM and are only ever dequantised in registers.
 *
 *  3. Asynchronous batched decode over device buffers, the serving path that
 *     the reference (batch 1, synchronous) has no counterpart for.
 *
 * Threading: every entry point takes a per-device lock; calls are ordered on
 * one CUDA stream per device (kq_b200_set_stream replaces it).
 */
#ifndef KQ_B200_H
#define KQ_B200_H

#include <stdint.h>

#include "kq_gdn.h"
#include "kq_layer.h"
#include "kq_model.h"
#include "kq_moe.h"
#include "kq_qsa.h"
#include "kq_status.h"
#include "kq_weight_provider.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- group 1 */

typedef struct kq_gdn_dimensions {
    uint32_t hidden_size;
    uint32_t key_head_count;
    uint32_t value_head_count;
    uint32_t key_head_dimension;
    uint32_t value_head_dimension;
    uint32_t conv_kernel_size;
    float rms_norm_epsilon;
    kq_gdn_activation_dtype activation_dtype;
} kq_gdn_dimensions;

typedef struct kq_qsa_dimensions {
    uint32_t hidden_size;
    uint32_t query_head_count;
    uint32_t key_value_head_count;
    uint32_t head_dimension;
    uint32_t index_query_head_count;
    uint32_t index_head_dimension;
    uint32_t block_size;
    uint32_t token_budget;
    uint32_t max_context;
    uint32_t rotary_dimension;
    float rms_norm_epsilon;
    float rope_theta;
    kq_qsa_activation_dtype activation_dtype;
} kq_qsa_dimensions;

typedef struct kq_moe_dimensions {
    uint32_t hidden_size;
    uint32_t expert_count;
    uint32_t top_k;
    uint32_t routed_intermediate_size;
    uint32_t shared_intermediate_size;
    kq_moe_activation_dtype activation_dtype;
} kq_moe_dimensions;

typedef struct kq_layer_dimensions {
    uint32_t layer_id;
    uint32_t hidden_size;
    uint32_t branch_count;
    uint32_t gr_rank;
    float rms_epsilon;
    kq_layer_family family;
} kq_layer_dimensions;

kq_status kq_gdn_test_config_create(const kq_gdn_dimensions *dimensions,
                                    kq_gdn_config **out_config,
                                    kq_diagnostic *diagnostic);
kq_status kq_qsa_test_config_create(const kq_qsa_dimensions *dimensions,
                                    kq_qsa_config **out_config,
                                    kq_diagnostic *diagnostic);

/* B200 limits on top of the reference's validation: top_k <= 32 and
 * expert_count <= 8192 (else KQ_STATUS_INCOMPATIBLE_MOE). */
kq_status kq_moe_test_config_create(const kq_moe_dimensions *dimensions,
                                    kq_moe_config **out_config,
                                    kq_diagnostic *diagnostic);

/* A layer over caller-owned sub-configs (closed by the caller after the
 * layer config): exactly one of gdn (families GDN) and qsa (QSA), and moe.
 * ple and ple_value must be NULL (the PLE_GDN family is refused with
 * KQ_STATUS_INCOMPATIBLE_LAYER). */
kq_status kq_layer_test_config_create(const kq_layer_dimensions *dimensions,
                                      kq_gdn_config *gdn,
                                      kq_qsa_config *qsa,
                                      kq_moe_config *moe,
                                      kq_ple_config *ple,
                                      kq_ple_value_config *ple_value,
                                      kq_layer_config **out_config,
                                      kq_diagnostic *diagnostic);

/* Undoes the state's last successful call of `token_count` tokens (once; a
 * second call, another count or a state without a commit is
 * KQ_STATUS_INVALID_LAYER_STATE). */
kq_status kq_layer_state_rollback_last(kq_layer_state *state,
                                       uint64_t token_count,
                                       kq_diagnostic *diagnostic);

/* Provider mode: weights are the tensors bound to the config with
 * kq_b200_gdn_config_bind / kq_b200_qsa_config_bind /
 * kq_b200_moe_config_bind.  weight_scratch keeps the reference's
 * minimum-size contract and is otherwise unused. */
kq_status kq_gdn_execute_quantized(const kq_gdn_config *config,
                                   kq_weight_provider *provider,
                                   const float *hidden_states,
                                   uint64_t sequence_length,
                                   const uint8_t *padding_mask,
                                   float *output,
                                   uint64_t output_capacity,
                                   kq_gdn_state *state,
                                   void *scratch,
                                   uint64_t scratch_bytes,
                                   void *weight_scratch,
                                   uint64_t weight_scratch_bytes,
                                   kq_gdn_checkpoint_observer observer,
                                   void *observer_user_data,
                                   kq_diagnostic *diagnostic);
kq_status kq_qsa_execute_quantized(const kq_qsa_config *config,
                                   kq_weight_provider *provider,
                                   const float *hidden_states,
                                   uint64_t sequence_length,
                                   float *output,
                                   uint64_t output_capacity,
                                   kq_qsa_state *state,
                                   void *scratch,
                                   uint64_t scratch_bytes,
                                   void *weight_scratch,
                                   uint64_t weight_scratch_bytes,
                                   kq_qsa_selection_observer selection_observer,
                                   kq_qsa_checkpoint_observer checkpoint_observer,
                                   void *observer_user_data,
                                   kq_diagnostic *diagnostic);

kq_status kq_moe_execute_quantized(const kq_moe_config *config,
                                   kq_weight_provider *provider,
                                   const float *hidden_states,
                                   uint64_t token_count,
                                   float *output,
                                   uint64_t output_capacity,
                                   void *scratch,
                                   uint64_t scratch_bytes,
                                   void *weight_scratch,
                                   uint64_t weight_scratch_bytes,
                                   kq_moe_route_observer route_observer,
                                   kq_moe_checkpoint_observer checkpoint_observer,
                                   void *observer_user_data,
                                   kq_diagnostic *diagnostic);

/* ---------------------------------------------------------------- group 2 */

/* Creates an empty device-resident provider on `device`. */
kq_status kq_b200_provider_create(int device,
                                  kq_weight_provider **out_provider,
                                  kq_diagnostic *diagnostic);

/* Uploads a rows x columns matrix stored as consecutive GGUF rows of
 * `type_id` blocks (F32, BF16, Q8_0, Q4_K or Q6_K; blocks run along the
 * columns).  `packed` is host memory of exactly rows * row_bytes bytes.
 * The returned descriptor is owned by the provider. */
kq_status kq_b200_provider_add_matrix(kq_weight_provider *provider,
                                      const char *semantic_id,
                                      kq_semantic_role role,
                                      uint32_t type_id,
                                      uint64_t rows,
                                      uint64_t columns,
                                      const void *packed,
                                      uint64_t packed_bytes,
                                      const kq_semantic_tensor **out_tensor,
                                      kq_diagnostic *diagnostic);

/* Uploads a small F32 vector (norm weights, conv taps, A_log, dt_bias). */
kq_status kq_b200_provider_add_vector_f32(kq_weight_provider *provider,
                                          const char *semantic_id,
                                          kq_semantic_role role,
                                          const float *values,
                                          uint64_t count,
                                          const kq_semantic_tensor **out_tensor,
                                          kq_diagnostic *diagnostic);

/* The model GGUF's storage of GDN tensors: value heads in tiled order (the
 * converter stores canonical value head g * R + r, key head g, as head
 * r * Hk + g).  The target model has 16 key heads, 3 value heads per key
 * head, 128 features per head. */
typedef struct kq_b200_gguf_layout {
    uint32_t gdn_key_heads;
    uint32_t gdn_value_repeat;
    uint32_t gdn_head_width;
} kq_b200_gguf_layout;

/* Uploads a matrix as the model's GGUF stores it and presents the canonical
 * tensor the operators read: the transforms of the reference provider
 * (src/kq_weight_provider.c:205-248,438-451) for `role`:
 *   KQ_ROLE_GDN_QKV    value rows (after the 2 Hk W q/k rows) reordered
 *   KQ_ROLE_GDN_GATE   rows reordered (head width W)
 *   KQ_ROLE_GDN_ALPHA, KQ_ROLE_GDN_BETA  rows reordered (one per head)
 *   KQ_ROLE_GDN_OUT    columns kept in tiled order: the GDN operator writes
 *                      its gated output in that order and the linear entry
 *                      points permute their canonical input
 *   other roles        stored as given (kq_b200_provider_add_matrix).
 * The allocation-free linear takes canonical-column tensors only. */
kq_status kq_b200_provider_add_gguf_matrix(kq_weight_provider *provider,
                                           const char *semantic_id,
                                           kq_semantic_role role,
                                           uint32_t type_id,
                                           uint64_t rows,
                                           uint64_t columns,
                                           const void *packed,
                                           uint64_t packed_bytes,
                                           const kq_b200_gguf_layout *layout,
                                           const kq_semantic_tensor **out_tensor,
                                           kq_diagnostic *diagnostic);

/* Uploads an F32 vector as the model's GGUF stores it, presented canonical
 * (src/kq_weight_provider.c:680-717): KQ_ROLE_GDN_A_LOG stored as -exp(A_log)
 * (canonical = logf(-stored), heads reordered), KQ_ROLE_GDN_DT_BIAS heads
 * reordered, KQ_ROLE_GDN_CONV channels reordered like the qkv rows, the QSA
 * q/k and index q/k norms stored as 1 + delta (canonical = stored - 1). */
kq_status kq_b200_provider_add_gguf_vector_f32(kq_weight_provider *provider,
                                               const char *semantic_id,
                                               kq_semantic_role role,
                                               const float *values,
                                               uint64_t count,
                                               const kq_b200_gguf_layout *layout,
                                               const kq_semantic_tensor **out_tensor,
                                               kq_diagnostic *diagnostic);

/* Uploads the QSA index projection the way the model's GGUF splits it: one
 * KQ_ROLE_QSA_INDEX_QK semantic with an INDEX_QUERY part (query_rows rows)
 * and an INDEX_KEY part (key_rows rows), in that order (src/kq_qsa.c:184-201).
 * kq_weight_provider_linear_f32 reads a part by its part role; pass the
 * semantic as both index_query and index_key of kq_b200_qsa_tensors. */
kq_status kq_b200_provider_add_index_qk(kq_weight_provider *provider,
                                        const char *semantic_id,
                                        uint32_t type_id,
                                        uint64_t query_rows,
                                        uint64_t key_rows,
                                        uint64_t columns,
                                        const void *query_packed,
                                        uint64_t query_bytes,
                                        const void *key_packed,
                                        uint64_t key_bytes,
                                        const kq_semantic_tensor **out_tensor,
                                        kq_diagnostic *diagnostic);

/* Uploads a routed-expert stack: `experts` matrices of rows x columns GGUF
 * rows, expert-major (the model GGUF's [experts][rows][columns] tensor,
 * e.g. blk.N.ffn_down_exps).  kq_weight_provider_linear_f32 reads one
 * expert's matrix by its expert id. */
kq_status kq_b200_provider_add_expert_stack(kq_weight_provider *provider,
                                            const char *semantic_id,
                                            kq_semantic_role role,
                                            uint32_t type_id,
                                            uint32_t experts,
                                            uint64_t rows,
                                            uint64_t columns,
                                            const void *packed,
                                            uint64_t packed_bytes,
                                            const kq_semantic_tensor **out_tensor,
                                            kq_diagnostic *diagnostic);

/* Uploads the routed gate/up projection the way the model's GGUF splits it:
 * one KQ_ROLE_ROUTED_GATE_UP semantic with a GATE part (ffn_gate_exps) and
 * an UP part (ffn_up_exps), each an expert stack of rows x columns
 * matrices (src/kq_model.c:1055-1096).  kq_weight_provider_linear_f32 reads
 * a part by its part role and expert id. */
kq_status kq_b200_provider_add_expert_gate_up(kq_weight_provider *provider,
                                             const char *semantic_id,
                                             uint32_t type_id,
                                             uint32_t experts,
                                             uint64_t rows,
                                             uint64_t columns,
                                             const void *gate_packed,
                                             uint64_t gate_bytes,
                                             const void *up_packed,
                                             uint64_t up_bytes,
                                             const kq_semantic_tensor **out_tensor,
                                             kq_diagnostic *diagnostic);

/* Batched form of kq_weight_provider_linear_f32:
 * y[b][r] = sum_c W[r][c] * x[b][c] for b < batch, with x [batch][columns]
 * and y [batch][rows] device arrays.  Batches above 8 run on the tensor
 * cores (three-term BF16 split, F32 accumulate); smaller ones on a warp
 * GEMV.  Asynchronous on the library stream (see kq_b200_synchronize). */
kq_status kq_b200_provider_linear_batch_f32(kq_weight_provider *provider,
                                            const kq_semantic_tensor *semantic,
                                            uint64_t rows,
                                            uint64_t columns,
                                            const float *x,
                                            uint32_t batch,
                                            float *y,
                                            kq_diagnostic *diagnostic);

/* Allocation-free form of kq_b200_provider_linear_batch_f32; it has no
 * counterpart in the reference.  For callers that cannot call cudaMalloc:
 * a serving loop whose HBM is fully committed (KV cache, fixed budget), a
 * host framework whose caching allocator owns device memory, or a
 * latency-bound loop where cudaMalloc/cudaFree would synchronise the device.
 * It allocates nothing: its scratch is one 4 MiB array compiled into the
 * library (held on every GPU that loads it until exit), and it calls no
 * cudaMalloc, cudaFree or other allocating routine.
 *   - Limit: on the tensor-core path (batches above 8, weight types it
 *     covers) a call needs ceil(batch/64) * ceil(columns/64) * 16 KiB of
 *     activation tiles, at most 4 MiB - 256 B; larger calls return
 *     KQ_STATUS_LIMIT_EXCEEDED.  The warp GEMV (batches up to 8) and the
 *     CUDA-core tiles use no scratch and have no such limit.
 *   - Runs on `cuda_stream` (NULL: the legacy default stream) and waits for
 *     it before returning, so non-finite input is reported by this call
 *     (KQ_STATUS_NUMERIC_DOMAIN).
 *   - kq_b200_provider_create looks up the array's device address on its
 *     device (cudaGetSymbolAddress), which makes the driver load the array
 *     there: create the provider before committing the rest of HBM.
 *   - Every call on a device shares the array (the last call's contents
 *     stay in it, and its first word is the call's error word): calls whose
 *     kernels overlap on the GPU race, on the tiles and on that word, so one
 *     such call can also report another's KQ_STATUS_NUMERIC_DOMAIN.
 * The caller's current device is restored on return. */
kq_status kq_b200_provider_linear_batch_f32_static(kq_weight_provider *provider,
                                                   const kq_semantic_tensor *semantic,
                                                   uint64_t rows,
                                                   uint64_t columns,
                                                   const float *x,
                                                   uint32_t batch,
                                                   float *y,
                                                   void *cuda_stream,
                                                   kq_diagnostic *diagnostic);

typedef struct kq_b200_gdn_tensors {
    const kq_semantic_tensor *a_log;    /* F32 [Hv] */
    const kq_semantic_tensor *conv;     /* F32 [C*K] */
    const kq_semantic_tensor *dt_bias;  /* F32 [Hv] */
    const kq_semantic_tensor *alpha;    /* matrix [Hv x H] */
    const kq_semantic_tensor *beta;     /* matrix [Hv x H] */
    const kq_semantic_tensor *qkv;      /* matrix [C x H] */
    const kq_semantic_tensor *gate;     /* matrix [Hv*dv x H] */
    const kq_semantic_tensor *norm;     /* F32 [dv] */
    const kq_semantic_tensor *output;   /* matrix [H x Hv*dv] */
} kq_b200_gdn_tensors;

/* MoE weights in the reference's role order (src/kq_moe.c:27-54). */
typedef struct kq_b200_moe_tensors {
    const kq_semantic_tensor *router;             /* matrix [E x H] */
    const kq_semantic_tensor *routed_down;        /* expert stack [E][H x I] */
    const kq_semantic_tensor *routed_gate_up;     /* gate/up expert stacks [E][I x H] */
    const kq_semantic_tensor *shared_down;        /* matrix [H x S] */
    const kq_semantic_tensor *shared_gate;        /* matrix [S x H] */
    const kq_semantic_tensor *shared_up;          /* matrix [S x H] */
    const kq_semantic_tensor *shared_gate_weight; /* matrix [1 x H] */
} kq_b200_moe_tensors;

typedef struct kq_b200_qsa_tensors {
    const kq_semantic_tensor *query;            /* [2*Hq*d x H], q/gate interleaved per head */
    const kq_semantic_tensor *key;              /* [Hkv*d x H] */
    const kq_semantic_tensor *value;            /* [Hkv*d x H] */
    const kq_semantic_tensor *output;           /* [H x Hq*d] */
    const kq_semantic_tensor *query_norm;       /* F32 [d], (1+w) form */
    const kq_semantic_tensor *key_norm;         /* F32 [d] */
    const kq_semantic_tensor *index_query;      /* [Hi*di x H] */
    const kq_semantic_tensor *index_key;        /* [di x H] */
    const kq_semantic_tensor *index_query_norm; /* F32 [di] */
    const kq_semantic_tensor *index_key_norm;   /* F32 [di] */
} kq_b200_qsa_tensors;

/* Gated-residual tensors of a layer in the reference's binding order
 * (src/kq_layer.c:100-120): per side inject [B x W], norm F32 vector [W]
 * (1 + w form), down [rank x W], up [W x rank]. */
typedef struct kq_b200_layer_tensors {
    const kq_semantic_tensor *attention_inject;
    const kq_semantic_tensor *attention_norm;
    const kq_semantic_tensor *attention_down;
    const kq_semantic_tensor *attention_up;
    const kq_semantic_tensor *moe_inject;
    const kq_semantic_tensor *moe_norm;
    const kq_semantic_tensor *moe_down;
    const kq_semantic_tensor *moe_up;
} kq_b200_layer_tensors;

/* Binds provider tensors to a config (what kq_*_config_create does from a
 * GGUF model in the reference).  Shapes are validated against the config. */
kq_status kq_b200_gdn_config_bind(kq_gdn_config *config,
                                  kq_weight_provider *provider,
                                  const kq_b200_gdn_tensors *tensors,
                                  kq_diagnostic *diagnostic);
kq_status kq_b200_qsa_config_bind(kq_qsa_config *config,
                                  kq_weight_provider *provider,
                                  const kq_b200_qsa_tensors *tensors,
                                  kq_diagnostic *diagnostic);
kq_status kq_b200_moe_config_bind(kq_moe_config *config,
                                  kq_weight_provider *provider,
                                  const kq_b200_moe_tensors *tensors,
                                  kq_diagnostic *diagnostic);
/* The layer's gated-residual tensors; its mixer and MoE configs are bound
 * to the same provider with their own bind calls. */
kq_status kq_b200_layer_config_bind(kq_layer_config *config,
                                    kq_weight_provider *provider,
                                    const kq_b200_layer_tensors *tensors,
                                    kq_diagnostic *diagnostic);

/* ---------------------------------------------------------------- group 3 */

/* Selects the device used by subsequently created objects (default 0). */
kq_status kq_b200_set_device(int device, kq_diagnostic *diagnostic);
/* Replaces the library's stream on the current device (cudaStream_t, or
 * NULL to restore the library's own non-blocking stream). */
kq_status kq_b200_set_stream(void *cuda_stream, kq_diagnostic *diagnostic);
void *kq_b200_get_stream(void);

/* One decode token for each of `batch` independent sequences.
 * `hidden` and `output` are device arrays [batch][hidden_size]; states are
 * distinct states of `config`.  Asynchronous on the library stream: errors
 * (non-finite values, capacity) surface at kq_b200_synchronize, which then
 * rolls every state back to its value after the last successful call. */
kq_status kq_b200_gdn_decode_batch(const kq_gdn_config *config,
                                   kq_gdn_state *const *states,
                                   uint32_t batch,
                                   const float *hidden,
                                   float *output,
                                   kq_diagnostic *diagnostic);
kq_status kq_b200_qsa_decode_batch(const kq_qsa_config *config,
                                   kq_qsa_state *const *states,
                                   uint32_t batch,
                                   const float *hidden,
                                   float *output,
                                   kq_diagnostic *diagnostic);

/* kq_moe_execute_quantized over device arrays hidden / output
 * [tokens][hidden_size] of a provider-bound config, without observers,
 * asynchronous on the library stream: non-finite values surface at
 * kq_b200_synchronize (output then undefined).  Every token is independent,
 * so a batch of decode tokens of many sequences is one call. */
kq_status kq_b200_moe_execute_async(const kq_moe_config *config,
                                    const float *hidden,
                                    uint64_t tokens,
                                    float *output,
                                    kq_diagnostic *diagnostic);

/* The decoder layer on device arrays of branches [tokens][B][H] of a
 * provider-bound config, asynchronous on the library stream: one token for
 * each of `batch` sequences (distinct states), or T tokens of one sequence.
 * Errors surface at kq_b200_synchronize, which rolls every state back. */
kq_status kq_b200_layer_decode_batch(const kq_layer_config *config,
                                     kq_layer_state *const *states,
                                     uint32_t batch,
                                     const float *branches,
                                     float *output,
                                     kq_diagnostic *diagnostic);
kq_status kq_b200_layer_prefill_async(const kq_layer_config *config,
                                      kq_layer_state *state,
                                      const float *branches,
                                      uint64_t T,
                                      float *output,
                                      kq_diagnostic *diagnostic);

/* T tokens of one sequence, like kq_gdn_execute_quantized /
 * kq_qsa_execute_quantized (src/kq_gdn_internal.h:81-96,
 * src/kq_qsa_internal.h:94-102) without a mask or observers, on device
 * arrays [T][hidden_size] and asynchronous on the library stream (errors and
 * the state roll-back as for the batched decode).  A tensor-parallel host
 * binds one config per head group (a GDN config over its value/key heads, a
 * QSA config over its query heads and their key/value head) and sums the
 * groups' outputs, which are partial sums of the output projection. */
kq_status kq_b200_gdn_prefill_async(const kq_gdn_config *config,
                                    kq_gdn_state *state,
                                    const float *hidden,
                                    uint64_t T,
                                    float *output,
                                    kq_diagnostic *diagnostic);
kq_status kq_b200_qsa_prefill_async(const kq_qsa_config *config,
                                    kq_qsa_state *state,
                                    const float *hidden,
                                    uint64_t T,
                                    float *output,
                                    kq_diagnostic *diagnostic);

/* Completes the token selections of a sharded QSA prefill across the ranks:
 * `words` is a device array of `count` uint32 (every token's selected block
 * ids, then every token's selection count) that is zero outside the calling
 * rank's chunks; the function must enqueue on `cuda_stream` a sum over all
 * ranks into `words` (for example ncclAllReduce) and return 0, or non-zero
 * on failure.  It is called once per call, on the calling thread. */
typedef int (*kq_b200_exchange_fn)(void *words, uint64_t count, void *cuda_stream, void *user);

/* kq_b200_qsa_prefill_async for one of `world` tensor-parallel ranks whose
 * configs hold the same indexer: the block scores and top-k of the 64-token
 * chunks c with c % world == rank are computed here, `exchange` shares them,
 * then every chunk's attention runs with its query heads.  world == 1 is
 * kq_b200_qsa_prefill_async (exchange may be NULL). */
kq_status kq_b200_qsa_prefill_sharded_async(const kq_qsa_config *config,
                                            kq_qsa_state *state,
                                            const float *hidden,
                                            uint64_t T,
                                            float *output,
                                            uint32_t rank,
                                            uint32_t world,
                                            kq_b200_exchange_fn exchange,
                                            void *user,
                                            kq_diagnostic *diagnostic);

/* kq_b200_qsa_prefill_sharded_async where more ranks than key/value heads
 * share the attention: `config` holds every query head of one key/value
 * head, and this rank runs the attention, gate and out-projection of token
 * part `token_part` of `token_parts` (contiguous ranges of whole 64-token
 * chunk groups), writing zero rows of `output` for the other tokens, so that
 * the sum over ranks is the layer's output.  token_parts == 1 is
 * kq_b200_qsa_prefill_sharded_async. */
kq_status kq_b200_qsa_prefill_split_async(const kq_qsa_config *config,
                                          kq_qsa_state *state,
                                          const float *hidden,
                                          uint64_t T,
                                          float *output,
                                          uint32_t rank,
                                          uint32_t world,
                                          uint32_t token_part,
                                          uint32_t token_parts,
                                          kq_b200_exchange_fn exchange,
                                          void *user,
                                          kq_diagnostic *diagnostic);

/* Waits for the library stream and reports the first device-side error
 * raised since the previous synchronize. */
kq_status kq_b200_synchronize(kq_diagnostic *diagnostic);

/* Number of kernels this library has launched on the current device. */
uint64_t kq_b200_kernel_launch_count(void);

/* Device timing of one kernel family with CUDA events recorded around each
 * of its launches on the launching stream ("gdn_recurrence", "proj",
 * "qsa_attend", "qsa_score", "qsa_select", "gdn_conv", "qsa_prepare",
 * "qsa_combine"; NULL or "" turns timing off).  Selecting a family resets
 * the totals; kq_b200_profile_read waits for the recorded events. */
void kq_b200_profile_kernel(const char *kernel_family);
void kq_b200_profile_read(uint64_t *launches, double *total_ms);

#ifdef __cplusplus
}
#endif

#endif
