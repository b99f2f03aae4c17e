/*
 * Weight provider: the semantic GEMV seam of the operator ABI.
 *
 * Replaces include/kq_weight_provider.h:14-94 of Kestrel-Q.  In the B200
 * library the provider is a device-resident store of GGUF-quantized
 * matrices and small F32 vectors (created by kq_b200_provider_create and
 * filled by kq_b200_provider_add_*, see kq_b200.h) instead of a view over a
 * memory-mapped GGUF file; kq_weight_provider_open therefore returns
 * KQ_STATUS_UNSUPPORTED_MODEL.  kq_weight_provider_linear_f32 and
 * kq_weight_provider_vector_f32 keep their signatures and error behaviour;
 * linear_f32 runs the dequant-fused GEMV kernel (host or device input and
 * output accepted).
 */
#ifndef KQ_WEIGHT_PROVIDER_H
#define KQ_WEIGHT_PROVIDER_H

#include <stdint.h>

#include "kq_gguf.h"
#include "kq_model.h"
#include "kq_status.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_WEIGHT_PROVIDER_NO_EXPERT UINT32_MAX

typedef struct kq_weight_provider kq_weight_provider;

typedef struct kq_weight_provider_metrics {
    uint64_t payload_budget_bytes;
    uint64_t logical_payload_bytes_touched;
    uint64_t quantized_blocks_touched;
    uint64_t linear_requests;
    uint64_t row_requests;
    uint64_t vector_requests;
    uint64_t selected_expert_requests;
    uint64_t ple_row_requests;
    uint64_t unique_semantic_tensors_touched;
    uint64_t maximum_f32_weight_bytes_materialized;
    uint64_t provider_owned_bytes;
    uint64_t linear_elapsed_nanoseconds;
} kq_weight_provider_metrics;

kq_status kq_weight_provider_open(const kq_gguf *gguf,
                                  const kq_model *model,
                                  uint64_t payload_budget_bytes,
                                  kq_weight_provider **out_provider,
                                  kq_diagnostic *diagnostic);
void kq_weight_provider_close(kq_weight_provider *provider);

/* Semantic matrix-vector product y = W x.  Output is committed only on
 * success. */
kq_status kq_weight_provider_linear_f32(kq_weight_provider *provider,
                                        const kq_semantic_tensor *semantic,
                                        kq_binding_part_role part_role,
                                        uint32_t expert_id,
                                        uint64_t rows,
                                        uint64_t columns,
                                        const float *input,
                                        float *output,
                                        uint64_t output_capacity,
                                        void *scratch,
                                        uint64_t scratch_bytes,
                                        kq_diagnostic *diagnostic);

/* Bounded small-vector materialisation (host output). */
kq_status kq_weight_provider_vector_f32(kq_weight_provider *provider,
                                        const kq_semantic_tensor *semantic,
                                        uint64_t element_count,
                                        float *output,
                                        uint64_t output_capacity,
                                        void *scratch,
                                        uint64_t scratch_bytes,
                                        kq_diagnostic *diagnostic);

const kq_weight_provider_metrics *kq_weight_provider_get_metrics(
    const kq_weight_provider *provider);

#ifdef __cplusplus
}
#endif

#endif
