/*
 * Quantized block geometry of the operator ABI.
 *
 * Replaces the geometry queries of include/kq_tensor_view.h:33-107 of
 * Kestrel-Q (kq_quant_geometry_for_type, kq_quant_packed_size,
 * kq_quant_element_to_block, kq_quant_range_to_blocks) with the same
 * signatures, and extends the type table with Q6_K (type 14: 256 values,
 * 210 bytes).  The GGUF-backed view objects (kq_tensor_view_open_*) are out
 * of scope.
 */
#ifndef KQ_TENSOR_VIEW_H
#define KQ_TENSOR_VIEW_H

#include <stdint.h>

#include "kq_gguf.h"
#include "kq_model.h"
#include "kq_status.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct kq_quant_geometry {
    uint32_t type_id;
    uint64_t block_elements;
    uint64_t bytes_per_block;
} kq_quant_geometry;

typedef struct kq_quant_block_span {
    uint64_t requested_element_offset;
    uint64_t requested_element_count;
    uint64_t first_block;
    uint64_t block_count;
    uint64_t physical_byte_offset;
    uint64_t physical_byte_length;
    uint64_t leading_elements;
    uint64_t trailing_elements;
} kq_quant_block_span;

kq_status kq_quant_geometry_for_type(uint32_t type_id,
                                     kq_quant_geometry *out_geometry,
                                     kq_diagnostic *diagnostic);
kq_status kq_quant_packed_size(uint32_t type_id,
                               uint64_t element_count,
                               uint64_t *out_packed_bytes,
                               kq_diagnostic *diagnostic);
kq_status kq_quant_element_to_block(uint32_t type_id,
                                    uint64_t total_elements,
                                    uint64_t element_index,
                                    uint64_t *out_block_index,
                                    uint64_t *out_element_in_block,
                                    kq_diagnostic *diagnostic);
kq_status kq_quant_range_to_blocks(uint32_t type_id,
                                   uint64_t total_elements,
                                   uint64_t element_offset,
                                   uint64_t element_count,
                                   kq_quant_block_span *out_span,
                                   kq_diagnostic *diagnostic);

#ifdef __cplusplus
}
#endif

#endif
