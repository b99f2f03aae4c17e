/*
 * GGUF block dequantisation and quantized row-dot on the B200.
 *
 * Replaces include/kq_numeric.h:19-43 of Kestrel-Q
 * (kq_dequantize_blocks_f32, kq_quantized_row_dot_f32) with the same
 * signatures.  Both run on the GPU: host buffers are staged, device buffers
 * are used in place.  Dequantised values are bit-identical to the
 * reference's (src/kq_numeric.c:176-295); the row-dot accumulates in the
 * reference's block-then-element order (src/kq_numeric.c:474-496) and is
 * therefore bit-identical too.  Supported types: F32, BF16, Q8_0, Q4_K and
 * Q6_K (Q6_K is not in the reference).  The F32 helper primitives of the
 * reference header (kq_f32_add ... kq_f32_renormalize) are CPU utilities of
 * the reference's layer code and are not exported.
 */
#ifndef KQ_NUMERIC_H
#define KQ_NUMERIC_H

#include <stdint.h>

#include "kq_status.h"
#include "kq_tensor_view.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_NUMERIC_MAX_BLOCK_ELEMENTS 256U

kq_status kq_dequantize_blocks_f32(uint32_t type_id,
                                   const void *packed,
                                   uint64_t packed_bytes,
                                   float *output,
                                   uint64_t output_capacity,
                                   uint64_t *output_count,
                                   kq_diagnostic *diagnostic);

kq_status kq_quantized_row_dot_f32(uint32_t type_id,
                                   const void *packed,
                                   uint64_t packed_bytes,
                                   const float *activation,
                                   uint64_t activation_count,
                                   float *output,
                                   kq_diagnostic *diagnostic);

#ifdef __cplusplus
}
#endif

#endif
