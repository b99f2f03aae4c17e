/*
 * GGUF tensor type ids used by the operator ABI.
 *
 * Subset of include/kq_gguf.h:14-23 of Kestrel-Q (the parser itself is out of
 * scope: weights reach the B200 library as in-memory GGUF blocks).  Q6_K
 * (GGUF type 14, 256 values in 210 bytes) is an addition: the reference has
 * no Q6_K decoder (src/kq_gguf.c:57-65) but the B200 path accepts it.
 */
#ifndef KQ_GGUF_H
#define KQ_GGUF_H

#include <stdint.h>

#include "kq_status.h"

#ifdef __cplusplus
extern "C" {
#endif

#define KQ_GGUF_MAX_DIMS 8U

enum {
    KQ_GGUF_TYPE_F32 = 0,
    KQ_GGUF_TYPE_Q5_1 = 7,
    KQ_GGUF_TYPE_Q8_0 = 8,
    KQ_GGUF_TYPE_Q4_K = 12,
    KQ_GGUF_TYPE_Q5_K = 13,
    KQ_GGUF_TYPE_Q6_K = 14,
    KQ_GGUF_TYPE_IQ4_NL = 20,
    KQ_GGUF_TYPE_BF16 = 30
};

/* Opaque here: the GGUF container is not parsed by the B200 library. */
typedef struct kq_gguf kq_gguf;
typedef struct kq_gguf_tensor kq_gguf_tensor;
typedef struct kq_gguf_metadata kq_gguf_metadata;

#ifdef __cplusplus
}
#endif

#endif
