/*
 * kq_oracle.c — CPU restatement of Kestrel-Q's token-mixing hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see kq_oracle.h).  Build: make -C oracle port.
 * Must be compiled with -fno-fast-math -ffp-contract=off: every product and
 * every sum below is a separately rounded F32 operation, in the reference's
 * order, so the results are bit-identical to the reference's scalar C.
 * File:line citations point into the Kestrel-Q source tree.
 */
#include "kq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ---------------------------------------------------------------- dequant */

/* f16 -> f32 with exact subnormal handling: src/kq_numeric.c:58-82. */
static float kqo_half(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000U) << 16;
    uint32_t exponent = ((uint32_t)h >> 10) & 0x1fU;
    uint32_t mantissa = (uint32_t)h & 0x3ffU;
    uint32_t bits;
    float value;
    if (exponent == 0U) {
        if (mantissa == 0U) {
            bits = sign;
        } else {
            /* normalise the subnormal: shift until the implicit bit appears */
            uint32_t e = 113U;
            while ((mantissa & 0x400U) == 0U) {
                mantissa <<= 1;
                e -= 1U;
            }
            bits = sign | (e << 23) | ((mantissa & 0x3ffU) << 13);
        }
    } else if (exponent == 31U) {
        bits = sign | 0x7f800000U | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112U) << 23) | (mantissa << 13);
    }
    memcpy(&value, &bits, sizeof(value));
    return value;
}

static uint16_t kqo_u16(const unsigned char *p) {
    return (uint16_t)(p[0] | (p[1] << 8));
}

int kqo_block_geometry(uint32_t type_id, uint64_t *block_elements,
                       uint64_t *bytes_per_block) {
    uint64_t e = 0, b = 0;
    switch (type_id) {
    case KQO_TYPE_F32: e = 1; b = 4; break;
    case KQO_TYPE_BF16: e = 1; b = 2; break;
    case KQO_TYPE_Q8_0: e = 32; b = 34; break;
    case KQO_TYPE_Q4_K: e = 256; b = 144; break;
    case KQO_TYPE_Q6_K: e = 256; b = 210; break;
    default: return KQO_UNSUPPORTED_TYPE;
    }
    if (block_elements) *block_elements = e;
    if (bytes_per_block) *bytes_per_block = b;
    return KQO_OK;
}

/* K-quant 6-bit scale/min unpack: src/kq_numeric.c:161-174. */
static void kqo_k_scale(uint32_t j, const unsigned char *s, uint8_t *sc,
                        uint8_t *mn) {
    if (j < 4U) {
        *sc = (uint8_t)(s[j] & 63U);
        *mn = (uint8_t)(s[j + 4U] & 63U);
    } else {
        *sc = (uint8_t)((s[j + 4U] & 15U) | ((s[j - 4U] >> 6) << 4));
        *mn = (uint8_t)((s[j + 4U] >> 4) | ((s[j] >> 6) << 4));
    }
}

static int kqo_decode_block(uint32_t type_id, const unsigned char *p,
                            float *out) {
    uint32_t i;
    if (type_id == KQO_TYPE_F32) {
        uint32_t bits = (uint32_t)p[0] | ((uint32_t)p[1] << 8) |
                        ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
        memcpy(out, &bits, 4);
        return KQO_OK;
    }
    if (type_id == KQO_TYPE_BF16) {
        uint32_t bits = (uint32_t)kqo_u16(p) << 16;
        memcpy(out, &bits, 4);
        return KQO_OK;
    }
    if (type_id == KQO_TYPE_Q8_0) {
        /* src/kq_numeric.c:210-222: out = (float)code * d */
        float d = kqo_half(kqo_u16(p));
        if (!isfinite(d)) return KQO_NUMERIC_DOMAIN;
        for (i = 0; i < 32U; ++i) {
            out[i] = (float)(int8_t)p[2U + i] * d;
        }
        return KQO_OK;
    }
    if (type_id == KQO_TYPE_Q4_K) {
        /* src/kq_numeric.c:223-277: two separately rounded products per
         * group, then (d*sc)*q - (dmin*m). */
        float d = kqo_half(kqo_u16(p));
        float dmin = kqo_half(kqo_u16(p + 2));
        const unsigned char *scales = p + 4;
        const unsigned char *q = p + 16;
        uint32_t g;
        if (!isfinite(d) || !isfinite(dmin)) return KQO_NUMERIC_DOMAIN;
        for (g = 0; g < 4U; ++g) {
            uint8_t s0, m0, s1, m1;
            float dl, ml, dh, mh;
            kqo_k_scale(2U * g, scales, &s0, &m0);
            kqo_k_scale(2U * g + 1U, scales, &s1, &m1);
            dl = d * (float)s0;
            ml = dmin * (float)m0;
            dh = d * (float)s1;
            mh = dmin * (float)m1;
            for (i = 0; i < 32U; ++i) {
                uint8_t byte = q[g * 32U + i];
                out[g * 64U + i] = dl * (float)(byte & 15U) - ml;
                out[g * 64U + 32U + i] = dh * (float)(byte >> 4) - mh;
            }
        }
        return KQO_OK;
    }
    if (type_id == KQO_TYPE_Q6_K) {
        /* Public GGUF Q6_K super-block (210 bytes, 256 values):
         *   ql[128]  low 4 bits of each 6-bit code
         *   qh[64]   high 2 bits, four codes per byte
         *   sc[16]   signed 8-bit sub-block scales (16 values each)
         *   d        fp16 super-block scale
         * Two halves of 128 values; within a half, value l (0..31) and its
         * neighbours at +32, +64, +96 take their low nibbles from
         * ql[l], ql[l+32], ql[l] >> 4, ql[l+32] >> 4 and their high bits
         * from qh[l] bit pairs 0-1, 2-3, 4-5, 6-7.  value = (d * sc) * (q - 32)
         * with each product rounded separately.  Not in the reference:
         * parity for this type is pinned only by this restatement. */
        const unsigned char *ql = p;
        const unsigned char *qh = p + 128;
        const signed char *sc = (const signed char *)(p + 192);
        float d = kqo_half(kqo_u16(p + 208));
        uint32_t half;
        if (!isfinite(d)) return KQO_NUMERIC_DOMAIN;
        for (half = 0; half < 2U; ++half) {
            const unsigned char *L = ql + half * 64U;
            const unsigned char *Hb = qh + half * 32U;
            const signed char *S = sc + half * 8U;
            float *o = out + half * 128U;
            for (i = 0; i < 32U; ++i) {
                uint32_t sub = i / 16U;
                int c0 = (int)((L[i] & 15U) | (((Hb[i] >> 0) & 3U) << 4)) - 32;
                int c1 = (int)((L[i + 32U] & 15U) | (((Hb[i] >> 2) & 3U) << 4)) - 32;
                int c2 = (int)((L[i] >> 4) | (((Hb[i] >> 4) & 3U) << 4)) - 32;
                int c3 = (int)((L[i + 32U] >> 4) | (((Hb[i] >> 6) & 3U) << 4)) - 32;
                float s0 = d * (float)S[sub + 0U];
                float s1 = d * (float)S[sub + 2U];
                float s2 = d * (float)S[sub + 4U];
                float s3 = d * (float)S[sub + 6U];
                o[i] = s0 * (float)c0;
                o[i + 32U] = s1 * (float)c1;
                o[i + 64U] = s2 * (float)c2;
                o[i + 96U] = s3 * (float)c3;
            }
        }
        return KQO_OK;
    }
    return KQO_UNSUPPORTED_TYPE;
}

int kqo_dequantize(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                   float *output, uint64_t output_capacity) {
    uint64_t be, bb, blocks, i;
    int st = kqo_block_geometry(type_id, &be, &bb);
    if (st != KQO_OK) return st;
    if (packed == NULL || output == NULL || packed_bytes % bb != 0U)
        return KQO_INVALID_ARGUMENT;
    blocks = packed_bytes / bb;
    if (output_capacity < blocks * be) return KQO_INVALID_ARGUMENT;
    for (i = 0; i < blocks; ++i) {
        st = kqo_decode_block(type_id, (const unsigned char *)packed + i * bb,
                              output + i * be);
        if (st != KQO_OK) return st;
    }
    return KQO_OK;
}

/* Quantized row dot: src/kq_numeric.c:420-503.  Block by block, sequential
 * F32 accumulation from 0.0f in element order. */
int kqo_row_dot(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                const float *x, uint64_t count, float *output) {
    float scratch[256];
    float acc = 0.0f;
    uint64_t be, bb, blocks, b, i;
    int st = kqo_block_geometry(type_id, &be, &bb);
    if (st != KQO_OK) return st;
    if (packed_bytes % bb != 0U || (packed_bytes / bb) * be != count)
        return KQO_INVALID_ARGUMENT;
    blocks = packed_bytes / bb;
    for (b = 0; b < blocks; ++b) {
        st = kqo_decode_block(type_id, (const unsigned char *)packed + b * bb,
                              scratch);
        if (st != KQO_OK) return st;
        for (i = 0; i < be; ++i) {
            float product = scratch[i] * x[b * be + i];
            acc = acc + product;
        }
    }
    if (!isfinite(acc)) return KQO_NUMERIC_DOMAIN;
    *output = acc;
    return KQO_OK;
}

int kqo_matvec(uint32_t type_id, const void *packed, uint64_t rows,
               uint64_t cols, const float *x, uint64_t batch, float *y) {
    uint64_t be, bb, row_bytes, r, b;
    int st = kqo_block_geometry(type_id, &be, &bb);
    if (st != KQO_OK) return st;
    if (cols % be != 0U) return KQO_INVALID_ARGUMENT;
    row_bytes = (cols / be) * bb;
    for (b = 0; b < batch; ++b) {
        for (r = 0; r < rows; ++r) {
            st = kqo_row_dot(type_id,
                             (const unsigned char *)packed + r * row_bytes,
                             row_bytes, x + b * cols, cols, &y[b * rows + r]);
            if (st != KQO_OK) return st;
        }
    }
    return KQO_OK;
}

/* ------------------------------------------------------------- primitives */

/* kq_f32_dot: src/kq_numeric.c:591-626 (sequential, from 0.0f). */
static float kqo_dot(const float *a, const float *b, uint64_t n) {
    float acc = 0.0f;
    uint64_t i;
    for (i = 0; i < n; ++i) {
        float product = a[i] * b[i];
        acc = acc + product;
    }
    return acc;
}

/* Branch-stable sigmoid: src/kq_numeric.c:628-638. */
static float kqo_sigmoid(float x) {
    if (x >= 0.0f) {
        float e = expf(-x);
        return 1.0f / (1.0f + e);
    } else {
        float e = expf(x);
        return e / (1.0f + e);
    }
}

/* ------------------------------------------------------------------- GDN */

/* One checkpoint to the callback (src/kq_gdn_qwen38.c:248-271). */
static void kqo_emit(kqo_checkpoint_fn cb, void *user, uint32_t kind, uint64_t token, uint32_t rank,
                     uint64_t d0, uint64_t d1, uint64_t d2, const float *values, uint64_t count) {
    uint64_t dims[4];
    if (cb == NULL) return;
    dims[0] = d0;
    dims[1] = d1;
    dims[2] = d2;
    dims[3] = 0;
    cb(kind, token, rank, dims, values, count, user);
}

int kqo_gdn_run(const kqo_gdn_dims *dm, const kqo_gdn_weights *w,
                const float *hidden, uint64_t tokens, const uint8_t *mask,
                float *output, float *conv_state, float *recurrent_state) {
    return kqo_gdn_run_observed(dm, w, hidden, tokens, mask, output, conv_state, recurrent_state, NULL, NULL);
}

/* Per-token loop of src/kq_gdn_qwen38.c:545-842 over F32 weights; the
 * checkpoint kinds follow include/kq_gdn.h:23-44 and are emitted where the
 * reference emits them. */
int kqo_gdn_run_observed(const kqo_gdn_dims *dm, const kqo_gdn_weights *w,
                         const float *hidden, uint64_t tokens, const uint8_t *mask,
                         float *output, float *conv_state, float *recurrent_state,
                         kqo_checkpoint_fn cb, void *user) {
    const uint64_t H = dm->hidden_size, Hv = dm->value_heads,
                   dk = dm->key_dim, dv = dm->value_dim, K = dm->conv_kernel;
    const uint64_t key_width = (uint64_t)dm->key_heads * dk;
    const uint64_t Vd = Hv * dv;
    const uint64_t C = 2U * key_width + Vd;
    const uint64_t repeat = Hv / dm->key_heads;
    const uint64_t conv_n = C * K, rec_n = Hv * dk * dv;
    const float query_scale = 1.0f / sqrtf((float)dk);
    float *ws, *conv, *rec, *xin, *proj, *gate, *pb, *pa, *co, *q, *k, *v,
          *beta, *g, *core, *sg, *y, *rd, *dl;
    uint64_t t, i, h, f, kf, c, j;
    int status = KQO_OK;

    if (dm->conv_kernel == 0U || dm->key_heads == 0U || Hv % dm->key_heads)
        return KQO_INVALID_ARGUMENT;
    ws = (float *)malloc(sizeof(float) *
                         (conv_n + rec_n + H + C + Vd + 2 * Hv + C +
                          2 * Hv * dk + Vd + 2 * Hv + Vd + Vd + H + 2 * Vd));
    if (ws == NULL) return KQO_INVALID_ARGUMENT;
    conv = ws;            rec = conv + conv_n;  xin = rec + rec_n;
    proj = xin + H;       gate = proj + C;      pb = gate + Vd;
    pa = pb + Hv;         co = pa + Hv;         q = co + C;
    k = q + Hv * dk;      v = k + Hv * dk;      beta = v + Vd;
    g = beta + Hv;        core = g + Hv;        sg = core + Vd;
    y = sg + Vd;          rd = y + H;           dl = rd + Vd;
    /* transactional: work on a copy (src/kq_gdn_qwen38.c:532-536) */
    memcpy(conv, conv_state, sizeof(float) * conv_n);
    memcpy(rec, recurrent_state, sizeof(float) * rec_n);

    for (t = 0; t < tokens && status == KQO_OK; ++t) {
        const float *x = hidden + t * H;
        float m = mask == NULL ? 1.0f : (float)mask[t];
        for (i = 0; i < H; ++i) xin[i] = x[i] * m;
        kqo_emit(cb, user, 0, t, 1, H, 0, 0, xin, H);                 /* MASKED_INPUT */
        /* projections (:558-579) */
        for (i = 0; i < C; ++i) proj[i] = kqo_dot(w->qkv + i * H, xin, H);
        for (i = 0; i < Vd; ++i) gate[i] = kqo_dot(w->gate + i * H, xin, H);
        for (i = 0; i < Hv; ++i) pb[i] = kqo_dot(w->beta + i * H, xin, H);
        for (i = 0; i < Hv; ++i) pa[i] = kqo_dot(w->alpha + i * H, xin, H);
        kqo_emit(cb, user, 1, t, 1, C, 0, 0, proj, C);                /* PROJECTED_QKV */
        kqo_emit(cb, user, 2, t, 2, Hv, dv, 0, gate, Vd);             /* PROJECTED_GATE */
        kqo_emit(cb, user, 3, t, 1, Hv, 0, 0, pb, Hv);                /* PROJECTED_BETA */
        kqo_emit(cb, user, 4, t, 1, Hv, 0, 0, pa, Hv);                /* PROJECTED_ALPHA */
        kqo_emit(cb, user, 5, t, 1, C, 0, 0, proj, C);                /* CONV_INPUT */
        /* causal conv over pre-activation history, then SiLU (:602-621) */
        for (c = 0; c < C; ++c) {
            float *hist = conv + c * K;
            float s;
            for (j = 1; j < K; ++j) hist[j - 1] = hist[j];
            hist[K - 1] = proj[c];
            s = kqo_dot(w->conv + c * K, hist, K);
            co[c] = s * kqo_sigmoid(s);
        }
        kqo_emit(cb, user, 6, t, 1, C, 0, 0, co, C);                  /* CONV_OUTPUT */
        kqo_emit(cb, user, 18, t, 2, C, K, 0, conv, conv_n);          /* CONV_STATE */
        /* head split with consecutive key-head repeat (:631-648) */
        for (h = 0; h < Hv; ++h) {
            uint64_t kh = h / repeat;
            memcpy(q + h * dk, co + kh * dk, sizeof(float) * dk);
            memcpy(k + h * dk, co + key_width + kh * dk, sizeof(float) * dk);
            memcpy(v + h * dv, co + 2 * key_width + h * dv, sizeof(float) * dv);
        }
        kqo_emit(cb, user, 7, t, 2, Hv, dk, 0, q, Hv * dk);           /* QUERY_BEFORE_NORM */
        kqo_emit(cb, user, 8, t, 2, Hv, dk, 0, k, Hv * dk);           /* KEY_BEFORE_NORM */
        kqo_emit(cb, user, 9, t, 2, Hv, dv, 0, v, Vd);                /* VALUE */
        /* beta, log-decay, L2 norms (:662-687) */
        for (h = 0; h < Hv; ++h) {
            float sp, a = pa[h] + w->dt_bias[h];
            float base = -expf(w->a_log[h]);
            float sum, inv;
            beta[h] = kqo_sigmoid(pb[h]);
            sp = a > 20.0f ? a : log1pf(expf(a));
            g[h] = base * sp;
            if (!isfinite(g[h]) || g[h] > 0.0f) { status = KQO_NUMERIC_DOMAIN; break; }
            sum = kqo_dot(q + h * dk, q + h * dk, dk);
            sum = sum + 1.0e-6f;
            inv = 1.0f / sqrtf(sum);
            for (i = 0; i < dk; ++i) {
                float nrm = q[h * dk + i] * inv;
                q[h * dk + i] = nrm * query_scale;
            }
            sum = kqo_dot(k + h * dk, k + h * dk, dk);
            sum = sum + 1.0e-6f;
            inv = 1.0f / sqrtf(sum);
            for (i = 0; i < dk; ++i) {
                float nrm = k[h * dk + i] * inv;
                k[h * dk + i] = nrm * 1.0f;
            }
        }
        if (status != KQO_OK) break;
        kqo_emit(cb, user, 10, t, 2, Hv, dk, 0, q, Hv * dk);          /* NORMALIZED_SCALED_QUERY */
        kqo_emit(cb, user, 11, t, 2, Hv, dk, 0, k, Hv * dk);          /* NORMALIZED_KEY */
        kqo_emit(cb, user, 12, t, 1, Hv, 0, 0, g, Hv);                /* LOG_DECAY */
        kqo_emit(cb, user, 13, t, 1, Hv, 0, 0, beta, Hv);             /* BETA */
        /* delta-rule recurrence (:705-761) */
        for (h = 0; h < Hv; ++h) {
            float decay = expf(g[h]);
            float *S = rec + h * dk * dv;
            const float *kh = k + h * dk, *qh = q + h * dk, *vh = v + h * dv;
            float *delta = dl + h * dv;
            for (i = 0; i < dk * dv; ++i) S[i] = S[i] * decay;
            for (f = 0; f < dv; ++f) {
                float sum = 0.0f;
                for (kf = 0; kf < dk; ++kf) {
                    float product = S[kf * dv + f] * kh[kf];
                    sum = sum + product;
                }
                rd[h * dv + f] = sum;
                delta[f] = (vh[f] - sum) * beta[h];
            }
            for (kf = 0; kf < dk; ++kf) {
                for (f = 0; f < dv; ++f) {
                    float update = kh[kf] * delta[f];
                    S[kf * dv + f] = S[kf * dv + f] + update;
                }
            }
            for (f = 0; f < dv; ++f) {
                float sum = 0.0f;
                for (kf = 0; kf < dk; ++kf) {
                    float product = S[kf * dv + f] * qh[kf];
                    sum = sum + product;
                }
                core[h * dv + f] = sum;
            }
        }
        for (i = 0; i < rec_n; ++i)
            if (!isfinite(rec[i])) { status = KQO_NUMERIC_DOMAIN; break; }
        if (status != KQO_OK) break;
        kqo_emit(cb, user, 14, t, 2, Hv, dv, 0, rd, Vd);              /* RECURRENT_READ */
        kqo_emit(cb, user, 15, t, 2, Hv, dv, 0, dl, Vd);              /* RECURRENT_DELTA */
        kqo_emit(cb, user, 16, t, 2, Hv, dv, 0, core, Vd);            /* RECURRENT_OUTPUT */
        kqo_emit(cb, user, 17, t, 3, Hv, dk, dv, rec, rec_n);         /* RECURRENT_STATE */
        /* gated RMSNorm (:787-815): norm weight applied directly */
        for (i = 0; i < Vd; ++i) sg[i] = kqo_sigmoid(gate[i]);
        for (h = 0; h < Hv; ++h) {
            float sum = 0.0f, inv;
            float *cr = core + h * dv;
            for (f = 0; f < dv; ++f) {
                float sq = cr[f] * cr[f];
                sum = sum + sq;
            }
            sum = sum / (float)dv;
            inv = 1.0f / sqrtf(sum + dm->rms_norm_epsilon);
            for (f = 0; f < dv; ++f) {
                float nrm = cr[f] * inv;
                float wt = w->norm[f] * nrm;
                cr[f] = wt * sg[h * dv + f];
            }
        }
        kqo_emit(cb, user, 19, t, 2, Hv, dv, 0, core, Vd);            /* GATED_NORM_OUTPUT */
        /* output projection (:826-831) */
        for (i = 0; i < H; ++i) {
            y[i] = kqo_dot(w->output + i * Vd, core, Vd);
            if (!isfinite(y[i])) { status = KQO_NUMERIC_DOMAIN; break; }
        }
        if (status != KQO_OK) break;
        memcpy(output + t * H, y, sizeof(float) * H);
        kqo_emit(cb, user, 20, t, 1, H, 0, 0, y, H);                  /* OPERATOR_OUTPUT */
    }
    if (status == KQO_OK) {
        memcpy(conv_state, conv, sizeof(float) * conv_n);
        memcpy(recurrent_state, rec, sizeof(float) * rec_n);
    }
    free(ws);
    return status;
}

/* ------------------------------------------------------------------- QSA */

/* (1 + w) RMSNorm: src/kq_qsa_qwen38.c:231-256. */
static int kqo_qsa_norm(float *x, uint64_t n, const float *dw, float eps) {
    float sum = 0.0f, inv;
    uint64_t i;
    for (i = 0; i < n; ++i) {
        float sq = x[i] * x[i];
        sum = sum + sq;
    }
    sum = sum / (float)n;
    inv = 1.0f / sqrtf(sum + eps);
    if (!isfinite(inv)) return KQO_NUMERIC_DOMAIN;
    for (i = 0; i < n; ++i) {
        x[i] = (x[i] * inv) * (1.0f + dw[i]);
        if (!isfinite(x[i])) return KQO_NUMERIC_DOMAIN;
    }
    return KQO_OK;
}

/* NeoX half rotation on the first `rot` dims: src/kq_qsa_qwen38.c:258-281. */
static int kqo_rope(float *x, uint32_t rot, float theta, uint64_t pos) {
    uint32_t half = rot / 2U, i;
    for (i = 0; i < half; ++i) {
        float e = (2.0f * (float)i) / (float)rot;
        float freq = 1.0f / powf(theta, e);
        float ang = (float)pos * freq;
        float cs = cosf(ang), sn = sinf(ang);
        float a = x[i], b = x[i + half];
        x[i] = a * cs - b * sn;
        x[i + half] = b * cs + a * sn;
        if (!isfinite(x[i]) || !isfinite(x[i + half])) return KQO_NUMERIC_DOMAIN;
    }
    return KQO_OK;
}

uint64_t kqo_select_blocks(const float *scores, uint64_t count, uint64_t limit,
                           uint32_t *sel) {
    uint64_t n = 0, cand;
    for (cand = 0; cand < count; ++cand) {
        uint64_t pos = 0;
        while (pos < n) {
            float cs = scores[cand], ps = scores[sel[pos]];
            int better = cs > ps || (cs == ps && (uint32_t)cand < sel[pos]);
            if (better) break;
            pos += 1;
        }
        if (pos < limit) {
            uint64_t end = n < limit ? n : limit - 1U;
            while (end > pos) { sel[end] = sel[end - 1]; end -= 1; }
            sel[pos] = (uint32_t)cand;
            if (n < limit) n += 1;
        }
    }
    return n;
}

int kqo_qsa_run(const kqo_qsa_dims *dm, const kqo_qsa_weights *w,
                const float *hidden, uint64_t tokens, float *output,
                float *kc, float *vc, float *rc, uint64_t capacity,
                uint64_t *length, uint32_t *sel_out, uint32_t *sel_counts,
                float *scores_out) {
    return kqo_qsa_run_observed(dm, w, hidden, tokens, output, kc, vc, rc, capacity, length, sel_out, sel_counts,
                                scores_out, NULL, NULL);
}

/* Per-token loop of src/kq_qsa_qwen38.c:524-828 over F32 weights; the
 * checkpoint kinds follow include/kq_qsa.h:23-36 and are emitted where the
 * reference emits them (:687-716 before the attention, :794-815 after the
 * output projection). */
int kqo_qsa_run_observed(const kqo_qsa_dims *dm, const kqo_qsa_weights *w,
                         const float *hidden, uint64_t tokens, float *output,
                         float *kc, float *vc, float *rc, uint64_t capacity,
                         uint64_t *length, uint32_t *sel_out, uint32_t *sel_counts,
                         float *scores_out, kqo_checkpoint_fn cb, void *user) {
    const uint64_t H = dm->hidden_size, Hq = dm->query_heads,
                   Hkv = dm->kv_heads, d = dm->head_dim, Hi = dm->index_heads,
                   di = dm->index_dim, blk = dm->block_size;
    const uint64_t qw = Hq * d, kvw = Hkv * d, iqw = Hi * di;
    const uint64_t topk = dm->token_budget / blk;
    const uint64_t sel_cap = dm->token_budget + blk - 1U;
    const uint64_t rep = Hq / Hkv;
    const uint64_t max_blocks = capacity / blk;
    uint64_t L0, t;
    float *qg, *q, *kk, *vv, *iq, *rk, *bk, *sc, *logit, *ctx, *y, *staged, *lg_all, *pr_all, *hctx;
    uint32_t *sel, *tok;
    int st = KQO_OK;

    if (length == NULL || *length + tokens > capacity || Hkv == 0U ||
        blk == 0U || Hq % Hkv)
        return KQO_LIMIT_EXCEEDED;
    L0 = *length;
    qg = (float *)malloc(sizeof(float) * (2 * qw + qw + kvw + kvw + iqw + di +
                                          max_blocks * di + max_blocks +
                                          sel_cap + qw + H + tokens * H + 2 * Hq * sel_cap + qw));
    sel = (uint32_t *)malloc(sizeof(uint32_t) * (topk + sel_cap + 1));
    if (qg == NULL || sel == NULL) { free(qg); free(sel); return KQO_INVALID_ARGUMENT; }
    tok = sel + topk;
    q = qg + 2 * qw;  kk = q + qw;   vv = kk + kvw;  iq = vv + kvw;
    rk = iq + iqw;    bk = rk + di;  sc = bk + max_blocks * di;
    logit = sc + max_blocks; ctx = logit + sel_cap; y = ctx + qw;
    staged = y + H;   lg_all = staged + tokens * H; pr_all = lg_all + Hq * sel_cap;
    hctx = pr_all + Hq * sel_cap;

    for (t = 0; t < tokens && st == KQO_OK; ++t) {
        const float *x = hidden + t * H;
        uint64_t pos = L0 + t, h, f, b, i, nblocks, tail, nsel, ntok = 0;
        /* projections (:539-565); pending rows are written straight into the
         * caches beyond the committed length, which is only advanced on
         * success (equivalent to the reference's pending buffers) */
        for (i = 0; i < 2 * qw; ++i) qg[i] = kqo_dot(w->query + i * H, x, H);
        for (i = 0; i < kvw; ++i) kk[i] = kqo_dot(w->key + i * H, x, H);
        for (i = 0; i < kvw; ++i) vv[i] = kqo_dot(w->value + i * H, x, H);
        for (i = 0; i < iqw; ++i) iq[i] = kqo_dot(w->index_query + i * H, x, H);
        for (i = 0; i < di; ++i) rk[i] = kqo_dot(w->index_key + i * H, x, H);
        /* norms + RoPE (:567-602) */
        for (h = 0; h < Hq && st == KQO_OK; ++h) {
            memcpy(q + h * d, qg + h * 2 * d, sizeof(float) * d);
            st = kqo_qsa_norm(q + h * d, d, w->query_norm, dm->rms_norm_epsilon);
            if (st == KQO_OK) st = kqo_rope(q + h * d, dm->rotary_dim, dm->rope_theta, pos);
        }
        for (h = 0; h < Hkv && st == KQO_OK; ++h) {
            st = kqo_qsa_norm(kk + h * d, d, w->key_norm, dm->rms_norm_epsilon);
            if (st == KQO_OK) st = kqo_rope(kk + h * d, dm->rotary_dim, dm->rope_theta, pos);
        }
        for (h = 0; h < Hi && st == KQO_OK; ++h) {
            st = kqo_qsa_norm(iq + h * di, di, w->index_query_norm, dm->rms_norm_epsilon);
            if (st == KQO_OK) st = kqo_rope(iq + h * di, dm->rotary_dim, dm->rope_theta, pos);
        }
        if (st != KQO_OK) break;
        memcpy(kc + pos * kvw, kk, sizeof(float) * kvw);
        memcpy(vc + pos * kvw, vv, sizeof(float) * kvw);
        memcpy(rc + pos * di, rk, sizeof(float) * di);
        /* block indexer over all complete blocks (:608-648) */
        nblocks = (pos + 1) / blk;
        tail = (pos + 1) % blk;
        for (b = 0; b < nblocks && st == KQO_OK; ++b) {
            float *key = bk + b * di, score = 0.0f;
            for (f = 0; f < di; ++f) {
                float sum = 0.0f;
                for (i = 0; i < blk; ++i) sum = sum + rc[(b * blk + i) * di + f];
                key[f] = sum / (float)blk;
            }
            st = kqo_qsa_norm(key, di, w->index_key_norm, dm->rms_norm_epsilon);
            if (st == KQO_OK) st = kqo_rope(key, dm->rotary_dim, dm->rope_theta, b * blk);
            if (st != KQO_OK) break;
            for (h = 0; h < Hi; ++h) {
                float dot = kqo_dot(iq + h * di, key, di);
                if (dot > 0.0f) score = score + dot;
            }
            score = score / sqrtf((float)di);
            if (!isfinite(score)) { st = KQO_NUMERIC_DOMAIN; break; }
            sc[b] = score;
        }
        if (st != KQO_OK) break;
        nsel = kqo_select_blocks(sc, nblocks, nblocks < topk ? nblocks : topk, sel);
        for (b = 0; b < nsel; ++b)
            for (i = 0; i < blk; ++i) tok[ntok++] = (uint32_t)(sel[b] * blk + i);
        for (i = 0; i < tail; ++i) tok[ntok++] = (uint32_t)(nblocks * blk + i);
        if (sel_out != NULL) {
            memset(sel_out + t * topk, 0, sizeof(uint32_t) * topk);
            memcpy(sel_out + t * topk, sel, sizeof(uint32_t) * nsel);
        }
        if (sel_counts != NULL) sel_counts[t] = (uint32_t)nsel;
        if (scores_out != NULL && nblocks > 0)
            memcpy(scores_out + t * max_blocks, sc, sizeof(float) * nblocks);
        kqo_emit(cb, user, 0, t, 2, Hi, di, 0, iq, iqw);                  /* INDEX_QUERY */
        kqo_emit(cb, user, 1, t, 1, di, 0, 0, rk, di);                    /* RAW_INDEX_KEY */
        kqo_emit(cb, user, 2, t, 2, nblocks, di, 0, bk, nblocks * di);    /* BLOCK_KEYS */
        kqo_emit(cb, user, 3, t, 1, nblocks, 0, 0, sc, nblocks);          /* CANDIDATE_SCORES */
        kqo_emit(cb, user, 4, t, 2, Hq, d, 0, q, qw);                     /* QUERY */
        kqo_emit(cb, user, 5, t, 2, Hkv, d, 0, kk, kvw);                  /* KEY */
        kqo_emit(cb, user, 6, t, 2, Hkv, d, 0, vv, kvw);                  /* VALUE */
        /* sparse softmax attention (:716-773) */
        for (h = 0; h < Hq; ++h) {
            uint64_t kvh = h / rep, s;
            float mx = -INFINITY, sum = 0.0f;
            for (s = 0; s < ntok; ++s) {
                const float *krow = kc + (uint64_t)tok[s] * kvw + kvh * d;
                float dot = 0.0f;
                for (f = 0; f < d; ++f) dot = dot + q[h * d + f] * krow[f];
                dot = dot / sqrtf((float)d);
                logit[s] = dot;
                lg_all[h * ntok + s] = dot;
                if (dot > mx) mx = dot;
            }
            for (s = 0; s < ntok; ++s) {
                float p = expf(logit[s] - mx);
                logit[s] = p;
                sum = sum + p;
            }
            if (!(sum > 0.0f) || !isfinite(sum)) { st = KQO_NUMERIC_DOMAIN; break; }
            for (s = 0; s < ntok; ++s) {
                logit[s] /= sum;
                pr_all[h * ntok + s] = logit[s];
            }
            for (f = 0; f < d; ++f) {
                float acc = 0.0f;
                for (s = 0; s < ntok; ++s)
                    acc = acc + logit[s] * vc[(uint64_t)tok[s] * kvw + kvh * d + f];
                ctx[h * d + f] = acc;
            }
        }
        if (st != KQO_OK) break;
        memcpy(hctx, ctx, sizeof(float) * qw);
        /* sigmoid output gate (:774-782), simple form */
        for (h = 0; h < Hq; ++h)
            for (f = 0; f < d; ++f) {
                float gt = qg[h * 2 * d + d + f];
                float sg = 1.0f / (1.0f + expf(-gt));
                ctx[h * d + f] = ctx[h * d + f] * sg;
            }
        for (i = 0; i < H; ++i) {
            y[i] = kqo_dot(w->output + i * qw, ctx, qw);
            if (!isfinite(y[i])) { st = KQO_NUMERIC_DOMAIN; break; }
        }
        if (st != KQO_OK) break;
        memcpy(staged + t * H, y, sizeof(float) * H);
        kqo_emit(cb, user, 7, t, 2, Hq, ntok, 0, lg_all, Hq * ntok);      /* ATTENTION_LOGITS */
        kqo_emit(cb, user, 8, t, 2, Hq, ntok, 0, pr_all, Hq * ntok);      /* ATTENTION_PROBABILITIES */
        kqo_emit(cb, user, 9, t, 2, Hq, d, 0, hctx, qw);                  /* HEAD_CONTEXT */
        kqo_emit(cb, user, 10, t, 2, Hq, d, 0, ctx, qw);                  /* GATED_CONTEXT */
        kqo_emit(cb, user, 11, t, 1, H, 0, 0, y, H);                      /* OPERATOR_OUTPUT */
    }
    if (st == KQO_OK) {
        memcpy(output, staged, sizeof(float) * tokens * H);
        *length = L0 + tokens;
    }
    free(qg);
    free(sel);
    return st;
}

/* ------------------------------------------------------------------- MoE */

/* Top-k of src/kq_moe_qwen38.c:211-245: the first k ids seed the set; a
 * later id replaces the set's worst entry (lowest value, the lowest id among
 * equal lowest values) only when strictly greater; the set is then ordered
 * by value descending, id ascending. */
static void kqo_moe_top_k(const float *p, uint32_t n, uint32_t k, uint32_t *ids) {
    uint32_t i;
    for (i = 0; i < k; ++i) ids[i] = i;
    for (i = k; i < n; ++i) {
        uint32_t pos, worst = 0;
        for (pos = 1; pos < k; ++pos) {
            uint32_t c = ids[pos], wv = ids[worst];
            if (p[c] < p[wv] || (p[c] == p[wv] && c < wv)) worst = pos;
        }
        if (p[i] > p[ids[worst]]) ids[worst] = i;
    }
    for (i = 1; i < k; ++i) {
        uint32_t v = ids[i], pos = i;
        while (pos > 0) {
            uint32_t prev = ids[pos - 1];
            if (p[prev] > p[v] || (p[prev] == p[v] && prev < v)) break;
            ids[pos] = prev;
            pos -= 1;
        }
        ids[pos] = v;
    }
}

/* SwiGLU of src/kq_numeric.c:700-728: silu(gate) * up, branch-stable sigmoid. */
static int kqo_swiglu(const float *g, const float *u, uint64_t n, float *out) {
    uint64_t i;
    for (i = 0; i < n; ++i) {
        float s = kqo_sigmoid(g[i]);
        float silu = g[i] * s;
        out[i] = silu * u[i];
        if (!isfinite(out[i])) return KQO_NUMERIC_DOMAIN;
    }
    return KQO_OK;
}

static int kqo_matvec_f32(const float *w, uint64_t rows, uint64_t cols, const float *x, float *y) {
    uint64_t r;
    for (r = 0; r < rows; ++r) {
        y[r] = kqo_dot(w + r * cols, x, cols);
        if (!isfinite(y[r])) return KQO_NUMERIC_DOMAIN;
    }
    return KQO_OK;
}

static void kqo_moe_emit(kqo_moe_checkpoint_fn cb, void *user, uint32_t kind, uint64_t token, uint32_t expert,
                         uint32_t position, uint64_t count, const float *values) {
    uint64_t dims[2];
    if (cb == NULL) return;
    dims[0] = count;
    dims[1] = 0;
    cb(kind, token, expert, position, 1, dims, values, count, user);
}

int kqo_moe_run(const kqo_moe_dims *dm, const kqo_moe_weights *w, const float *hidden, uint64_t tokens,
                float *output, float *logits_out, float *probs_out, uint32_t *ids_out, float *weights_out) {
    return kqo_moe_run_observed(dm, w, hidden, tokens, output, logits_out, probs_out, ids_out, weights_out,
                                NULL, NULL);
}

/* Per-token loop of src/kq_moe_qwen38.c:604-867 over F32 weights: router
 * logits (kq_f32_dot per expert), softmax (src/kq_numeric.c:776-813), top-k,
 * renormalised selected weights (:247-274), the selected experts in
 * ascending id order accumulated as routed_sum + weight * output, then the
 * shared expert scaled by sigmoid(shared_gate_weight . x).  Checkpoint
 * kinds follow include/kq_moe.h:24-41 in the reference's emission order.
 * The output is written only when every token succeeded. */
int kqo_moe_run_observed(const kqo_moe_dims *dm, const kqo_moe_weights *w, const float *hidden,
                         uint64_t tokens, float *output, float *logits_out, float *probs_out,
                         uint32_t *ids_out, float *weights_out, kqo_moe_checkpoint_fn cb, void *user) {
    const uint64_t H = dm->hidden_size, E = dm->expert_count, K = dm->top_k,
                   I = dm->routed_intermediate_size, S = dm->shared_intermediate_size;
    float *buf, *lg, *pr, *sw, *gate, *up, *act, *eo, *wo, *rsum, *sg, *su, *sa, *so, *gs, *staged;
    uint32_t *ids;
    uint64_t t, i;
    int st = KQO_OK;
    if (H == 0 || E == 0 || K == 0 || K > E || I == 0 || S == 0) return KQO_INVALID_ARGUMENT;
    for (i = 0; i < tokens * H; ++i)
        if (!isfinite(hidden[i])) return KQO_NUMERIC_DOMAIN;
    buf = (float *)malloc(sizeof(float) * (2 * E + K + 3 * I + 3 * H + 3 * S + 2 * H + tokens * H));
    ids = (uint32_t *)malloc(sizeof(uint32_t) * K);
    if (buf == NULL || ids == NULL) { free(buf); free(ids); return KQO_INVALID_ARGUMENT; }
    lg = buf; pr = lg + E; sw = pr + E; gate = sw + K; up = gate + I; act = up + I;
    eo = act + I; wo = eo + H; rsum = wo + H; sg = rsum + H; su = sg + S; sa = su + S;
    so = sa + S; gs = so + H; staged = gs + H;
    for (t = 0; t < tokens && st == KQO_OK; ++t) {
        const float *x = hidden + t * H;
        float *y = staged + t * H;
        float mx, sum = 0.0f, ssum = 0.0f, logit, scale;
        uint64_t e;
        st = kqo_matvec_f32(w->router, E, H, x, lg);
        if (st != KQO_OK) break;
        mx = lg[0];
        for (e = 1; e < E; ++e) if (lg[e] > mx) mx = lg[e];
        for (e = 0; e < E; ++e) {
            pr[e] = expf(lg[e] - mx);
            sum = sum + pr[e];
        }
        if (!isfinite(sum) || sum <= 0.0f) { st = KQO_NUMERIC_DOMAIN; break; }
        for (e = 0; e < E; ++e) pr[e] = pr[e] / sum;
        kqo_moe_top_k(pr, (uint32_t)E, (uint32_t)K, ids);
        for (i = 0; i < K; ++i) {
            sw[i] = pr[ids[i]];
            ssum = ssum + sw[i];
        }
        if (!(ssum > 0.0f) || !isfinite(ssum)) { st = KQO_NUMERIC_DOMAIN; break; }
        for (i = 0; i < K; ++i) {
            sw[i] = sw[i] / ssum;
            if (!isfinite(sw[i])) { st = KQO_NUMERIC_DOMAIN; break; }
        }
        if (st != KQO_OK) break;
        if (logits_out) memcpy(logits_out + t * E, lg, sizeof(float) * E);
        if (probs_out) memcpy(probs_out + t * E, pr, sizeof(float) * E);
        if (ids_out) memcpy(ids_out + t * K, ids, sizeof(uint32_t) * K);
        if (weights_out) memcpy(weights_out + t * K, sw, sizeof(float) * K);
        kqo_moe_emit(cb, user, 0, t, UINT32_MAX, UINT32_MAX, E, lg);   /* ROUTER_LOGITS */
        kqo_moe_emit(cb, user, 1, t, UINT32_MAX, UINT32_MAX, E, pr);   /* ROUTER_PROBABILITIES */
        kqo_moe_emit(cb, user, 2, t, UINT32_MAX, UINT32_MAX, K, sw);   /* SELECTED_WEIGHTS */
        for (i = 0; i < H; ++i) rsum[i] = 0.0f;
        for (e = 0; e < E && st == KQO_OK; ++e) {
            uint64_t pos;
            for (pos = 0; pos < K; ++pos) if (ids[pos] == e) break;
            if (pos == K) continue;
            st = kqo_matvec_f32(w->routed_gate + e * I * H, I, H, x, gate);
            if (st == KQO_OK) st = kqo_matvec_f32(w->routed_up + e * I * H, I, H, x, up);
            if (st == KQO_OK) st = kqo_swiglu(gate, up, I, act);
            if (st == KQO_OK) st = kqo_matvec_f32(w->routed_down + e * H * I, H, I, act, eo);
            if (st != KQO_OK) break;
            kqo_moe_emit(cb, user, 3, t, (uint32_t)e, (uint32_t)pos, I, gate);   /* ROUTED_GATE */
            kqo_moe_emit(cb, user, 4, t, (uint32_t)e, (uint32_t)pos, I, up);     /* ROUTED_UP */
            kqo_moe_emit(cb, user, 5, t, (uint32_t)e, (uint32_t)pos, I, act);    /* ROUTED_ACTIVATED */
            kqo_moe_emit(cb, user, 6, t, (uint32_t)e, (uint32_t)pos, H, eo);     /* ROUTED_EXPERT_OUTPUT */
            for (i = 0; i < H; ++i) {
                wo[i] = eo[i] * sw[pos];
                if (!isfinite(wo[i])) { st = KQO_NUMERIC_DOMAIN; break; }
            }
            if (st != KQO_OK) break;
            kqo_moe_emit(cb, user, 7, t, (uint32_t)e, (uint32_t)pos, H, wo);     /* ROUTED_WEIGHTED_OUTPUT */
            for (i = 0; i < H; ++i) {
                rsum[i] = rsum[i] + wo[i];
                if (!isfinite(rsum[i])) { st = KQO_NUMERIC_DOMAIN; break; }
            }
        }
        if (st != KQO_OK) break;
        kqo_moe_emit(cb, user, 8, t, UINT32_MAX, UINT32_MAX, H, rsum);   /* ROUTED_WEIGHTED_SUM */
        st = kqo_matvec_f32(w->shared_gate, S, H, x, sg);
        if (st == KQO_OK) st = kqo_matvec_f32(w->shared_up, S, H, x, su);
        if (st == KQO_OK) st = kqo_swiglu(sg, su, S, sa);
        if (st == KQO_OK) st = kqo_matvec_f32(w->shared_down, H, S, sa, so);
        if (st != KQO_OK) break;
        logit = kqo_dot(w->shared_gate_weight, x, H);
        if (!isfinite(logit)) { st = KQO_NUMERIC_DOMAIN; break; }
        scale = kqo_sigmoid(logit);
        if (!isfinite(scale)) { st = KQO_NUMERIC_DOMAIN; break; }
        for (i = 0; i < H; ++i) {
            gs[i] = so[i] * scale;
            y[i] = rsum[i] + gs[i];
            if (!isfinite(gs[i]) || !isfinite(y[i])) { st = KQO_NUMERIC_DOMAIN; break; }
        }
        if (st != KQO_OK) break;
        kqo_moe_emit(cb, user, 9, t, UINT32_MAX, UINT32_MAX, S, sg);     /* SHARED_GATE_PROJECTION */
        kqo_moe_emit(cb, user, 10, t, UINT32_MAX, UINT32_MAX, S, su);    /* SHARED_UP_PROJECTION */
        kqo_moe_emit(cb, user, 11, t, UINT32_MAX, UINT32_MAX, S, sa);    /* SHARED_ACTIVATED */
        kqo_moe_emit(cb, user, 12, t, UINT32_MAX, UINT32_MAX, H, so);    /* SHARED_OUTPUT */
        kqo_moe_emit(cb, user, 13, t, UINT32_MAX, UINT32_MAX, 1, &logit); /* SHARED_SCALE_LOGIT */
        kqo_moe_emit(cb, user, 14, t, UINT32_MAX, UINT32_MAX, 1, &scale); /* SHARED_SCALE */
        kqo_moe_emit(cb, user, 15, t, UINT32_MAX, UINT32_MAX, H, gs);    /* GATED_SHARED_OUTPUT */
        kqo_moe_emit(cb, user, 16, t, UINT32_MAX, UINT32_MAX, H, y);     /* OPERATOR_OUTPUT */
    }
    if (st == KQO_OK) memcpy(output, staged, sizeof(float) * tokens * H);
    free(buf);
    free(ids);
    return st;
}

/* ----------------------------------------------------------------- layer */

/* Gated-residual read of src/kq_layer_qwen38.c:37-165 over F32 weights:
 * per-branch (1 + w) RMSNorm, rank = silu(down . n / B), read gate =
 * sigmoid(up . rank), mixed = sum_b gate * n / B, write gate =
 * 2 sigmoid(inject . n / B). */
static int kqo_gr_read(const kqo_layer_dims *dm, const kqo_gr_weights *w, const float *br, float *nm, float *rg,
                       float *mixed, float *rank, float *wg) {
    const uint64_t H = dm->hidden_size, B = dm->branch_count, R = dm->gr_rank, W = H * B;
    uint64_t b, i, j;
    for (b = 0; b < B; ++b) {
        /* kq_f32_rms_norm: src/kq_numeric.c:730-774 */
        float sum = 0.0f, mean, inv;
        const float *x = br + b * H;
        for (i = 0; i < H; ++i) {
            float sq = x[i] * x[i];
            sum = sum + sq;
        }
        mean = sum / (float)H;
        inv = 1.0f / sqrtf(mean + dm->rms_epsilon);
        if (!isfinite(inv)) return KQO_NUMERIC_DOMAIN;
        for (i = 0; i < H; ++i) {
            float n = x[i] * inv;
            float wt = 1.0f + w->norm[b * H + i];
            nm[b * H + i] = n * wt;
            if (!isfinite(nm[b * H + i])) return KQO_NUMERIC_DOMAIN;
        }
    }
    for (i = 0; i < R; ++i) {
        float sum = 0.0f;
        for (j = 0; j < W; ++j) sum += w->down[i * W + j] * nm[j];
        rank[i] = sum;
    }
    for (i = 0; i < R; ++i) rank[i] /= (float)B;
    for (i = 0; i < R; ++i) rank[i] *= kqo_sigmoid(rank[i]);
    for (i = 0; i < W; ++i) {
        float sum = 0.0f;
        for (j = 0; j < R; ++j) sum += w->up[i * R + j] * rank[j];
        rg[i] = sum;
    }
    for (i = 0; i < W; ++i) rg[i] = kqo_sigmoid(rg[i]);
    for (i = 0; i < H; ++i) {
        float sum = 0.0f;
        for (b = 0; b < B; ++b) sum += rg[b * H + i] * nm[b * H + i];
        mixed[i] = sum / (float)B;
    }
    for (b = 0; b < B; ++b) {
        float sum = 0.0f;
        for (j = 0; j < W; ++j) sum += w->inject[b * W + j] * nm[j];
        wg[b] = sum;
    }
    for (b = 0; b < B; ++b) wg[b] /= (float)B;
    for (b = 0; b < B; ++b) wg[b] = 2.0f * kqo_sigmoid(wg[b]);
    return KQO_OK;
}

/* kq_layer_gr_write_f32: src/kq_layer_qwen38.c:196-209. */
static void kqo_gr_write(const kqo_layer_dims *dm, const float *br, const float *block, const float *wg, float *out) {
    uint64_t b, i;
    for (b = 0; b < dm->branch_count; ++b)
        for (i = 0; i < dm->hidden_size; ++i) {
            uint64_t o = b * dm->hidden_size + i;
            out[o] = br[o] + block[i] * wg[b];
        }
}

/* One decoder layer over T tokens (src/kq_layer.c:639-827 without PLE):
 * attention gated-residual read per token, the mixer over all T tokens
 * (GDN with the padding mask, or QSA), write, MoE gated-residual read, the
 * MoE over all T tokens, write.  The mixer's state arrays are updated only
 * on success (the layer's transactional contract); checkpoints follow
 * include/kq_layer.h's kinds in the reference's order (rank 2 ones with
 * dims (branches, hidden)). */
int kqo_layer_run_observed(const kqo_layer_dims *dm, const kqo_gr_weights *attn_gr, const kqo_gr_weights *moe_gr,
                           const kqo_gdn_dims *gd, const kqo_gdn_weights *gw, float *conv, float *rec,
                           const kqo_qsa_dims *qd, const kqo_qsa_weights *qw, float *kc, float *vc, float *rc,
                           uint64_t capacity, uint64_t *length, const kqo_moe_dims *md, const kqo_moe_weights *mw,
                           const float *input, uint64_t tokens, const uint8_t *mask, float *output,
                           kqo_checkpoint_fn cb, void *user) {
    const uint64_t H = dm->hidden_size, B = dm->branch_count, W = H * B, R = dm->gr_rank;
    float *buf, *nm, *rg, *rank, *mixed, *awg, *block, *after, *moe_in, *mwg, *moe_out, *staged;
    float *conv2 = NULL, *rec2 = NULL;
    uint64_t t, len = length ? *length : 0;
    int st = KQO_OK;
    if (H == 0 || B == 0 || R == 0 || (dm->family == 1) == (gd == NULL)) return KQO_INVALID_ARGUMENT;
    buf = (float *)malloc(sizeof(float) * (2 * W + R + tokens * (2 * H + B + W + H + B + H + W)));
    if (buf == NULL) return KQO_INVALID_ARGUMENT;
    nm = buf; rg = nm + W; rank = rg + W; mixed = rank + R; awg = mixed + tokens * H; block = awg + tokens * B;
    after = block + tokens * H; moe_in = after + tokens * W; mwg = moe_in + tokens * H; moe_out = mwg + tokens * B;
    staged = moe_out + tokens * H;
    for (t = 0; t < tokens; ++t) kqo_emit(cb, user, 0, t, 2, B, H, 0, input + t * W, W);   /* INPUT */
    for (t = 0; t < tokens && st == KQO_OK; ++t) {
        st = kqo_gr_read(dm, attn_gr, input + t * W, nm, rg, mixed + t * H, rank, awg + t * B);
        if (st != KQO_OK) break;
        kqo_emit(cb, user, 3, t, 2, B, H, 0, nm, W);             /* ATTN_GR_NORMALIZED */
        kqo_emit(cb, user, 4, t, 2, B, H, 0, rg, W);             /* ATTN_GR_READ_GATE */
        kqo_emit(cb, user, 5, t, 1, H, 0, 0, mixed + t * H, H);  /* MIXER_INPUT */
    }
    if (st == KQO_OK) {
        if (gd != NULL) {
            const uint64_t nc = ((uint64_t)2 * gd->key_heads * gd->key_dim +
                                 (uint64_t)gd->value_heads * gd->value_dim) * gd->conv_kernel;
            const uint64_t nr = (uint64_t)gd->value_heads * gd->key_dim * gd->value_dim;
            conv2 = (float *)malloc(sizeof(float) * nc);
            rec2 = (float *)malloc(sizeof(float) * nr);
            if (conv2 == NULL || rec2 == NULL) st = KQO_INVALID_ARGUMENT;
            else {
                memcpy(conv2, conv, sizeof(float) * nc);
                memcpy(rec2, rec, sizeof(float) * nr);
                st = kqo_gdn_run(gd, gw, mixed, tokens, mask, block, conv2, rec2);
                if (st == KQO_OK) {
                    memcpy(conv, conv2, sizeof(float) * nc);
                    memcpy(rec, rec2, sizeof(float) * nr);
                }
            }
        } else {
            st = kqo_qsa_run(qd, qw, mixed, tokens, block, kc, vc, rc, capacity, &len, NULL, NULL, NULL);
        }
    }
    for (t = 0; t < tokens && st == KQO_OK; ++t) {
        kqo_emit(cb, user, 6, t, 1, H, 0, 0, block + t * H, H);   /* MIXER_OUTPUT */
        kqo_emit(cb, user, 7, t, 1, B, 0, 0, awg + t * B, B);     /* ATTN_GR_WRITE_GATE */
        kqo_gr_write(dm, input + t * W, block + t * H, awg + t * B, after + t * W);
        kqo_emit(cb, user, 8, t, 2, B, H, 0, after + t * W, W);   /* AFTER_MIXER_RESIDUAL */
        st = kqo_gr_read(dm, moe_gr, after + t * W, nm, rg, moe_in + t * H, rank, mwg + t * B);
        if (st != KQO_OK) break;
        kqo_emit(cb, user, 9, t, 2, B, H, 0, nm, W);              /* MOE_GR_NORMALIZED */
        kqo_emit(cb, user, 10, t, 2, B, H, 0, rg, W);             /* MOE_GR_READ_GATE */
        kqo_emit(cb, user, 11, t, 1, H, 0, 0, moe_in + t * H, H); /* MOE_INPUT */
    }
    if (st == KQO_OK) st = kqo_moe_run(md, mw, moe_in, tokens, moe_out, NULL, NULL, NULL, NULL);
    for (t = 0; t < tokens && st == KQO_OK; ++t) {
        kqo_emit(cb, user, 12, t, 1, H, 0, 0, moe_out + t * H, H);  /* MOE_OUTPUT */
        kqo_emit(cb, user, 13, t, 1, B, 0, 0, mwg + t * B, B);      /* MOE_GR_WRITE_GATE */
        kqo_gr_write(dm, after + t * W, moe_out + t * H, mwg + t * B, staged + t * W);
        kqo_emit(cb, user, 14, t, 2, B, H, 0, staged + t * W, W);   /* OUTPUT */
    }
    if (st == KQO_OK) {
        memcpy(output, staged, sizeof(float) * tokens * W);
        if (length) *length = len;
    }
    free(conv2);
    free(rec2);
    free(buf);
    return st;
}
