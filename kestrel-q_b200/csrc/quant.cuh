// Device-side GGUF block decoding, bit-identical to the reference's scalar C.
//
// Every product / difference is an explicitly rounded F32 operation
// (__fmul_rn / __fsub_rn), so nvcc cannot contract them into FMAs: the
// reference is compiled with -ffp-contract=off and rounds each step
// (src/kq_numeric.c:210-277 of Kestrel-Q).  Q6_K follows the public GGUF
// block format (the reference has no Q6_K).
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace kqb {

enum : uint32_t {
    kTypeF32 = 0,
    kTypeQ8_0 = 8,
    kTypeQ4_K = 12,
    kTypeQ6_K = 14,
    kTypeBF16 = 30,
};

// f16 bits -> f32, exact for normals, subnormals, inf and NaN payloads
// (src/kq_numeric.c:58-82).
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exponent = (h >> 10) & 0x1fu;
    uint32_t mantissa = h & 0x3ffu;
    uint32_t bits;
    if (exponent == 0u) {
        if (mantissa == 0u) {
            bits = sign;
        } else {
            // subnormal: the leading one sits at bit (31 - clz); shift it to
            // bit 10 and lower the exponent accordingly.
            int lead = 31 - __clz(mantissa);   // 0..9
            int shift = 10 - lead;
            mantissa = (mantissa << shift) & 0x3ffu;
            bits = sign | ((uint32_t)(113 - shift) << 23) | (mantissa << 13);
        }
    } else if (exponent == 31u) {
        bits = sign | 0x7f800000u | (mantissa << 13);
    } else {
        bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t load_u16(const uint8_t *p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8);
}

// 6-bit scale/min pair j (0..7) of a Q4_K super-block (src/kq_numeric.c:161-174).
__device__ __forceinline__ void q4k_scale_min(const uint8_t *s, int j,
                                              uint32_t &sc, uint32_t &mn) {
    if (j < 4) {
        sc = s[j] & 63u;
        mn = s[j + 4] & 63u;
    } else {
        sc = (s[j + 4] & 15u) | ((uint32_t)(s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

// Geometry of a supported type; returns false for unsupported ids.
__host__ __device__ __forceinline__ bool block_geometry(uint32_t type, uint32_t &elems,
                                                        uint32_t &bytes) {
    switch (type) {
    case kTypeF32: elems = 1; bytes = 4; return true;
    case kTypeBF16: elems = 1; bytes = 2; return true;
    case kTypeQ8_0: elems = 32; bytes = 34; return true;
    case kTypeQ4_K: elems = 256; bytes = 144; return true;
    case kTypeQ6_K: elems = 256; bytes = 210; return true;
    default: elems = 0; bytes = 0; return false;
    }
}

// Decodes elements [first, first + count) of one row of `cols` columns.
// `row` points at the row's first packed byte.  `count` and `first` must
// stay inside one 32-element group for the K-quants (first % 32 + count <= 32
// is not required for F32/BF16/Q8_0).  Used where a thread owns a run of up
// to 32 consecutive elements.
__device__ __forceinline__ void decode_run(uint32_t type, const uint8_t *row,
                                           uint32_t first, uint32_t count,
                                           float *out) {
    if (type == kTypeF32) {
        const float *p = reinterpret_cast<const float *>(row) + first;
        for (uint32_t i = 0; i < count; ++i) out[i] = p[i];
    } else if (type == kTypeBF16) {
        const uint16_t *p = reinterpret_cast<const uint16_t *>(row) + first;
        for (uint32_t i = 0; i < count; ++i) out[i] = __uint_as_float((uint32_t)p[i] << 16);
    } else if (type == kTypeQ8_0) {
        for (uint32_t i = 0; i < count; ++i) {
            uint32_t e = first + i;
            const uint8_t *b = row + (e >> 5) * 34u;
            float d = half_bits_to_float(load_u16(b));
            out[i] = __fmul_rn((float)(int8_t)b[2 + (e & 31u)], d);
        }
    } else if (type == kTypeQ4_K) {
        // all `count` elements share one super-block and one 32-group
        const uint8_t *b = row + (first >> 8) * 144u;
        uint32_t within = first & 255u;
        uint32_t group = within >> 6;          // 0..3
        uint32_t high = (within >> 5) & 1u;    // low or high nibble half
        uint32_t idx0 = within & 31u;
        float d = half_bits_to_float(load_u16(b));
        float dmin = half_bits_to_float(load_u16(b + 2));
        uint32_t sc, mn;
        q4k_scale_min(b + 4, (int)(2u * group + high), sc, mn);
        float dl = __fmul_rn(d, (float)sc);
        float ml = __fmul_rn(dmin, (float)mn);
        const uint8_t *q = b + 16 + group * 32u;
        for (uint32_t i = 0; i < count; ++i) {
            uint32_t byte = q[idx0 + i];
            uint32_t code = high ? (byte >> 4) : (byte & 15u);
            out[i] = __fsub_rn(__fmul_rn(dl, (float)code), ml);
        }
    } else if (type == kTypeQ6_K) {
        const uint8_t *b = row + (first >> 8) * 210u;
        uint32_t within = first & 255u;
        uint32_t half = within >> 7;            // 0..1
        uint32_t v = within & 127u;
        uint32_t s = v >> 5;                    // which of the 4 interleaved runs
        uint32_t l0 = v & 31u;
        const uint8_t *ql = b + half * 64u;
        const uint8_t *qh = b + 128u + half * 32u;
        const int8_t *sc = reinterpret_cast<const int8_t *>(b + 192u) + half * 8u;
        float d = half_bits_to_float(load_u16(b + 208u));
        for (uint32_t i = 0; i < count; ++i) {
            uint32_t l = l0 + i;
            uint32_t lowbyte = ql[l + ((s & 1u) << 5)];
            uint32_t lo = (s & 2u) ? (lowbyte >> 4) : (lowbyte & 15u);
            uint32_t hi = (qh[l] >> (2u * s)) & 3u;
            int code = (int)(lo | (hi << 4)) - 32;
            float scale = __fmul_rn(d, (float)sc[(l >> 4) + 2u * s]);
            out[i] = __fmul_rn(scale, (float)code);
        }
    }
}

// ------------------------------------------------------------------ fast path
//
// decode32: 32 consecutive elements starting at `first` (a multiple of 32,
// first + 32 <= cols) of one row, with 16-byte vector loads.  Same
// arithmetic as decode_run (bit-identical results).  `row` must be 16-byte
// aligned and the row length a multiple of 16 bytes for the planar and Q4_K
// layouts; callers fall back to decode_run otherwise.

__device__ __forceinline__ void bytes16(uint4 v, uint8_t *b) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        b[4 * i + 0] = (uint8_t)(w[i]);
        b[4 * i + 1] = (uint8_t)(w[i] >> 8);
        b[4 * i + 2] = (uint8_t)(w[i] >> 16);
        b[4 * i + 3] = (uint8_t)(w[i] >> 24);
    }
}

template <uint32_t TYPE, uint32_t LAYOUT>
__device__ __forceinline__ void decode32_t(const uint8_t *row, uint32_t cols, uint32_t first, float *out) {
    if constexpr (TYPE == kTypeQ4_K) {
        const uint8_t *b = row + (first >> 8) * 144u;
        const uint32_t w = first & 255u, group = w >> 6, high = (w >> 5) & 1u;
        uint8_t hdr[16], q[32];
        bytes16(*reinterpret_cast<const uint4 *>(b), hdr);
        bytes16(*reinterpret_cast<const uint4 *>(b + 16 + group * 32), q);
        bytes16(*reinterpret_cast<const uint4 *>(b + 32 + group * 32), q + 16);
        const float d = half_bits_to_float((uint32_t)hdr[0] | ((uint32_t)hdr[1] << 8));
        const float dmin = half_bits_to_float((uint32_t)hdr[2] | ((uint32_t)hdr[3] << 8));
        uint32_t sc, mn;
        q4k_scale_min(hdr + 4, (int)(2u * group + high), sc, mn);
        const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dmin, (float)mn);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t code = high ? (q[i] >> 4) : (q[i] & 15u);
            out[i] = __fsub_rn(__fmul_rn(dl, (float)code), ml);
        }
    } else if constexpr (TYPE == kTypeQ6_K && LAYOUT == 1) {
        const uint32_t nsb = cols >> 8, sb = first >> 8, w = first & 255u;
        const uint32_t half = w >> 7, s = (w & 127u) >> 5;
        const uint8_t *ql = row + sb * 128u + half * 64u + 32u * (s & 1u);
        const uint8_t *qh = row + nsb * 128u + sb * 64u + half * 32u;
        const int8_t *sc = reinterpret_cast<const int8_t *>(row + nsb * 192u + sb * 16u + half * 8u + 2u * s);
        const uint8_t *dp = row + nsb * 208u + sb * 2u;
        uint8_t lo[32], hi[32];
        bytes16(*reinterpret_cast<const uint4 *>(ql), lo);
        bytes16(*reinterpret_cast<const uint4 *>(ql + 16), lo + 16);
        bytes16(*reinterpret_cast<const uint4 *>(qh), hi);
        bytes16(*reinterpret_cast<const uint4 *>(qh + 16), hi + 16);
        const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
        const float s0 = __fmul_rn(d, (float)sc[0]), s1 = __fmul_rn(d, (float)sc[1]);
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const uint32_t nib = (s & 2u) ? (lo[l] >> 4) : (lo[l] & 15u);
            const int code = (int)(nib | (((hi[l] >> (2u * s)) & 3u) << 4)) - 32;
            out[l] = __fmul_rn(l < 16 ? s0 : s1, (float)code);
        }
    } else if constexpr (TYPE == kTypeQ8_0 && LAYOUT == 1) {
        const uint32_t nb = cols >> 5, blk = first >> 5;
        const uint8_t *codes = row + blk * 32u;
        const uint8_t *dp = row + nb * 32u + blk * 2u;
        uint8_t c[32];
        bytes16(*reinterpret_cast<const uint4 *>(codes), c);
        bytes16(*reinterpret_cast<const uint4 *>(codes + 16), c + 16);
        const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
#pragma unroll
        for (int i = 0; i < 32; ++i) out[i] = __fmul_rn((float)(int8_t)c[i], d);
    } else if constexpr (TYPE == kTypeBF16) {
        const uint4 *p = reinterpret_cast<const uint4 *>(row + (size_t)first * 2u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint4 v = p[j];
            const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                out[8 * j + 2 * i] = __uint_as_float(w4[i] << 16);
                out[8 * j + 2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
            }
        }
    } else {   // F32
        const float4 *p = reinterpret_cast<const float4 *>(row + (size_t)first * 4u);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 v = p[j];
            out[4 * j] = v.x; out[4 * j + 1] = v.y; out[4 * j + 2] = v.z; out[4 * j + 3] = v.w;
        }
    }
}

// Scalar decode of `count` elements of a planar-layout row (tails).
__device__ __forceinline__ void decode_run_planar(uint32_t type, const uint8_t *row, uint32_t cols,
                                                  uint32_t first, uint32_t count, float *out) {
    if (type == kTypeQ8_0) {
        const uint32_t nb = cols >> 5;
        for (uint32_t i = 0; i < count; ++i) {
            const uint32_t e = first + i, blk = e >> 5;
            const uint8_t *dp = row + nb * 32u + blk * 2u;
            const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
            out[i] = __fmul_rn((float)(int8_t)row[blk * 32u + (e & 31u)], d);
        }
    } else {   // Q6_K
        const uint32_t nsb = cols >> 8;
        for (uint32_t i = 0; i < count; ++i) {
            const uint32_t e = first + i, sb = e >> 8, w = e & 255u;
            const uint32_t half = w >> 7, s = (w & 127u) >> 5, l = w & 31u;
            const uint8_t lob = row[sb * 128u + half * 64u + 32u * (s & 1u) + l];
            const uint8_t hib = row[nsb * 128u + sb * 64u + half * 32u + l];
            const int8_t scv = (int8_t)row[nsb * 192u + sb * 16u + half * 8u + 2u * s + (l >> 4)];
            const uint8_t *dp = row + nsb * 208u + sb * 2u;
            const float d = half_bits_to_float((uint32_t)dp[0] | ((uint32_t)dp[1] << 8));
            const uint32_t nib = (s & 2u) ? (lob >> 4) : (lob & 15u);
            const int code = (int)(nib | (((hib >> (2u * s)) & 3u) << 4)) - 32;
            out[i] = __fmul_rn(__fmul_rn(d, (float)scv), (float)code);
        }
    }
}

// Any run of a provider matrix (layout-aware).  A 32-element aligned run
// of an aligned row takes the vectorised path.
template <typename M>
__device__ __forceinline__ void decode_any(const M &m, const uint8_t *row, uint32_t first, uint32_t count,
                                           float *out) {
    const bool fast = count == 32u && (first & 31u) == 0u && (m.row_bytes & 15u) == 0u &&
                      (reinterpret_cast<uintptr_t>(row) & 15u) == 0u;
    if (fast) {
        switch (m.type) {
        case kTypeQ4_K: decode32_t<kTypeQ4_K, 0>(row, m.cols, first, out); return;
        case kTypeQ6_K:
            if (m.layout == 1) { decode32_t<kTypeQ6_K, 1>(row, m.cols, first, out); return; }
            break;
        case kTypeQ8_0:
            if (m.layout == 1) { decode32_t<kTypeQ8_0, 1>(row, m.cols, first, out); return; }
            break;
        case kTypeBF16: decode32_t<kTypeBF16, 0>(row, m.cols, first, out); return;
        case kTypeF32: decode32_t<kTypeF32, 0>(row, m.cols, first, out); return;
        default: break;
        }
    }
    if (m.layout == 1 && (m.type == kTypeQ6_K || m.type == kTypeQ8_0))
        decode_run_planar(m.type, row, m.cols, first, count, out);
    else
        decode_run(m.type, row, first, count, out);
}

// Exactly 32 values (zero past the row end) with static indexing only, so
// `out` stays in registers.  Fast vector path when aligned, element-wise
// otherwise.
template <typename M>
__device__ __forceinline__ void decode32_any(const M &m, const uint8_t *row, uint32_t first, float (&out)[32]) {
    const bool fast = (first & 31u) == 0u && first + 32u <= m.cols && (m.row_bytes & 15u) == 0u &&
                      (reinterpret_cast<uintptr_t>(row) & 15u) == 0u;
    if (fast) {
        switch (m.type) {
        case kTypeQ4_K: decode32_t<kTypeQ4_K, 0>(row, m.cols, first, out); return;
        case kTypeQ6_K:
            if (m.layout == 1) { decode32_t<kTypeQ6_K, 1>(row, m.cols, first, out); return; }
            break;
        case kTypeQ8_0:
            if (m.layout == 1) { decode32_t<kTypeQ8_0, 1>(row, m.cols, first, out); return; }
            break;
        case kTypeBF16: decode32_t<kTypeBF16, 0>(row, m.cols, first, out); return;
        case kTypeF32: decode32_t<kTypeF32, 0>(row, m.cols, first, out); return;
        default: break;
        }
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) {
        float v[1] = {0.0f};
        if (first + i < m.cols) {
            if (m.layout == 1 && (m.type == kTypeQ6_K || m.type == kTypeQ8_0))
                decode_run_planar(m.type, row, m.cols, first + i, 1, v);
            else
                decode_run(m.type, row, first + i, 1, v);
        }
        out[i] = v[0];
    }
}

// Two-phase form of decode32_any for software pipelining: load_raw32 issues
// the 16-byte loads of a run (no use of the data), decode_raw32 decodes it
// later.  Runs that are not vector-aligned, and F32 rows, are decoded
// directly from memory by decode_raw32.
struct Raw32 {
    uint4 v[4];
    uint32_t e;
    uint32_t fast;
};

__device__ __forceinline__ uint4 ld16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

template <typename M>
__device__ __forceinline__ void load_raw32(const M &m, const uint8_t *row, uint32_t first, Raw32 &r) {
    r.fast = ((first & 31u) == 0u && first + 32u <= m.cols && (m.row_bytes & 15u) == 0u &&
              (reinterpret_cast<uintptr_t>(row) & 15u) == 0u) ? 1u : 0u;
    if (!r.fast) return;
    if (m.type == kTypeQ4_K) {
        const uint8_t *b = row + (first >> 8) * 144u;
        const uint32_t g = (first & 255u) >> 6;
        r.v[0] = ld16(b);
        r.v[1] = ld16(b + 16 + g * 32);
        r.v[2] = ld16(b + 32 + g * 32);
    } else if (m.type == kTypeQ6_K && m.layout == 1) {
        const uint32_t nsb = m.cols >> 8, sb = first >> 8, w = first & 255u;
        const uint32_t half = w >> 7, s = (w & 127u) >> 5;
        const uint8_t *ql = row + sb * 128u + half * 64u + 32u * (s & 1u);
        const uint8_t *qh = row + nsb * 128u + sb * 64u + half * 32u;
        r.v[0] = ld16(ql);
        r.v[1] = ld16(ql + 16);
        r.v[2] = ld16(qh);
        r.v[3] = ld16(qh + 16);
        const uint32_t scp = *reinterpret_cast<const uint16_t *>(row + nsb * 192u + sb * 16u + half * 8u + 2u * s);
        const uint32_t dp = *reinterpret_cast<const uint16_t *>(row + nsb * 208u + sb * 2u);
        r.e = scp | (dp << 16);
    } else if (m.type == kTypeQ8_0 && m.layout == 1) {
        const uint32_t nb = m.cols >> 5, blk = first >> 5;
        r.v[0] = ld16(row + blk * 32u);
        r.v[1] = ld16(row + blk * 32u + 16);
        r.e = *reinterpret_cast<const uint16_t *>(row + nb * 32u + blk * 2u);
    } else if (m.type == kTypeBF16) {
        const uint8_t *p = row + (size_t)first * 2u;
        r.v[0] = ld16(p); r.v[1] = ld16(p + 16); r.v[2] = ld16(p + 32); r.v[3] = ld16(p + 48);
    } else {
        r.fast = 0u;
    }
}

template <typename M>
__device__ __forceinline__ void decode_raw32(const M &m, const Raw32 &r, const uint8_t *row, uint32_t first,
                                             float (&out)[32]) {
    if (!r.fast) {
        decode32_any(m, row, first, out);
        return;
    }
    if (m.type == kTypeQ4_K) {
        uint8_t hdr[16], q[32];
        bytes16(r.v[0], hdr);
        bytes16(r.v[1], q);
        bytes16(r.v[2], q + 16);
        const uint32_t w = first & 255u, group = w >> 6, high = (w >> 5) & 1u;
        const float d = half_bits_to_float((uint32_t)hdr[0] | ((uint32_t)hdr[1] << 8));
        const float dmin = half_bits_to_float((uint32_t)hdr[2] | ((uint32_t)hdr[3] << 8));
        uint32_t sc, mn;
        q4k_scale_min(hdr + 4, (int)(2u * group + high), sc, mn);
        const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dmin, (float)mn);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t code = high ? (q[i] >> 4) : (q[i] & 15u);
            out[i] = __fsub_rn(__fmul_rn(dl, (float)code), ml);
        }
    } else if (m.type == kTypeQ6_K) {
        uint8_t lo[32], hi[32];
        bytes16(r.v[0], lo);
        bytes16(r.v[1], lo + 16);
        bytes16(r.v[2], hi);
        bytes16(r.v[3], hi + 16);
        const uint32_t s = ((first & 255u) & 127u) >> 5;
        const float d = half_bits_to_float(r.e >> 16);
        const float s0 = __fmul_rn(d, (float)(int8_t)(r.e & 0xFFu));
        const float s1 = __fmul_rn(d, (float)(int8_t)((r.e >> 8) & 0xFFu));
#pragma unroll
        for (int l = 0; l < 32; ++l) {
            const uint32_t nib = (s & 2u) ? (lo[l] >> 4) : (lo[l] & 15u);
            const int code = (int)(nib | (((hi[l] >> (2u * s)) & 3u) << 4)) - 32;
            out[l] = __fmul_rn(l < 16 ? s0 : s1, (float)code);
        }
    } else if (m.type == kTypeQ8_0) {
        uint8_t c[32];
        bytes16(r.v[0], c);
        bytes16(r.v[1], c + 16);
        const float d = half_bits_to_float(r.e & 0xFFFFu);
#pragma unroll
        for (int i = 0; i < 32; ++i) out[i] = __fmul_rn((float)(int8_t)c[i], d);
    } else {   // BF16
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t w4[4] = {r.v[j].x, r.v[j].y, r.v[j].z, r.v[j].w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                out[8 * j + 2 * i] = __uint_as_float(w4[i] << 16);
                out[8 * j + 2 * i + 1] = __uint_as_float(w4[i] & 0xFFFF0000u);
            }
        }
    }
}

}  // namespace kqb
