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

}  // namespace kqb
