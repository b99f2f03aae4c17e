// Dequant-fused projection GEMM on the 5th-generation tensor cores.
//
//   y[b][n] = sum_k W[n][k] * x[b][k]      (W: GGUF blocks in HBM, x: F32)
//
// One CTA computes a 128 (weight rows, MMA M) x 64 (batch rows, MMA N) tile
// of y^T with tcgen05.mma (kind::f16, FP16 operands, F32 accumulator in
// TMEM).  F32 accuracy is kept with a three-term split: w = wh + wl and
// x = xh + xl (fp16 each, both parts rounded to nearest, so each pair holds
// 22 significant bits), y ~= wh*xh + wh*xl + wl*xh; the dropped wl*xl term
// and the rounding of the low parts are ~2^-22 relative per product (a
// bf16 split, 8 bits per part, left ~2^-16, which over K = 4096 products of
// outputs of a few hundred exceeded a 2e-3 absolute tolerance).  fp16's
// range is kept by exact power-of-two scales: the weights of a matrix by
// 2^scale_exp (chosen at upload from the block headers so that every value
// is below 2^14), the activations by 2^-2 (inputs must stay below 2^18 in
// magnitude; larger ones raise a range error); the epilogue undoes both.
//
// Warp roles (608 threads, one CTA per SM):
//   TMA warp     per K chunk of 64: 2-D TMA loads of the chunk's raw GGUF
//                bytes (16-byte columns x 128 rows: Q4_K header + quants,
//                Q6_K/Q8_0 planes, BF16 values) and a 1-D bulk copy of the
//                chunk's activation tile, which a small kernel converted
//                once per launch into bf16 hi/lo in the 128-byte-swizzled
//                K-major image the MMA reads.  Ring of 6 (Q6_K, BF16) to
//                9 (Q4_K) slots in 200 KB of shared memory.
//   16 decode    each thread owns one weight row (its TMEM lane) and 16 K
//   warps        values of the chunk: decodes them from shared memory with
//                exact arithmetic (an FMA on a byte-to-float bit pattern,
//                same values as the reference decoder, src/kq_numeric.c),
//                splits them into bf16 hi/lo and stores both
//                straight into TMEM with tcgen05.st: the A operand never
//                touches shared memory.  Six A buffers in TMEM.
//   MMA warp     per K-step of 16, one thread issues an N=128 MMA
//                wh * [xh | xl] (the activation tile's hi and lo halves are
//                adjacent, so one instruction covers both terms) and an N=64
//                MMA wl * xh into the first 64 columns of the same
//                accumulator; A from TMEM, B from shared memory.  It commits
//                to the chunk's mbarrier, which frees the ring slot and the
//                TMEM A buffer.  (An M=128 tcgen05.mma costs about the same
//                issue time for N=64 and N=128.)
// Epilogue: the decode warps read the three partial products with
// tcgen05.ld and add them.
// Split-K runs as a thread-block cluster along gridDim.z: every CTA leaves
// its accumulator tile in shared memory and each CTA sums one slice of the
// rows over all CTAs of the cluster in rank order (distributed shared
// memory, deterministic, no second kernel and no partials in HBM).
//
// Every mbarrier wait is bounded.  A wait that gives up records an error in
// the call's error word and raises a CTA-wide abort flag; every role then
// leaves its loop, waits (bounded) for MMAs in flight, frees TMEM and the
// CTA still reaches the cluster barriers, so no CTA is left waiting.
#include "kernels.hpp"
#include "quant.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace kqb {

namespace {

constexpr int kUM = 128;                  // weight rows per CTA (MMA M)
constexpr int kUN = 64;                   // batch rows per CTA, small batches (MMA N)
constexpr int kUNWide = 256;              // batch rows per CTA, large batches (prefill)
constexpr int kUK = 64;                   // K per chunk (one 128-byte swizzle row of bf16)
constexpr int kMaxXRing = 10;
constexpr int kMaxRawRing = 3;
constexpr int kMaxABufs = 6;
constexpr int kDecodeWarps = 16;
// The single-thread roles sit on different schedulers (scheduler = warp % 4),
// because their TMA / MMA instructions take issue time from the decode warps
// that share a scheduler with them: warp 16 (scheduler 0) owns TMEM, 17
// (scheduler 1) issues the MMAs, 18 (scheduler 2) the TMA loads.
constexpr int kAllocWarp = kDecodeWarps;
constexpr int kMmaWarp = kDecodeWarps + 1;
constexpr int kTmaWarp = kDecodeWarps + 2;
constexpr int kThreads = (kDecodeWarps + 3) * 32;
constexpr int kAccStride = kUN + 1;       // floats per row of the split-K exchange tile
constexpr uint32_t kTmemCols = 512;
// Activations enter the MMA as fp16 hi/lo parts of x * kXScale (exact);
// |x| must stay below kXRangeLimit, where x / 4 would round to fp16 infinity
// beyond 65504.  The epilogue multiplies by 2^(2 - scale_exp).
constexpr float kXScale = 0.25f;
constexpr float kXRangeLimit = 262016.0f;
constexpr uint32_t kXmSlotBytes = 16384;   // minimum-term activation tile (factored kernel)

// Geometry of a tile of NT batch rows.
//  NT = 64: TMEM columns [0, 128) hold the accumulator: wh * [xh | xl]
//           (N = 128) with wl * xh (N = 64) added into its first 64 columns;
//           six A buffers follow.
//  NT = 256: the activation tile is [xh (256 rows) | xl (256 rows)] and all
//           three products go into one accumulator of 256 columns (three
//           N = 256 MMAs per K step); four A buffers follow.  Each decoded
//           weight chunk then feeds four times the MMA work, which is what
//           a prefill needs (decode time per chunk is the same).
// An A buffer is 64 columns: hi 32 | lo 32 (64 bf16 K values each).
template <uint32_t NT> struct Tile {
    static_assert(NT == 64 || NT == 256, "tile widths");
    static constexpr uint32_t xslot = 2u * NT * kUK * 2u;       // bytes: [xh | xl]
    static constexpr uint32_t raw_ring = NT == 64 ? 3u : 2u;    // raw super-block slots
    static constexpr uint32_t budget = (NT == 64 ? 200u : 220u) * 1024u;
    static constexpr uint32_t dcols = NT == 64 ? 128u : NT;
    static constexpr uint32_t abase = dcols;
    static constexpr uint32_t abufs = (kTmemCols - dcols) / 64u < (uint32_t)kMaxABufs
                                          ? (kTmemCols - dcols) / 64u : (uint32_t)kMaxABufs;
    static_assert(abase + 64u * abufs <= kTmemCols, "TMEM budget");
};
constexpr uint32_t kWaitLimit = 1u << 26;           // mbarrier polls before giving up
constexpr uint64_t kWaitNs = 2000000000ull;          // or 2 s of global time, whichever comes first

// Wait sites, recorded in the abort flag by the first wait that gives up
// and reported in the error code (kErrTimeout | site << 8).
enum WaitSite : uint32_t {
    kSiteRawFree = 1, kSiteXFree, kSiteAReady, kSiteXFull, kSiteRawFull, kSiteADone, kSiteAccum,
    kSiteDFree, kSiteDFull, kSiteXmFull, kSiteXmFree, kSiteScale
};

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Bounded wait for the phase with parity `parity` to complete.  Gives up
// early when another role has raised the CTA's abort flag; raises it itself
// (with its site) when the poll limit or the time limit is reached.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile uint32_t *abort,
                                          uint32_t site) {
    const uint32_t addr = smem_u32(bar);
    uint64_t t0 = 0;   // the clock is read only once a wait is slow
    for (uint32_t i = 0; i < kWaitLimit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.b32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((i & 63u) == 63u) {
            if (*abort) return false;
            const uint64_t now = global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kWaitNs) break;
        }
    }
    atomicCAS(const_cast<uint32_t *>(abort), 0u, site);
    return false;
}

// Warp-uniform form: lane 0 waits, the result is broadcast.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, volatile uint32_t *abort,
                                               uint32_t site) {
    uint32_t ok = 0;
    if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, abort, site) ? 1u : 0u;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    return ok != 0;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

// 2-D TMA tile load (no multicast) completing on `bar`.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// 1-D bulk copy global -> shared (no multicast) completing on `bar`.
__device__ __forceinline__ void bulk_load(uint32_t dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// K-major, 128B-swizzled shared-memory matrix descriptor (sm_100 format:
// start >> 4 in [0,14), LBO (16 B, ignored for swizzled K-major) in
// [16,30), SBO = 1024 B between 8-row groups in [32,46), version 1 in
// [46,48), layout SWIZZLE_128B = 2 in [61,64)).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor: F32 accumulate (c_format 1, bits [4,6)), FP16 A
// and B (a_format = b_format = 0, bits [7,10) and [10,13)), both K-major,
// N >> 3 in [17,23), M >> 4 in [24,29).
constexpr uint32_t idesc_for(uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((uint32_t)(kUM >> 4) << 24);
}

// D (TMEM) += A (TMEM, 128 lanes x 16 K) * B (shared memory descriptor).
template <uint32_t N>
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(tmem_d), "r"(tmem_a), "l"(b), "n"(idesc_for(N)), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// Splits two F32 values into fp16 hi = RN(w) and fp16 lo = RN(w - hi) (the
// residual is exact in F32), packed with w0 in the low half of each word:
// |w - hi - lo| <= 2^-22 |w| for |w| in the fp16 normal range, and at most
// 2^-25 absolute below it.
__device__ __forceinline__ void split_f16(float w0, float w1, uint32_t &hi, uint32_t &lo) {
    const __half2 h = __floats2half2_rn(w0, w1);
    const float2 hf = __half22float2(h);
    const __half2 l = __floats2half2_rn(__fsub_rn(w0, hf.x), __fsub_rn(w1, hf.y));
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = *reinterpret_cast<const uint32_t *>(&l);
}

// Packs 8 values into two 16-byte chunks (hi, lo) of fp16.
__device__ __forceinline__ void pack8(const float *v, uint4 &hi, uint4 &lo) {
    split_f16(v[0], v[1], hi.x, lo.x);
    split_f16(v[2], v[3], hi.y, lo.y);
    split_f16(v[4], v[5], hi.z, lo.z);
    split_f16(v[6], v[7], hi.w, lo.w);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `r` in a SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t chunk) {
    return r * 128u + ((chunk ^ (r & 7u)) << 4);
}


__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Load from the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ float ld_dsmem(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote));
    return v;
}

// ---- exact decode into bf16 hi/lo pairs (f32x2 arithmetic)

__device__ __forceinline__ uint64_t f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void unf2(uint64_t v, float &a, float &b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

// fp16 hi/lo split of a pair of (already scaled) decoded weights.
__device__ __forceinline__ void split_pair(uint64_t w, uint32_t &hi, uint32_t &lo) {
    float w0, w1;
    unf2(w, w0, w1);
    split_f16(w0, w1, hi, lo);
}

// f = 0.5 + u / 256 for the byte u = byte b of w (u < 128): one PRMT builds
// the bit pattern 0x3Fuu0000 (exponent of 0.5, u in the mantissa's top 7
// bits).
__device__ __forceinline__ float half_plus_byte(uint32_t w, uint32_t b) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7054u | (b << 8)));
}
// f = 0.5 + u / 65536 for any byte u = byte b of w (bit pattern 0x3F00uu00).
__device__ __forceinline__ float half_plus_byte16(uint32_t w, uint32_t b) {
    return __uint_as_float(__byte_perm(w, 0x3F000000u, 0x7504u | (b << 4)));
}

// f16 bits -> F32 with the hardware conversion (exact for every f16 value,
// the same result as the reference's bit-level conversion).
__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)bits));
}

__device__ __forceinline__ uint32_t word_of(const uint4 &v, uint32_t i) {
    return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// Raw bytes of one super-block step (SC chunks of 64) for 128 rows, as the
// TMA boxes leave them in shared memory.  Wide boxes keep the TMA engine
// efficient; 128- and 64-byte boxes use the TMA swizzle so that a warp
// reading 32 consecutive rows at the same column is free of bank conflicts.
//   Q4_K (SC 4): [128][144]            whole super-blocks, no swizzle
//   Q6_K (SC 4): ql [128][128] SW128 | qh [128][64] SW64 | sc [128][16] |
//                d window [128][16]
//   Q8_0 (SC 4): codes 2 x [128][128] SW128 | d [128][16]
//   BF16 (SC 2): values 2 x [128][128] SW128
template <uint32_t T> struct TypeCfg;
template <> struct TypeCfg<kTypeQ4_K> { static constexpr uint32_t sc = 4, raw = 128 * 144; };
template <> struct TypeCfg<kTypeQ6_K> { static constexpr uint32_t sc = 4, raw = 128 * 224; };
template <> struct TypeCfg<kTypeQ8_0> { static constexpr uint32_t sc = 4, raw = 128 * 272; };
template <> struct TypeCfg<kTypeBF16> { static constexpr uint32_t sc = 2, raw = 128 * 256; };

// Ring depths per type and tile width within the shared-memory budget.
template <uint32_t T, uint32_t NT> struct Ring {
    static constexpr uint32_t raw = TypeCfg<T>::raw;
    static constexpr uint32_t rr = Tile<NT>::raw_ring;
    static constexpr uint32_t xdepth_fit = (Tile<NT>::budget - rr * raw) / Tile<NT>::xslot;
    static constexpr uint32_t xdepth = xdepth_fit < (uint32_t)kMaxXRing ? xdepth_fit : kMaxXRing;
    static constexpr uint32_t smem = rr * raw + xdepth * Tile<NT>::xslot + 1024 /*align*/;
    static_assert(xdepth >= 2, "double-buffered activations");
    static_assert(rr <= (uint32_t)kMaxRawRing, "raw ring");
    static_assert(raw % 1024 == 0, "slots keep the 1024-byte swizzle alignment");
    static_assert(smem <= 227u * 1024u, "shared memory per CTA");
};

__device__ __forceinline__ uint4 lds16(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
// 16-byte chunk j of row r in a TMA 128B-swizzled box of 128-byte rows.
__device__ __forceinline__ uint32_t sw128_at(uint32_t r, uint32_t j) { return r * 128u + ((j ^ (r & 7u)) << 4); }
// 16-byte chunk j of row r in a TMA 64B-swizzled box of 64-byte rows.
__device__ __forceinline__ uint32_t sw64_at(uint32_t r, uint32_t j) { return r * 64u + ((j ^ ((r >> 1) & 3u)) << 4); }

// Decodes the 16 values [16q, 16q + 16) of chunk c of one staged row, scaled
// by `wscale` (the matrix's power of two), into packed fp16 hi/lo pairs.  The
// decoded F32 values equal the reference decoder's (src/kq_numeric.c) times
// wscale: each is one correctly rounded FMA of exactly representable
// operands, for example Q4_K: dl*code - ml = (256 dl) * f - (128 dl + ml)
// with f = 0.5 + code/256, and scaling both operands by a power of two
// scales the rounded result exactly.
template <uint32_t T>
__device__ __forceinline__ void decode16(const uint8_t *raw, uint32_t row, uint32_t cols, uint32_t c, uint32_t q,
                                         float wscale, uint32_t (&hi)[8], uint32_t (&lo)[8]) {
    if constexpr (T == kTypeQ4_K) {
        // quants: nibble (q >> 1) of bytes 16*(q&1).. of the 64-group
        const uint8_t *blk = raw + row * 144u;
        const uint4 hdr = lds16(blk);
        const uint4 qs = lds16(blk + 16u + (c & 3u) * 32u + 16u * (q & 1u));
        const uint32_t high = q >> 1, j = 2u * (c & 3u) + high;
        const float d = h2f(hdr.x & 0xFFFFu);
        const float dmin = h2f(hdr.x >> 16);
        auto sbyte = [&](uint32_t k) { return (word_of(hdr, 1u + (k >> 2)) >> (8u * (k & 3u))) & 0xFFu; };
        uint32_t sc, mn;
        if (j < 4) {
            sc = sbyte(j) & 63u;
            mn = sbyte(j + 4) & 63u;
        } else {
            sc = (sbyte(j + 4) & 15u) | ((sbyte(j - 4) >> 6) << 4);
            mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
        }
        const float dl = __fmul_rn(d, (float)sc), ml = __fmul_rn(dmin, (float)mn);
        const float a = __fmul_rn(__fmul_rn(dl, 256.0f), wscale);
        const float c0 = __fmul_rn(__fadd_rn(__fmul_rn(dl, 128.0f), ml), wscale);
        const uint64_t A = f2(a, a), C0 = f2(-c0, -c0);
        const uint32_t wq[4] = {qs.x, qs.y, qs.z, qs.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t nib = high ? (wq[k] >> 4) & 0x0F0F0F0Fu : wq[k] & 0x0F0F0F0Fu;
            split_pair(fma2(A, f2(half_plus_byte(nib, 0), half_plus_byte(nib, 1)), C0), hi[2 * k], lo[2 * k]);
            split_pair(fma2(A, f2(half_plus_byte(nib, 2), half_plus_byte(nib, 3)), C0), hi[2 * k + 1],
                       lo[2 * k + 1]);
        }
    } else if constexpr (T == kTypeQ6_K) {
        // code = (ql nibble | qh 2 bits << 4) - 32, value = (d * sc) * code
        const uint32_t nsb = cols >> 8, sb = c >> 2, half = (c & 3u) >> 1;
        const uint32_t h = q >> 1, s = 2u * (c & 1u) + h, part = q & 1u;
        const uint4 ql = lds16(raw + sw128_at(row, 4u * half + 2u * h + part));
        const uint4 qh = lds16(raw + 16384u + sw64_at(row, 2u * half + part));
        const uint32_t scb = raw[24576u + row * 16u + half * 8u + 2u * s + part];
        const uint32_t dbits =
            *reinterpret_cast<const uint16_t *>(raw + 26624u + row * 16u + ((nsb * 208u + sb * 2u) & 15u));
        const float scale = __fmul_rn(h2f(dbits), (float)(int8_t)scb);
        const float a = __fmul_rn(__fmul_rn(scale, 256.0f), wscale);   // all exact
        const float c0 = __fmul_rn(__fmul_rn(scale, 160.0f), wscale);
        const uint64_t A = f2(a, a), C0 = f2(-c0, -c0);
        const uint32_t wl[4] = {ql.x, ql.y, ql.z, ql.w}, wh[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t nib = (c & 1u) ? (wl[k] >> 4) & 0x0F0F0F0Fu : wl[k] & 0x0F0F0F0Fu;
            const uint32_t bw = nib | (((wh[k] >> (2u * s)) & 0x03030303u) << 4);
            split_pair(fma2(A, f2(half_plus_byte(bw, 0), half_plus_byte(bw, 1)), C0), hi[2 * k], lo[2 * k]);
            split_pair(fma2(A, f2(half_plus_byte(bw, 2), half_plus_byte(bw, 3)), C0), hi[2 * k + 1],
                       lo[2 * k + 1]);
        }
    } else if constexpr (T == kTypeQ8_0) {
        // value = code * d with code = (byte ^ 0x80) - 128
        const uint32_t nb = cols >> 5, h = q >> 1, blk = 2u * c + h;
        const uint4 cw = lds16(raw + ((c & 3u) >> 1) * 16384u + sw128_at(row, 4u * (c & 1u) + 2u * h + (q & 1u)));
        const uint32_t dbits =
            *reinterpret_cast<const uint16_t *>(raw + 32768u + row * 16u + ((nb * 32u + blk * 2u) & 15u));
        const float d = h2f(dbits);
        const float a = __fmul_rn(__fmul_rn(d, 65536.0f), wscale);   // all exact
        const float c0 = __fmul_rn(__fmul_rn(d, 32896.0f), wscale);
        const uint64_t A = f2(a, a), C0 = f2(-c0, -c0);
        const uint32_t wc[4] = {cw.x ^ 0x80808080u, cw.y ^ 0x80808080u, cw.z ^ 0x80808080u, cw.w ^ 0x80808080u};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            split_pair(fma2(A, f2(half_plus_byte16(wc[k], 0), half_plus_byte16(wc[k], 1)), C0), hi[2 * k],
                       lo[2 * k]);
            split_pair(fma2(A, f2(half_plus_byte16(wc[k], 2), half_plus_byte16(wc[k], 3)), C0), hi[2 * k + 1],
                       lo[2 * k + 1]);
        }
    } else {   // BF16: each value is its bits << 16 as F32, scaled exactly
        const uint8_t *box = raw + (c & 1u) * 16384u;
        const uint4 v0 = lds16(box + sw128_at(row, 2u * q)), v1 = lds16(box + sw128_at(row, 2u * q + 1u));
        const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int i = 0; i < 8; ++i)
            split_f16(__fmul_rn(__uint_as_float(w[i] << 16), wscale),
                      __fmul_rn(__uint_as_float(w[i] & 0xFFFF0000u), wscale), hi[i], lo[i]);
    }
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                   "r"(r[7])
                 : "memory");
}


}  // namespace

// Tensor maps of the segments' raw bytes: 2-D uint8 [rows][row_bytes],
// boxes of (width, box_rows); up to three widths per type (see TypeCfg).
struct TmapSet {
    CUtensorMap map[kMaxSegments][3];
    uint32_t box_rows[kMaxSegments];
};

// Activations x 2^-2 to fp16 hi/lo tiles in the MMA's shared-memory image:
// out[btile][chunk] = { hi: NT rows x 128 B swizzled, lo: same }.
// One CTA converts 16 rows of one chunk; one thread 8 values.
// With `xm` (64-row tiles whose weights include Q4_K), also the minimum-term
// tiles of the factored kernel: per batch tile and group of 4 super-blocks a
// 128-row SW128 image whose K step u (16 values) holds, for super-block 4g+u
// and batch row r, [Xh_0..7 | Xh_0..7] in row r and [Xl_0..7 | 0] in row
// 64 + r, X_s = (sum of sub-block s's 32 values of x / 4) / 32.
template <uint32_t NT>
__global__ void __launch_bounds__(128)
xconv_kernel(const float *__restrict__ x, uint32_t ldx, uint32_t batch, uint32_t cols, uint32_t nchunks,
             uint8_t *__restrict__ out, uint8_t *__restrict__ xm, uint32_t nxm, ErrorWord err) {
    pdl_wait();
    constexpr uint32_t kGroups = NT / 16u;
    const uint32_t c = blockIdx.x / kGroups, bt = blockIdx.y;
    const uint32_t r = (blockIdx.x % kGroups) * 16u + (threadIdx.x >> 3), q8 = threadIdx.x & 7u;
    const uint32_t b = bt * NT + r, k0 = c * kUK + q8 * 8u;
    float v[8];
    const float *src = x + (size_t)b * ldx + k0;
    if (b < batch && k0 + 8 <= cols && ((reinterpret_cast<uintptr_t>(src) & 15u) == 0)) {
        const float4 a = *reinterpret_cast<const float4 *>(src);
        const float4 e = *reinterpret_cast<const float4 *>(src + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = e.x; v[5] = e.y; v[6] = e.z; v[7] = e.w;
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = (b < batch && k0 + i < cols) ? src[i] : 0.0f;
    }
    // the projection's input check (non-finite input -> NUMERIC_DOMAIN), and
    // the fp16 range of the scaled activations (|x| / 4 < 65504)
    bool bad = false, big = false;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        bad |= !isfinite(v[i]);
        big |= isfinite(v[i]) && !(fabsf(v[i]) < kXRangeLimit);
        v[i] = __fmul_rn(v[i], kXScale);
    }
    if (__any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0)
        atomicCAS(err.word, 0ull, ((unsigned long long)kErrNonFinite << 32) | err.call_id);
    if (__any_sync(0xffffffffu, big) && (threadIdx.x & 31) == 0)
        atomicCAS(err.word, 0ull, ((unsigned long long)kErrRange << 32) | err.call_id);
    if (NT == kUN && xm != nullptr) {
        // sub-block of 32 = 4 neighbouring lanes (q8 0..3 or 4..7 of a row)
        float t = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) t = __fadd_rn(t, v[i]);
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 1));
        t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, 2));
        if ((q8 & 3u) == 0) {
            uint32_t h, l;
            split_f16(__fmul_rn(t, 0.03125f), 0.0f, h, l);
            const uint32_t sb = c >> 2, s = 2u * (c & 3u) + (q8 >> 2), ks = (sb & 3u) * 16u + s;
            uint8_t *mt = xm + ((size_t)bt * nxm + (sb >> 2)) * kXmSlotBytes;
            auto at = [](uint32_t R, uint32_t k) {   // fp16 element k of row R, SW128
                const uint32_t byte = 2u * k;
                return R * 128u + ((((byte >> 4) ^ (R & 7u))) << 4) + (byte & 15u);
            };
            *reinterpret_cast<uint16_t *>(mt + at(r, ks)) = (uint16_t)h;
            *reinterpret_cast<uint16_t *>(mt + at(r, ks + 8u)) = (uint16_t)h;
            *reinterpret_cast<uint16_t *>(mt + at(64u + r, ks)) = (uint16_t)l;
            *reinterpret_cast<uint16_t *>(mt + at(64u + r, ks + 8u)) = 0;
        }
    }
    uint4 hi, lo;
    pack8(v, hi, lo);
    uint8_t *tile = out + ((size_t)bt * nchunks + c) * Tile<NT>::xslot;
    const uint32_t off = sw128_off(r, q8);
    *reinterpret_cast<uint4 *>(tile + off) = hi;
    *reinterpret_cast<uint4 *>(tile + Tile<NT>::xslot / 2 + off) = lo;
}


// TMA loads of super-block step `sb` (SC chunks) of 128 rows from row0.
template <uint32_t T>
__device__ __forceinline__ void load_raw(uint32_t dst, const CUtensorMap *maps, uint32_t cols, uint32_t sb,
                                         int row0, uint64_t *bar) {
    if constexpr (T == kTypeQ4_K) {
        tma_load_2d(dst, &maps[0], (int)(sb * 144u), row0, bar);
    } else if constexpr (T == kTypeQ6_K) {
        const uint32_t nsb = cols >> 8;
        tma_load_2d(dst, &maps[0], (int)(sb * 128u), row0, bar);                          // ql
        tma_load_2d(dst + 16384u, &maps[1], (int)(nsb * 128u + sb * 64u), row0, bar);    // qh
        tma_load_2d(dst + 24576u, &maps[2], (int)(nsb * 192u + sb * 16u), row0, bar);    // scales
        tma_load_2d(dst + 26624u, &maps[2], (int)((nsb * 208u + sb * 2u) & ~15u), row0, bar);   // d window
    } else if constexpr (T == kTypeQ8_0) {
        const uint32_t nb = cols >> 5;
        tma_load_2d(dst, &maps[0], (int)(sb * 256u), row0, bar);                          // codes, blocks 8sb..
        tma_load_2d(dst + 16384u, &maps[0], (int)(sb * 256u + 128u), row0, bar);
        tma_load_2d(dst + 32768u, &maps[1], (int)(nb * 32u + sb * 16u), row0, bar);       // d of 8 blocks
    } else {
        tma_load_2d(dst, &maps[0], (int)(sb * 256u), row0, bar);                          // 2 chunks of values
        tma_load_2d(dst + 16384u, &maps[0], (int)(sb * 256u + 128u), row0, bar);
    }
}

// Bytes one load_raw delivers (full boxes, out-of-range rows zero-filled).
template <uint32_t T>
__device__ __forceinline__ uint32_t raw_tx(uint32_t box_rows) {
    if constexpr (T == kTypeQ4_K) return 144u * box_rows;
    else if constexpr (T == kTypeQ6_K) return 224u * box_rows;
    else if constexpr (T == kTypeQ8_0) return 272u * box_rows;
    else return 256u * box_rows;
}

template <uint32_t T, uint32_t NT>
__global__ void __launch_bounds__(kThreads, 1)
proj_umma_kernel(const __grid_constant__ TmapSet tmaps, ProjSegments segs, const uint8_t *__restrict__ xtiles,
                 uint32_t nchunks_x, float *__restrict__ y, uint32_t ldy, uint32_t batch,
                 uint32_t kchunks_per_split, ErrorWord err) {
    using R = Ring<T, NT>;
    constexpr uint32_t SC = TypeCfg<T>::sc, kRawBytes = R::raw, kX = R::xdepth, kRawRing = R::rr;
    constexpr uint32_t kXSlot = Tile<NT>::xslot, kABufs = Tile<NT>::abufs, kABase = Tile<NT>::abase;
    constexpr uint32_t kIssuers = 1u;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t rfull[kMaxRawRing], rfree[kMaxRawRing], xfull[kMaxXRing], mdone[kMaxXRing];
    __shared__ uint64_t aready[kMaxABufs], adone[kMaxABufs], accum;
    __shared__ uint32_t tmem_base_slot, skip_slot;
    __shared__ volatile uint32_t abort_flag;
    static_assert(NT != 64 || kUM * kAccStride * 4 <= kX * kXSlot, "exchange tile does not fit");
    // No early return anywhere: every CTA of a split-K cluster must reach
    // both cluster barriers.

    uint8_t *raw_ring = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *x_ring = raw_ring + kRawRing * kRawBytes;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    // decoded weights x 2^scale_exp, result x 2^(2 - scale_exp): exact powers
    // of two built from their exponent bits (scale_exp is within [-64, 64])
    const float wscale = __uint_as_float((uint32_t)(127 + m.scale_exp) << 23);
    const float oscale = __uint_as_float((uint32_t)(127 + 2 - m.scale_exp) << 23);
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kUM;
    const uint32_t b0 = blockIdx.y * NT;
    const uint32_t nchunks_total = (m.cols + kUK - 1) / kUK;
    // kchunks_per_split is a multiple of SC, so c_begin starts a super-block step
    const uint32_t c_begin = blockIdx.z * kchunks_per_split;
    const uint32_t c_end = min(nchunks_total, c_begin + kchunks_per_split);
    const uint32_t nchunks_planned = c_end > c_begin ? c_end - c_begin : 0;

    if (tid == 0) {
        for (uint32_t s = 0; s < kRawRing; ++s) mbar_init(&rfull[s], 1);
        for (uint32_t s = 0; s < kX; ++s) {
            mbar_init(&xfull[s], 1);
            mbar_init(&mdone[s], kIssuers);
        }
        for (uint32_t s = 0; s < kRawRing; ++s) mbar_init(&rfree[s], kIssuers);
        for (uint32_t b = 0; b < kABufs; ++b) {
            mbar_init(&aready[b], kDecodeWarps);
            mbar_init(&adone[b], kIssuers);
        }
        mbar_init(&accum, kIssuers);
        abort_flag = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kAllocWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_slot;

    // The weights of the first raw slots are requested before the wait: they
    // are uploaded by the host and never written by a kernel.
    uint32_t prefetched = 0;   // raw steps already issued (producer thread)
    const CUtensorMap *maps = tmaps.map[seg];
    const uint32_t rtx = raw_tx<T>(tmaps.box_rows[seg]);
    const uint32_t sb0 = c_begin / SC;
    if (warp == kTmaWarp && lane == 0 && nchunks_planned > 0) {
        prefetched = min((nchunks_planned + SC - 1) / SC, kRawRing);
        for (uint32_t j = 0; j < prefetched; ++j) {
            mbar_expect_tx(&rfull[j], rtx);
            load_raw<T>(smem_u32(raw_ring + j * kRawBytes), maps, m.cols, sb0 + j, (int)row0, &rfull[j]);
        }
    }
    pdl_wait();
    // one read of the error word for the whole CTA, so that every role
    // agrees on the chunk count
    if (tid == 0) skip_slot = *reinterpret_cast<volatile unsigned long long *>(err.word) != 0ull ? 1u : 0u;
    __syncthreads();
    const bool skip = skip_slot != 0u;
    const uint32_t nchunks = skip ? 0u : nchunks_planned;

    if (warp == kTmaWarp) {
        // ---- producer: one thread issues every copy
        if (lane == 0 && skip) {
            // an earlier kernel failed: only let the weight loads already in
            // flight land before the CTA exits
            for (uint32_t j = 0; j < prefetched; ++j)
                if (!mbar_wait(&rfull[j], 0u, &abort_flag, kSiteRawFull)) break;
        }
        if (lane == 0 && nchunks > 0) {
            for (uint32_t it = 0; it < nchunks; ++it) {
                if (it % SC == 0) {
                    // raw slot of step j was last used by step j - kRawRing;
                    // steps below `prefetched` were issued before the wait
                    const uint32_t j = it / SC, rs = j % kRawRing;
                    if (j >= prefetched) {
                        if (j >= kRawRing &&
                            !mbar_wait(&rfree[rs], ((j - kRawRing) / kRawRing) & 1u, &abort_flag, kSiteRawFree))
                            break;
                        mbar_expect_tx(&rfull[rs], rtx);
                        load_raw<T>(smem_u32(raw_ring + rs * kRawBytes), maps, m.cols, sb0 + j, (int)row0,
                                    &rfull[rs]);
                    }
                }
                const uint32_t xs = it % kX;
                if (it >= kX && !mbar_wait(&mdone[xs], ((it - kX) / kX) & 1u, &abort_flag, kSiteXFree)) break;
                mbar_expect_tx(&xfull[xs], kXSlot);
                bulk_load(smem_u32(x_ring + xs * kXSlot),
                          xtiles + ((size_t)blockIdx.y * nchunks_x + c_begin + it) * kXSlot, kXSlot, &xfull[xs]);
            }
        }
    } else if (warp == kMmaWarp) {
        // ---- MMA issue: one thread
        if (lane == 0) {
            // x slot i's descriptor = slot 0's + i * kXSlot / 16 in the
            // address field (shared addresses stay below 256 KB: no carry)
            const uint64_t desc0 = sw128_desc(smem_u32(x_ring));
            for (uint32_t it = 0; it < nchunks; ++it) {
                const uint32_t xs = it % kX, b = it % kABufs;
                if (!mbar_wait(&aready[b], (it / kABufs) & 1u, &abort_flag, kSiteAReady)) break;
                if (!mbar_wait(&xfull[xs], (it / kX) & 1u, &abort_flag, kSiteXFull)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                // B: the slot's swizzled rows are [xh (NT rows) | xl (NT rows)]
                const uint64_t db = desc0 + (uint64_t)(xs * (kXSlot >> 4));
                const uint32_t ah = tmem + kABase + b * 64u, al = ah + 32u;
                const uint32_t first = it == 0 ? 0u : 1u;
#pragma unroll
                for (uint32_t kk = 0; kk < kUK / 16; ++kk) {   // +32 bytes of K per step = +2 in the address field
                    if constexpr (NT == 64) {
                        umma_ts<2 * NT>(tmem, ah + kk * 8u, db + 2u * kk, kk == 0 ? first : 1u);
                        umma_ts<NT>(tmem, al + kk * 8u, db + 2u * kk, 1u);
                    } else {
                        const uint64_t dlo = db + (uint64_t)((kXSlot / 2) >> 4);
                        umma_ts<NT>(tmem, ah + kk * 8u, db + 2u * kk, kk == 0 ? first : 1u);
                        umma_ts<NT>(tmem, ah + kk * 8u, dlo + 2u * kk, 1u);
                        umma_ts<NT>(tmem, al + kk * 8u, db + 2u * kk, 1u);
                    }
                }
                umma_commit(&mdone[xs]);
                umma_commit(&adone[b]);
                if (it % SC == SC - 1) umma_commit(&rfree[(it / SC) % kRawRing]);
            }
            umma_commit(&accum);   // completes once every MMA this thread issued has
        }
    } else if (warp < kDecodeWarps) {
        // ---- decode warps: lane = weight row within the warp's TMEM quarter
        const uint32_t quarter = warp & 3, q = warp >> 2;
        const uint32_t row = quarter * 32u + lane;
        const uint32_t lane_addr = (quarter * 32u) << 16;
        for (uint32_t it = 0; it < nchunks; ++it) {
            const uint32_t j = it / SC, rs = j % kRawRing, b = it % kABufs;
            if (!mbar_wait_warp(&rfull[rs], (j / kRawRing) & 1u, &abort_flag, kSiteRawFull)) break;
            // A buffer b was last read by the MMAs of chunk it - kABufs
            if (it >= kABufs && !mbar_wait_warp(&adone[b], ((it - kABufs) / kABufs) & 1u, &abort_flag, kSiteADone))
                break;
            uint32_t hi[8], lo[8];
            decode16<T>(raw_ring + rs * kRawBytes, row, m.cols, c_begin + it, q, wscale, hi, lo);
            const uint32_t ta = tmem + lane_addr + kABase + b * 64u + q * 8u;
            tmem_st8(ta, hi);
            tmem_st8(ta + 32u, lo);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            __syncwarp();
            if (lane == 0) mbar_arrive(&aready[b]);
        }
    }

    // ---- epilogue
    bool ok = false;
    if (warp < kDecodeWarps) {
        ok = mbar_wait_warp(&accum, 0, &abort_flag, kSiteAccum);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    }
    const bool all_ok = __syncthreads_and(warp >= kDecodeWarps || ok) && abort_flag == 0u;
    if (!all_ok && tid == 0)
        atomicCAS(err.word, 0ull, ((unsigned long long)(kErrTimeout | (abort_flag << 8)) << 32) | err.call_id);

    // accumulator: decode warp w reads TMEM lanes 32*(w&3).., its quarter of the columns
    const uint32_t lane_base = 32u * (warp & 3);
    const uint32_t trow = lane_base + lane;
    const bool write = all_ok && !skip;
    bool out_bad = false;   // the projection's output check
    if constexpr (NT != 64) {
        // one accumulator holds all three products; no split-K
        const uint32_t col_base = (uint32_t)(warp >> 2) * (NT / 4u);
        const uint32_t row = row0 + trow;
        // warp-uniform condition: tcgen05.ld is a .sync.aligned warp
        // instruction; rows past the matrix only skip their stores
        if (warp < kDecodeWarps && write && nchunks > 0) {
#pragma unroll 1
            for (uint32_t g = 0; g < NT / 4u; g += 16u) {
                uint32_t r0[16];
                tmem_ld16(tmem + (lane_base << 16) + col_base + g, r0);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const uint32_t b = b0 + col_base + g + j;
                    const float v = __fmul_rn(__uint_as_float(r0[j]), oscale);
                    if (b < batch && row < m.rows) {
                        out_bad |= !isfinite(v);
                        y[(size_t)b * ldy + segs.out_offset[seg] + row] = v;
                    }
                }
            }
        }
    } else {
    const uint32_t col_base = (uint32_t)(warp >> 2) * 16u;
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.0f;   // empty split: contributes zero
    if (warp < kDecodeWarps && all_ok && nchunks > 0) {
        // y = (wh*xh + wl*xh) + wh*xl
        uint32_t r0[16], r1[16];
        const uint32_t taddr = tmem + (lane_base << 16) + col_base;
        tmem_ld16(taddr, r0);
        tmem_ld16(taddr + kUN, r1);
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < 16; ++j)
            acc[j] = __fmul_rn(__fadd_rn(__uint_as_float(r0[j]), __uint_as_float(r1[j])), oscale);
    }
    const uint32_t nsplit = gridDim.z;
    if (nsplit == 1) {
        const uint32_t row = row0 + trow;
        if (warp < kDecodeWarps && write && row < m.rows) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const uint32_t b = b0 + col_base + j;
                if (b < batch) {
                    out_bad |= !isfinite(acc[j]);
                    y[(size_t)b * ldy + segs.out_offset[seg] + row] = acc[j];
                }
            }
        }
    } else {
        // exchange tile in the drained activation ring: [128 rows][kAccStride]
        float *xt = reinterpret_cast<float *>(x_ring);
        if (warp < kDecodeWarps) {
#pragma unroll
            for (int j = 0; j < 16; ++j) xt[trow * kAccStride + col_base + j] = acc[j];
        }
        cluster_sync();
        const uint32_t rank = cluster_rank();
        const uint32_t rows_per = kUM / nsplit;
        const uint32_t base = smem_u32(xt);
        for (uint32_t i = tid; i < rows_per * kUN; i += kThreads) {
            const uint32_t rr = i % rows_per, bb = i / rows_per;
            const uint32_t lr = rank * rows_per + rr;
            const uint32_t off = base + (lr * kAccStride + bb) * 4u;
            float v[8];
#pragma unroll
            for (uint32_t z = 0; z < 8; ++z) v[z] = z < nsplit ? ld_dsmem(off, z) : 0.0f;
            float sum = v[0];
#pragma unroll
            for (uint32_t z = 1; z < 8; ++z)
                if (z < nsplit) sum = __fadd_rn(sum, v[z]);
            const uint32_t row = row0 + lr, b = b0 + bb;
            if (write && row < m.rows && b < batch) {
                out_bad |= !isfinite(sum);
                y[(size_t)b * ldy + segs.out_offset[seg] + row] = sum;
            }
        }
        cluster_sync();   // peers finish reading this CTA's tile before it exits
    }
    }
    if (out_bad) atomicCAS(err.word, 0ull, ((unsigned long long)kErrNonFinite << 32) | err.call_id);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == kAllocWarp) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ---- factored-scale projection (Q4_K, Q6_K; batch tiles of 64)
//
// The kernel above turns every weight into F32 and splits it into two fp16
// terms: about 15 instructions per weight on the CUDA cores.  A K-quant
// weight is a small integer times per-block scales, so the scales can leave
// the MMA operand:
//   Q4_K  w = d*sc_s*q - dmin*m_s   (s: sub-block of 32; sc, m 6-bit; q 4-bit)
//         sum_k w x = sum_sb d_sb * sum_{k in sb} (sc*q) x
//                     - sum_{sb,s} (dmin*m_s) * X_s,  X_s = sum of the
//         sub-block's 32 activations.  sc*q <= 945 is an exact fp16
//         integer: one A term.
//   Q6_K  w = d*sc_s*(q - 32)       (s: sub-block of 16; sc int8; q 6-bit)
//         sc*(q - 32) lies in [-4096, 4096] and needs up to 12 bits:
//         A = RN16(sc*(q - 32)) plus its residual e in {-1, 0, 1} (exact
//         fp16 FMA): two A terms.
// The activations keep the fp16 hi/lo split of x / 4.  The MMAs of one
// super-block (256 K) accumulate A*[xh | xl] (Q6_K also e*xh) into one of
// two TMEM accumulators; epilogue warps add the halves, scale by the
// super-block's d and accumulate in F32 registers while the MMAs of the next
// super-block run into the other accumulator.  Q4_K's minimum term is a
// second, K/32-sized product accumulated over the CTA's whole K range:
// A' = dmin*m*2^scale_exp (17 significant bits, exact as fp16 hi | lo over
// the 8 sub-blocks = one K step of 16) times X/32 as [Xh | Xh] and [Xl | 0]
// (two N = 64 MMAs; tiles written by the activation kernel).  A' and the
// F32 d of every super-block are built once at upload (q4k_build_aux) and
// arrive by TMA, 4 super-blocks per tile, with the minimum-term activations.
//
// Decode: Q4_K one PRMT per two weights (a nibble pair as fp16 1024 + q) and
// one fp16 FMA ((1024 + q)*sc - 1024*sc = sc*q, exact); Q6_K one PRMT, one
// subtraction (q - 32), one multiply (RN) and one FMA (residual) per pair.
//
// Pipelining.  mbarrier operations by many warps on one barrier serialise
// (measured: hundreds of cycles per hand-off with 16 arriving warps), so
// each role group meets on a hardware named barrier and one leader thread
// does the group's single mbarrier wait and arrive.  The ring works in units
// of U chunks of 64 K; each unit has ONE readiness barrier (the decode
// leader + the TMA's activation bytes) and ONE consumed barrier (the MMA
// commit that frees both its A buffer and its activation slot), so the
// activation ring has as many slots as there are A buffers.
//
// Warp roles (864 threads, one CTA per SM):
//   0       TMEM owner; weight producer (raw super-blocks and the Q4_K group
//           tiles), which runs up to three super-blocks ahead
//   1       MMA issue
//   2       activation producer (one unit per slot, gated by the MMAs), kept
//           apart from the weight loads so that their HBM latency stays hidden
//   3..18   decode, Fact::groups groups taking units in turn, so that a
//           group's hand-off latency overlaps the others' decoding; lane =
//           weight row in TMEM quarter (warp & 3), 16 * groups K values of
//           each chunk
//   19..26  epilogue: lane = weight row, 32 of the 64 batch columns
// TMEM columns: accumulators 2 x 128 at 0.  Q4_K: minimum term 64 at 256,
// three A buffers of 2 x 32 at 320.  Q6_K: A buffers of U x (32 RN + 32
// residual) at 256.
constexpr int kFTmaWarp = 0;      // weight producer; also owns TMEM
constexpr int kFAllocWarp = 0;
constexpr int kFMmaWarp = 1;
constexpr int kFXWarp = 2;        // activation producer
constexpr int kFDecode0 = 3;      // first decode warp
constexpr int kFDecodeWarps = 16;
constexpr int kFEpi0 = kFDecode0 + kFDecodeWarps;
constexpr int kFEpiWarps = 8;
constexpr int kFThreads = (kFEpi0 + kFEpiWarps) * 32;
constexpr uint32_t kXmSlot = kXmSlotBytes;   // 4 super-blocks x 16 K, 128 rows
constexpr uint32_t kMlSlot = 16384;          // Q4_K A': 128 rows x 4 super-blocks x 16 K
constexpr uint32_t kDgSlot = 2048;           // Q4_K d: 128 rows x 4 super-blocks, F32

template <uint32_t T> struct Fact {
    static constexpr bool q4 = T == kTypeQ4_K;
    static constexpr uint32_t U = 2u;                           // chunks per unit
    static constexpr uint32_t kU = q4 ? 3u : 2u;                // units in flight
    // Decode groups.  A group's consecutive units are `groups` apart and the
    // group waits on the consumed barrier of unit u + groups - kU; that
    // barrier's previous phase (unit u + groups - 2 kU) must already be
    // complete, or the parity test would accept a phase from two completions
    // ago.  The group waited for unit u - kU before unit u, so groups <= kU.
    // (Four groups measured no faster than two.)
    static constexpr uint32_t groups = 2u;
    static constexpr uint32_t dm = 256u;                        // Q4_K minimum term (64 columns)
    static constexpr uint32_t abase = q4 ? 320u : 256u;
    static constexpr uint32_t ecols = q4 ? 0u : U * 32u;        // residual offset in a buffer
    static constexpr uint32_t astride = q4 ? U * 32u : U * 64u;
    static constexpr uint32_t raw = TypeCfg<T>::raw;
    static constexpr uint32_t rr = 3u;
    static constexpr uint32_t xm = q4 ? 2u : 0u;                // minimum-term activation tiles
    static constexpr uint32_t ml = q4 ? 2u : 0u;                // A' tiles
    static constexpr uint32_t dg = q4 ? 2u : 0u;                // d tiles
    static constexpr uint32_t xslot = U * Tile<kUN>::xslot;     // one unit of activations
    static constexpr uint32_t smem =
        rr * raw + xm * kXmSlot + ml * kMlSlot + dg * kDgSlot + kU * xslot + 1024u;
    static_assert(abase + kU * astride <= kTmemCols, "TMEM budget");
    static_assert(smem <= 227u * 1024u - 4096u, "shared memory per CTA");
    static_assert(kUM * kUN * 4u <= kU * xslot, "exchange tile");
    static_assert(4u % U == 0u, "units tile a super-block");
    static_assert(groups <= kU && kFDecodeWarps % (4 * groups) == 0, "decode groups");
};

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// Scale and minimum (6-bit each) of Q4_K sub-block j (0..7) from the
// super-block header (d, dmin, 12 packed bytes).
__device__ __forceinline__ void q4k_scale_min(const uint4 &hdr, uint32_t j, uint32_t &sc, uint32_t &mn) {
    auto sbyte = [&](uint32_t k) { return (word_of(hdr, 1u + (k >> 2)) >> (8u * (k & 3u))) & 0xFFu; };
    if (j < 4) {
        sc = sbyte(j) & 63u;
        mn = sbyte(j + 4) & 63u;
    } else {
        sc = (sbyte(j + 4) & 15u) | ((sbyte(j - 4) >> 6) << 4);
        mn = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
    }
}

// Q6_K: the integer A operand of the 16 values [16q, 16q + 16) of chunk c of
// one staged row (same staging as decode16) as fp16 pairs: RN16(sc*(q - 32))
// in a and the exact residual in e.
__device__ __forceinline__ void fact_decode_q6k16(const uint8_t *raw, uint32_t row, uint32_t c, uint32_t q,
                                                  uint32_t (&a)[8], uint32_t (&e)[8]) {
    const uint32_t half = (c & 3u) >> 1;
    const uint32_t h = q >> 1, s = 2u * (c & 1u) + h, part = q & 1u;
    const uint4 ql = lds16(raw + sw128_at(row, 4u * half + 2u * h + part));
    const uint4 qh = lds16(raw + 16384u + sw64_at(row, 2u * half + part));
    const uint32_t scb = raw[24576u + row * 16u + half * 8u + 2u * s + part];
    const __half2 s2 = __half2half2(__int2half_rn((int)(int8_t)scb));      // exact
    const __half2 off = __half2half2(__ushort_as_half((unsigned short)0x6420u));   // 1056
    const uint32_t wl[4] = {ql.x, ql.y, ql.z, ql.w}, wh[4] = {qh.x, qh.y, qh.z, qh.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t nib = (c & 1u) ? (wl[k] >> 4) & 0x0F0F0F0Fu : wl[k] & 0x0F0F0F0Fu;
        const uint32_t bw = nib | (((wh[k] >> (2u * s)) & 0x03030303u) << 4);
        // bytes {q, 0x64, q', 0x64}: the fp16 pair (1024 + q, 1024 + q'); minus 1056 = q - 32, exact
        const __half2 t0 = __hsub2(bits_h2(__byte_perm(bw, 0x64u, 0x4140u)), off);
        const __half2 t1 = __hsub2(bits_h2(__byte_perm(bw, 0x64u, 0x4342u)), off);
        const __half2 r0 = __hmul2(t0, s2), r1 = __hmul2(t1, s2);
        a[2 * k] = h2_bits(r0);
        a[2 * k + 1] = h2_bits(r1);
        e[2 * k] = h2_bits(__hfma2(t0, s2, __hneg2(r0)));       // sc*(q-32) - RN(...), exact
        e[2 * k + 1] = h2_bits(__hfma2(t1, s2, __hneg2(r1)));
    }
}

// Q4_K: the 32 values [32p, 32p + 32) of chunk c of one staged row (one
// sub-block: the low (p = 0) or high (p = 1) nibbles of the chunk's 32 quant
// bytes) as 16 fp16 pairs sc*q, with one header read and scale unpack.
__device__ __forceinline__ void fact_decode_q4k32(const uint8_t *raw, uint32_t row, uint32_t c, uint32_t p,
                                                  uint32_t (&a)[16]) {
    const uint8_t *blk = raw + row * 144u;
    const uint4 hdr = lds16(blk);
    const uint4 q0 = lds16(blk + 16u + (c & 3u) * 32u), q1 = lds16(blk + 32u + (c & 3u) * 32u);
    uint32_t sc, mn;
    q4k_scale_min(hdr, 2u * (c & 3u) + p, sc, mn);
    const __half2 s2 = __half2half2(__uint2half_rn(sc));                 // exact
    const __half2 n2 = __hneg2(__half2half2(__uint2half_rn(sc << 10)));  // -1024 sc, exact
    const uint32_t wq[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        const uint32_t nib = p ? (wq[k] >> 4) & 0x0F0F0F0Fu : wq[k] & 0x0F0F0F0Fu;
        // bytes {q, 0x64, q', 0x64}: the fp16 pair (1024 + q, 1024 + q'), then
        // (1024 + q)*sc - 1024*sc = sc*q exactly
        a[2 * k] = h2_bits(__hfma2(bits_h2(__byte_perm(nib, 0x64u, 0x4140u)), s2, n2));
        a[2 * k + 1] = h2_bits(__hfma2(bits_h2(__byte_perm(nib, 0x64u, 0x4342u)), s2, n2));
    }
}

// Q6_K: the super-block scale d of chunk c's super-block.
__device__ __forceinline__ float q6k_scale(const uint8_t *raw, uint32_t row, uint32_t cols, uint32_t c) {
    const uint32_t nsb = cols >> 8, sb = c >> 2;
    return h2f(*reinterpret_cast<const uint16_t *>(raw + 26624u + row * 16u + ((nsb * 208u + sb * 2u) & 15u)));
}

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
    return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// Hardware named barriers among a subset of the CTA's warps.
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
__device__ __forceinline__ void named_arrive(uint32_t id, uint32_t threads) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(threads) : "memory");
}
enum NamedBarrier : uint32_t { kBarEpiIn = 1, kBarEpiOut, kBarDecIn, kBarDecOut };   // decode: 2 per group
constexpr uint32_t kFMaxGroups = 4;   // decode groups (kBarDecIn + 2 * groups - 1 <= 15)

// D (TMEM) += A (shared-memory descriptor) * B (shared-memory descriptor).
template <uint32_t N>
__device__ __forceinline__ void umma_ss(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "n"(idesc_for(N)), "r"(accumulate));
}

// 16-byte load from the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ float4 ld_dsmem4(uint32_t local_addr, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(remote));
    return v;
}

// Split-K exchange tile: 128 rows x 64 floats, 16-byte chunk c of row r at
// chunk c ^ (r & 15) (conflict-free for a warp of consecutive rows).
__device__ __forceinline__ uint32_t xchg_off(uint32_t r, uint32_t c) { return r * 256u + ((c ^ (r & 15u)) << 4); }

template <uint32_t T>
__global__ void __launch_bounds__(kFThreads, 1)
proj_fact_kernel(const __grid_constant__ TmapSet tmaps, ProjSegments segs, const uint8_t *__restrict__ xtiles,
                 uint32_t nchunks_x, const uint8_t *__restrict__ xmtiles, uint32_t nxm, float *__restrict__ y,
                 uint32_t ldy, uint32_t batch, uint32_t kchunks_per_split, ErrorWord err) {
    using F = Fact<T>;
    constexpr bool kQ4 = F::q4;
    constexpr uint32_t U = F::U, kU = F::kU, kRR = F::rr, kRaw = F::raw, kXSlot = F::xslot;
    constexpr uint32_t kPerSb = 4u / U;   // units per super-block
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t rfull[kRR], rfree[kRR], ready[kU], ucons[kU];
    __shared__ uint64_t dfull[2], dfree[2], xmfull[2], xmfree[2], dready[4], accum;
    __shared__ float dscale[4][kUM];
    __shared__ uint32_t tmem_base_slot, skip_slot;
    __shared__ volatile uint32_t abort_flag, dec_stop[kFMaxGroups], epi_stop;
    // No early return anywhere: every CTA of a split-K cluster must reach
    // the cluster barriers.

    uint8_t *raw_ring = align1024(smem_raw);
    uint8_t *xm_ring = raw_ring + kRR * kRaw;
    uint8_t *ml_ring = xm_ring + F::xm * kXmSlot;
    uint8_t *dg_ring = ml_ring + F::ml * kMlSlot;
    uint8_t *x_ring = dg_ring + F::dg * kDgSlot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kUM;
    const uint32_t b0 = blockIdx.y * kUN;
    const uint32_t nchunks_total = m.cols / kUK;
    // kchunks_per_split is a multiple of 4: every CTA starts a super-block
    const uint32_t c_begin = blockIdx.z * kchunks_per_split;
    const uint32_t c_end = min(nchunks_total, c_begin + kchunks_per_split);
    const uint32_t nchunks_planned = c_end > c_begin ? c_end - c_begin : 0;
    const uint32_t sb0 = c_begin >> 2;

    if (tid == 0) {
        for (uint32_t s = 0; s < kRR; ++s) {
            mbar_init(&rfull[s], 1);
            mbar_init(&rfree[s], 1);
        }
        for (uint32_t u = 0; u < kU; ++u) {
            mbar_init(&ready[u], 2);   // decode leader + the TMA's activation bytes
            mbar_init(&ucons[u], 1);
        }
        for (uint32_t i = 0; i < 2; ++i) {
            mbar_init(&dfull[i], 1);
            mbar_init(&dfree[i], 1);    // epilogue leader
            mbar_init(&xmfull[i], 1);
            mbar_init(&xmfree[i], 2);   // MMA commit + epilogue leader (d tile)
        }
        for (uint32_t i = 0; i < 4; ++i) mbar_init(&dready[i], 1);
        mbar_init(&accum, 1);
        abort_flag = 0u;
        for (uint32_t i = 0; i < kFMaxGroups; ++i) dec_stop[i] = 0u;
        epi_stop = 0u;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kFAllocWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_slot;

    // weights of the first raw slots before the wait (never written by a kernel)
    uint32_t prefetched = 0;
    const CUtensorMap *maps = tmaps.map[seg];
    const uint32_t rtx = raw_tx<T>(tmaps.box_rows[seg]);
    if (warp == kFTmaWarp && lane == 0 && nchunks_planned > 0) {
        prefetched = min(nchunks_planned / 4u, kRR);
        for (uint32_t j = 0; j < prefetched; ++j) {
            mbar_expect_tx(&rfull[j], rtx);
            load_raw<T>(smem_u32(raw_ring + j * kRaw), maps, m.cols, sb0 + j, (int)row0, &rfull[j]);
        }
    }
    pdl_wait();
    if (tid == 0) skip_slot = *reinterpret_cast<volatile unsigned long long *>(err.word) != 0ull ? 1u : 0u;
    __syncthreads();
    const bool skip = skip_slot != 0u;
    const uint32_t nchunks = skip ? 0u : nchunks_planned;
    const uint32_t nsb = nchunks >> 2, nunits = nchunks / U;

    float acc[32];   // epilogue warps only (initialised there)
    bool epi_ok = true;
    const bool epi = warp >= kFEpi0;

    if (warp == kFTmaWarp) {
        // ---- weight producer: raw super-blocks (three ahead) and group tiles
        if (lane == 0 && skip) {
            for (uint32_t j = 0; j < prefetched; ++j)
                if (!mbar_wait(&rfull[j], 0u, &abort_flag, kSiteRawFull)) break;
        }
        if (lane == 0 && nsb > 0) {
            for (uint32_t j = 0; j < nsb; ++j) {
                if constexpr (kQ4) {
                    const uint32_t sb = sb0 + j, lt = (sb >> 2) - (sb0 >> 2);
                    if (j == 0 || (sb & 3u) == 0) {
                        const uint32_t slot = lt & 1u;
                        if (lt >= 2 && !mbar_wait(&xmfree[slot], ((lt - 2) >> 1) & 1u, &abort_flag, kSiteXmFree))
                            break;
                        const uint32_t brows = tmaps.box_rows[seg];
                        mbar_expect_tx(&xmfull[slot], kXmSlot + 128u * brows + 16u * brows);
                        bulk_load(smem_u32(xm_ring + slot * kXmSlot),
                                  xmtiles + ((size_t)blockIdx.y * nxm + (sb >> 2)) * kXmSlot, kXmSlot, &xmfull[slot]);
                        tma_load_2d(smem_u32(ml_ring + slot * kMlSlot), &maps[1], (int)((sb >> 2) * 128u), (int)row0,
                                    &xmfull[slot]);
                        tma_load_2d(smem_u32(dg_ring + slot * kDgSlot), &maps[2], (int)((sb >> 2) * 16u), (int)row0,
                                    &xmfull[slot]);
                    }
                }
                if (j >= prefetched) {
                    const uint32_t rs = j % kRR;
                    if (j >= kRR && !mbar_wait(&rfree[rs], ((j - kRR) / kRR) & 1u, &abort_flag, kSiteRawFree)) break;
                    mbar_expect_tx(&rfull[rs], rtx);
                    load_raw<T>(smem_u32(raw_ring + rs * kRaw), maps, m.cols, sb0 + j, (int)row0, &rfull[rs]);
                }
            }
        }
    } else if (warp == kFXWarp) {
        // ---- activation producer: the unit's slot was last read by the MMAs of unit u - kU
        if (lane == 0) {
            for (uint32_t u = 0; u < nunits; ++u) {
                const uint32_t us = u % kU;
                if (u >= kU && !mbar_wait(&ucons[us], ((u - kU) / kU) & 1u, &abort_flag, kSiteXFree)) break;
                mbar_expect_tx(&ready[us], kXSlot);
                bulk_load(smem_u32(x_ring + us * kXSlot),
                          xtiles + ((size_t)blockIdx.y * nchunks_x + c_begin + u * U) * Tile<kUN>::xslot, kXSlot,
                          &ready[us]);
            }
        }
    } else if (warp == kFMmaWarp) {
        // ---- MMA issue: one thread
        if (lane == 0) {
            const uint64_t desc0 = sw128_desc(smem_u32(x_ring));
            const uint64_t descm = sw128_desc(smem_u32(xm_ring));
            const uint64_t descl = sw128_desc(smem_u32(ml_ring));
            for (uint32_t u = 0; u < nunits; ++u) {
                const uint32_t j = u / kPerSb, us = u % kU, dbuf = j & 1u;
                const bool first = u % kPerSb == 0, last = u % kPerSb == kPerSb - 1;
                const uint32_t sb = sb0 + j, lt = (sb >> 2) - (sb0 >> 2);
                // accumulator dbuf was last read by the epilogue of super-block j - 2
                if (first && j >= 2 && !mbar_wait(&dfree[dbuf], ((j - 2) >> 1) & 1u, &abort_flag, kSiteDFree))
                    break;
                if constexpr (kQ4) {
                    if (first && (j == 0 || (sb & 3u) == 0) &&
                        !mbar_wait(&xmfull[lt & 1u], (lt >> 1) & 1u, &abort_flag, kSiteXmFull))
                        break;
                }
                if (!mbar_wait(&ready[us], (u / kU) & 1u, &abort_flag, kSiteAReady)) break;
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t dacc = tmem + dbuf * 128u;
#pragma unroll
                for (uint32_t c2 = 0; c2 < U; ++c2) {
                    const uint64_t db = desc0 + (uint64_t)((us * kXSlot + c2 * Tile<kUN>::xslot) >> 4);
                    const uint32_t a = tmem + F::abase + us * F::astride + c2 * 32u;
#pragma unroll
                    for (uint32_t kk = 0; kk < kUK / 16; ++kk) {
                        umma_ts<2 * kUN>(dacc, a + kk * 8u, db + 2u * kk, (first && c2 == 0 && kk == 0) ? 0u : 1u);
                        if constexpr (!kQ4) umma_ts<kUN>(dacc, a + F::ecols + kk * 8u, db + 2u * kk, 1u);
                    }
                }
                if constexpr (kQ4) {
                    if (first) {
                        // minimum term: A' rows x [Xh | Xh], then x [Xl | 0]
                        const uint64_t da = descl + (uint64_t)((lt & 1u) * (kMlSlot >> 4)) + 2u * (sb & 3u);
                        const uint64_t dx = descm + (uint64_t)((lt & 1u) * (kXmSlot >> 4)) + 2u * (sb & 3u);
                        umma_ss<kUN>(tmem + F::dm, da, dx, j == 0 ? 0u : 1u);
                        umma_ss<kUN>(tmem + F::dm, da, dx + (uint64_t)((64u * 128u) >> 4), 1u);
                    }
                }
                umma_commit(&ucons[us]);
                if (last) {
                    umma_commit(&rfree[j % kRR]);
                    umma_commit(&dfull[dbuf]);
                    if constexpr (kQ4) {
                        if ((sb & 3u) == 3u || j + 1 == nsb) umma_commit(&xmfree[lt & 1u]);
                    }
                }
            }
            umma_commit(&accum);   // completes once every MMA this thread issued has
        }
    } else if (warp < kFEpi0) {
        // ---- decode warps: group g takes units g, g + groups, ...; lane =
        // weight row within the warp's TMEM quarter
        constexpr uint32_t kFGroups = F::groups;
        constexpr uint32_t kGroupWarps = kFDecodeWarps / kFGroups, kGroupThreads = kGroupWarps * 32;
        constexpr uint32_t kParts = 16u / kGroupWarps;   // 16-value parts of a chunk per thread
        const uint32_t g = (uint32_t)(warp - kFDecode0) / kGroupWarps;
        const uint32_t quarter = warp & 3, part0 = ((uint32_t)(warp - kFDecode0) % kGroupWarps >> 2) * kParts;
        const uint32_t row = quarter * 32u + lane;
        const uint32_t lane_addr = (quarter * 32u) << 16;
        const bool leader = (uint32_t)(warp - kFDecode0) % kGroupWarps == 0;
        const uint32_t bar_in = kBarDecIn + 2u * g, bar_out = kBarDecOut + 2u * g;
        for (uint32_t u = g; u < nunits; u += kFGroups) {
            const uint32_t j = u / kPerSb, rs = j % kRR, us = u % kU;
            const bool first = u % kPerSb == 0;
            if (leader) {
                // the super-block's raw slot landed; the A buffer was last
                // read by the MMAs of unit u - kU
                bool ok = mbar_wait_warp(&rfull[rs], (j / kRR) & 1u, &abort_flag, kSiteRawFull);
                ok = ok && (u < kU || mbar_wait_warp(&ucons[us], ((u - kU) / kU) & 1u, &abort_flag, kSiteADone));
                if (!ok && lane == 0) dec_stop[g] = 1u;
            }
            named_sync(bar_in, kGroupThreads);
            if (dec_stop[g]) break;
            const uint8_t *rawp = raw_ring + rs * kRaw;
#pragma unroll
            for (uint32_t c2 = 0; c2 < U; ++c2) {
                const uint32_t ta0 = tmem + lane_addr + F::abase + us * F::astride + c2 * 32u;
                if constexpr (kQ4) {
#pragma unroll
                    for (uint32_t h = 0; h < kParts; h += 2) {
                        uint32_t a[16];
                        fact_decode_q4k32(rawp, row, c_begin + u * U + c2, (part0 + h) >> 1, a);
                        tmem_st16(ta0 + (part0 + h) * 8u, a);
                    }
                } else {
#pragma unroll
                    for (uint32_t h = 0; h < kParts; ++h) {
                        uint32_t a[8], e[8];
                        fact_decode_q6k16(rawp, row, c_begin + u * U + c2, part0 + h, a, e);
                        tmem_st8(ta0 + (part0 + h) * 8u, a);
                        tmem_st8(ta0 + (part0 + h) * 8u + F::ecols, e);
                    }
                }
            }
            // Q6_K: the super-block's d for the epilogue (Q4_K's comes by TMA)
            const bool head = !kQ4 && first;
            if (head && part0 == 0) dscale[j & 3u][row] = q6k_scale(rawp, row, m.cols, c_begin + u * U);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            if (leader) {
                named_sync(bar_out, kGroupThreads);   // every warp of the group stored unit u
                if (lane == 0) {
                    mbar_arrive(&ready[us]);
                    if (head) mbar_arrive(&dready[j & 3u]);
                }
            } else {
                named_arrive(bar_out, kGroupThreads);
            }
        }
    } else if (epi) {
        // ---- epilogue warps: per super-block acc += d * (A*xh + A*xl)
        const uint32_t eq = warp & 3, eh = (uint32_t)(warp - kFEpi0) >> 2;
        const uint32_t row = eq * 32u + lane;
        const uint32_t lane_addr = (eq * 32u) << 16;
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.0f;
        constexpr uint32_t kEpiThreads = kFEpiWarps * 32;
        const bool eleader = warp == kFEpi0;
        for (uint32_t j = 0; j < nsb; ++j) {
            const uint32_t sb = sb0 + j, lt = (sb >> 2) - (sb0 >> 2);
            if (eleader) {
                bool ok = mbar_wait_warp(&dfull[j & 1u], (j >> 1) & 1u, &abort_flag, kSiteDFull);
                if constexpr (kQ4) {
                    // the group's d tile (loaded with its minimum-term tiles)
                    if (ok && (j == 0 || (sb & 3u) == 0))
                        ok = mbar_wait_warp(&xmfull[lt & 1u], (lt >> 1) & 1u, &abort_flag, kSiteXmFull);
                } else {
                    ok = ok && mbar_wait_warp(&dready[j & 3u], (j >> 2) & 1u, &abort_flag, kSiteScale);
                }
                if (!ok && lane == 0) epi_stop = 1u;
            }
            named_sync(kBarEpiIn, kEpiThreads);
            if (epi_stop) {
                epi_ok = false;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            float d;
            if constexpr (kQ4)
                d = reinterpret_cast<const float *>(dg_ring + (lt & 1u) * kDgSlot)[row * 4u + (sb & 3u)];
            else
                d = dscale[j & 3u][row];
            const uint32_t base = tmem + lane_addr + (j & 1u) * 128u + eh * 32u;
#pragma unroll
            for (uint32_t g = 0; g < 4; ++g) {
                uint32_t h[8], l[8];
                tmem_ld8(base + g * 8u, h);
                tmem_ld8(base + kUN + g * 8u, l);
                asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    acc[g * 8 + i] =
                        __fmaf_rn(d, __fadd_rn(__uint_as_float(h[i]), __uint_as_float(l[i])), acc[g * 8 + i]);
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
            if (eleader) {
                named_sync(kBarEpiOut, kEpiThreads);   // every epilogue warp has read the accumulator
                if (lane == 0) {
                    mbar_arrive(&dfree[j & 1u]);
                    if (kQ4 && ((sb & 3u) == 3u || j + 1 == nsb)) mbar_arrive(&xmfree[lt & 1u]);
                }
            } else {
                named_arrive(kBarEpiOut, kEpiThreads);
            }
        }
        // every MMA of the CTA complete before TMEM is read again or freed
        epi_ok = mbar_wait_warp(&accum, 0, &abort_flag, kSiteAccum) && epi_ok;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        // minus 2^(5 - scale_exp) * the minimum term
        if constexpr (kQ4) {
            if (epi_ok && nsb > 0) {
                const float mscale = __uint_as_float((uint32_t)(127 + 5 - m.scale_exp) << 23);
                const uint32_t base = tmem + lane_addr + F::dm + eh * 32u;
#pragma unroll
                for (uint32_t g = 0; g < 4; ++g) {
                    uint32_t v[8];
                    tmem_ld8(base + g * 8u, v);
                    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
                    for (int i = 0; i < 8; ++i) acc[g * 8 + i] = __fmaf_rn(-mscale, __uint_as_float(v[i]), acc[g * 8 + i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = __fmul_rn(acc[i], 4.0f);   // x was scaled by 1/4
    }

    const bool all_ok = __syncthreads_and(!epi || epi_ok) && abort_flag == 0u;
    if (!all_ok && tid == 0)
        atomicCAS(err.word, 0ull, ((unsigned long long)(kErrTimeout | (abort_flag << 8)) << 32) | err.call_id);
    const bool write = all_ok && !skip;
    bool out_bad = false;

    const uint32_t eh = (uint32_t)(warp - kFEpi0) >> 2;
    const uint32_t erow = (warp & 3) * 32u + lane;
    const uint32_t nsplit = gridDim.z;
    if (nsplit == 1) {
        const uint32_t row = row0 + erow;
        if (epi && write && row < m.rows) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t b = b0 + eh * 32u + i;
                if (b < batch) {
                    out_bad |= !isfinite(acc[i]);
                    y[(size_t)b * ldy + segs.out_offset[seg] + row] = acc[i];
                }
            }
        }
    } else {
        // exchange tile in the drained activation ring (xchg_off layout);
        // each CTA then sums a slice of the rows over the cluster, in rank
        // order, with 16-byte loads
        uint8_t *xt = x_ring;
        if (epi) {
#pragma unroll
            for (uint32_t c = 0; c < 8; ++c)
                *reinterpret_cast<float4 *>(xt + xchg_off(erow, eh * 8u + c)) =
                    make_float4(acc[4 * c], acc[4 * c + 1], acc[4 * c + 2], acc[4 * c + 3]);
        }
        cluster_sync();
        const uint32_t rank = cluster_rank();
        const uint32_t rows_per = kUM / nsplit;
        const uint32_t base = smem_u32(xt);
        for (uint32_t i = tid; i < rows_per * (kUN / 4u); i += kFThreads) {
            const uint32_t rr = i % rows_per, g = i / rows_per;
            const uint32_t lr = rank * rows_per + rr;
            const uint32_t off = base + xchg_off(lr, g);
            float4 v[8];
#pragma unroll
            for (uint32_t z = 0; z < 8; ++z)
                if (z < nsplit) v[z] = ld_dsmem4(off, z);
            float4 sum = v[0];
#pragma unroll
            for (uint32_t z = 1; z < 8; ++z)
                if (z < nsplit) {
                    sum.x = __fadd_rn(sum.x, v[z].x);
                    sum.y = __fadd_rn(sum.y, v[z].y);
                    sum.z = __fadd_rn(sum.z, v[z].z);
                    sum.w = __fadd_rn(sum.w, v[z].w);
                }
            const uint32_t row = row0 + lr, b = b0 + 4u * g;
            if (write && row < m.rows) {
                const float s4[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
                for (uint32_t k = 0; k < 4; ++k)
                    if (b + k < batch) {
                        out_bad |= !isfinite(s4[k]);
                        y[(size_t)(b + k) * ldy + segs.out_offset[seg] + row] = s4[k];
                    }
            }
        }
        cluster_sync();   // peers finish reading this CTA's tile before it exits
    }
    if (out_bad) atomicCAS(err.word, 0ull, ((unsigned long long)kErrNonFinite << 32) | err.call_id);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == kFAllocWarp) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ---- Q4_K side data (host, at upload)

uint32_t q4k_aux_pitch_a(uint32_t cols) { return (cols / 256u + 3u) / 4u * 128u; }
uint32_t q4k_aux_pitch_d(uint32_t cols) { return (cols / 256u + 3u) / 4u * 16u; }
size_t q4k_aux_bytes(uint32_t rows, uint32_t cols) {
    return (size_t)rows * (q4k_aux_pitch_a(cols) + q4k_aux_pitch_d(cols));
}

static float host_half(const uint8_t *p) {
    __half_raw r;
    r.x = (unsigned short)(p[0] | (p[1] << 8));
    return __half2float(__half(r));
}

void q4k_build_aux(const uint8_t *packed, uint32_t rows, uint32_t cols, int32_t scale_exp, uint8_t *out) {
    const uint32_t nsb = cols / 256u, pa = q4k_aux_pitch_a(cols), pd = q4k_aux_pitch_d(cols);
    std::memset(out, 0, q4k_aux_bytes(rows, cols));
    uint8_t *plane_d = out + (size_t)rows * pa;
    const float wscale = std::ldexp(1.0f, scale_exp);
    for (uint32_t r = 0; r < rows; ++r) {
        for (uint32_t sb = 0; sb < nsb; ++sb) {
            const uint8_t *blk = packed + ((size_t)r * nsb + sb) * 144u;
            const float d = host_half(blk), dmin = host_half(blk + 2) * wscale;   // exact power of two
            const uint8_t *sc = blk + 4;
            uint16_t hl[16];
            for (uint32_t j = 0; j < 8; ++j) {
                const uint32_t mn = j < 4 ? (sc[j + 4] & 63u) : ((sc[j + 4] >> 4) | ((sc[j] >> 6) << 4));
                const float v = dmin * (float)mn;   // exact: 11 x 6 significant bits
                const __half h = __float2half_rn(v);
                const __half l = __float2half_rn(v - __half2float(h));
                hl[j] = __half_raw(h).x;
                hl[8 + j] = __half_raw(l).x;
            }
            std::memcpy(out + (size_t)r * pa + sb * 32u, hl, sizeof(hl));
            std::memcpy(plane_d + (size_t)r * pd + sb * 4u, &d, 4);
        }
    }
}

bool umma_supported(const QMatrix &m) {
    const bool aligned = (m.row_bytes & 15u) == 0u && (reinterpret_cast<uintptr_t>(m.data) & 15u) == 0u;
    if (!aligned) return false;
    switch (m.type) {
    case kTypeQ4_K: return true;
    case kTypeQ6_K: return m.layout == 1 && m.cols % 256 == 0;
    case kTypeQ8_0: return m.layout == 1 && m.cols % 64 == 0;
    case kTypeBF16: return m.cols % 64 == 0;
    default: return false;
    }
}

// Narrow activation tiles, followed by the factored kernel's minimum-term
// tiles (one per batch tile and group of 16 chunks).
static size_t narrow_xtile_bytes(uint32_t batch, uint32_t cols) {
    const size_t nch = (cols + kUK - 1) / kUK;
    return (size_t)((batch + kUN - 1) / kUN) * nch * Tile<kUN>::xslot;
}
static uint32_t xm_tiles(uint32_t nchunks) { return (nchunks + 15u) / 16u; }

size_t umma_xtile_bytes(uint32_t batch, uint32_t cols, bool allow_wide) {
    const size_t nch = (cols + kUK - 1) / kUK;
    const size_t narrow = narrow_xtile_bytes(batch, cols) +
                          (size_t)((batch + kUN - 1) / kUN) * xm_tiles((uint32_t)nch) * kXmSlotBytes;
    if (batch <= (uint32_t)kUN || !allow_wide) return narrow;
    const size_t wide = (size_t)((batch + kUNWide - 1) / kUNWide) * nch * Tile<kUNWide>::xslot;
    return std::max(narrow, wide);
}


// ---- tensor maps (host)

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
        (void)cudaGetLastError();
    });
    return fn;
}

struct MapKey {
    const uint8_t *data;
    uint32_t rows, row_bytes, width, swizzle;
    bool operator==(const MapKey &o) const {
        return data == o.data && rows == o.rows && row_bytes == o.row_bytes && width == o.width &&
               swizzle == o.swizzle;
    }
};
struct MapKeyHash {
    size_t operator()(const MapKey &k) const {
        return std::hash<const void *>()(k.data) ^ ((size_t)k.rows << 20) ^ ((size_t)k.row_bytes << 40) ^
               ((size_t)k.width << 8) ^ (size_t)k.swizzle;
    }
};

// Tensor map of a matrix's raw bytes with boxes `width` bytes wide, cached
// when `cache` is set (provider matrices live as long as the provider, and a
// reused address with the same shape encodes the same map); without it the
// map is encoded straight into *out and no host memory is allocated.
static bool tensor_map(const QMatrix &m, uint32_t width, CUtensorMapSwizzle swizzle, CUtensorMap *out,
                       bool cache_maps = true) {
    static std::mutex mu;
    static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
    const MapKey key{m.data, m.rows, m.row_bytes, width, (uint32_t)swizzle};
    std::unique_lock<std::mutex> lk(mu, std::defer_lock);
    if (cache_maps) {
        lk.lock();
        auto itr = cache.find(key);
        if (itr != cache.end()) {
            *out = itr->second;
            return true;
        }
    }
    EncodeTiledFn fn = encode_fn();
    if (fn == nullptr) return false;
    CUtensorMap map;
    const cuuint64_t dims[2] = {m.row_bytes, m.rows};
    const cuuint64_t strides[1] = {m.row_bytes};
    const cuuint32_t box[2] = {width, std::min<uint32_t>(m.rows, kUM)};
    const cuuint32_t estr[2] = {1u, 1u};
    if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(m.data), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return false;
    if (cache_maps) {
        if (cache.size() > 4096) cache.clear();
        cache.emplace(key, map);
    }
    *out = map;
    return true;
}

// The maps one segment of type T needs (the box widths of TypeCfg).
template <uint32_t T>
static bool segment_maps(const QMatrix &m, CUtensorMap (&maps)[3], bool cache = true) {
    if constexpr (T == kTypeQ4_K) {
        if (!tensor_map(m, 144, CU_TENSOR_MAP_SWIZZLE_NONE, &maps[0], cache)) return false;
        if (m.aux == nullptr) return true;
        // side planes: A' rows (128-byte boxes = 4 super-blocks, swizzled as
        // the MMA reads them) and d
        QMatrix pa = m, pd = m;
        pa.data = m.aux;
        pa.row_bytes = q4k_aux_pitch_a(m.cols);
        pd.data = m.aux + (size_t)m.rows * pa.row_bytes;
        pd.row_bytes = q4k_aux_pitch_d(m.cols);
        return tensor_map(pa, 128, CU_TENSOR_MAP_SWIZZLE_128B, &maps[1], cache) &&
               tensor_map(pd, 16, CU_TENSOR_MAP_SWIZZLE_NONE, &maps[2], cache);
    } else if constexpr (T == kTypeQ6_K) {
        return tensor_map(m, 128, CU_TENSOR_MAP_SWIZZLE_128B, &maps[0], cache) &&
               tensor_map(m, 64, CU_TENSOR_MAP_SWIZZLE_64B, &maps[1], cache) &&
               tensor_map(m, 16, CU_TENSOR_MAP_SWIZZLE_NONE, &maps[2], cache);
    } else if constexpr (T == kTypeQ8_0) {
        return tensor_map(m, 128, CU_TENSOR_MAP_SWIZZLE_128B, &maps[0], cache) &&
               tensor_map(m, 16, CU_TENSOR_MAP_SWIZZLE_NONE, &maps[1], cache);
    } else {
        return tensor_map(m, 128, CU_TENSOR_MAP_SWIZZLE_128B, &maps[0], cache);
    }
}

static bool maps_for(const QMatrix &m, CUtensorMap (&maps)[3], bool cache = true) {
    switch (m.type) {
    case kTypeQ4_K: return segment_maps<kTypeQ4_K>(m, maps, cache);
    case kTypeQ6_K: return segment_maps<kTypeQ6_K>(m, maps, cache);
    case kTypeQ8_0: return segment_maps<kTypeQ8_0>(m, maps, cache);
    default: return segment_maps<kTypeBF16>(m, maps, cache);
    }
}

// Split count: 1, 2, 4 or 8 (a cluster of that many CTAs along z, at most
// `max_splits`), chosen to minimise waves x (chunks per CTA + ~8 chunks of
// pipeline fill and epilogue) + 2 per cluster member for the
// distributed-shared-memory reduction, with one CTA per SM.  The constants
// are fitted to measured B200 times of the in-/out-projection shapes.
// Split-count cost constants of the factored kernel: chunks cost about a
// quarter of the two-term kernel's, so fill and the cluster reduction weigh
// more (fitted to measured in-/out-projection times).
constexpr double kFactFill = 16.0;
constexpr double kFactMember = 3.0;

static int sm_count() {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (sms <= 0) sms = 148;
    }
    return sms;
}

static uint32_t choose_splits(uint32_t tiles, uint32_t nchunks, uint32_t max_splits, double *cost_out = nullptr,
                              double fill = 8.0, double per_member = 2.0) {
    const int sms = sm_count();
    uint32_t best = 1;
    double best_cost = 1e30;
    for (uint32_t s = 1; s <= max_splits; s *= 2) {
        if (s > 1 && nchunks < 4 * s) break;
        const double waves = std::ceil((double)tiles * s / sms);
        const double cost = waves * ((nchunks + s - 1) / s + fill) + (s > 1 ? per_member * s : 0.0);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = s; }
    }
    if (cost_out) *cost_out = best_cost;
    return best;
}

// The wide tile (256 batch rows per CTA, no split) against the narrow one
// (64 rows, split-K): a CTA spends about the same time per weight chunk
// either way (the decode of the weights bounds it), so the wide tile wins
// once it still fills the SMs; 1.15 covers its longer MMA issue per chunk.
static bool choose_wide(uint32_t tiles, uint32_t nchunks, uint32_t batch) {
    const char *env = getenv("KQ_B200_PROJ_WIDE");   // tuning and tests: 0 narrow, 1 wide
    const int forced = env ? atoi(env) : -1;
    if (batch <= (uint32_t)kUN) return false;
    if (forced == 0 || forced == 1) return forced == 1;
    double narrow;
    choose_splits(tiles * ((batch + kUN - 1) / kUN), nchunks, 8, &narrow);
    const double waves = std::ceil((double)tiles * ((batch + kUNWide - 1) / kUNWide) / sm_count());
    return waves * (nchunks + 8.0) * 1.15 < narrow;
}

// Largest split cluster (8, 4, 2 or 1) the device can co-schedule for this
// kernel; queried once per type and device (the attribute it sets belongs to
// the current device).
template <typename Kernel>
static uint32_t probe_splits(Kernel kernel, uint32_t threads, uint32_t smem) {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    uint32_t best = 1;
    for (uint32_t s = 8; s >= 2; s /= 2) {
        cudaLaunchConfig_t cfg{};
        cfg.gridDim = dim3(1, 1, s);
        cfg.blockDim = dim3(threads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = 1;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = s;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) == cudaSuccess && n > 0) {
            best = s;
            break;
        }
    }
    (void)cudaGetLastError();
    return best;
}

// The same for the factored kernel (its own shared memory and block size).
template <uint32_t T>
static uint32_t max_splits_fact() {
    static std::atomic<uint32_t> per_device[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 63;
    uint32_t cached = per_device[dev].load(std::memory_order_acquire);
    if (cached == 0) {
        cached = probe_splits(proj_fact_kernel<T>, kFThreads, Fact<T>::smem);
        per_device[dev].store(cached, std::memory_order_release);
    }
    return cached;
}

// Factored kernel for Q4_K / Q6_K batch tiles of 64 (KQ_B200_PROJ_FACT=0
// selects the two-term kernel instead; tuning and tests).
static bool fact_enabled() {
    const char *e = getenv("KQ_B200_PROJ_FACT");
    return !(e && e[0] == '0');
}

template <uint32_t T>
static uint32_t max_splits_for() {
    static std::atomic<uint32_t> per_device[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 63;
    uint32_t cached = per_device[dev].load(std::memory_order_acquire);
    if (cached == 0) {
        cudaFuncSetAttribute(proj_umma_kernel<T, kUN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             Ring<T, kUN>::smem);
        uint32_t best = 1;
        for (uint32_t s = 8; s >= 2; s /= 2) {
            cudaLaunchConfig_t cfg{};
            cfg.gridDim = dim3(1, 1, s);
            cfg.blockDim = dim3(kThreads);
            cfg.dynamicSmemBytes = Ring<T, kUN>::smem;
            cudaLaunchAttribute at[1];
            at[0].id = cudaLaunchAttributeClusterDimension;
            at[0].val.clusterDim.x = 1;
            at[0].val.clusterDim.y = 1;
            at[0].val.clusterDim.z = s;
            cfg.attrs = at;
            cfg.numAttrs = 1;
            int n = 0;
            if (cudaOccupancyMaxActiveClusters(&n, proj_umma_kernel<T, kUN>, &cfg) == cudaSuccess && n > 0) {
                best = s;
                break;
            }
        }
        (void)cudaGetLastError();
        cached = best;
        per_device[dev].store(cached, std::memory_order_release);
    }
    return cached;
}

template <uint32_t T>
static bool launch_typed(uint32_t tiles, uint32_t nchunks, const ProjSegments &segs, const uint8_t *xt,
                         uint32_t nchunks_x, const uint8_t *xm, float *y, uint32_t ldy, uint32_t batch, bool wide,
                         ErrorWord err, cudaStream_t stream, bool cache_maps) {
    TmapSet maps;
    for (int i = 0; i < segs.count; ++i) {
        if (!segment_maps<T>(segs.m[i], maps.map[i], cache_maps)) return false;
        maps.box_rows[i] = std::min<uint32_t>(segs.m[i].rows, kUM);
    }
    cudaLaunchConfig_t cfg{};
    cfg.blockDim = dim3(kThreads);
    cfg.stream = stream;
    cudaLaunchAttribute at[2];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // see launch_pdl
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    if (wide) {
        static DeviceOnce attr;
        attr.run([] {
            cudaFuncSetAttribute(proj_umma_kernel<T, kUNWide>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Ring<T, kUNWide>::smem);
        });
        cfg.gridDim = dim3(tiles, (batch + kUNWide - 1) / kUNWide, 1);
        cfg.dynamicSmemBytes = Ring<T, kUNWide>::smem;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, proj_umma_kernel<T, kUNWide>, maps, segs, xt, nchunks_x, y, ldy, batch, nchunks,
                           err);
        return true;
    }
    const uint32_t btiles = (batch + kUN - 1) / kUN;
    const char *forced_env = getenv("KQ_B200_PROJ_SPLITS");   // tuning: fixed split count
    const int forced = forced_env ? atoi(forced_env) : 0;
    if constexpr (T == kTypeQ4_K || T == kTypeQ6_K) {
        bool aux = true;   // Q4_K: every segment carries its side data
        for (int i = 0; i < segs.count; ++i) aux &= T != kTypeQ4_K || segs.m[i].aux != nullptr;
        if (fact_enabled() && aux && (T != kTypeQ4_K || xm != nullptr)) {
            static DeviceOnce attr;
            attr.run([] {
                cudaFuncSetAttribute(proj_fact_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     Fact<T>::smem);
            });
            const uint32_t cap = max_splits_fact<T>();
            uint32_t splits = choose_splits(tiles * btiles, nchunks, cap, nullptr, kFactFill, kFactMember);
            if (forced == 1 || forced == 2 || forced == 4 || forced == 8) splits = std::min<uint32_t>((uint32_t)forced, cap);
            const uint32_t per = ((nchunks + splits - 1) / splits + 3u) / 4u * 4u;
            cfg.gridDim = dim3(tiles, btiles, splits);
            cfg.blockDim = dim3(kFThreads);
            cfg.dynamicSmemBytes = Fact<T>::smem;
            at[1].id = cudaLaunchAttributeClusterDimension;
            at[1].val.clusterDim.x = 1;
            at[1].val.clusterDim.y = 1;
            at[1].val.clusterDim.z = splits;
            cfg.numAttrs = 2;
            cudaLaunchKernelEx(&cfg, proj_fact_kernel<T>, maps, segs, xt, nchunks_x, xm, xm_tiles(nchunks_x), y,
                               ldy, batch, per, err);
            return true;
        }
    }
    uint32_t splits = choose_splits(tiles * btiles, nchunks, max_splits_for<T>());
    if (forced == 1 || forced == 2 || forced == 4 || forced == 8)
        splits = std::min<uint32_t>((uint32_t)forced, max_splits_for<T>());
    // chunks per split: whole super-block steps
    constexpr uint32_t SC = TypeCfg<T>::sc;
    const uint32_t per = ((nchunks + splits - 1) / splits + SC - 1) / SC * SC;
    cfg.gridDim = dim3(tiles, btiles, splits);
    cfg.dynamicSmemBytes = Ring<T, kUN>::smem;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = 1;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = splits;
    cfg.numAttrs = 2;
    cudaLaunchKernelEx(&cfg, proj_umma_kernel<T, kUN>, maps, segs, xt, nchunks_x, y, ldy, batch, per, err);
    return true;
}

// Launches one group of segments that share a weight type.
static bool launch_group(uint32_t type, ProjSegments segs, const uint8_t *xt, uint32_t nchunks_x,
                         const uint8_t *xm, float *y, uint32_t ldy, uint32_t batch, bool wide, ErrorWord err,
                         cudaStream_t stream, bool cache_maps) {
    uint32_t acc = 0, cols = 0;
    for (int i = 0; i < segs.count; ++i) {
        segs.tile_start[i] = acc;
        acc += (segs.m[i].rows + kUM - 1) / kUM;
        cols = std::max(cols, segs.m[i].cols);
    }
    segs.tile_start[segs.count] = acc;
    const uint32_t nchunks = (cols + kUK - 1) / kUK;
    bool ok;
    switch (type) {
    case kTypeQ4_K: ok = launch_typed<kTypeQ4_K>(acc, nchunks, segs, xt, nchunks_x, xm, y, ldy, batch, wide, err, stream, cache_maps); break;
    case kTypeQ6_K: ok = launch_typed<kTypeQ6_K>(acc, nchunks, segs, xt, nchunks_x, xm, y, ldy, batch, wide, err, stream, cache_maps); break;
    case kTypeQ8_0: ok = launch_typed<kTypeQ8_0>(acc, nchunks, segs, xt, nchunks_x, xm, y, ldy, batch, wide, err, stream, cache_maps); break;
    default: ok = launch_typed<kTypeBF16>(acc, nchunks, segs, xt, nchunks_x, xm, y, ldy, batch, wide, err, stream, cache_maps); break;
    }
    if (ok) count_launch();
    return ok;
}

bool launch_projection_umma(const ProjSegments &in, const float *x, uint32_t ldx, float *y, uint32_t ldy,
                            uint32_t batch, uint8_t *xtiles, size_t xtile_bytes, ErrorWord err,
                            cudaStream_t stream, bool cache_maps, bool allow_wide) {
    uint32_t cols = 0;
    for (int i = 0; i < in.count; ++i) {
        if (!umma_supported(in.m[i])) return false;
        cols = std::max(cols, in.m[i].cols);
    }
    for (int i = 1; i < in.count; ++i)
        if (in.m[i].cols != cols) return false;
    if (xtiles == nullptr || xtile_bytes < umma_xtile_bytes(batch, cols, allow_wide)) return false;
    // tensor maps first, so that a failure launches nothing
    for (int i = 0; i < in.count; ++i) {
        CUtensorMap maps[3];
        if (!maps_for(in.m[i], maps, cache_maps)) return false;
    }
    const uint32_t nchunks = (cols + kUK - 1) / kUK;
    uint32_t tiles = 0;
    for (int i = 0; i < in.count; ++i) tiles += (in.m[i].rows + kUM - 1) / kUM;
    const bool wide = allow_wide && choose_wide(tiles, nchunks, batch);
    // the factored Q4_K kernel also reads the sub-block sums of the activations
    bool q4 = false;
    for (int i = 0; i < in.count; ++i) q4 |= in.m[i].type == kTypeQ4_K;
    uint8_t *xm = (!wide && q4 && fact_enabled()) ? xtiles + narrow_xtile_bytes(batch, cols) : nullptr;
    if (wide) {
        const dim3 xg(nchunks * (kUNWide / 16), (batch + kUNWide - 1) / kUNWide);
        launch_pdl(xconv_kernel<kUNWide>, xg, 128, 0, stream, x, ldx, batch, cols, nchunks, xtiles,
                   (uint8_t *)nullptr, 0u, err);
    } else {
        const dim3 xg(nchunks * (kUN / 16), (batch + kUN - 1) / kUN);
        launch_pdl(xconv_kernel<kUN>, xg, 128, 0, stream, x, ldx, batch, cols, nchunks, xtiles, xm,
                   xm_tiles(nchunks), err);
    }
    count_launch();
    // one launch per weight type present
    bool done[kMaxSegments] = {};
    for (int i = 0; i < in.count; ++i) {
        if (done[i]) continue;
        ProjSegments g{};
        for (int j = i; j < in.count; ++j) {
            if (done[j] || in.m[j].type != in.m[i].type) continue;
            g.m[g.count] = in.m[j];
            g.out_offset[g.count] = in.out_offset[j];
            ++g.count;
            done[j] = true;
        }
        launch_group(in.m[i].type, g, xtiles, nchunks, xm, y, ldy, batch, wide, err, stream, cache_maps);
    }
    return true;
}

}  // namespace kqb
