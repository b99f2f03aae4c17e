// Dequant-fused projection GEMM on the 5th-generation tensor cores.
//
//   y[b][n] = sum_k W[n][k] * x[b][k]      (W: GGUF blocks in HBM, x: F32)
//
// One CTA computes a 128 (weight rows, MMA M) x 64 (batch rows, MMA N) tile
// of y^T with tcgen05.mma (kind::f16, BF16 operands, F32 accumulator in
// TMEM).  F32 accuracy is kept with a three-term split: w = wh + wl and
// x = xh + xl (bf16 each, the low part rounded from the residual), and
// y ~= wh*xh + wh*xl + wl*xh, the dropped wl*xl term being ~2^-16 relative.
//
// Pipeline per K chunk of 64 (all 256 threads take part in every phase):
//   1. cp.async stages, two chunks ahead, the chunk's raw GGUF bytes of the
//      128 weight rows (16-byte pieces of each row: Q4_K header + quants,
//      Q6_K/Q8_0 planes, BF16 values) and the chunk's activation tile, which
//      a small kernel converted once per launch into bf16 hi/lo already in
//      the shared-memory image the MMA reads (4-slot ring).
//   2. The raw bytes are decoded from shared memory (quant.cuh, bit-exact
//      with the reference decoder), split into bf16 hi/lo and stored in the
//      canonical K-major 128-byte-swizzle layout (row r at r*128 B, 16-byte
//      chunk c stored at chunk c ^ (r & 7)).  Dequantised weights never
//      reach HBM.
//   3. Thread 0 issues the 4 x 3 tcgen05.mma of the chunk and commits them
//      to the ring slot's mbarrier.
// Epilogue: tcgen05.ld 32x32b from TMEM.  One kernel instance per weight
// type keeps the code small.
// Split-K over gridDim.z writes partial tiles that a second kernel sums in
// a fixed order (deterministic results).
//
// Every mbarrier wait is bounded; on time-out the kernel records an error
// in the call's error word, waits (bounded) for its own MMAs, frees TMEM and
// returns.
#include "kernels.hpp"
#include "quant.cuh"

#include <algorithm>

#include <cuda_bf16.h>

namespace kqb {

namespace {

constexpr int kUM = 128;         // weight rows per CTA (MMA M)
constexpr int kUN = 64;          // batch rows per CTA (MMA N)
constexpr int kUK = 64;          // K per stage (one 128-byte swizzle row of bf16)
constexpr int kRing = 4;                  // raw + activation slots (2 chunks ahead)
constexpr int kDec = 2;                   // decoded weight tiles
constexpr int kATile = kUM * kUK * 2;     // bytes of one bf16 A tile (16 KB)
constexpr int kBTile = kUN * kUK * 2;     // bytes of one bf16 B tile (8 KB)
constexpr int kRawBytes = 16 * 1024;      // raw weight bytes of one chunk (max over types)
constexpr int kSlotBytes = kRawBytes + 2 * kBTile;
constexpr int kSmemBytes = kRing * kSlotBytes + kDec * 2 * kATile + 1024 /*align*/;
constexpr uint32_t kTmemCols = 64;
constexpr uint32_t kWaitLimit = 1u << 26;  // mbarrier polls before giving up
constexpr uint32_t kErrTimeout = 4;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

// Bounded wait for the phase with parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
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
    }
    return false;
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

// Instruction descriptor: F32 accumulate, BF16 A and B, both K-major,
// N = kUN, M = kUM.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kUN >> 3) << 17) |
                            ((uint32_t)(kUM >> 4) << 24);

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(a), "l"(b), "r"(kIdesc), "r"(accumulate));
}

__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// Splits an F32 value into bf16 hi (round to nearest) and bf16 lo of the
// exact residual.  Returns (lo << 16) | hi.
__device__ __forceinline__ uint32_t split_bf16(float v) {
    __nv_bfloat16 hi = __float2bfloat16_rn(v);
    float r = v - __bfloat162float(hi);
    __nv_bfloat16 lo = __float2bfloat16_rn(r);
    return (uint32_t)__bfloat16_as_ushort(hi) | ((uint32_t)__bfloat16_as_ushort(lo) << 16);
}

// Packs 8 values into two 16-byte chunks (hi, lo) of bf16.
__device__ __forceinline__ void pack8(const float *v, uint4 &hi, uint4 &lo) {
    uint32_t s[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = split_bf16(v[i]);
    hi.x = (s[0] & 0xFFFFu) | (s[1] << 16);
    hi.y = (s[2] & 0xFFFFu) | (s[3] << 16);
    hi.z = (s[4] & 0xFFFFu) | (s[5] << 16);
    hi.w = (s[6] & 0xFFFFu) | (s[7] << 16);
    lo.x = (s[0] >> 16) | (s[1] & 0xFFFF0000u);
    lo.y = (s[2] >> 16) | (s[3] & 0xFFFF0000u);
    lo.z = (s[4] >> 16) | (s[5] & 0xFFFF0000u);
    lo.w = (s[6] >> 16) | (s[7] & 0xFFFF0000u);
}

// Byte offset of 16-byte chunk `chunk` (0..7) of row `r` in a SW128 tile.
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t chunk) {
    return r * 128u + ((chunk ^ (r & 7u)) << 4);
}


// Raw bytes per weight row and chunk staged in shared memory.
template <uint32_t T> struct RawRow;
template <> struct RawRow<kTypeQ4_K> { static constexpr uint32_t bytes = 48; };   // header 16 + quants 32
template <> struct RawRow<kTypeQ6_K> { static constexpr uint32_t bytes = 128; };  // ql 64, qh 32, sc 16, d 16
template <> struct RawRow<kTypeQ8_0> { static constexpr uint32_t bytes = 80; };   // codes 64, d 16
template <> struct RawRow<kTypeBF16> { static constexpr uint32_t bytes = 128; };  // 64 values

__device__ __forceinline__ void cp16(uint32_t smem_addr, const void *gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr), "l"(gmem) : "memory");
}

// 16-byte piece `p` of row `row` for chunk `c` (same piece numbering as the
// raw row layout above).  Returns false past the last piece.
template <uint32_t T>
__device__ __forceinline__ const uint8_t *raw_piece(const uint8_t *row, uint32_t cols, uint32_t c, uint32_t p) {
    if constexpr (T == kTypeQ4_K) {
        const uint8_t *b = row + (c >> 2) * 144u;           // 4 chunks per super-block
        if (p == 0) return b;                               // d, dmin, scales
        return b + 16u + (c & 3u) * 32u + (p - 1u) * 16u;   // quants of the 64-group
    } else if constexpr (T == kTypeQ6_K) {
        const uint32_t nsb = cols >> 8, sb = c >> 2, half = (c & 3u) >> 1;
        if (p < 4) return row + sb * 128u + half * 64u + p * 16u;            // ql
        if (p < 6) return row + nsb * 128u + sb * 64u + half * 32u + (p - 4u) * 16u;  // qh
        if (p == 6) return row + nsb * 192u + sb * 16u;                     // scales
        return row + ((nsb * 208u + sb * 2u) & ~15u);                        // d chunk
    } else if constexpr (T == kTypeQ8_0) {
        const uint32_t nb = cols >> 5;
        if (p < 4) return row + (2u * c) * 32u + p * 16u;                    // codes of 2 blocks
        return row + ((nb * 32u + 2u * c * 2u) & ~15u);                      // d chunk
    } else {   // BF16
        return row + (size_t)c * 128u + p * 16u;
    }
}

// Matrix description with the weight type fixed at compile time, so the
// decoders keep only the branch of that type.
template <uint32_t T> struct TypedQ {
    static constexpr uint32_t type = T;
    uint32_t layout, cols, row_bytes;
};

template <uint32_t T>
__device__ __forceinline__ void raw_to_regs(const uint8_t *raw, uint32_t cols, uint32_t c, uint32_t half_,
                                            Raw32 &r) {
    r.fast = 1u;
    if constexpr (T == kTypeQ4_K) {
        r.v[0] = *reinterpret_cast<const uint4 *>(raw);
        r.v[1] = *reinterpret_cast<const uint4 *>(raw + 16);
        r.v[2] = *reinterpret_cast<const uint4 *>(raw + 32);
    } else if constexpr (T == kTypeQ6_K) {
        const uint32_t nsb = cols >> 8, sb = c >> 2, half = (c & 3u) >> 1;
        const uint32_t s = 2u * (c & 1u) + half_;
        r.v[0] = *reinterpret_cast<const uint4 *>(raw + 32u * half_);
        r.v[1] = *reinterpret_cast<const uint4 *>(raw + 32u * half_ + 16u);
        r.v[2] = *reinterpret_cast<const uint4 *>(raw + 64);
        r.v[3] = *reinterpret_cast<const uint4 *>(raw + 80);
        const uint32_t scp = *reinterpret_cast<const uint16_t *>(raw + 96u + half * 8u + 2u * s);
        const uint32_t dp = *reinterpret_cast<const uint16_t *>(raw + 112u + ((nsb * 208u + sb * 2u) & 15u));
        r.e = scp | (dp << 16);
    } else if constexpr (T == kTypeQ8_0) {
        const uint32_t nb = cols >> 5, blk = 2u * c + half_;
        r.v[0] = *reinterpret_cast<const uint4 *>(raw + 32u * half_);
        r.v[1] = *reinterpret_cast<const uint4 *>(raw + 32u * half_ + 16u);
        r.e = *reinterpret_cast<const uint16_t *>(raw + 64u + ((nb * 32u + blk * 2u) & 15u));
    } else {
        const uint8_t *p = raw + 64u * half_;
        r.v[0] = *reinterpret_cast<const uint4 *>(p);
        r.v[1] = *reinterpret_cast<const uint4 *>(p + 16);
        r.v[2] = *reinterpret_cast<const uint4 *>(p + 32);
        r.v[3] = *reinterpret_cast<const uint4 *>(p + 48);
    }
}

}  // namespace

// Activations to bf16 hi/lo tiles in the MMA's shared-memory image:
// out[btile][chunk] = { hi: 64 rows x 128 B swizzled, lo: same }.
__global__ void xconv_kernel(const float *__restrict__ x, uint32_t ldx, uint32_t batch, uint32_t cols,
                             uint32_t nchunks, uint8_t *__restrict__ out) {
    const uint32_t bt = blockIdx.y, c = blockIdx.x;
    const uint32_t r = threadIdx.x >> 2, q = threadIdx.x & 3;   // 64 rows x 4 quarters of 16
    const uint32_t b = bt * kUN + r;
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const uint32_t k = c * kUK + q * 16 + i;
        v[i] = (b < batch && k < cols) ? x[(size_t)b * ldx + k] : 0.0f;
    }
    uint8_t *tile = out + ((size_t)bt * nchunks + c) * (2 * kBTile);
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        uint4 hi, lo;
        pack8(v + 8 * j, hi, lo);
        const uint32_t off = sw128_off(r, q * 2 + j);
        *reinterpret_cast<uint4 *>(tile + off) = hi;
        *reinterpret_cast<uint4 *>(tile + kBTile + off) = lo;
    }
}

template <uint32_t T>
__global__ void __launch_bounds__(256, 1)
proj_umma_kernel(ProjSegments segs, const uint8_t *__restrict__ xtiles, uint32_t nchunks_x,
                 float *__restrict__ y, uint32_t ldy, uint32_t batch,
                 float *__restrict__ partial, uint32_t kchunks_per_split, ErrorWord err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[kRing];
    __shared__ uint32_t tmem_base_slot;
    if (*reinterpret_cast<volatile unsigned long long *>(err.word) != 0ull) return;
    static_assert(RawRow<T>::bytes * kUM <= kRawBytes, "raw slot too small");

    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *ring = smem;                                   // kRing x [B hi | B lo | raw]
    uint8_t *dec = smem + kRing * kSlotBytes;               // kDec x [A hi | A lo]
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kUM;
    const uint32_t b0 = blockIdx.y * kUN;
    const uint32_t nchunks_total = (m.cols + kUK - 1) / kUK;
    const uint32_t c_begin = blockIdx.z * kchunks_per_split;
    const uint32_t c_end = min(nchunks_total, c_begin + kchunks_per_split);
    const uint32_t nchunks = c_end > c_begin ? c_end - c_begin : 0;

    if (tid == 0) {
        for (int s = 0; s < kRing; ++s) mbar_init(&bars[s], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_base_slot)), "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = tmem_base_slot;

    // staging roles: pieces of the 128 raw rows, then the 16 KB x tile
    constexpr uint32_t kPieces = RawRow<T>::bytes / 16;
    auto stage_chunk = [&](uint32_t it) {
        const uint32_t c = c_begin + it;
        uint8_t *slot = ring + (it % kRing) * kSlotBytes;
        const uint32_t raw_base = smem_u32(slot + 2 * kBTile);
        for (uint32_t i = tid; i < kUM * kPieces; i += blockDim.x) {
            const uint32_t r = i / kPieces, p = i % kPieces;
            const uint32_t grow = min(row0 + r, m.rows - 1);   // rows past the end decode unused data
            cp16(raw_base + r * RawRow<T>::bytes + p * 16u,
                 raw_piece<T>(m.data + (size_t)grow * m.row_bytes, m.cols, c, p));
        }
        const uint8_t *xsrc = xtiles + ((size_t)blockIdx.y * nchunks_x + c) * (2 * kBTile);
        const uint32_t xdst = smem_u32(slot);
        for (uint32_t i = tid; i < 2 * kBTile / 16; i += blockDim.x) cp16(xdst + i * 16u, xsrc + i * 16u);
    };
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };

    const uint32_t a_row = tid >> 1, a_half = tid & 1;
    const bool a_live = row0 + a_row < m.rows;
    bool ok = true;
    uint32_t issued = 0;
    if (nchunks > 0) stage_chunk(0);
    commit();
    if (nchunks > 1) stage_chunk(1);
    commit();
    for (uint32_t it = 0; it < nchunks; ++it) {
        if (it >= 2) {
            // MMAs of chunk it-2 read decode tile it%2 and ring slot (it+2)%4
            const bool got = mbar_wait(&bars[(it - 2) % kRing], ((it - 2) / kRing) & 1u);
            if (!__syncthreads_and(got)) { ok = false; break; }
        }
        if (it + 2 < nchunks) stage_chunk(it + 2);
        commit();
        asm volatile("cp.async.wait_group 2;" ::: "memory");
        __syncthreads();
        const uint32_t c = c_begin + it;
        uint8_t *slot = ring + (it % kRing) * kSlotBytes;
        uint8_t *A_hi = dec + (it % kDec) * 2 * kATile;
        uint8_t *A_lo = A_hi + kATile;
        {
            float w[32];
            if (a_live) {
                Raw32 r;
                raw_to_regs<T>(slot + 2 * kBTile + a_row * RawRow<T>::bytes, m.cols, c, a_half, r);
                const TypedQ<T> tq{m.layout, m.cols, m.row_bytes};
                decode_raw32(tq, r, nullptr, c * kUK + a_half * 32, w);
            } else {
#pragma unroll
                for (int i = 0; i < 32; ++i) w[i] = 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                uint4 hi, lo;
                pack8(w + 8 * j, hi, lo);
                const uint32_t off = sw128_off(a_row, a_half * 4 + j);
                *reinterpret_cast<uint4 *>(A_hi + off) = hi;
                *reinterpret_cast<uint4 *>(A_lo + off) = lo;
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ah = smem_u32(A_hi), al = smem_u32(A_lo);
            const uint32_t bh = smem_u32(slot), bl = smem_u32(slot + kBTile);
#pragma unroll
            for (int kk = 0; kk < kUK / 16; ++kk) {
                const uint32_t koff = kk * 32;
                const uint64_t dah = sw128_desc(ah + koff), dal = sw128_desc(al + koff);
                const uint64_t dbh = sw128_desc(bh + koff), dbl = sw128_desc(bl + koff);
                umma_bf16(tmem, dah, dbh, (it > 0 || kk > 0) ? 1u : 0u);
                umma_bf16(tmem, dah, dbl, 1u);
                umma_bf16(tmem, dal, dbh, 1u);
            }
            umma_commit(&bars[it % kRing]);
        }
        ++issued;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    if (ok && issued > 0) {
        const uint32_t last = issued - 1;
        if (!mbar_wait(&bars[last % kRing], (last / kRing) & 1u)) ok = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool all_ok = __syncthreads_and(ok);

    const uint32_t lane_base = 32u * (warp & 3);
    const uint32_t col_base = (uint32_t)(warp >> 2) * 32u;
    const uint32_t row = row0 + lane_base + lane;
    float *dst = partial ? partial + (size_t)blockIdx.z * batch * ldy : y;
    if (all_ok && issued > 0) {
        uint32_t r[32];
        const uint32_t taddr = tmem + (lane_base << 16) + col_base;
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
            "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
            "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
            : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
              "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
              "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
              "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
              "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
            : "r"(taddr));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (row < m.rows) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t b = b0 + col_base + j;
                if (b < batch) dst[(size_t)b * ldy + segs.out_offset[seg] + row] = __uint_as_float(r[j]);
            }
        }
    } else if (all_ok && partial != nullptr && row < m.rows) {
        // an empty split still owns its slice of the partial buffer
        for (int j = 0; j < 32; ++j) {
            const uint32_t b = b0 + col_base + j;
            if (b < batch) dst[(size_t)b * ldy + segs.out_offset[seg] + row] = 0.0f;
        }
    }
    if (!all_ok && tid == 0) {
        atomicCAS(err.word, 0ull, ((unsigned long long)kErrTimeout << 32) | err.call_id);
        for (uint32_t s = 0; s < kRing; ++s) (void)mbar_wait(&bars[s], 0), (void)mbar_wait(&bars[s], 1);
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// Sums the split-K partial tiles in split order (deterministic).
__global__ void splitk_reduce_kernel(const float *__restrict__ partial, uint32_t splits, uint32_t batch,
                                     uint32_t ldy, float *__restrict__ y, uint32_t col0, uint32_t cols) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)batch * cols) return;
    const uint32_t b = (uint32_t)(i / cols), c = col0 + (uint32_t)(i % cols);
    const size_t off = (size_t)b * ldy + c;
    float s = partial[off];
    for (uint32_t z = 1; z < splits; ++z) s += partial[(size_t)z * batch * ldy + off];
    y[off] = s;
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

size_t umma_xtile_bytes(uint32_t batch, uint32_t cols) {
    return (size_t)((batch + kUN - 1) / kUN) * ((cols + kUK - 1) / kUK) * 2 * kBTile;
}

// Launches one group of segments that share a weight type.
static void launch_group(uint32_t type, ProjSegments segs, const uint8_t *xt, uint32_t nchunks_x, float *y,
                         uint32_t ldy, uint32_t batch, float *partial, size_t partial_floats, ErrorWord err,
                         cudaStream_t stream) {
    uint32_t acc = 0, cols = 0, col_lo = UINT32_MAX, col_hi = 0, covered = 0;
    for (int i = 0; i < segs.count; ++i) {
        segs.tile_start[i] = acc;
        acc += (segs.m[i].rows + kUM - 1) / kUM;
        cols = std::max(cols, segs.m[i].cols);
        col_lo = std::min(col_lo, segs.out_offset[i]);
        col_hi = std::max(col_hi, segs.out_offset[i] + segs.m[i].rows);
        covered += segs.m[i].rows;
    }
    segs.tile_start[segs.count] = acc;
    const uint32_t btiles = (batch + kUN - 1) / kUN;
    const uint32_t nchunks = (cols + kUK - 1) / kUK;
    // split K until there are about two CTAs per SM, keeping >= 4 chunks
    uint32_t splits = 1;
    while (splits < kProjPartialSplits && acc * btiles * splits < 2 * 148 && nchunks / (splits * 2) >= 4)
        splits *= 2;
    if (splits > 1 && (partial == nullptr || partial_floats < (size_t)splits * batch * ldy)) splits = 1;
    if (covered != col_hi - col_lo) splits = 1;   // the reduce covers one contiguous range
    const uint32_t per = (nchunks + splits - 1) / splits;
    dim3 grid(acc, btiles, splits);
    float *part = splits > 1 ? partial : nullptr;
#define KQB_LAUNCH(TT)                                                                              \
    cudaFuncSetAttribute(proj_umma_kernel<TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes); \
    proj_umma_kernel<TT><<<grid, 256, kSmemBytes, stream>>>(segs, xt, nchunks_x, y, ldy, batch, part, per, err)
    switch (type) {
    case kTypeQ4_K: KQB_LAUNCH(kTypeQ4_K); break;
    case kTypeQ6_K: KQB_LAUNCH(kTypeQ6_K); break;
    case kTypeQ8_0: KQB_LAUNCH(kTypeQ8_0); break;
    default: KQB_LAUNCH(kTypeBF16); break;
    }
#undef KQB_LAUNCH
    count_launch();
    if (splits > 1) {
        const uint64_t n = (uint64_t)batch * (col_hi - col_lo);
        splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(partial, splits, batch, ldy, y,
                                                                            col_lo, col_hi - col_lo);
        count_launch();
    }
}

bool launch_projection_umma(const ProjSegments &in, const float *x, uint32_t ldx, float *y, uint32_t ldy,
                            uint32_t batch, float *partial, size_t partial_floats, uint8_t *xtiles,
                            size_t xtile_bytes, ErrorWord err, cudaStream_t stream) {
    uint32_t cols = 0;
    for (int i = 0; i < in.count; ++i) {
        if (!umma_supported(in.m[i])) return false;
        cols = std::max(cols, in.m[i].cols);
    }
    for (int i = 1; i < in.count; ++i)
        if (in.m[i].cols != cols) return false;
    if (xtiles == nullptr || xtile_bytes < umma_xtile_bytes(batch, cols)) return false;
    const uint32_t nchunks = (cols + kUK - 1) / kUK;
    dim3 xg(nchunks, (batch + kUN - 1) / kUN);
    xconv_kernel<<<xg, 256, 0, stream>>>(x, ldx, batch, cols, nchunks, xtiles);
    count_launch();
    // one launch per weight type; the partial buffer is reused in order
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
        launch_group(in.m[i].type, g, xtiles, nchunks, y, ldy, batch, partial, partial_floats, err, stream);
    }
    return true;
}

}  // namespace kqb
