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
// Producer: all 256 threads decode the GGUF blocks of the K chunk in
// registers (quant.cuh, bit-exact with the reference decoder), split them,
// and store bf16 hi/lo tiles in shared memory in the canonical K-major
// 128-byte-swizzle layout (row r at r*128 B, 16-byte chunk c stored at
// chunk c ^ (r & 7)).  The weights never reach HBM in dequantised form.
// MMA issue: thread 0, four K=16 steps per 64-wide K chunk, committed to an
// mbarrier per shared-memory stage (two stages: decode of chunk c+1
// overlaps the MMAs of chunk c).  Epilogue: tcgen05.ld 32x32b from TMEM.
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
constexpr int kStages = 2;
constexpr int kATile = kUM * kUK * 2;     // bytes of one bf16 A tile (16 KB)
constexpr int kBTile = kUN * kUK * 2;     // bytes of one bf16 B tile (8 KB)
constexpr int kStageBytes = 2 * kATile + 2 * kBTile;
constexpr int kSmemBytes = kStages * kStageBytes + 1024 /*align*/ + 64;
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

}  // namespace

__global__ void __launch_bounds__(256, 1)
proj_umma_kernel(ProjSegments segs, const float *__restrict__ x, uint32_t ldx,
                 float *__restrict__ y, uint32_t ldy, uint32_t batch,
                 float *__restrict__ partial, uint32_t kchunks_per_split, ErrorWord err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ uint64_t bars[kStages];
    __shared__ uint32_t tmem_base_slot;
    if (*reinterpret_cast<volatile unsigned long long *>(err.word) != 0ull) return;

    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kUM;
    const uint32_t b0 = blockIdx.y * kUN;
    const uint32_t nchunks_total = (m.cols + kUK - 1) / kUK;
    const uint32_t c_begin = blockIdx.z * kchunks_per_split;
    const uint32_t c_end = min(nchunks_total, c_begin + kchunks_per_split);

    if (tid == 0) {
        for (int s = 0; s < kStages; ++s) mbar_init(&bars[s], 1);
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

    // producer roles
    const uint32_t a_row = tid >> 1;              // 0..127
    const uint32_t a_half = tid & 1;              // 32-element half of the K chunk
    const uint32_t wrow = row0 + a_row;
    const uint8_t *wptr = m.data + (size_t)min(wrow, m.rows - 1) * m.row_bytes;
    const uint32_t b_row = tid >> 2;              // 0..63
    const uint32_t b_quarter = tid & 3;           // 16-element quarter
    const uint32_t xb = b0 + b_row;

    bool ok = true;
    uint32_t issued = 0;
    // software pipeline: the raw bytes of chunk c+1 are loaded into
    // registers while chunk c is decoded and stored
    const bool a_live = wrow < m.rows;
    const bool x_vec = (ldx & 3u) == 0u && (reinterpret_cast<uintptr_t>(x) & 15u) == 0u;
    Raw32 raw_cur, raw_nxt;
    float4 x_cur[4], x_nxt[4];
    auto load_chunk = [&](uint32_t c, Raw32 &raw, float4 (&xv)[4]) {
        const uint32_t k0 = c * kUK;
        const uint32_t fa = k0 + a_half * 32;
        raw.fast = 0u;
        if (a_live && fa < m.cols) load_raw32(m, wptr, fa, raw);
        const uint32_t fb = k0 + b_quarter * 16;
        if (xb < batch && fb + 16 <= m.cols && x_vec) {
            const float4 *src = reinterpret_cast<const float4 *>(x + (size_t)xb * ldx + fb);
#pragma unroll
            for (int i = 0; i < 4; ++i) xv[i] = src[i];
        } else {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                float t[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t k = fb + 4 * i + j;
                    t[j] = (xb < batch && k < m.cols) ? x[(size_t)xb * ldx + k] : 0.0f;
                }
                xv[i] = make_float4(t[0], t[1], t[2], t[3]);
            }
        }
    };
    if (c_begin < c_end) load_chunk(c_begin, raw_cur, x_cur);
    for (uint32_t c = c_begin; c < c_end; ++c) {
        const uint32_t it = c - c_begin;
        const int stage = it % kStages;
        uint8_t *A_hi = smem + stage * kStageBytes;
        uint8_t *A_lo = A_hi + kATile;
        uint8_t *B_hi = A_lo + kATile;
        uint8_t *B_lo = B_hi + kBTile;
        if (it >= kStages) {
            // the MMAs that read this stage (chunk it - kStages) must be done;
            // the decision to continue is made uniformly by the whole CTA
            const bool got = mbar_wait(&bars[stage], ((it - kStages) / kStages) & 1u);
            if (!__syncthreads_and(got)) { ok = false; break; }
        }
        if (c + 1 < c_end) load_chunk(c + 1, raw_nxt, x_nxt);
        const uint32_t k0 = c * kUK;
        // A: weights, 32 elements per thread
        {
            float w[32];
            const uint32_t first = k0 + a_half * 32;
            if (a_live && first < m.cols) {
                decode_raw32(m, raw_cur, wptr, first, w);
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
        // B: activations, 16 elements per thread
        {
            float v[16];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[4 * i] = x_cur[i].x; v[4 * i + 1] = x_cur[i].y;
                v[4 * i + 2] = x_cur[i].z; v[4 * i + 3] = x_cur[i].w;
            }
#pragma unroll
            for (int j = 0; j < 2; ++j) {
                uint4 hi, lo;
                pack8(v + 8 * j, hi, lo);
                const uint32_t off = sw128_off(b_row, b_quarter * 2 + j);
                *reinterpret_cast<uint4 *>(B_hi + off) = hi;
                *reinterpret_cast<uint4 *>(B_lo + off) = lo;
            }
        }
        raw_cur = raw_nxt;
#pragma unroll
        for (int i = 0; i < 4; ++i) x_cur[i] = x_nxt[i];
        // make the generic-proxy stores visible to the tensor core (async proxy)
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t ah = smem_u32(A_hi), al = smem_u32(A_lo);
            const uint32_t bh = smem_u32(B_hi), bl = smem_u32(B_lo);
#pragma unroll
            for (int kk = 0; kk < kUK / 16; ++kk) {
                const uint32_t koff = kk * 32;   // 16 bf16 = 32 bytes along K
                const uint64_t dah = sw128_desc(ah + koff), dal = sw128_desc(al + koff);
                const uint64_t dbh = sw128_desc(bh + koff), dbl = sw128_desc(bl + koff);
                umma_bf16(tmem, dah, dbh, (it > 0 || kk > 0) ? 1u : 0u);
                umma_bf16(tmem, dah, dbl, 1u);
                umma_bf16(tmem, dal, dbh, 1u);
            }
            umma_commit(&bars[stage]);
        }
        ++issued;
    }
    // all issued MMAs complete (the last commit covers every earlier MMA)
    if (ok && issued > 0) {
        const uint32_t last = issued - 1;
        if (!mbar_wait(&bars[last % kStages], (last / kStages) & 1u)) ok = false;
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const bool all_ok = __syncthreads_and(ok);

    if (all_ok && issued > 0) {
        // epilogue: warp w reads TMEM lanes 32*(w%4).. and columns (w/4)*32..
        const uint32_t lane_base = 32u * (warp & 3);
        const uint32_t col_base = (uint32_t)(warp >> 2) * 32u;
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
        const uint32_t row = row0 + lane_base + lane;
        if (row < m.rows) {
            float *dst = partial ? partial + (size_t)blockIdx.z * batch * ldy : y;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const uint32_t b = b0 + col_base + j;
                if (b < batch) dst[(size_t)b * ldy + segs.out_offset[seg] + row] = __uint_as_float(r[j]);
            }
        }
    }
    if (all_ok && issued == 0 && partial != nullptr) {
        // an empty split still owns its slice of the partial buffer
        const uint32_t row = row0 + 32u * (warp & 3) + lane;
        const uint32_t col_base = (uint32_t)(warp >> 2) * 32u;
        if (row < m.rows)
            for (int j = 0; j < 32; ++j) {
                const uint32_t b = b0 + col_base + j;
                if (b < batch)
                    partial[(size_t)blockIdx.z * batch * ldy + (size_t)b * ldy + segs.out_offset[seg] + row] = 0.0f;
            }
    }
    if (!all_ok && tid == 0) {
        atomicCAS(err.word, 0ull, ((unsigned long long)kErrTimeout << 32) | err.call_id);
        // bounded wait for MMAs still in flight before TMEM is released
        for (uint32_t s = 0; s < kStages; ++s) (void)mbar_wait(&bars[s], 0), (void)mbar_wait(&bars[s], 1);
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

bool launch_projection_umma(const ProjSegments &in, const float *x, uint32_t ldx, float *y, uint32_t ldy,
                            uint32_t batch, float *partial, size_t partial_floats, ErrorWord err,
                            cudaStream_t stream) {
    ProjSegments segs = in;
    uint32_t acc = 0, cols = 0, col_lo = UINT32_MAX, col_hi = 0;
    for (int i = 0; i < segs.count; ++i) {
        segs.tile_start[i] = acc;
        acc += (segs.m[i].rows + kUM - 1) / kUM;
        cols = std::max(cols, segs.m[i].cols);
        col_lo = std::min(col_lo, segs.out_offset[i]);
        col_hi = std::max(col_hi, segs.out_offset[i] + segs.m[i].rows);
    }
    segs.tile_start[segs.count] = acc;
    const uint32_t btiles = (batch + kUN - 1) / kUN;
    const uint32_t nchunks = (cols + kUK - 1) / kUK;
    // split K until there are about two CTAs per SM (148 SMs), keeping at
    // least 8 chunks per split
    uint32_t splits = 1;
    while (splits < kProjPartialSplits && acc * btiles * splits < 2 * 148 && nchunks / (splits * 2) >= 4)
        splits *= 2;
    if (splits > 1 && (partial == nullptr || partial_floats < (size_t)splits * batch * ldy)) splits = 1;
    // the split-K reduce covers one contiguous column range
    uint32_t covered = 0;
    for (int i = 0; i < segs.count; ++i) covered += segs.m[i].rows;
    if (covered != col_hi - col_lo) splits = 1;
    cudaFuncSetAttribute(proj_umma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    const uint32_t per = (nchunks + splits - 1) / splits;
    dim3 grid(acc, btiles, splits);
    proj_umma_kernel<<<grid, 256, kSmemBytes, stream>>>(segs, x, ldx, y, ldy, batch,
                                                        splits > 1 ? partial : nullptr, per, err);
    count_launch();
    if (splits > 1) {
        const uint64_t n = (uint64_t)batch * (col_hi - col_lo);
        splitk_reduce_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(partial, splits, batch, ldy, y,
                                                                            col_lo, col_hi - col_lo);
        count_launch();
    }
    return true;
}

}  // namespace kqb
