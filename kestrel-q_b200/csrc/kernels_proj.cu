// Dequant-fused projections: y = W x for GGUF-quantized W held in HBM.
//
// Replaces the row loop of kq_weight_provider_linear_f32
// (src/kq_weight_provider.c:464-475 of Kestrel-Q), which calls
// kq_quantized_row_dot_f32 (src/kq_numeric.c:420-503) once per row.
// Weights are decoded in registers (quant.cuh) and never written back to HBM.
#include "kernels.hpp"
#include "quant.cuh"

#include <algorithm>
#include <atomic>
#include <cstdlib>

namespace kqb {

namespace {
std::atomic<uint64_t> g_launches{0};
}

uint64_t launches_total() { return g_launches.load(); }

// KQ_B200_SIMT_PROJECTION=1 selects the CUDA-core tiled GEMM for batches
// above 8 (used by the tests to cross-check the tensor-core path).
bool force_simt_projection() {
    static int v = -1;
    if (v < 0) {
        const char *e = getenv("KQ_B200_SIMT_PROJECTION");
        v = (e != nullptr && e[0] == '1') ? 1 : 0;
    }
    return v == 1;
}
void count_launch() { g_launches.fetch_add(1); }

__device__ __forceinline__ bool error_raised(const ErrorWord &e) {
    return *reinterpret_cast<volatile unsigned long long *>(e.word) != 0ull;
}

__device__ __forceinline__ void raise_error(const ErrorWord &e, uint32_t code) {
    unsigned long long v = ((unsigned long long)code << 32) | e.call_id;
    atomicCAS(e.word, 0ull, v);
}

// ------------------------------------------------------------ tiled GEMM
//
// Tile: 64 output rows x 64 batch rows, K consumed 64 at a time.  Each of the
// 256 threads owns a 4 x 4 register tile.  The weight tile is dequantised by
// all threads into shared memory (k-major), the activation tile is staged
// transposed; both then feed 16 FMAs per pair of 128-bit shared loads.

constexpr int kTileR = 64;
constexpr int kTileB = 64;
constexpr int kTileK = 64;
constexpr int kLd = kTileR + 4;   // padded leading dimension (floats)

__global__ void __launch_bounds__(256)
proj_tiled_kernel(ProjSegments segs, const float *__restrict__ x, uint32_t ldx,
                  float *__restrict__ y, uint32_t ldy, uint32_t batch,
                  ErrorWord err) {
    pdl_wait();
    __shared__ __align__(16) float ws[kTileK][kLd];
    __shared__ __align__(16) float xs[kTileK][kLd];
    if (error_raised(err)) return;

    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kTileR;
    const uint32_t b0 = blockIdx.y * kTileB;
    const int t = threadIdx.x;
    const int tr = t & 15, tb = t >> 4;
    float acc[4][4] = {};

    // loader roles
    const int lr = t & 63;            // weight row within the tile
    const int lrun = (t >> 6) * 16;   // 16-element run within the K chunk
    const uint32_t wrow = row0 + lr;
    const uint8_t *wptr = m.data + (size_t)min(wrow, m.rows - 1) * m.row_bytes;

    for (uint32_t k0 = 0; k0 < m.cols; k0 += kTileK) {
        // weights: 64 rows x 64 k, dequantised into ws[k][r]
        {
            float vals[16];
            uint32_t first = k0 + lrun;
            uint32_t count = 0;
            if (first < m.cols) count = min(16u, m.cols - first);
            if (wrow < m.rows && count > 0) {
                decode_any(m, wptr, first, count, vals);
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                ws[lrun + i][lr] = (wrow < m.rows && (uint32_t)i < count) ? vals[i] : 0.0f;
            }
        }
        // activations: 64 batch x 64 k, transposed into xs[k][b]
        for (int idx = t; idx < kTileB * kTileK; idx += 256) {
            int bb = idx / kTileK, kk = idx % kTileK;
            uint32_t gb = b0 + bb, gk = k0 + kk;
            xs[kk][bb] = (gb < batch && gk < m.cols) ? x[(size_t)gb * ldx + gk] : 0.0f;
        }
        __syncthreads();
#pragma unroll 8
        for (int kk = 0; kk < kTileK; ++kk) {
            float4 w4 = *reinterpret_cast<const float4 *>(&ws[kk][tr * 4]);
            float4 x4 = *reinterpret_cast<const float4 *>(&xs[kk][tb * 4]);
            float wv[4] = {w4.x, w4.y, w4.z, w4.w};
            float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(wv[i], xv[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint32_t r = row0 + tr * 4 + i;
        if (r >= m.rows) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t b = b0 + tb * 4 + j;
            if (b < batch) y[(size_t)b * ldy + segs.out_offset[seg] + r] = acc[i][j];
        }
    }
}

// ------------------------------------------------------------ warp GEMV
//
// Small batches (<= 8): one warp per row; lane l decodes 32-element runs
// l*32 + j*1024 of the row and keeps one partial sum per batch row, reduced
// with warp shuffles at the end.

template <int BMAX>
__global__ void __launch_bounds__(256)
proj_warp_kernel(ProjSegments segs, const float *__restrict__ x, uint32_t ldx,
                 float *__restrict__ y, uint32_t ldy, uint32_t batch,
                 ErrorWord err) {
    pdl_wait();
    if (error_raised(err)) return;
    const int lane = threadIdx.x & 31;
    const uint32_t warp_global = blockIdx.x * 8 + (threadIdx.x >> 5);
    // segment lookup in units of rows (tile_start holds row starts here)
    int seg = 0;
    while (seg + 1 < segs.count && warp_global >= segs.tile_start[seg + 1]) ++seg;
    if (warp_global >= segs.tile_start[segs.count]) return;
    const QMatrix m = segs.m[seg];
    const uint32_t row = warp_global - segs.tile_start[seg];
    const uint8_t *wptr = m.data + (size_t)row * m.row_bytes;
    float acc[BMAX];
#pragma unroll
    for (int b = 0; b < BMAX; ++b) acc[b] = 0.0f;
    for (uint32_t base = (uint32_t)lane * 32u; base < m.cols; base += 1024u) {
        float w[32];
        uint32_t count = min(32u, m.cols - base);
        decode_any(m, wptr, base, count, w);
        const bool vec_ok = count == 32u && (ldx & 3u) == 0u &&
                            (reinterpret_cast<uintptr_t>(x) & 15u) == 0u;
        if (vec_ok) {
#pragma unroll
            for (int b = 0; b < BMAX; ++b) {
                if ((uint32_t)b >= batch) break;
                const float4 *xp = reinterpret_cast<const float4 *>(x + (size_t)b * ldx + base);
                float s = acc[b];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    float4 xv = xp[i];
                    s = fmaf(w[4 * i + 0], xv.x, s);
                    s = fmaf(w[4 * i + 1], xv.y, s);
                    s = fmaf(w[4 * i + 2], xv.z, s);
                    s = fmaf(w[4 * i + 3], xv.w, s);
                }
                acc[b] = s;
            }
        } else {
            for (int b = 0; b < BMAX; ++b) {
                if ((uint32_t)b >= batch) break;
                const float *xp = x + (size_t)b * ldx + base;
                for (uint32_t i = 0; i < count; ++i) acc[b] = fmaf(w[i], xp[i], acc[b]);
            }
        }
    }
#pragma unroll
    for (int b = 0; b < BMAX; ++b) {
        float s = acc[b];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0 && (uint32_t)b < batch) y[(size_t)b * ldy + segs.out_offset[seg] + row] = s;
    }
}

// ------------------------------------------------------------ exact GEMV
//
// Every output is accumulated k = 0..K-1 from 0.0f as acc = acc + w*x with
// both operations rounded separately: the reference's kq_f32_dot order
// (src/kq_numeric.c:616-619).  Used for the QSA indexer projections so that
// block selection is bit-identical to the reference.
//
// Layout: a CTA owns 16 rows x 32 batch rows; lane = batch row, so the
// sequential chain of each output lives in one lane and a warp keeps four
// independent chains (four rows) in flight.  Per 128-column chunk the
// weights are decoded once into shared memory (read back as broadcasts) and
// the activations are staged transposed (one conflict-free load per lane).

// Exact projection: every output is the reference's sequential F32 row dot,
// acc = acc + w[k]*x[k] for k = 0..cols-1 with separately rounded products and
// sums (src/kq_numeric.c:420-503), so results are bit-identical.  The chain is
// inherently serial; throughput comes from running many chains at once and
// from keeping their operands in flight.  A CTA owns 8 weight rows x 64 batch
// rows (512 chains); each thread two chains (a row pair, one batch row), so
// two independent add chains hide the add latency.  K chunks of 128 are staged
// in shared memory by cp.async four chunks deep (raw F32 or BF16 weight bytes,
// F32 activations) and read as 16-byte vectors, four chain steps per load.
// Other weight types are decoded into the stage synchronously (slow path).
constexpr int kExK = 128;             // K per staged chunk
constexpr int kExXStride = kExK + 4;  // padded activation row (conflict-free float4 reads)

// Tile of TR weight rows x BB batch rows.  TR = 4 (decode batches): a
// thread owns 1 row x 1 batch row; BB = 16 makes four times the CTAs of a
// 64-row batch span, small enough that all of a decode launch's CTAs are
// resident at once, about evenly over the SMs.  TR = 8: 2 rows x 1 batch
// row; TR = 32 (large batches): 4 rows x 2 batch rows, eight independent
// sequential chains per thread, each weight value read from shared memory
// feeding two of them.
template <int TR, int BB = 64> struct ExTile {
    static constexpr int stages = TR == 8 ? 4 : 3;
    static constexpr int rpt = TR == 4 ? 1 : TR == 8 ? 2 : 4;    // rows per thread
    static constexpr int bpt = TR == 32 ? 2 : 1;                  // batch rows per thread
    static constexpr int batch = BB;
    static constexpr int threads = TR / rpt * (BB / bpt);
    static constexpr size_t xbytes = (size_t)BB * kExXStride * 4;   // per stage
    static constexpr size_t wbytes = (size_t)TR * kExK * 4;         // per stage (F32 room)
    static constexpr size_t smem = stages * (xbytes + wbytes);
    static_assert(TR != 32 || (BB == 64 && threads == 256), "the 32-row tile spans 64 batch rows");
};


__device__ __forceinline__ void cp_async16(void *smem, const void *gmem) {
    const uint32_t a = (uint32_t)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(a), "l"(gmem) : "memory");
}

// MODE 0: F32 weights, 1: BF16 weights (both staged raw by cp.async);
// 2: any type, decoded into F32 by the staging threads.  Every output is one
// sequential F32 chain over K in the reference's order (products and sums
// rounded separately).
template <int MODE, int TR, int BB>
__global__ void __launch_bounds__(ExTile<TR, BB>::threads)
proj_exact_kernel(ProjSegments segs, const float *__restrict__ x, uint32_t ldx,
                  float *__restrict__ y, uint32_t ldy, uint32_t batch,
                  ErrorWord err) {
    using TT = ExTile<TR, BB>;
    constexpr int kStages = TT::stages, RPT = TT::rpt, BPT = TT::bpt, kThreads = TT::threads;
    constexpr size_t kExXBytes = TT::xbytes;
    pdl_wait();
    extern __shared__ __align__(16) uint8_t ex_smem[];
    if (error_raised(err)) return;
    float *xs_base = reinterpret_cast<float *>(ex_smem);
    uint8_t *ws_base = ex_smem + kStages * kExXBytes;
    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * TR;
    const uint32_t b0 = blockIdx.y * BB;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // the thread's rows rb .. rb + RPT - 1 (weight reads broadcast to the
    // threads of a row) and batch rows bb + 32 j
    const int rb = TR == 32 ? 4 * warp : RPT * (tid / BB);
    const int bb = TR == 32 ? lane : tid % BB;
    const uint32_t nchunks = (m.cols + kExK - 1) / kExK;
    const bool xvec = (ldx % 4u) == 0u && (reinterpret_cast<uintptr_t>(x) & 15u) == 0u;
    constexpr uint32_t kElem = MODE == 1 ? 2u : 4u;   // staged weight bytes per value

    auto stage = [&](uint32_t c) {
        const int buf = c % kStages;
        const uint32_t k0 = c * kExK;
        float *xs = xs_base + (size_t)buf * BB * kExXStride;
        uint8_t *ws = ws_base + (size_t)buf * TT::wbytes;
        // weights: TR rows x 128 values
        if constexpr (MODE == 2) {
            for (int i = tid; i < TR * (kExK / 4); i += kThreads) {
                const int r = i / (kExK / 4), kk = (i % (kExK / 4)) * 4;
                const uint32_t grow = row0 + r;
                float w[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (grow < m.rows && k0 + kk < m.cols)
                    decode_any(m, m.data + (size_t)grow * m.row_bytes, k0 + kk, min(4u, m.cols - (k0 + kk)), w);
                for (int e = 0; e < 4; ++e)
                    reinterpret_cast<float *>(ws)[r * kExK + kk + e] = (k0 + kk + e < m.cols) ? w[e] : 0.0f;
            }
        } else {
            constexpr int kPieces = kExK * kElem / 16;   // 16-byte pieces per row
            for (int i = tid; i < TR * kPieces; i += kThreads) {
                const int r = i / kPieces, pc = i % kPieces;
                const uint32_t grow = row0 + r, k = k0 + pc * (16 / kElem);
                uint8_t *dst = ws + (size_t)r * kExK * kElem + pc * 16;
                if (grow < m.rows && k + 16 / kElem <= m.cols) {
                    cp_async16(dst, m.data + (size_t)grow * m.row_bytes + (size_t)k * kElem);
                } else {
                    for (uint32_t e = 0; e < 16 / kElem; ++e) {
                        const bool in = grow < m.rows && k + e < m.cols;
                        if constexpr (MODE == 1) {
                            reinterpret_cast<uint16_t *>(dst)[e] =
                                in ? reinterpret_cast<const uint16_t *>(m.data + (size_t)grow * m.row_bytes)[k + e] : 0;
                        } else {
                            reinterpret_cast<float *>(dst)[e] =
                                in ? reinterpret_cast<const float *>(m.data + (size_t)grow * m.row_bytes)[k + e] : 0.0f;
                        }
                    }
                }
            }
        }
        // activations: 64 rows x 128 values
        for (int i = tid; i < BB * (kExK / 4); i += kThreads) {
            const int br = i / (kExK / 4), q4 = (i % (kExK / 4)) * 4;
            const uint32_t gb = b0 + br, k = k0 + q4;
            float *dst = xs + (size_t)br * kExXStride + q4;
            if (xvec && gb < batch && k + 4 <= m.cols) {
                cp_async16(dst, x + (size_t)gb * ldx + k);
            } else {
                for (int e = 0; e < 4; ++e)
                    dst[e] = (gb < batch && k + e < m.cols) ? x[(size_t)gb * ldx + k + e] : 0.0f;
            }
        }
    };
    auto commit = [] { asm volatile("cp.async.commit_group;" ::: "memory"); };

    float acc[RPT][BPT];
#pragma unroll
    for (int r = 0; r < RPT; ++r)
#pragma unroll
        for (int j = 0; j < BPT; ++j) acc[r][j] = 0.0f;
    for (uint32_t c = 0; c < (uint32_t)kStages - 1; ++c) {
        if (c < nchunks) stage(c);
        commit();
    }
    for (uint32_t c = 0; c < nchunks; ++c) {
        if (c + kStages - 1 < nchunks) stage(c + kStages - 1);
        commit();
        asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
        __syncthreads();
        const int buf = c % kStages;
        const uint32_t kc = min((uint32_t)kExK, m.cols - c * kExK);
        const float *xv = xs_base + (size_t)buf * BB * kExXStride + (size_t)bb * kExXStride;
        const uint8_t *ws = ws_base + (size_t)buf * TT::wbytes + (size_t)rb * kExK * kElem;
        auto wq = [&](int r, int k) {   // 4 F32 weights of row rb + r at k
            const uint8_t *row = ws + (size_t)r * kExK * kElem;
            if constexpr (MODE == 1) {
                const uint2 u = *reinterpret_cast<const uint2 *>(row + (size_t)k * 2);
                return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                   __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
            } else {
                return *reinterpret_cast<const float4 *>(row + (size_t)k * 4);
            }
        };
        if (kc == (uint32_t)kExK) {   // fully unrolled: every operand address is an immediate offset
#pragma unroll
            for (int k = 0; k < kExK; k += 4) {
                float xv4[BPT][4];
#pragma unroll
                for (int j = 0; j < BPT; ++j) {
                    const float4 v = *reinterpret_cast<const float4 *>(xv + (size_t)j * 32 * kExXStride + k);
                    xv4[j][0] = v.x; xv4[j][1] = v.y; xv4[j][2] = v.z; xv4[j][3] = v.w;
                }
#pragma unroll
                for (int r = 0; r < RPT; ++r) {
                    const float4 a = wq(r, k);
                    const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                    for (int e = 0; e < 4; ++e)
#pragma unroll
                        for (int j = 0; j < BPT; ++j) acc[r][j] = __fadd_rn(acc[r][j], __fmul_rn(av[e], xv4[j][e]));
                }
            }
        } else {
            for (uint32_t k = 0; k < kc; k += 4) {
                for (uint32_t e = 0; e < 4 && k + e < kc; ++e) {
#pragma unroll
                    for (int r = 0; r < RPT; ++r) {
                        const float4 a = wq(r, (int)k);
                        const float av[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
                        for (int j = 0; j < BPT; ++j)
                            acc[r][j] = __fadd_rn(acc[r][j],
                                                  __fmul_rn(av[e], xv[(size_t)j * 32 * kExXStride + k + e]));
                    }
                }
            }
        }
        __syncthreads();
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
    for (int j = 0; j < BPT; ++j) {
        const uint32_t b = b0 + bb + 32 * j;
        if (b >= batch) continue;
#pragma unroll
        for (int r = 0; r < RPT; ++r) {
            const uint32_t row = row0 + rb + r;
            if (row < m.rows) y[(size_t)b * ldy + segs.out_offset[seg] + row] = acc[r][j];
        }
    }
}

static void fill_tile_starts(ProjSegments &s, uint32_t unit) {
    uint32_t acc = 0;
    for (int i = 0; i < s.count; ++i) {
        s.tile_start[i] = acc;
        acc += (s.m[i].rows + unit - 1) / unit;
    }
    s.tile_start[s.count] = acc;
}

size_t projection_workspace_floats(uint32_t batch, uint32_t /*ldy*/, uint32_t cols) {
    if (batch <= 8) return 0;
    return ((umma_xtile_bytes(batch, cols) + 255) & ~size_t(255)) / 4;
}

bool launch_projection(const ProjSegments &in, const float *x, uint32_t ldx,
                       float *y, uint32_t ldy, uint32_t batch, ErrorWord err,
                       cudaStream_t stream, float *partial, size_t partial_floats) {
    ProjSegments segs = in;
    KernelTimer timer("proj", stream);
    if (batch > 8 && !force_simt_projection() && partial != nullptr &&
        launch_projection_umma(segs, x, ldx, y, ldy, batch, reinterpret_cast<uint8_t *>(partial),
                               partial_floats * 4, err, stream))
        return true;
    if (batch <= 8) {
        fill_tile_starts(segs, 1);
        uint32_t rows = segs.tile_start[segs.count];
        dim3 grid((rows + 7) / 8);
        if (batch <= 1)
            launch_pdl(proj_warp_kernel<1>, grid, 256, 0, stream, segs, x, ldx, y, ldy, batch, err);
        else if (batch <= 4)
            launch_pdl(proj_warp_kernel<4>, grid, 256, 0, stream, segs, x, ldx, y, ldy, batch, err);
        else
            launch_pdl(proj_warp_kernel<8>, grid, 256, 0, stream, segs, x, ldx, y, ldy, batch, err);
    } else {
        fill_tile_starts(segs, kTileR);
        dim3 grid(segs.tile_start[segs.count], (batch + kTileB - 1) / kTileB);
        launch_pdl(proj_tiled_kernel, grid, 256, 0, stream, segs, x, ldx, y, ldy, batch, err);
    }
    count_launch();
    return false;
}

template <int TR, int BB>
static void launch_exact_tiles(const ProjSegments &in, const float *x, uint32_t ldx, float *y, uint32_t ldy,
                               uint32_t batch, ErrorWord err, cudaStream_t stream) {
    using TT = ExTile<TR, BB>;
    ProjSegments segs = in;
    fill_tile_starts(segs, TR);
    dim3 grid(segs.tile_start[segs.count], (batch + BB - 1) / BB);
    // one launch per mode; segments of mixed types go through the generic mode
    int mode = 0;
    for (int i = 0; i < segs.count; ++i) {
        const QMatrix &q = segs.m[i];
        const bool aligned = (q.row_bytes % 16u) == 0u && (reinterpret_cast<uintptr_t>(q.data) & 15u) == 0u;
        const int mi = !aligned ? 2 : q.type == kTypeF32 ? 0 : q.type == kTypeBF16 ? 1 : 2;
        mode = i == 0 ? mi : (mode == mi ? mode : 2);
    }
    constexpr size_t smem = TT::smem;
    static DeviceOnce attr;
    attr.run([] {
        cudaFuncSetAttribute(proj_exact_kernel<0, TR, BB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(proj_exact_kernel<1, TR, BB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        cudaFuncSetAttribute(proj_exact_kernel<2, TR, BB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    });
    if (mode == 0)
        launch_pdl(proj_exact_kernel<0, TR, BB>, grid, TT::threads, smem, stream, segs, x, ldx, y, ldy, batch, err);
    else if (mode == 1)
        launch_pdl(proj_exact_kernel<1, TR, BB>, grid, TT::threads, smem, stream, segs, x, ldx, y, ldy, batch, err);
    else
        launch_pdl(proj_exact_kernel<2, TR, BB>, grid, TT::threads, smem, stream, segs, x, ldx, y, ldy, batch, err);
}

void launch_projection_exact(const ProjSegments &in, const float *x,
                             uint32_t ldx, float *y, uint32_t ldy,
                             uint32_t batch, ErrorWord err,
                             cudaStream_t stream) {
    KernelTimer timer("proj_exact", stream);
    // 32-row tiles once the batch alone gives several CTAs per SM; 4-row x
    // 16-batch-row tiles for decode batches (up to 64), so that the rows
    // and batch spans together fill the SMs evenly
    if (batch >= 1024)
        launch_exact_tiles<32, 64>(in, x, ldx, y, ldy, batch, err, stream);
    else if (batch <= 64u)
        launch_exact_tiles<4, 16>(in, x, ldx, y, ldy, batch, err, stream);
    else
        launch_exact_tiles<8, 64>(in, x, ldx, y, ldy, batch, err, stream);
    count_launch();
}

// ------------------------------------------------------------ validation

__global__ void dequantize_kernel(uint32_t type, const uint8_t *packed,
                                  uint64_t elements, float *out) {
    pdl_wait();
    uint64_t run = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t first = run * 32u;
    if (first >= elements) return;
    uint32_t count = (uint32_t)min((uint64_t)32u, elements - first);
    float w[32];
    // decode_run indexes blocks from `first`; offsets fit 32 bits per call
    // by rebasing on the super-block / block that contains `first`.
    uint32_t be, bb;
    block_geometry(type, be, bb);
    uint64_t block = first / be;
    const uint8_t *base = packed + block * bb;
    decode_run(type, base, (uint32_t)(first - block * be), count, w);
    for (uint32_t i = 0; i < count; ++i) out[first + i] = w[i];
}

void launch_dequantize(uint32_t type, const uint8_t *packed, uint64_t elements,
                       float *out, cudaStream_t stream) {
    uint64_t runs = (elements + 31) / 32;
    launch_pdl(dequantize_kernel, (unsigned)((runs + 255) / 256), 256, 0, stream, type, packed, elements, out);
    count_launch();
}

__global__ void row_dot_kernel(uint32_t type, const uint8_t *packed,
                               uint64_t elements, const float *x, float *out,
                               int *status) {
    pdl_wait();
    uint32_t be, bb;
    block_geometry(type, be, bb);
    float acc = 0.0f;
    bool finite = true;
    for (uint64_t first = 0; first < elements; first += 32u) {
        float w[32];
        uint32_t count = (uint32_t)min((uint64_t)32u, elements - first);
        uint64_t block = first / be;
        decode_run(type, packed + block * bb, (uint32_t)(first - block * be), count, w);
        for (uint32_t i = 0; i < count; ++i) {
            float xv = x[first + i];
            if (!isfinite(xv)) finite = false;
            acc = __fadd_rn(acc, __fmul_rn(w[i], xv));
        }
    }
    *out = acc;
    *status = (!finite) ? 1 : (isfinite(acc) ? 0 : 2);
}

void launch_row_dot(uint32_t type, const uint8_t *packed, uint64_t elements,
                    const float *x, float *out, int *status,
                    cudaStream_t stream) {
    launch_pdl(row_dot_kernel, 1, 1, 0, stream, type, packed, elements, x, out, status);
    count_launch();
}

__global__ void check_finite_kernel(const float *x, uint64_t count, ErrorWord err) {
    pdl_wait();
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (; i < count; i += stride) bad |= !isfinite(x[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0) raise_error(err, kErrNonFinite);
}

__global__ void permute_column_heads_kernel(const float *__restrict__ x, uint32_t batch, uint32_t cols,
                                            uint32_t width, const int32_t *__restrict__ heads, uint32_t nheads,
                                            float *__restrict__ y) {
    pdl_wait();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)batch * nheads * width) return;
    const uint64_t b = i / ((uint64_t)nheads * width);
    const uint32_t h = (uint32_t)(i / width % nheads), f = (uint32_t)(i % width);
    y[b * cols + (uint64_t)heads[h] * width + f] = x[b * cols + (uint64_t)h * width + f];
}

void launch_permute_column_heads(const float *x, uint32_t batch, uint32_t cols, uint32_t width,
                                 const int32_t *heads, uint32_t nheads, float *y, cudaStream_t stream) {
    const uint64_t n = (uint64_t)batch * nheads * width;
    launch_pdl(permute_column_heads_kernel, (unsigned)((n + 255) / 256), 256, 0, stream, x, batch, cols, width,
               heads, nheads, y);
    count_launch();
}

void launch_check_finite(const float *x, uint64_t count, ErrorWord err,
                         cudaStream_t stream) {
    uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 1184);
    if (blocks == 0) blocks = 1;
    launch_pdl(check_finite_kernel, (unsigned)blocks, 256, 0, stream, x, count, err);
    count_launch();
}

__global__ void mask_rows_kernel(const float *x, const uint8_t *mask, uint32_t rows,
                                 uint32_t cols, float *y) {
    pdl_wait();
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)rows * cols) return;
    y[i] = x[i] * (float)mask[i / cols];
}

void launch_mask_rows(const float *x, const uint8_t *mask, uint32_t rows,
                      uint32_t cols, float *y, cudaStream_t stream) {
    uint64_t n = (uint64_t)rows * cols;
    launch_pdl(mask_rows_kernel, (unsigned)((n + 255) / 256), 256, 0, stream, x, mask, rows, cols, y);
    count_launch();
}

}  // namespace kqb
