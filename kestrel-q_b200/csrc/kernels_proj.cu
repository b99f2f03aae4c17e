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

constexpr int kExRows = 16;          // rows per CTA (4 per warp)
constexpr int kExBatch = 32;         // batch rows per CTA (one per lane)
constexpr int kExK = 128;            // columns per chunk

__global__ void __launch_bounds__(128)
proj_exact_kernel(ProjSegments segs, const float *__restrict__ x, uint32_t ldx,
                  float *__restrict__ y, uint32_t ldy, uint32_t batch,
                  ErrorWord err) {
    __shared__ __align__(16) float ws[kExRows][kExK];
    __shared__ float xs[kExK][kExBatch + 1];
    if (error_raised(err)) return;
    int seg = 0;
    while (seg + 1 < segs.count && blockIdx.x >= segs.tile_start[seg + 1]) ++seg;
    const QMatrix m = segs.m[seg];
    const uint32_t row0 = (blockIdx.x - segs.tile_start[seg]) * kExRows;
    const uint32_t b0 = blockIdx.y * kExBatch;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (uint32_t k0 = 0; k0 < m.cols; k0 += kExK) {
        const uint32_t kc = min((uint32_t)kExK, m.cols - k0);
        // decode: thread t owns row t/8, 16-element run (t%8)*16 of the chunk
        {
            const int r = threadIdx.x >> 3, run = (threadIdx.x & 7) * 16;
            const uint32_t grow = row0 + r;
            float w[16];
            uint32_t cnt = 0;
            if ((uint32_t)run < kc) cnt = min(16u, kc - run);
            if (grow < m.rows && cnt > 0)
                decode_any(m, m.data + (size_t)grow * m.row_bytes, k0 + run, cnt, w);
            for (int i = 0; i < 16; ++i) ws[r][run + i] = (grow < m.rows && (uint32_t)i < cnt) ? w[i] : 0.0f;
        }
        // activations, transposed: xs[k][b]
        for (int idx = threadIdx.x; idx < kExBatch * kExK; idx += blockDim.x) {
            const int bb = idx / kExK, kk = idx % kExK;
            const uint32_t gb = b0 + bb;
            xs[kk][bb] = (gb < batch && (uint32_t)kk < kc) ? x[(size_t)gb * ldx + k0 + kk] : 0.0f;
        }
        __syncthreads();
        const float *w0 = ws[warp * 4 + 0], *w1 = ws[warp * 4 + 1];
        const float *w2 = ws[warp * 4 + 2], *w3 = ws[warp * 4 + 3];
        for (uint32_t k = 0; k < kc; ++k) {
            const float xv = xs[k][lane];
            acc[0] = __fadd_rn(acc[0], __fmul_rn(w0[k], xv));
            acc[1] = __fadd_rn(acc[1], __fmul_rn(w1[k], xv));
            acc[2] = __fadd_rn(acc[2], __fmul_rn(w2[k], xv));
            acc[3] = __fadd_rn(acc[3], __fmul_rn(w3[k], xv));
        }
        __syncthreads();
    }
    const uint32_t b = b0 + lane;
    if (b >= batch) return;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t row = row0 + warp * 4 + i;
        if (row < m.rows) y[(size_t)b * ldy + segs.out_offset[seg] + row] = acc[i];
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

void launch_projection(const ProjSegments &in, const float *x, uint32_t ldx,
                       float *y, uint32_t ldy, uint32_t batch, ErrorWord err,
                       cudaStream_t stream, float *partial, size_t partial_floats) {
    ProjSegments segs = in;
    KernelTimer timer("proj", stream);
    if (batch > 8 && !force_simt_projection() && partial != nullptr &&
        launch_projection_umma(segs, x, ldx, y, ldy, batch, reinterpret_cast<uint8_t *>(partial),
                               partial_floats * 4, err, stream))
        return;
    if (batch <= 8) {
        fill_tile_starts(segs, 1);
        uint32_t rows = segs.tile_start[segs.count];
        dim3 grid((rows + 7) / 8);
        if (batch <= 1)
            proj_warp_kernel<1><<<grid, 256, 0, stream>>>(segs, x, ldx, y, ldy, batch, err);
        else if (batch <= 4)
            proj_warp_kernel<4><<<grid, 256, 0, stream>>>(segs, x, ldx, y, ldy, batch, err);
        else
            proj_warp_kernel<8><<<grid, 256, 0, stream>>>(segs, x, ldx, y, ldy, batch, err);
    } else {
        fill_tile_starts(segs, kTileR);
        dim3 grid(segs.tile_start[segs.count], (batch + kTileB - 1) / kTileB);
        proj_tiled_kernel<<<grid, 256, 0, stream>>>(segs, x, ldx, y, ldy, batch, err);
    }
    count_launch();
}

void launch_projection_exact(const ProjSegments &in, const float *x,
                             uint32_t ldx, float *y, uint32_t ldy,
                             uint32_t batch, ErrorWord err,
                             cudaStream_t stream) {
    ProjSegments segs = in;
    KernelTimer timer("proj_exact", stream);
    fill_tile_starts(segs, kExRows);
    dim3 grid(segs.tile_start[segs.count], (batch + kExBatch - 1) / kExBatch);
    proj_exact_kernel<<<grid, 128, 0, stream>>>(segs, x, ldx, y, ldy, batch, err);
    count_launch();
}

// ------------------------------------------------------------ validation

__global__ void dequantize_kernel(uint32_t type, const uint8_t *packed,
                                  uint64_t elements, float *out) {
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
    dequantize_kernel<<<(unsigned)((runs + 255) / 256), 256, 0, stream>>>(type, packed, elements, out);
    count_launch();
}

__global__ void row_dot_kernel(uint32_t type, const uint8_t *packed,
                               uint64_t elements, const float *x, float *out,
                               int *status) {
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
    row_dot_kernel<<<1, 1, 0, stream>>>(type, packed, elements, x, out, status);
    count_launch();
}

__global__ void check_finite_kernel(const float *x, uint64_t count, ErrorWord err) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (; i < count; i += stride) bad |= !isfinite(x[i]);
    if (__syncthreads_or(bad) && threadIdx.x == 0) raise_error(err, kErrNonFinite);
}

void launch_check_finite(const float *x, uint64_t count, ErrorWord err,
                         cudaStream_t stream) {
    uint64_t blocks = std::min<uint64_t>((count + 255) / 256, 1184);
    if (blocks == 0) blocks = 1;
    check_finite_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, count, err);
    count_launch();
}

__global__ void mask_rows_kernel(const float *x, const uint8_t *mask, uint32_t rows,
                                 uint32_t cols, float *y) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)rows * cols) return;
    y[i] = x[i] * (float)mask[i / cols];
}

void launch_mask_rows(const float *x, const uint8_t *mask, uint32_t rows,
                      uint32_t cols, float *y, cudaStream_t stream) {
    uint64_t n = (uint64_t)rows * cols;
    mask_rows_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(x, mask, rows, cols, y);
    count_launch();
}

}  // namespace kqb
