// Internal launch interface between the host ABI layer and the CUDA kernels.
#pragma once

#include <atomic>
#include <cstdint>
#include <mutex>

#include <cuda_runtime.h>

namespace kqb {

// Runs a set-up step (cudaFuncSetAttribute and the like) once per device.
// Function attributes belong to the current device's context, so a launcher
// used on several devices of one process must set them on each; the step
// has completed on a device before any caller on that device goes past run().
struct DeviceOnce {
    std::atomic<uint64_t> done{0};
    std::mutex mu;
    template <typename F>
    void run(F &&f) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
            f();
            return;
        }
        const uint64_t bit = 1ull << dev;
        if (done.load(std::memory_order_acquire) & bit) return;
        std::lock_guard<std::mutex> lk(mu);
        if (done.load(std::memory_order_relaxed) & bit) return;
        f();
        done.fetch_or(bit, std::memory_order_release);
    }
};

// Programmatic dependent launch: every kernel of the library is launched
// with launch_pdl (or the same attribute), which lets the GPU set it up while
// the previous kernel on the stream is still finishing, and every kernel
// calls pdl_wait() before it touches anything the previous kernel may write;
// pdl_wait() blocks until that kernel has completed and its writes are
// visible.  Only data no kernel writes (uploaded weights) is requested before
// the wait: the tensor-core projection issues its first weight loads there.
// (Triggering dependents early, right after the wait, and loading the GDN
// recurrent state before it were both measured slower on the decode step.)
template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kernel, static_cast<Args &&>(args)...);
}

#ifdef __CUDACC__
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
#endif

// Error word shared by every kernel of one device.  0 = no error; otherwise
// the id of the first failing call (see Runtime::next_call_id) in the low
// 32 bits and a kernel error code in the high 32 bits.
enum DeviceError : uint32_t {
    kErrNone = 0,
    kErrNonFinite = 1,   // non-finite input, state or result
    kErrDecay = 2,       // GDN log-decay not finite or positive
    kErrSelection = 3,   // QSA selected-token count invalid
    kErrTimeout = 4,     // a bounded wait gave up (wait site in bits 8..15)
    kErrRange = 5,       // an activation beyond the tensor-core projection's range (|x| >= 2^18)
};

// One quantized (or F32/BF16) matrix in HBM: `rows` consecutive GGUF rows.
//
// layout 0: the GGUF byte stream as given.  layout 1 ("planar"): each row's
// blocks are split into aligned planes with the same byte count, so that a
// 32-element run loads with 16-byte vector loads:
//   Q6_K: [ql nsb*128][qh nsb*64][scales nsb*16][d nsb*2]
//   Q8_0: [codes nb*32][d nb*2]
// and the row pitch `row_bytes` is rounded up to a multiple of 16 bytes.
// (Q4_K's 144-byte super-blocks are already 16-byte aligned and stay GGUF.)
// `scale_exp`: the tensor-core projection multiplies the decoded weights by
// 2^scale_exp (exact) before splitting them into fp16 hi/lo parts, so that
// every value of the matrix lies inside the fp16 range, and divides the
// result by it again (weight_scale_exponent() picks it at upload).
struct QMatrix {
    const uint8_t *data;
    uint32_t type;
    uint32_t rows;
    uint32_t cols;
    uint32_t row_bytes;
    uint32_t layout;
    int32_t scale_exp;
    // Q4_K only (may be null): per-super-block side data of the factored
    // tensor-core kernel, built at upload by q4k_build_aux.
    const uint8_t *aux = nullptr;
};

// Q4_K side data, per row and super-block sb (pitches padded to groups of 4
// super-blocks):
//   plane A  [rows][q4k_aux_pitch_a]  16 fp16 at byte 32*sb: dmin*m_s*2^e
//            rounded to fp16 (s = 0..7), then the 8 residuals (exact F32
//            minus the rounded value, rounded to fp16)
//   plane D  [rows][q4k_aux_pitch_d]  F32 d at byte 4*sb
// e = scale_exp.  Plane D follows plane A at offset rows * pitch_a.
uint32_t q4k_aux_pitch_a(uint32_t cols);
uint32_t q4k_aux_pitch_d(uint32_t cols);
size_t q4k_aux_bytes(uint32_t rows, uint32_t cols);
void q4k_build_aux(const uint8_t *packed, uint32_t rows, uint32_t cols, int32_t scale_exp, uint8_t *out);

// Power-of-two exponent e for a matrix whose decoded values are bounded by
// |w| <= bound: bound * 2^e < 2^14, clamped to [-64, 64] (0 for a zero or
// non-finite bound).
int32_t weight_scale_exponent(double bound);
// Upper bound of |decoded value| over `rows` GGUF rows of `type` blocks
// (read from the block headers: scales, minima, codes' ranges).
double weight_abs_bound(uint32_t type, const uint8_t *packed, uint64_t rows, uint64_t row_bytes);

constexpr int kMaxSegments = 6;

// Several matrices applied to the same input, outputs concatenated:
// y[b][offset_s + r] = sum_k W_s[r][k] * x[b][k].
struct ProjSegments {
    QMatrix m[kMaxSegments];
    uint32_t out_offset[kMaxSegments];
    uint32_t tile_start[kMaxSegments + 1];  // filled by the launcher
    int count;
};

struct ErrorWord {
    unsigned long long *word;   // device
    uint32_t call_id;
};

// ---- projections (kernels_proj.cu)
// `partial` (may be null) is work space of partial_floats floats; the
// tensor-core path runs when it holds projection_workspace_floats().  Returns
// true when the tensor-core path ran: it checks its input and its output for
// non-finite values on the device, so callers need no separate check.
bool launch_projection(const ProjSegments &segs, const float *x, uint32_t ldx,
                       float *y, uint32_t ldy, uint32_t batch, ErrorWord err,
                       cudaStream_t stream, float *partial = nullptr,
                       size_t partial_floats = 0);
// Tensor-core path (kernels_umma.cu), used for batches above 8.  Returns
// false (nothing launched) for shapes / types it does not cover (true: the
// input and output were checked for non-finite values).  `xtiles`
// is work space of umma_xtile_bytes(batch, cols, allow_wide) bytes.
// `cache_maps` false encodes the TMA descriptors on the stack instead of the
// host-side descriptor cache (no host allocation).  `allow_wide` false keeps
// the 64-row activation tile for every batch (smaller work space).
bool launch_projection_umma(const ProjSegments &segs, const float *x, uint32_t ldx,
                            float *y, uint32_t ldy, uint32_t batch, uint8_t *xtiles,
                            size_t xtile_bytes, ErrorWord err, cudaStream_t stream,
                            bool cache_maps = true, bool allow_wide = true);
size_t umma_xtile_bytes(uint32_t batch, uint32_t cols, bool allow_wide = true);
// True when the tensor-core path covers this matrix's type and layout.
bool umma_supported(const QMatrix &m);
// Work space (in floats) that launch_projection uses for `batch` rows of
// input with `cols` columns: the activation tiles of the tensor-core path.
size_t projection_workspace_floats(uint32_t batch, uint32_t ldy, uint32_t cols);
// Sequential-order product: each output is accumulated k = 0..K-1 from 0.0f
// with separately rounded products and sums, i.e. bit-identical to the
// reference's kq_f32_dot / kq_quantized_row_dot_f32.
void launch_projection_exact(const ProjSegments &segs, const float *x,
                             uint32_t ldx, float *y, uint32_t ldy,
                             uint32_t batch, ErrorWord err,
                             cudaStream_t stream);
void launch_dequantize(uint32_t type, const uint8_t *packed, uint64_t elements,
                       float *out, cudaStream_t stream);
void launch_row_dot(uint32_t type, const uint8_t *packed, uint64_t elements,
                    const float *x, float *out, int *status,
                    cudaStream_t stream);
void launch_check_finite(const float *x, uint64_t count, ErrorWord err,
                         cudaStream_t stream);
// y[b][heads[h] * width + f] = x[b][h * width + f] for the `nheads` heads of
// each of `batch` rows of `cols` values (canonical -> tiled column order).
void launch_permute_column_heads(const float *x, uint32_t batch, uint32_t cols, uint32_t width,
                                 const int32_t *heads, uint32_t nheads, float *y, cudaStream_t stream);
// y[t][i] = x[t][i] * (float)mask[t] (padding mask of src/kq_gdn_qwen38.c:548-553)
void launch_mask_rows(const float *x, const uint8_t *mask, uint32_t rows,
                      uint32_t cols, float *y, cudaStream_t stream);

// ---- GDN (kernels_gdn.cu)
constexpr int kMaxBatch = 64;

struct GdnDims {
    uint32_t hidden, key_heads, value_heads, key_dim, value_dim, kernel;
    uint32_t conv_channels, key_width, value_width, repeat;
    float eps;
};

struct GdnBatchPtrs {
    const float *conv_in[kMaxBatch];
    float *conv_out[kMaxBatch];
    const float *rec_in[kMaxBatch];
    float *rec_out[kMaxBatch];
};

struct GdnWeightsDev {
    const float *a_log, *conv, *dt_bias, *norm;
    // The output projection's column order, by value head: the gated output
    // of canonical head h is stored at head position gated_head[h] (a model
    // GGUF keeps GDN value heads in tiled order, so its out-projection reads
    // its input in that order); null: canonical order.
    const int32_t *gated_head = nullptr;
};

#ifdef __CUDACC__
// Head position of value head h in the gated output.
__device__ __forceinline__ uint32_t gated_head_pos(const GdnWeightsDev &w, uint32_t h) {
    return w.gated_head != nullptr ? (uint32_t)w.gated_head[h] : h;
}
#endif

// proj: [B*T][ldp] (qkv | gate | beta | alpha), item = b*T + t.
// `logdecay` (may be null) receives g as well as decay = exp(g).
void launch_gdn_conv_gates(const GdnDims &d, const GdnWeightsDev &w,
                           const GdnBatchPtrs &p, uint32_t batch,
                           uint32_t tokens, const float *proj, uint32_t ldp,
                           float *qk, float *v, float *beta, float *decay,
                           ErrorWord err, cudaStream_t stream, float *logdecay = nullptr);
void launch_gdn_recurrence(const GdnDims &d, const GdnWeightsDev &w,
                           const GdnBatchPtrs &p, uint32_t batch,
                           uint32_t tokens, const float *qk, const float *v,
                           const float *beta, const float *decay,
                           const float *proj, uint32_t ldp, float *gated,
                           ErrorWord err, cudaStream_t stream);

// Decode (one token per sequence) with the conv / gate stage fused into the
// recurrence, for dk = dv = 128 and conv kernel 4.
bool gdn_decode_fused_supported(const GdnDims &d);
void launch_gdn_decode_fused(const GdnDims &d, const GdnWeightsDev &w, const GdnBatchPtrs &p, uint32_t batch,
                             const float *proj, uint32_t ldp, float *gated, ErrorWord err, cudaStream_t stream);

// Checkpoint path (an observer is attached): one token of one sequence with
// every intermediate the reference's observer sees kept in device arrays.
// The recurrent and conv states go from *_in to *_out as in the other paths.
struct GdnDebugBufs {
    float *conv_out;              // [C]     SiLU(conv)
    float *conv_state;            // [C][K]  history after this token's shift
    float *q_raw, *k_raw;         // [Hv][dk] before the L2 norm (key heads repeated)
    float *v;                     // [Hv][dv]
    float *q_norm, *k_norm;       // [Hv][dk] normalised (q also scaled by 1/sqrt(dk))
    float *log_decay, *beta;      // [Hv]
    float *read, *delta, *core;   // [Hv][dv] recurrence read, delta and output
    float *gated;                 // [Hv][dv] gated RMSNorm output, canonical head order
    float *gated_proj;            // the same in the out-projection's head order (may equal gated)
};
void launch_gdn_debug_token(const GdnDims &d, const GdnWeightsDev &w, const float *conv_in, float *conv_out,
                            const float *rec_in, float *rec_out, const float *proj, const GdnDebugBufs &b,
                            ErrorWord err, cudaStream_t stream);

// Chunked (WY-form) prefill of one sequence (kernels_gdn_chunk.cu), for
// dk = dv = 128: same inputs as the recurrence plus the log decays; `work`
// holds gdn_chunk_workspace_floats(d, tokens) floats.
bool gdn_chunked_supported(const GdnDims &d);
size_t gdn_chunk_workspace_floats(const GdnDims &d, uint32_t tokens);
void launch_gdn_chunked(const GdnDims &d, const GdnWeightsDev &w, const GdnBatchPtrs &p, uint32_t tokens,
                        const float *qk, const float *v, const float *beta, const float *logdecay,
                        const float *proj, uint32_t ldp, float *gated, float *work, ErrorWord err,
                        cudaStream_t stream);

// ---- QSA (kernels_qsa.cu)
struct QsaDims {
    uint32_t hidden, q_heads, kv_heads, head_dim, index_heads, index_dim;
    uint32_t block, budget, topk, rotary, repeat, sel_capacity;
    float eps;
    float inv_sqrt_head;       // not used for exact paths
    float sqrt_index_dim;      // sqrtf((float)index_dim), host-computed
    float sqrt_head_dim;       // sqrtf((float)head_dim)
};

struct QsaSeq {
    float *key;          // [capacity][Hkv*d]
    float *value;        // [capacity][Hkv*d]
    float *raw;          // [capacity][di]
    float *block_keys;   // [di][capacity/block] feature-major
    uint32_t length;     // committed length before this token
    uint32_t capacity;
    // bf16 hi / lo copies of the key and value rows (v = hi + lo), written
    // beside the F32 rows, KV-head major: [Hkv][capacity][kQsaSplitRow]
    // uint16 with a row = [hi 256 | lo 256 | 8 unused]; null when the
    // tensor-core attention does not cover the geometry (head_dim != 256)
    uint16_t *key_split = nullptr;
    uint16_t *value_split = nullptr;
};

// uint16 elements per row of the split cache: 1040 bytes, so that rows
// copied back to back into shared memory start in 8 different bank groups
constexpr uint32_t kQsaSplitRow = 520;

// Entries of one launch: up to kMaxBatch independent sequences, or (uniform
// != 0) any number of consecutive tokens of one sequence: entry b is s[0]
// with length s[0].length + b (a prefill; every entry shares the cache).
struct QsaBatch {
    QsaSeq s[kMaxBatch];
    uint32_t uniform = 0;
};

__host__ __device__ inline QsaSeq batch_seq(const QsaBatch &bt, uint32_t b) {
    if (bt.uniform) {
        QsaSeq s = bt.s[0];
        s.length += b;
        return s;
    }
    return bt.s[b];
}

// Row stride (in blocks) of a sequence's feature-major block-key cache
// [di][ld]: the block count rounded up to a multiple of 4, so that four
// consecutive blocks of one feature are one aligned 16-byte load.
__host__ __device__ inline uint32_t block_key_ld(uint32_t capacity, uint32_t block) {
    return ((capacity / block) + 3u) & ~3u;
}

struct QsaWeightsDev {
    const float *q_norm, *k_norm, *iq_norm, *ik_norm;
    const float *rope_cos, *rope_sin;   // [positions][rotary/2]
    uint32_t rope_positions;
};

// proj: [B][2*Hq*d + 2*Hkv*d] (q/gate interleaved | k | v);
// iproj: [B][Hi*di + di] (index query | raw index key), exact order.
// `inline_block_key`: an entry whose token completes a block also caches
// that block's key.  Entries that share one cache (a prefill chunk) pass
// false and run launch_qsa_block_keys afterwards, because the block's other
// raw rows are written by other CTAs of the same launch.
// `index_queries` false: the entries' index queries are neither read nor
// written (their scores are computed on another rank); `queries` false: the
// same for the attention queries (their attention runs on another rank).
void launch_qsa_prepare(const QsaDims &d, const QsaWeightsDev &w,
                        const QsaBatch &b, uint32_t batch, const float *proj,
                        uint32_t ldp, const float *iproj, uint32_t ldi,
                        float *q_out, float *iq_out, bool inline_block_key,
                        bool index_queries, bool queries, ErrorWord err,
                        cudaStream_t stream);
// `shared_sequence`: every entry is a token of the same sequence (one
// cache, consecutive positions), so the entries share the block keys.
void launch_qsa_score(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                      const float *iq, float *scores, uint32_t ld_scores,
                      uint32_t max_blocks, bool shared_sequence, ErrorWord err,
                      cudaStream_t stream);
// `rank_order`: the selected ids in the reference's rank order (score
// descending, id ascending), else in ascending id order (same set).
void launch_qsa_select(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                       const float *scores, uint32_t ld_scores,
                       uint32_t *selected, uint32_t *selected_count,
                       bool rank_order, ErrorWord err, cudaStream_t stream);
void launch_qsa_attend(const QsaDims &d, const QsaBatch &b, uint32_t batch,
                       const float *q, const uint32_t *selected,
                       const uint32_t *selected_count, float *partial_o,
                       float *partial_ml, uint32_t splits,
                       ErrorWord err, cudaStream_t stream);
void launch_qsa_combine(const QsaDims &d, uint32_t batch,
                        const float *partial_o, const float *partial_ml,
                        uint32_t splits, const float *proj, uint32_t ldp,
                        float *gated, ErrorWord err, cudaStream_t stream);
// Checkpoint path: the attention of entry 0 of `b` (one token) for every
// query head over its selected tokens in the reference's rank order (the
// selection written with rank_order), with the logits [Hq][ntok], the
// probabilities [Hq][ntok] and the ungated context [Hq][d] written out
// (ntok = selected blocks x block + the tail; rows packed with that stride).
void launch_qsa_debug_attention(const QsaDims &d, const QsaBatch &b, const float *q, const uint32_t *selected,
                                const uint32_t *selected_count, float *logits, float *probs, float *context,
                                ErrorWord err, cudaStream_t stream);
// True when the attention runs on the tensor cores (head_dim 256, at most 8
// query heads per KV head), which reads the bf16 hi / lo copies of the
// cache rows; the state then keeps them.
bool qsa_split_cache_used(const QsaDims &d);
bool force_simt_attention();
// Writes the hi / lo copies of tokens [0, length) of an F32 cache
// [token][kv_heads][256] into the split layout of a `capacity`-token cache.
void launch_qsa_split_rows(const float *src, uint16_t *dst, uint64_t length, uint32_t kv_heads,
                           uint64_t capacity, cudaStream_t stream);
// Recomputes the block-key cache entries [first_block, end_block) of one
// sequence from its raw index keys (after an import).
void launch_qsa_block_keys(const QsaDims &d, const QsaWeightsDev &w,
                           const QsaSeq &s, uint32_t first_block,
                           uint32_t end_block, ErrorWord err,
                           cudaStream_t stream);

// ---- MoE (kernels_moe.cu)
constexpr uint32_t kMoeMaxTopK = 32;
constexpr uint32_t kMoeMaxExperts = 8192;

struct MoeDims {
    uint32_t hidden, experts, top_k, routed, shared;
};

// Device weights: router [E x H] and shared gate weight [1 x H] (exact
// products), expert stacks gate / up [E*I x H] and down [E*H x I]
// (expert-major rows), shared gate / up [S x H], shared down [H x S].
struct MoeWeightsDev {
    QMatrix router, gate, up, down, shared_gate, shared_up, shared_down, shared_gate_weight;
};

// Intermediate values kept for the checkpoint observer (all null when not
// observed): routed gate / up [picks][I] and weighted outputs [picks][H] by
// slot, routed sum and gated shared output [T][H], (shared logit, scale)
// [T][2].
struct MoeDebug {
    float *gate, *up, *weighted, *routed_sum, *gated_shared, *scale;
};

// Work space of one call over T tokens (moe_carve).  Picks p = t*K + k;
// slots are expert-major.
struct MoeBuffers {
    float *logits;          // [T][E+1]: router logits, then the shared gate logit
    float *probs;           // [T][E]
    uint32_t *sel_ids;      // [T][K], top-k order
    float *sel_w;           // [T][K]
    uint32_t *counts;       // [E]
    uint32_t *offsets;      // [E+1]
    uint32_t *active;       // [1+E]: active expert count, then their ids
    uint32_t *rank;         // [picks] position among the expert's picks
    uint32_t *slot;         // [picks] pick -> slot
    uint32_t *pick_of_slot; // [picks] slot -> pick
    float *act;             // [picks][I] by slot
    float *eout;            // [picks][H] by slot
    float *shared_gu;       // [T][2S]
    float *shared_act;      // [T][S]
    float *shared_out;      // [T][H]
    float *proj_gu, *proj_down;   // tensor-core projection work space
    size_t proj_floats_gu, proj_floats_down;
    MoeDebug dbg;
};

size_t moe_workspace_bytes(const MoeDims &d, uint32_t T, bool debug);
void moe_carve(const MoeDims &d, uint32_t T, bool debug, void *ws, MoeBuffers &b);
// The whole operator on device arrays x [T][H] -> y [T][H].
void launch_moe(const MoeDims &d, const MoeWeightsDev &w, const float *x, uint32_t T, float *y, MoeBuffers &b,
                ErrorWord err, cudaStream_t stream);
// Its stages (launch_moe runs router, route, dispatch, experts, shared
// expert, combine).
void launch_moe_route(const MoeDims &d, const float *logits, uint32_t ldl, uint32_t T, MoeBuffers &b,
                      ErrorWord err, cudaStream_t stream);
void launch_moe_dispatch(const MoeDims &d, uint32_t T, MoeBuffers &b, ErrorWord err, cudaStream_t stream);
void launch_moe_experts(const MoeDims &d, const MoeWeightsDev &w, const float *x, uint32_t ldx, uint32_t T,
                        MoeBuffers &b, ErrorWord err, cudaStream_t stream);

// ---- layer gated residual (kernels_layer.cu)
struct GrDims {
    uint32_t hidden, branches, rank;
    float eps;
};

// norm: device F32 [B*H] (1 + w form); down [rank x W], up [W x rank],
// inject [B x W] (W = B*H), any projection type.
struct GrWeightsDev {
    const float *norm;
    QMatrix down, up, inject;
};

// Work space of one read over T tokens (gr_carve); after launch_gr_read,
// `normalized` and `read` hold every token's normalised branches and read
// gates [T][W].
struct GrBuffers {
    float *normalized, *proj, *rank, *read;
    float *ws_down, *ws_up;
    size_t ws_down_floats, ws_up_floats;
};

size_t gr_workspace_bytes(const GrDims &d, uint32_t T);
void gr_carve(const GrDims &d, uint32_t T, void *ws, GrBuffers &b);
// Branches [T][B][H] -> mixed [T][H] and write gates [T][B].
void launch_gr_read(const GrDims &d, const GrWeightsDev &w, const float *branches, uint32_t T, float *mixed,
                    float *write_gate, GrBuffers &b, ErrorWord err, cudaStream_t stream);
// out[t][b][h] = branches[t][b][h] + block[t][h] * write_gate[t][b]
void launch_gr_write(const GrDims &d, const float *branches, const float *block, const float *write_gate, uint32_t T,
                     float *out, ErrorWord err, cudaStream_t stream);

uint64_t launches_total();
bool force_simt_projection();
void count_launch();

// Optional CUDA-event timing of one named kernel family (kq_b200_profile_*):
// construct before the launch, destroy after it.
struct KernelTimer {
    KernelTimer(const char *name, cudaStream_t stream);
    ~KernelTimer();
    int slot;
    cudaStream_t stream;
};

}  // namespace kqb
