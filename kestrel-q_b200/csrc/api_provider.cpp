// Device-resident weight provider: the GEMV seam of the operator ABI
// (kq_weight_provider_linear_f32, src/kq_weight_provider.c:378-509 of
// Kestrel-Q) over GGUF blocks uploaded once to HBM.
#include <algorithm>
#include <cfenv>
#include <functional>
#include <string>
#include <cmath>
#include <cstring>
#include <vector>

#include "kq_b200.h"
#include "kq_tensor_view.h"
#include "provider.hpp"
#include "quant.cuh"

using namespace kqb;

namespace kqb {

// |value| of an IEEE half stored little-endian at p (inf for inf / NaN).
static double half_abs(const uint8_t *p) {
    const uint32_t h = (uint32_t)p[0] | ((uint32_t)p[1] << 8);
    const uint32_t e = (h >> 10) & 31u, m = h & 0x3ffu;
    if (e == 31u) return INFINITY;
    return e == 0u ? std::ldexp((double)m, -24) : std::ldexp((double)(m | 0x400u), (int)e - 25);
}

double weight_abs_bound(uint32_t type, const uint8_t *p, uint64_t rows, uint64_t row_bytes) {
    const uint64_t total = rows * row_bytes;
    double b = 0.0;
    switch (type) {
    case kTypeQ4_K:   // d * sc * q - dmin * m, sc and m 6-bit, q 4-bit
        for (uint64_t o = 0; o + 144 <= total; o += 144)
            b = std::max(b, half_abs(p + o) * 63.0 * 15.0 + half_abs(p + o + 2) * 63.0);
        break;
    case kTypeQ6_K:   // d * sc * (q - 32), sc int8, q 6-bit
        for (uint64_t o = 0; o + 210 <= total; o += 210) b = std::max(b, half_abs(p + o + 208) * 128.0 * 32.0);
        break;
    case kTypeQ8_0:   // d * code, code int8
        for (uint64_t o = 0; o + 34 <= total; o += 34) b = std::max(b, half_abs(p + o) * 128.0);
        break;
    case kTypeBF16:
        for (uint64_t o = 0; o + 2 <= total; o += 2) {
            const uint32_t bits = ((uint32_t)p[o] | ((uint32_t)p[o + 1] << 8)) << 16;
            float v;
            std::memcpy(&v, &bits, 4);
            b = std::max(b, std::fabs((double)v));
        }
        break;
    default:
        for (uint64_t o = 0; o + 4 <= total; o += 4) {
            float v;
            std::memcpy(&v, p + o, 4);
            b = std::max(b, std::fabs((double)v));
        }
        break;
    }
    return b;
}

int32_t weight_scale_exponent(double bound) {
    if (!(bound > 0.0) || !std::isfinite(bound)) return 0;
    int k = 0;
    std::frexp(bound, &k);   // bound < 2^k
    return std::min(64, std::max(-64, 14 - k));
}

}  // namespace kqb

ProviderTensor *provider_lookup(const kq_weight_provider *provider,
                                const kq_semantic_tensor *semantic) {
    if (provider == nullptr || semantic == nullptr || provider->magic != kProviderMagic) return nullptr;
    for (const auto &t : provider->tensors)
        if (&t->desc == semantic) return t.get();
    return nullptr;
}

ProviderTensor *provider_part(const kq_weight_provider *provider, const kq_semantic_tensor *semantic,
                              kq_binding_part_role part_role) {
    ProviderTensor *t = provider_lookup(provider, semantic);
    if (t == nullptr) return nullptr;
    if (t->parts[0] == nullptr) return part_role == KQ_BINDING_PART_WHOLE ? t : nullptr;
    const kq_binding_part_role first = t->desc.bindings[0].part_role, second = t->desc.bindings[1].part_role;
    if (part_role == first) return t->parts[0];
    if (part_role == second) return t->parts[1];
    return nullptr;
}

namespace {

// Canonical (grouped) index of a GDN value-head-major element -> its
// position in the model GGUF's tiled order: canonical head g * R + r is
// stored as head r * Hk + g (src/kq_weight_provider.c:205-211; the
// converter's reordering, docs/MODEL-GGUF-MAPPING.md of Kestrel-Q).
uint64_t grouped_to_tiled(uint64_t canonical, uint64_t width, const kq_b200_gguf_layout &g) {
    const uint64_t group = canonical / (g.gdn_value_repeat * width);
    const uint64_t within = canonical % (g.gdn_value_repeat * width);
    const uint64_t repeat = within / width, feature = within % width;
    return (repeat * g.gdn_key_heads + group) * width + feature;
}

bool layout_valid(const kq_b200_gguf_layout *g) {
    return g != nullptr && g->gdn_key_heads > 0 && g->gdn_value_repeat > 0 && g->gdn_head_width > 0 &&
           (uint64_t)g->gdn_key_heads * g->gdn_value_repeat * g->gdn_head_width <= UINT32_MAX;
}

// QSA norms the converter stores as 1 + delta (src/kq_weight_provider.c:218-230)
bool folded_gamma(kq_semantic_role role) {
    return role == KQ_ROLE_QSA_Q_NORM || role == KQ_ROLE_QSA_K_NORM || role == KQ_ROLE_QSA_INDEX_Q_NORM ||
           role == KQ_ROLE_QSA_INDEX_K_NORM;
}

}  // namespace

static ProviderTensor *new_tensor(kq_weight_provider *p, const char *id, kq_semantic_role role) {
    auto t = std::make_unique<ProviderTensor>();
    std::memset(&t->desc, 0, sizeof(t->desc));
    if (id) std::strncpy(t->desc.semantic_id, id, KQ_SEMANTIC_ID_CAPACITY - 1);
    t->desc.role = role;
    t->desc.relation = KQ_BINDING_DIRECT_ONE_TO_ONE;
    t->desc.runtime_scope = KQ_SCOPE_REQUIRED_INITIAL_TEXT;
    t->desc.canonical_dtype = KQ_CANONICAL_DTYPE_BF16;
    t->desc.layer_id = KQ_MODEL_NO_LAYER;
    t->desc.canonical_expert_axis = KQ_MODEL_NO_AXIS;
    t->desc.binding_count = 1;
    t->desc.bindings[0].part_role = KQ_BINDING_PART_WHOLE;
    t->desc.bindings[0].part_count = 1;
    ProviderTensor *raw = t.get();
    p->tensors.push_back(std::move(t));
    return raw;
}

extern "C" {

kq_status kq_weight_provider_open(const kq_gguf *, const kq_model *, uint64_t,
                                  kq_weight_provider **out_provider, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_provider) *out_provider = nullptr;
    return fail(diagnostic, KQ_STATUS_UNSUPPORTED_MODEL,
                "GGUF-backed providers are not supported by the B200 library; "
                "use kq_b200_provider_create");
}

kq_status kq_b200_provider_create(int device, kq_weight_provider **out, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "provider output is required");
    *out = nullptr;
    kq_status st = kq_b200_set_device(device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    DeviceContext *c;
    st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    st = static_scratch_prepare(device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    auto *p = new kq_weight_provider();
    p->device = device;
    *out = p;
    return KQ_STATUS_OK;
}

void kq_weight_provider_close(kq_weight_provider *provider) {
    if (provider == nullptr || provider->magic != kProviderMagic) return;
    cudaSetDevice(provider->device);
    cudaDeviceSynchronize();
    for (auto &t : provider->tensors) {
        if (t->owned) cudaFree(t->owned);
        if (t->col_heads_dev) cudaFree(t->col_heads_dev);
    }
    provider->magic = 0;
    delete provider;
}

}  // extern "C"

// Uploads rows x columns GGUF rows (see kq_b200_provider_add_matrix).
// `side_data` builds the Q4_K side data of the factored tensor-core kernel
// (not for expert stacks, whose experts the grouped MoE kernels read).
static kq_status upload_matrix(kq_weight_provider *provider, const char *semantic_id, kq_semantic_role role,
                               uint32_t type_id, uint64_t rows, uint64_t columns, const void *packed,
                               uint64_t packed_bytes, bool side_data, ProviderTensor **out,
                               kq_diagnostic *diagnostic) {
    *out = nullptr;
    if (provider == nullptr || provider->magic != kProviderMagic || packed == nullptr || rows == 0 || columns == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, data and output are required");
    uint32_t be, bb;
    if (!block_geometry(type_id, be, bb))
        return fail(diagnostic, KQ_STATUS_UNSUPPORTED_TENSOR_TYPE,
                    "matrix type must be F32, BF16, Q8_0, Q4_K or Q6_K");
    if (columns % be != 0)
        return fail(diagnostic, KQ_STATUS_INVALID_QUANTIZED_GEOMETRY, "columns are not whole blocks");
    uint64_t row_bytes = columns / be * bb, total;
    if (!mul_ok(rows, row_bytes, &total) || rows > UINT32_MAX || columns > UINT32_MAX ||
        row_bytes > UINT32_MAX)
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "matrix size overflows");
    if (packed_bytes != total)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "packed byte count does not match the shape");
    kq_status st = kq_b200_set_device(provider->device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    // Q6_K and Q8_0 rows are stored as aligned planes (same bytes, see
    // kernels.hpp QMatrix) so the kernels can use 16-byte loads; a row whose
    // byte count is not a multiple of 16 (Q8_0 rows of 640 values: 680 B)
    // is padded to the next multiple, so every row starts 16-byte aligned
    const uint8_t *src = static_cast<const uint8_t *>(packed);
    std::vector<uint8_t> planar;
    uint32_t layout = 0;
    uint64_t pitch = row_bytes, stored = total;
    if (type_id == KQ_GGUF_TYPE_Q6_K || type_id == KQ_GGUF_TYPE_Q8_0) {
        pitch = (row_bytes + 15) & ~uint64_t(15);
        if (!mul_ok(rows, pitch, &stored))
            return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "matrix size overflows");
        planar.assign(stored, 0);
        const uint64_t nblk = columns / be;
        for (uint64_t r = 0; r < rows; ++r) {
            const uint8_t *in = src + r * row_bytes;
            uint8_t *out = planar.data() + r * pitch;
            for (uint64_t b = 0; b < nblk; ++b) {
                const uint8_t *blk = in + b * bb;
                if (type_id == KQ_GGUF_TYPE_Q6_K) {
                    std::memcpy(out + b * 128, blk, 128);                     // ql
                    std::memcpy(out + nblk * 128 + b * 64, blk + 128, 64);    // qh
                    std::memcpy(out + nblk * 192 + b * 16, blk + 192, 16);    // scales
                    std::memcpy(out + nblk * 208 + b * 2, blk + 208, 2);      // d
                } else {
                    std::memcpy(out + b * 32, blk + 2, 32);                   // codes
                    std::memcpy(out + nblk * 32 + b * 2, blk, 2);             // d
                }
            }
        }
        src = planar.data();
        layout = 1;
    }
    const int32_t scale_exp =
        weight_scale_exponent(weight_abs_bound(type_id, static_cast<const uint8_t *>(packed), rows, row_bytes));
    // Q4_K: the factored tensor-core kernel's per-super-block side data
    // (kernels.hpp q4k_build_aux) follows the blocks in the same allocation
    const uint64_t aux_offset = (stored + 255) & ~uint64_t(255);
    std::vector<uint8_t> aux;
    if (type_id == KQ_GGUF_TYPE_Q4_K && side_data) {
        aux.resize(q4k_aux_bytes((uint32_t)rows, (uint32_t)columns));
        q4k_build_aux(static_cast<const uint8_t *>(packed), (uint32_t)rows, (uint32_t)columns, scale_exp,
                      aux.data());
    }
    const uint64_t alloc = aux.empty() ? stored : aux_offset + aux.size();
    void *dev = nullptr;
    KQB_CUDA(cudaMalloc(&dev, alloc), diagnostic, "weight allocation");
    cudaError_t e = cudaMemcpy(dev, src, stored, cudaMemcpyHostToDevice);
    if (e == cudaSuccess && !aux.empty())
        e = cudaMemcpy(static_cast<uint8_t *>(dev) + aux_offset, aux.data(), aux.size(), cudaMemcpyHostToDevice);
    // a pageable upload may return before its DMA lands; the library's
    // streams do not wait for the legacy stream, so finish it here
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
        cudaFree(dev);
        return cuda_fail(diagnostic, e, "weight upload");
    }
    ProviderTensor *t = new_tensor(provider, semantic_id, role);
    t->owned = dev;
    t->bytes = total;   // logical payload (the side data is not part of it)
    t->m.data = static_cast<const uint8_t *>(dev);
    t->m.type = type_id;
    t->m.rows = (uint32_t)rows;
    t->m.cols = (uint32_t)columns;
    t->m.row_bytes = (uint32_t)pitch;
    t->m.layout = layout;
    t->m.scale_exp = scale_exp;
    t->m.aux = aux.empty() ? nullptr : static_cast<const uint8_t *>(dev) + aux_offset;
    t->desc.canonical_rank = 2;
    t->desc.canonical_dimensions[0] = rows;
    t->desc.canonical_dimensions[1] = columns;
    provider->metrics.provider_owned_bytes += alloc;
    *out = t;
    return KQ_STATUS_OK;
}

extern "C" {

kq_status kq_b200_provider_add_matrix(kq_weight_provider *provider, const char *semantic_id,
                                      kq_semantic_role role, uint32_t type_id, uint64_t rows,
                                      uint64_t columns, const void *packed, uint64_t packed_bytes,
                                      const kq_semantic_tensor **out_tensor,
                                      kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (out_tensor == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "output is required");
    ProviderTensor *t;
    kq_status st = upload_matrix(provider, semantic_id, role, type_id, rows, columns, packed, packed_bytes, true, &t,
                                 diagnostic);
    if (st != KQ_STATUS_OK) return st;
    *out_tensor = &t->desc;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_add_expert_stack(kq_weight_provider *provider, const char *semantic_id,
                                            kq_semantic_role role, uint32_t type_id, uint32_t experts,
                                            uint64_t rows, uint64_t columns, const void *packed,
                                            uint64_t packed_bytes, const kq_semantic_tensor **out_tensor,
                                            kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    uint64_t total_rows;
    if (out_tensor == nullptr || experts == 0 || rows == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "experts, rows and output are required");
    if (!mul_ok(rows, experts, &total_rows) || rows > UINT32_MAX)
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "expert stack size overflows");
    ProviderTensor *t;
    kq_status st = upload_matrix(provider, semantic_id, role, type_id, total_rows, columns, packed, packed_bytes,
                                 false, &t, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    t->experts = experts;
    t->expert_rows = (uint32_t)rows;
    t->desc.canonical_rank = 3;
    t->desc.canonical_dimensions[0] = experts;
    t->desc.canonical_dimensions[1] = rows;
    t->desc.canonical_dimensions[2] = columns;
    t->desc.canonical_expert_axis = 0;
    t->desc.expert_count = experts;
    *out_tensor = &t->desc;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_add_expert_gate_up(kq_weight_provider *provider, const char *semantic_id,
                                             uint32_t type_id, uint32_t experts, uint64_t rows, uint64_t columns,
                                             const void *gate_packed, uint64_t gate_bytes, const void *up_packed,
                                             uint64_t up_bytes, const kq_semantic_tensor **out_tensor,
                                             kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (provider == nullptr || provider->magic != kProviderMagic || out_tensor == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider and output are required");
    const kq_semantic_tensor *g = nullptr, *u = nullptr;
    const std::string base = semantic_id ? semantic_id : "gate_up";
    kq_status st = kq_b200_provider_add_expert_stack(provider, (base + ".gate").c_str(), KQ_ROLE_ROUTED_GATE_UP,
                                                     type_id, experts, rows, columns, gate_packed, gate_bytes, &g,
                                                     diagnostic);
    if (st != KQ_STATUS_OK) return st;
    st = kq_b200_provider_add_expert_stack(provider, (base + ".up").c_str(), KQ_ROLE_ROUTED_GATE_UP, type_id,
                                           experts, rows, columns, up_packed, up_bytes, &u, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    // one semantic, two bindings: GATE (part 0 of 2), UP (part 1 of 2), the
    // order of src/kq_model.c:1083-1094 and src/kq_tensor_view.c:333-334
    ProviderTensor *t = new_tensor(provider, semantic_id, KQ_ROLE_ROUTED_GATE_UP);
    t->parts[0] = provider_lookup(provider, g);
    t->parts[1] = provider_lookup(provider, u);
    t->desc.relation = KQ_BINDING_ONE_CANONICAL_TO_MULTIPLE_PHYSICAL;
    t->desc.canonical_rank = 3;
    t->desc.canonical_dimensions[0] = experts;
    t->desc.canonical_dimensions[1] = 2 * rows;
    t->desc.canonical_dimensions[2] = columns;
    t->desc.canonical_expert_axis = 0;
    t->desc.expert_count = experts;
    t->desc.binding_count = 2;
    t->desc.bindings[0].part_role = KQ_BINDING_PART_GATE;
    t->desc.bindings[0].part_index = 0;
    t->desc.bindings[0].part_count = 2;
    t->desc.bindings[1].part_role = KQ_BINDING_PART_UP;
    t->desc.bindings[1].part_index = 1;
    t->desc.bindings[1].part_count = 2;
    *out_tensor = &t->desc;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_add_vector_f32(kq_weight_provider *provider, const char *semantic_id,
                                          kq_semantic_role role, const float *values,
                                          uint64_t count, const kq_semantic_tensor **out_tensor,
                                          kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (provider == nullptr || provider->magic != kProviderMagic || values == nullptr ||
        out_tensor == nullptr || count == 0 || count > (1ull << 28))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, values and output are required");
    for (uint64_t i = 0; i < count; ++i)
        if (!std::isfinite(values[i]))
            return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "vector values must be finite");
    kq_status st = kq_b200_set_device(provider->device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    void *dev = nullptr;
    KQB_CUDA(cudaMalloc(&dev, count * sizeof(float)), diagnostic, "vector allocation");
    cudaError_t e = cudaMemcpy(dev, values, count * sizeof(float), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaStreamSynchronize(cudaStreamLegacy);
    if (e != cudaSuccess) {
        cudaFree(dev);
        return cuda_fail(diagnostic, e, "vector upload");
    }
    ProviderTensor *t = new_tensor(provider, semantic_id, role);
    t->is_vector = true;
    t->owned = dev;
    t->vec_dev = static_cast<float *>(dev);
    t->vec_host.assign(values, values + count);
    t->bytes = count * sizeof(float);
    t->desc.canonical_rank = 1;
    t->desc.canonical_dimensions[0] = count;
    provider->metrics.provider_owned_bytes += t->bytes;
    *out_tensor = &t->desc;
    return KQ_STATUS_OK;
}

kq_status kq_weight_provider_linear_f32(kq_weight_provider *provider,
                                        const kq_semantic_tensor *semantic,
                                        kq_binding_part_role part_role, uint32_t expert_id,
                                        uint64_t rows, uint64_t columns, const float *input,
                                        float *output, uint64_t output_capacity, void *scratch,
                                        uint64_t scratch_bytes, kq_diagnostic *diagnostic) {
    (void)scratch;
    (void)scratch_bytes;
    kq_diagnostic_clear(diagnostic);
    ProviderTensor *t = provider_lookup(provider, semantic);
    if (t == nullptr || input == nullptr || output == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, semantic and buffers are required");
    // a split semantic is read by part (src/kq_weight_provider.c:250-262)
    t = provider_part(provider, semantic, part_role);
    if (t == nullptr || t->is_vector)
        return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH, "requested semantic binding part is absent");
    // an expert stack is read one expert at a time (src/kq_weight_provider.c:250-272)
    QMatrix m = t->m;
    if (expert_id != KQ_WEIGHT_PROVIDER_NO_EXPERT) {
        if (t->experts == 0 || expert_id >= t->experts)
            return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "selected expert ID is outside the semantic stack");
        m.data += (size_t)expert_id * t->expert_rows * m.row_bytes;
        m.rows = t->expert_rows;
        m.aux = nullptr;
    } else if (t->experts != 0) {
        return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH, "routed expert stack requires an explicit expert ID");
    }
    if (rows != m.rows || columns != m.cols)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "linear shape does not match the semantic");
    if (output_capacity < rows) return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "linear output is too small");
    if (ranges_overlap(input, columns * 4, output, rows * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "linear input and output overlap");
    if (std::fegetround() != FE_TONEAREST)
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "round-to-nearest floating mode is required");
    kq_status st = kq_b200_set_device(provider->device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    DeviceContext *c;
    st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    st = c->synchronize(diagnostic);   // settle earlier asynchronous work first
    if (st != KQ_STATUS_OK) return st;
    const bool dev_in = is_device_pointer(input), dev_out = is_device_pointer(output);
    void *ws;
    st = c->workspace(Carve::round(columns * 4) + Carve::round(rows * 4) + 512, &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    const float *x = input;
    std::vector<float> permuted;
    if (!t->col_heads.empty()) {
        // tiled columns: the canonical input goes to the physical column
        // positions first (src/kq_weight_provider.c:438-451)
        std::vector<float> canonical(columns);
        KQB_CUDA(cudaMemcpy(canonical.data(), input, columns * 4, cudaMemcpyDefault), diagnostic, "input read");
        permuted.resize(columns);
        const uint64_t w = t->head_width;
        for (uint64_t h = 0; h < t->col_heads.size(); ++h)
            std::memcpy(permuted.data() + (uint64_t)t->col_heads[h] * w, canonical.data() + h * w, w * 4);
        float *p = cv.take<float>(columns);
        KQB_CUDA(cudaMemcpyAsync(p, permuted.data(), columns * 4, cudaMemcpyHostToDevice, c->stream), diagnostic,
                 "H2D");
        KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "H2D");
        x = p;
    } else if (!dev_in) {
        float *p = cv.take<float>(columns);
        KQB_CUDA(cudaMemcpyAsync(p, input, columns * 4, cudaMemcpyHostToDevice, c->stream), diagnostic, "H2D");
        x = p;
    }
    float *y = cv.take<float>(rows);
    ErrorWord err = c->begin_call();
    launch_check_finite(x, columns, err, c->stream);
    ProjSegments segs{};
    segs.count = 1;
    segs.m[0] = m;
    segs.out_offset[0] = 0;
    launch_projection(segs, x, (uint32_t)columns, y, (uint32_t)rows, 1, err, c->stream);
    launch_check_finite(y, rows, err, c->stream);
    KQB_CUDA(cudaGetLastError(), diagnostic, "linear launch");
    st = c->synchronize(diagnostic);
    if (st != KQ_STATUS_OK) return st;
    KQB_CUDA(cudaMemcpy(output, y, rows * 4, dev_out ? cudaMemcpyDeviceToDevice : cudaMemcpyDeviceToHost),
             diagnostic, "linear output");
    provider->metrics.linear_requests += 1;
    provider->metrics.row_requests += rows;
    provider->metrics.logical_payload_bytes_touched += (uint64_t)m.rows * m.row_bytes;
    if (expert_id != KQ_WEIGHT_PROVIDER_NO_EXPERT) provider->metrics.selected_expert_requests += 1;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_linear_batch_f32(kq_weight_provider *provider,
                                            const kq_semantic_tensor *semantic, uint64_t rows,
                                            uint64_t columns, const float *x, uint32_t batch, float *y,
                                            kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    ProviderTensor *t = provider_lookup(provider, semantic);
    if (t == nullptr || x == nullptr || y == nullptr || batch == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, semantic and buffers are required");
    if (t->is_vector || t->parts[0] != nullptr || t->experts != 0)
        return fail(diagnostic, KQ_STATUS_TENSOR_LAYOUT_MISMATCH, "semantic is not a whole matrix");
    if (rows != t->m.rows || columns != t->m.cols)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "linear shape does not match the semantic");
    if (!is_device_pointer(x) || !is_device_pointer(y))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "batched linear takes device buffers");
    if (ranges_overlap(x, (uint64_t)batch * columns * 4, y, (uint64_t)batch * rows * 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "linear input and output overlap");
    kq_status st = kq_b200_set_device(provider->device, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    DeviceContext *c;
    st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    const size_t partial_floats = projection_workspace_floats(batch, (uint32_t)rows, (uint32_t)columns);
    const size_t perm_bytes = t->col_heads.empty() ? 0 : Carve::round((size_t)batch * columns * 4);
    void *ws;
    st = c->workspace(Carve::round(partial_floats * 4) + perm_bytes + 256, &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    float *partial = partial_floats ? cv.take<float>(partial_floats) : nullptr;
    ErrorWord err = c->begin_call();
    launch_check_finite(x, (uint64_t)batch * columns, err, c->stream);
    if (!t->col_heads.empty()) {
        // tiled columns: the canonical input rows go to the physical column positions
        float *xp = cv.take<float>((size_t)batch * columns);
        launch_permute_column_heads(x, batch, (uint32_t)columns, t->head_width, t->col_heads_dev,
                                    (uint32_t)t->col_heads.size(), xp, c->stream);
        x = xp;
    }
    ProjSegments segs{};
    segs.count = 1;
    segs.m[0] = t->m;
    launch_projection(segs, x, (uint32_t)columns, y, (uint32_t)rows, batch, err, c->stream, partial,
                      partial_floats);
    KQB_CUDA(cudaGetLastError(), diagnostic, "linear launch");
    provider->metrics.linear_requests += 1;
    return KQ_STATUS_OK;
}

kq_status kq_weight_provider_vector_f32(kq_weight_provider *provider,
                                        const kq_semantic_tensor *semantic,
                                        uint64_t element_count, float *output,
                                        uint64_t output_capacity, void *, uint64_t,
                                        kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    ProviderTensor *t = provider_lookup(provider, semantic);
    if (t == nullptr || output == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider, semantic and output are required");
    if (!t->is_vector) return fail(diagnostic, KQ_STATUS_LIMIT_EXCEEDED, "complete matrices are not materialised");
    if (element_count != t->vec_host.size())
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "vector element count mismatch");
    if (output_capacity < element_count) return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "vector output is too small");
    std::memcpy(output, t->vec_host.data(), element_count * sizeof(float));
    provider->metrics.vector_requests += 1;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_add_gguf_matrix(kq_weight_provider *provider, const char *semantic_id,
                                           kq_semantic_role role, uint32_t type_id, uint64_t rows,
                                           uint64_t columns, const void *packed, uint64_t packed_bytes,
                                           const kq_b200_gguf_layout *layout,
                                           const kq_semantic_tensor **out_tensor, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (!layout_valid(layout) || packed == nullptr || rows == 0 || columns == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid GGUF layout and tensor are required");
    const kq_b200_gguf_layout &g = *layout;
    const uint64_t W = g.gdn_head_width, Hv = (uint64_t)g.gdn_key_heads * g.gdn_value_repeat;
    const uint64_t qk = 2ull * g.gdn_key_heads * W;
    uint32_t be, bb;
    if (!block_geometry(type_id, be, bb) || columns % be != 0)
        return fail(diagnostic, KQ_STATUS_INVALID_QUANTIZED_GEOMETRY, "columns are not whole blocks of the type");
    const uint64_t row_bytes = columns / be * bb;
    if (rows > UINT32_MAX || row_bytes > UINT32_MAX || packed_bytes != rows * row_bytes)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "packed byte count does not match the shape");
    // canonical row r is stored at physical row phys(r)
    // (src/kq_weight_provider.c:232-248)
    std::function<uint64_t(uint64_t)> phys;
    if (role == KQ_ROLE_GDN_QKV) {
        if (rows != qk + Hv * W)
            return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN qkv rows do not match the layout");
        phys = [&](uint64_t r) { return r < qk ? r : qk + grouped_to_tiled(r - qk, W, g); };
    } else if (role == KQ_ROLE_GDN_GATE) {
        if (rows != Hv * W)
            return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN gate rows do not match the layout");
        phys = [&](uint64_t r) { return grouped_to_tiled(r, W, g); };
    } else if (role == KQ_ROLE_GDN_ALPHA || role == KQ_ROLE_GDN_BETA) {
        if (rows != Hv)
            return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN alpha/beta rows do not match the layout");
        phys = [&](uint64_t r) { return grouped_to_tiled(r, 1, g); };
    }
    const uint8_t *src = static_cast<const uint8_t *>(packed);
    std::vector<uint8_t> canonical;
    if (phys) {
        canonical.resize(packed_bytes);
        for (uint64_t r = 0; r < rows; ++r)
            std::memcpy(canonical.data() + r * row_bytes, src + phys(r) * row_bytes, row_bytes);
        src = canonical.data();
    }
    if (role == KQ_ROLE_GDN_OUT && columns != Hv * W)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN output columns do not match the layout");
    const kq_semantic_tensor *desc = nullptr;
    kq_status st = kq_b200_provider_add_matrix(provider, semantic_id, role, type_id, rows, columns, src,
                                               packed_bytes, &desc, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (role == KQ_ROLE_GDN_OUT) {
        // tiled columns stay as stored: the operator writes its gated output
        // in this order and the linear seam permutes its input
        // (src/kq_weight_provider.c:438-451)
        ProviderTensor *t = provider_lookup(provider, desc);
        t->head_width = (uint32_t)W;
        t->col_heads.resize(Hv);
        for (uint64_t h = 0; h < Hv; ++h) t->col_heads[h] = (int32_t)(grouped_to_tiled(h * W, W, g) / W);
        KQB_CUDA(cudaMalloc(&t->col_heads_dev, Hv * sizeof(int32_t)), diagnostic, "column head map");
        KQB_CUDA(cudaMemcpy(t->col_heads_dev, t->col_heads.data(), Hv * sizeof(int32_t), cudaMemcpyHostToDevice),
                 diagnostic, "column head map");
    }
    *out_tensor = desc;
    return KQ_STATUS_OK;
}

kq_status kq_b200_provider_add_gguf_vector_f32(kq_weight_provider *provider, const char *semantic_id,
                                               kq_semantic_role role, const float *values, uint64_t count,
                                               const kq_b200_gguf_layout *layout,
                                               const kq_semantic_tensor **out_tensor, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (!layout_valid(layout) || values == nullptr || count == 0 || count > (1ull << 28))
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid GGUF layout and values are required");
    const kq_b200_gguf_layout &g = *layout;
    const uint64_t W = g.gdn_head_width, Hv = (uint64_t)g.gdn_key_heads * g.gdn_value_repeat;
    const uint64_t qk = 2ull * g.gdn_key_heads * W;
    std::vector<float> out(values, values + count);
    // src/kq_weight_provider.c:680-717
    if (role == KQ_ROLE_GDN_A_LOG || role == KQ_ROLE_GDN_DT_BIAS) {
        if (count != Hv)
            return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN per-head vector does not match the layout");
        for (uint64_t i = 0; i < count; ++i) {
            const float v = values[grouped_to_tiled(i, 1, g)];
            // A_log is stored as -exp(A_log)
            out[i] = role == KQ_ROLE_GDN_A_LOG ? logf(-v) : v;
            if (!std::isfinite(out[i]))
                return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "stored GDN A_log must be negative and finite");
        }
    } else if (role == KQ_ROLE_GDN_CONV) {
        if (count % 4 != 0 || count / 4 != qk + Hv * W)
            return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "GDN conv channels do not match the layout");
        for (uint64_t c = 0; c < count / 4; ++c) {
            const uint64_t p = c < qk ? c : qk + grouped_to_tiled(c - qk, W, g);
            std::memcpy(out.data() + c * 4, values + p * 4, 4 * sizeof(float));
        }
    } else if (folded_gamma(role)) {
        for (uint64_t i = 0; i < count; ++i) out[i] = values[i] - 1.0f;   // stored as 1 + delta
    }
    return kq_b200_provider_add_vector_f32(provider, semantic_id, role, out.data(), count, out_tensor, diagnostic);
}

kq_status kq_b200_provider_add_index_qk(kq_weight_provider *provider, const char *semantic_id, uint32_t type_id,
                                        uint64_t query_rows, uint64_t key_rows, uint64_t columns,
                                        const void *query_packed, uint64_t query_bytes, const void *key_packed,
                                        uint64_t key_bytes, const kq_semantic_tensor **out_tensor,
                                        kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_tensor) *out_tensor = nullptr;
    if (provider == nullptr || provider->magic != kProviderMagic || out_tensor == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "valid provider and output are required");
    const kq_semantic_tensor *q = nullptr, *k = nullptr;
    const std::string base = semantic_id ? semantic_id : "index_qk";
    kq_status st = kq_b200_provider_add_matrix(provider, (base + ".index_query").c_str(), KQ_ROLE_QSA_INDEX_QK,
                                               type_id, query_rows, columns, query_packed, query_bytes, &q,
                                               diagnostic);
    if (st != KQ_STATUS_OK) return st;
    st = kq_b200_provider_add_matrix(provider, (base + ".index_key").c_str(), KQ_ROLE_QSA_INDEX_QK, type_id, key_rows,
                                     columns, key_packed, key_bytes, &k, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    // one semantic, two bindings: INDEX_QUERY (part 0 of 2), INDEX_KEY
    // (part 1 of 2), the order src/kq_qsa.c:184-201 requires
    ProviderTensor *t = new_tensor(provider, semantic_id, KQ_ROLE_QSA_INDEX_QK);
    t->parts[0] = provider_lookup(provider, q);
    t->parts[1] = provider_lookup(provider, k);
    t->desc.canonical_rank = 2;
    t->desc.canonical_dimensions[0] = query_rows + key_rows;
    t->desc.canonical_dimensions[1] = columns;
    t->desc.binding_count = 2;
    t->desc.bindings[0].part_role = KQ_BINDING_PART_INDEX_QUERY;
    t->desc.bindings[0].part_index = 0;
    t->desc.bindings[0].part_count = 2;
    t->desc.bindings[1].part_role = KQ_BINDING_PART_INDEX_KEY;
    t->desc.bindings[1].part_index = 1;
    t->desc.bindings[1].part_count = 2;
    *out_tensor = &t->desc;
    return KQ_STATUS_OK;
}

const kq_weight_provider_metrics *kq_weight_provider_get_metrics(const kq_weight_provider *provider) {
    if (provider == nullptr || provider->magic != kProviderMagic) return nullptr;
    return &provider->metrics;
}

}  // extern "C"
