// Status strings, quantized geometry and the GPU dequant / row-dot entry
// points of the operator ABI.
#include <cfenv>
#include <cmath>
#include <cstring>
#include <vector>

#include "kq_numeric.h"
#include "kq_status.h"
#include "kq_tensor_view.h"
#include "quant.cuh"
#include "runtime.hpp"

using namespace kqb;

extern "C" {

// Status text: the same wording as src/kq_status.c:9-126 of Kestrel-Q,
// because callers print and compare it.
const char *kq_status_string(kq_status status) {
    switch (status) {
    case KQ_STATUS_OK: return "ok";
    case KQ_STATUS_INVALID_ARGUMENT: return "invalid argument";
    case KQ_STATUS_OUT_OF_MEMORY: return "out of memory";
    case KQ_STATUS_FILE_OPEN_FAILED: return "file open failed";
    case KQ_STATUS_FILE_SIZE_FAILED: return "file size failed";
    case KQ_STATUS_FILE_MAP_FAILED: return "file mapping failed";
    case KQ_STATUS_TRUNCATED: return "truncated file";
    case KQ_STATUS_BAD_MAGIC: return "bad GGUF magic";
    case KQ_STATUS_UNSUPPORTED_VERSION: return "unsupported GGUF version";
    case KQ_STATUS_MALFORMED_METADATA: return "malformed GGUF metadata";
    case KQ_STATUS_UNSUPPORTED_METADATA: return "unsupported GGUF metadata";
    case KQ_STATUS_MALFORMED_TENSOR: return "malformed GGUF tensor";
    case KQ_STATUS_UNSUPPORTED_TENSOR_TYPE: return "unsupported GGUF tensor type";
    case KQ_STATUS_ARITHMETIC_OVERFLOW: return "arithmetic overflow";
    case KQ_STATUS_LIMIT_EXCEEDED: return "defensive limit exceeded";
    case KQ_STATUS_INVALID_ALIGNMENT: return "invalid GGUF alignment";
    case KQ_STATUS_SPAN_OUT_OF_RANGE: return "tensor span out of range";
    case KQ_STATUS_DUPLICATE_METADATA: return "duplicate GGUF metadata key";
    case KQ_STATUS_DUPLICATE_TENSOR: return "duplicate GGUF tensor name";
    case KQ_STATUS_INCONSISTENT_DATA_SECTION: return "inconsistent GGUF data section";
    case KQ_STATUS_UNSUPPORTED_MODEL: return "unsupported model";
    case KQ_STATUS_MODEL_TOPOLOGY_MISMATCH: return "model topology mismatch";
    case KQ_STATUS_SEMANTIC_MAPPING_FAILED: return "semantic tensor mapping failed";
    case KQ_STATUS_UNKNOWN_PHYSICAL_TENSOR: return "unknown physical tensor";
    case KQ_STATUS_NO_TENSOR_PAYLOAD: return "semantic has no tensor payload";
    case KQ_STATUS_INVALID_QUANTIZED_GEOMETRY: return "invalid quantized tensor geometry";
    case KQ_STATUS_NONCONTIGUOUS_TENSOR_VIEW: return "tensor member is not physically contiguous";
    case KQ_STATUS_TENSOR_LAYOUT_MISMATCH: return "tensor layout does not satisfy the requested access";
    case KQ_STATUS_TENSOR_OWNERSHIP_MISMATCH: return "tensor descriptor does not belong to the GGUF";
    case KQ_STATUS_INCOMPATIBLE_TOKENIZER: return "incompatible tokenizer metadata";
    case KQ_STATUS_INVALID_UTF8: return "invalid UTF-8";
    case KQ_STATUS_INVALID_TOKEN_ID: return "invalid tokenizer token ID";
    case KQ_STATUS_BUFFER_TOO_SMALL: return "output buffer too small";
    case KQ_STATUS_UNSUPPORTED_TOKENIZER_OPTION: return "unsupported tokenizer option";
    case KQ_STATUS_UNSUPPORTED_CHAT: return "unsupported chat role, content, or option";
    case KQ_STATUS_MALFORMED_CHAT: return "malformed chat input";
    case KQ_STATUS_INCOMPATIBLE_PLE: return "incompatible PLE configuration";
    case KQ_STATUS_INVALID_PLE_STATE: return "invalid PLE stream state";
    case KQ_STATUS_MALFORMED_QUANTIZED_DATA: return "malformed quantized data";
    case KQ_STATUS_NUMERIC_DOMAIN: return "invalid numeric domain";
    case KQ_STATUS_DIMENSION_MISMATCH: return "numeric dimension mismatch";
    case KQ_STATUS_ALIASING_VIOLATION: return "forbidden numeric buffer aliasing";
    case KQ_STATUS_INCOMPATIBLE_GDN: return "incompatible GDN configuration";
    case KQ_STATUS_INVALID_GDN_STATE: return "invalid GDN stream state";
    case KQ_STATUS_INCOMPATIBLE_QSA: return "incompatible QSA configuration";
    case KQ_STATUS_INVALID_QSA_STATE: return "invalid QSA stream state";
    case KQ_STATUS_INCOMPATIBLE_MOE: return "incompatible MoE configuration";
    case KQ_STATUS_INCOMPATIBLE_PLE_VALUE: return "incompatible PLE value configuration";
    case KQ_STATUS_INVALID_PLE_VALUE_STATE: return "invalid PLE value stream state";
    case KQ_STATUS_PLE_LOOKUP_FAILED: return "PLE value lookup failed";
    case KQ_STATUS_INCOMPATIBLE_LAYER: return "incompatible transformer-layer configuration";
    case KQ_STATUS_INVALID_LAYER_STATE: return "invalid transformer-layer stream state";
    case KQ_STATUS_INCOMPATIBLE_MODEL_EXEC: return "incompatible model execution configuration";
    case KQ_STATUS_INVALID_MODEL_STATE: return "invalid model execution state";
    case KQ_STATUS_INCOMPATIBLE_SAMPLING: return "incompatible sampling policy";
    case KQ_STATUS_INVALID_RNG_STATE: return "invalid sampling RNG state";
    default: return "unknown status";
    }
}

void kq_diagnostic_clear(kq_diagnostic *diagnostic) {
    if (diagnostic == nullptr) return;
    diagnostic->status = KQ_STATUS_OK;
    diagnostic->message[0] = '\0';
}

// Type table of src/kq_gguf.c:57-65 of Kestrel-Q plus Q6_K.
kq_status kq_quant_geometry_for_type(uint32_t type_id, kq_quant_geometry *out,
                                     kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "output quantized geometry is required");
    std::memset(out, 0, sizeof(*out));
    uint64_t elems = 0, bytes = 0;
    switch (type_id) {
    case KQ_GGUF_TYPE_F32: elems = 1; bytes = 4; break;
    case KQ_GGUF_TYPE_Q5_1: elems = 32; bytes = 24; break;
    case KQ_GGUF_TYPE_Q8_0: elems = 32; bytes = 34; break;
    case KQ_GGUF_TYPE_Q4_K: elems = 256; bytes = 144; break;
    case KQ_GGUF_TYPE_Q5_K: elems = 256; bytes = 176; break;
    case KQ_GGUF_TYPE_Q6_K: elems = 256; bytes = 210; break;
    case KQ_GGUF_TYPE_IQ4_NL: elems = 32; bytes = 18; break;
    case KQ_GGUF_TYPE_BF16: elems = 1; bytes = 2; break;
    default: return fail(diagnostic, KQ_STATUS_UNSUPPORTED_TENSOR_TYPE, "GGUF tensor type is unsupported");
    }
    out->type_id = type_id;
    out->block_elements = elems;
    out->bytes_per_block = bytes;
    return KQ_STATUS_OK;
}

kq_status kq_quant_packed_size(uint32_t type_id, uint64_t element_count,
                               uint64_t *out_packed_bytes, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_packed_bytes == nullptr) return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "output packed byte count is required");
    *out_packed_bytes = 0;
    kq_quant_geometry g;
    kq_status st = kq_quant_geometry_for_type(type_id, &g, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (element_count == 0 || element_count % g.block_elements != 0)
        return fail(diagnostic, KQ_STATUS_INVALID_QUANTIZED_GEOMETRY,
                    "element count is not a non-zero whole number of quant blocks");
    if (!mul_ok(element_count / g.block_elements, g.bytes_per_block, out_packed_bytes))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "packed byte count overflows uint64");
    return KQ_STATUS_OK;
}

kq_status kq_quant_element_to_block(uint32_t type_id, uint64_t total_elements,
                                    uint64_t element_index, uint64_t *out_block_index,
                                    uint64_t *out_element_in_block, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out_block_index == nullptr || out_element_in_block == nullptr)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "block index and intra-block outputs are required");
    *out_block_index = 0;
    *out_element_in_block = 0;
    kq_quant_geometry g;
    uint64_t packed;
    kq_status st = kq_quant_geometry_for_type(type_id, &g, diagnostic);
    if (st == KQ_STATUS_OK) st = kq_quant_packed_size(type_id, total_elements, &packed, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (element_index >= total_elements)
        return fail(diagnostic, KQ_STATUS_SPAN_OUT_OF_RANGE, "logical element index is outside the tensor");
    *out_block_index = element_index / g.block_elements;
    *out_element_in_block = element_index % g.block_elements;
    return KQ_STATUS_OK;
}

kq_status kq_quant_range_to_blocks(uint32_t type_id, uint64_t total_elements,
                                   uint64_t element_offset, uint64_t element_count,
                                   kq_quant_block_span *out, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (out == nullptr || element_count == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "non-zero logical range and output span are required");
    std::memset(out, 0, sizeof(*out));
    kq_quant_geometry g;
    uint64_t packed, end;
    kq_status st = kq_quant_geometry_for_type(type_id, &g, diagnostic);
    if (st == KQ_STATUS_OK) st = kq_quant_packed_size(type_id, total_elements, &packed, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    if (!add_ok(element_offset, element_count, &end))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "logical element range overflows uint64");
    if (element_offset >= total_elements || end > total_elements)
        return fail(diagnostic, KQ_STATUS_SPAN_OUT_OF_RANGE, "logical element range is outside the tensor");
    uint64_t first = element_offset / g.block_elements;
    uint64_t last_excl = (end - 1) / g.block_elements + 1;
    out->requested_element_offset = element_offset;
    out->requested_element_count = element_count;
    out->first_block = first;
    out->block_count = last_excl - first;
    uint64_t block_elem_off, block_elem_end;
    if (!mul_ok(first, g.bytes_per_block, &out->physical_byte_offset) ||
        !mul_ok(out->block_count, g.bytes_per_block, &out->physical_byte_length) ||
        !mul_ok(first, g.block_elements, &block_elem_off) ||
        !mul_ok(last_excl, g.block_elements, &block_elem_end))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "quantized block span arithmetic overflows uint64");
    out->leading_elements = element_offset - block_elem_off;
    out->trailing_elements = block_elem_end - end;
    return KQ_STATUS_OK;
}

// GPU block dequantisation, bit-identical to src/kq_numeric.c:297-359.
kq_status kq_dequantize_blocks_f32(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                                   float *output, uint64_t output_capacity,
                                   uint64_t *output_count, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (output_count == nullptr || packed == nullptr || packed_bytes == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "packed input and output count are required");
    *output_count = 0;
    kq_quant_geometry g;
    kq_status st = kq_quant_geometry_for_type(type_id, &g, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    uint32_t e32, b32;
    if (!block_geometry(type_id, e32, b32))
        return fail(diagnostic, KQ_STATUS_UNSUPPORTED_TENSOR_TYPE,
                    "the B200 decoder supports F32, BF16, Q8_0, Q4_K and Q6_K");
    if (packed_bytes % g.bytes_per_block != 0)
        return fail(diagnostic, KQ_STATUS_MALFORMED_QUANTIZED_DATA, "packed bytes are not a bounded whole-block span");
    uint64_t blocks = packed_bytes / g.bytes_per_block, required, out_bytes;
    if (!mul_ok(blocks, g.block_elements, &required) || !mul_ok(required, 4, &out_bytes))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "decoded output count overflows");
    *output_count = required;
    if (output == nullptr || output_capacity < required)
        return fail(diagnostic, KQ_STATUS_BUFFER_TOO_SMALL, "decoded output capacity is too small");
    if (ranges_overlap(packed, packed_bytes, output, out_bytes))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "packed input and decoded output overlap");
    if (std::fegetround() != FE_TONEAREST)
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "round-to-nearest floating mode is required");
    DeviceContext *c;
    st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    const bool dev_in = is_device_pointer(packed), dev_out = is_device_pointer(output);
    void *ws = nullptr;
    size_t need = (dev_in ? 0 : Carve::round(packed_bytes)) + (dev_out ? 0 : Carve::round(out_bytes));
    st = c->workspace(need + 256, &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    const uint8_t *din = static_cast<const uint8_t *>(packed);
    float *dout = output;
    if (!dev_in) {
        uint8_t *p = cv.take<uint8_t>(packed_bytes);
        KQB_CUDA(cudaMemcpyAsync(p, packed, packed_bytes, cudaMemcpyHostToDevice, c->stream), diagnostic, "H2D");
        din = p;
    }
    if (!dev_out) dout = cv.take<float>(required);
    launch_dequantize(type_id, din, required, dout, c->stream);
    KQB_CUDA(cudaGetLastError(), diagnostic, "dequantize launch");
    if (!dev_out)
        KQB_CUDA(cudaMemcpyAsync(output, dout, out_bytes, cudaMemcpyDeviceToHost, c->stream), diagnostic, "D2H");
    KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "dequantize");
    // non-finite scales are malformed data (src/kq_numeric.c:212-216,235-239)
    if (type_id == KQ_GGUF_TYPE_Q8_0 || type_id == KQ_GGUF_TYPE_Q4_K || type_id == KQ_GGUF_TYPE_Q6_K) {
        const unsigned char *host = nullptr;
        std::vector<unsigned char> copy;
        if (dev_in) {
            copy.resize(packed_bytes);
            KQB_CUDA(cudaMemcpy(copy.data(), packed, packed_bytes, cudaMemcpyDeviceToHost), diagnostic, "scale check");
            host = copy.data();
        } else {
            host = static_cast<const unsigned char *>(packed);
        }
        for (uint64_t b = 0; b < blocks; ++b) {
            const unsigned char *blk = host + b * g.bytes_per_block;
            uint32_t offs[2] = {0, 2};
            int n = type_id == KQ_GGUF_TYPE_Q4_K ? 2 : 1;
            if (type_id == KQ_GGUF_TYPE_Q6_K) offs[0] = 208;
            for (int i = 0; i < n; ++i) {
                uint32_t h = blk[offs[i]] | (blk[offs[i] + 1] << 8);
                if (((h >> 10) & 0x1f) == 0x1f)
                    return fail(diagnostic, KQ_STATUS_MALFORMED_QUANTIZED_DATA, "quantized block scale is non-finite");
            }
        }
    }
    return KQ_STATUS_OK;
}

// GPU row dot in the reference's sequential order (src/kq_numeric.c:420-503).
kq_status kq_quantized_row_dot_f32(uint32_t type_id, const void *packed, uint64_t packed_bytes,
                                   const float *activation, uint64_t activation_count,
                                   float *output, kq_diagnostic *diagnostic) {
    kq_diagnostic_clear(diagnostic);
    if (packed == nullptr || activation == nullptr || output == nullptr || packed_bytes == 0 ||
        activation_count == 0)
        return fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT, "row-dot inputs and scalar output are required");
    kq_quant_geometry g;
    kq_status st = kq_quant_geometry_for_type(type_id, &g, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    uint32_t e32, b32;
    if (!block_geometry(type_id, e32, b32))
        return fail(diagnostic, KQ_STATUS_UNSUPPORTED_TENSOR_TYPE,
                    "the B200 decoder supports F32, BF16, Q8_0, Q4_K and Q6_K");
    if (packed_bytes % g.bytes_per_block != 0)
        return fail(diagnostic, KQ_STATUS_MALFORMED_QUANTIZED_DATA, "row is not a bounded whole-block span");
    uint64_t expected;
    if (!mul_ok(packed_bytes / g.bytes_per_block, g.block_elements, &expected))
        return fail(diagnostic, KQ_STATUS_ARITHMETIC_OVERFLOW, "row element count overflows");
    if (expected != activation_count)
        return fail(diagnostic, KQ_STATUS_DIMENSION_MISMATCH, "quantized row and activation lengths differ");
    if (ranges_overlap(packed, packed_bytes, output, 4) ||
        ranges_overlap(activation, activation_count * 4, output, 4))
        return fail(diagnostic, KQ_STATUS_ALIASING_VIOLATION, "row-dot scalar output overlaps an input");
    if (std::fegetround() != FE_TONEAREST)
        return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "round-to-nearest floating mode is required");
    DeviceContext *c;
    st = context(&c, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    std::lock_guard<std::recursive_mutex> lk(c->mu);
    void *ws = nullptr;
    st = c->workspace(Carve::round(packed_bytes) + Carve::round(activation_count * 4) + 512, &ws, diagnostic);
    if (st != KQ_STATUS_OK) return st;
    Carve cv(ws);
    const uint8_t *din = static_cast<const uint8_t *>(packed);
    const float *dx = activation;
    if (!is_device_pointer(packed)) {
        uint8_t *p = cv.take<uint8_t>(packed_bytes);
        KQB_CUDA(cudaMemcpyAsync(p, packed, packed_bytes, cudaMemcpyHostToDevice, c->stream), diagnostic, "H2D");
        din = p;
    }
    if (!is_device_pointer(activation)) {
        float *p = cv.take<float>(activation_count);
        KQB_CUDA(cudaMemcpyAsync(p, activation, activation_count * 4, cudaMemcpyHostToDevice, c->stream),
                 diagnostic, "H2D");
        dx = p;
    }
    float *dres = cv.take<float>(1);
    int *dstatus = cv.take<int>(1);
    launch_row_dot(type_id, din, expected, dx, dres, dstatus, c->stream);
    KQB_CUDA(cudaGetLastError(), diagnostic, "row-dot launch");
    float result = 0.0f;
    int status = 0;
    KQB_CUDA(cudaMemcpyAsync(&result, dres, 4, cudaMemcpyDeviceToHost, c->stream), diagnostic, "D2H");
    KQB_CUDA(cudaMemcpyAsync(&status, dstatus, 4, cudaMemcpyDeviceToHost, c->stream), diagnostic, "D2H");
    KQB_CUDA(cudaStreamSynchronize(c->stream), diagnostic, "row dot");
    if (status == 1) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "numeric primitive input must be finite");
    if (status == 2) return fail(diagnostic, KQ_STATUS_NUMERIC_DOMAIN, "row-dot produced a non-finite result");
    if (is_device_pointer(output)) {
        KQB_CUDA(cudaMemcpy(output, &result, 4, cudaMemcpyHostToDevice), diagnostic, "result store");
    } else {
        *output = result;
    }
    return KQ_STATUS_OK;
}

}  // extern "C"
