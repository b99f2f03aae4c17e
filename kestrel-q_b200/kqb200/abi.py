"""ctypes declarations of the B200 operator ABI (include/*.h).

Loads ``kestrel-q_b200/lib/libkqb200.so``; there is no fallback: a missing
library raises, and every compute entry point reports an error status when no
GPU is present.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libkqb200.so"

u32, u64, f32, vp = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p

# kq_status values used by the host code (include/kq_status.h)
OK = 0
INVALID_ARGUMENT = 1
OUT_OF_MEMORY = 2
UNSUPPORTED_TENSOR_TYPE = 12
ARITHMETIC_OVERFLOW = 13
LIMIT_EXCEEDED = 14
SPAN_OUT_OF_RANGE = 16
UNSUPPORTED_MODEL = 20
SEMANTIC_MAPPING_FAILED = 22
INVALID_QUANTIZED_GEOMETRY = 25
TENSOR_LAYOUT_MISMATCH = 27
BUFFER_TOO_SMALL = 32
MALFORMED_QUANTIZED_DATA = 38
NUMERIC_DOMAIN = 39
DIMENSION_MISMATCH = 40
ALIASING_VIOLATION = 41
INCOMPATIBLE_GDN = 42
INVALID_GDN_STATE = 43
INCOMPATIBLE_QSA = 44
INVALID_QSA_STATE = 45
INCOMPATIBLE_MOE = 46
INCOMPATIBLE_LAYER = 50
INVALID_LAYER_STATE = 51

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_BF16 = 0, 8, 12, 14, 30


class Diagnostic(C.Structure):
    _fields_ = [("status", C.c_int), ("message", C.c_char * 256)]

    def text(self) -> str:
        return self.message.decode(errors="replace")


class GdnDimensions(C.Structure):
    _fields_ = [("hidden_size", u32), ("key_head_count", u32), ("value_head_count", u32),
                ("key_head_dimension", u32), ("value_head_dimension", u32),
                ("conv_kernel_size", u32), ("rms_norm_epsilon", f32), ("activation_dtype", C.c_int)]


class QsaDimensions(C.Structure):
    _fields_ = [("hidden_size", u32), ("query_head_count", u32), ("key_value_head_count", u32),
                ("head_dimension", u32), ("index_query_head_count", u32),
                ("index_head_dimension", u32), ("block_size", u32), ("token_budget", u32),
                ("max_context", u32), ("rotary_dimension", u32), ("rms_norm_epsilon", f32),
                ("rope_theta", f32), ("activation_dtype", C.c_int)]


GDN_WEIGHT_FIELDS = ["a_log", "conv", "dt_bias", "alpha", "beta", "qkv", "gate", "norm", "output"]
QSA_WEIGHT_FIELDS = ["query", "key", "value", "output", "query_norm", "key_norm", "index_query",
                     "index_key", "index_query_norm", "index_key_norm"]


def _pair_fields(names):
    out = []
    for n in names:
        out += [(n, vp), (n + "_count", u64)]
    return out


MOE_WEIGHT_FIELDS = ["router", "routed_gate", "routed_up", "routed_down", "shared_gate", "shared_up",
                     "shared_down", "shared_gate_weight"]
MOE_TENSOR_FIELDS = ["router", "routed_down", "routed_gate_up", "shared_down", "shared_gate", "shared_up",
                     "shared_gate_weight"]


class MoeDimensions(C.Structure):   # include/kq_b200.h kq_moe_dimensions
    _fields_ = [("hidden_size", u32), ("expert_count", u32), ("top_k", u32), ("routed_intermediate_size", u32),
                ("shared_intermediate_size", u32), ("activation_dtype", C.c_int)]


class GdnWeightsF32(C.Structure):
    _fields_ = _pair_fields(GDN_WEIGHT_FIELDS)


class QsaWeightsF32(C.Structure):
    _fields_ = _pair_fields(QSA_WEIGHT_FIELDS)


class MoeWeightsF32(C.Structure):
    _fields_ = _pair_fields(MOE_WEIGHT_FIELDS)


class MoeExpertWeightsF32(C.Structure):
    _fields_ = _pair_fields(["gate", "up", "down"])


class MoeTensors(C.Structure):
    _fields_ = [(n, vp) for n in MOE_TENSOR_FIELDS]


GR_FIELDS = ["norm", "down", "up", "inject"]
LAYER_TENSOR_FIELDS = ["attention_inject", "attention_norm", "attention_down", "attention_up", "moe_inject",
                       "moe_norm", "moe_down", "moe_up"]


class LayerDimensions(C.Structure):   # include/kq_b200.h kq_layer_dimensions
    _fields_ = [("layer_id", u32), ("hidden_size", u32), ("branch_count", u32), ("gr_rank", u32),
                ("rms_epsilon", f32), ("family", C.c_int)]


class LayerGrWeightsF32(C.Structure):   # include/kq_layer.h kq_layer_gr_weights_f32
    _fields_ = _pair_fields(GR_FIELDS)


class LayerWeightsF32(C.Structure):   # include/kq_layer.h kq_layer_weights_f32
    _fields_ = [("attention_gr", LayerGrWeightsF32), ("moe_gr", LayerGrWeightsF32), ("gdn", vp), ("qsa", vp),
                ("moe", vp), ("ple_value", vp), ("ple_provider", vp)]


class LayerMetrics(C.Structure):   # include/kq_layer.h kq_layer_metrics
    _fields_ = [(n, u64) for n in ["elapsed_nanoseconds", "tokens_processed", "scratch_bytes", "gr_workspace_bytes",
                                   "transaction_staging_bytes", "qsa_selection_events", "qsa_candidate_blocks",
                                   "qsa_selected_blocks", "qsa_selected_tokens"]]


class LayerTensors(C.Structure):
    _fields_ = [(n, vp) for n in LAYER_TENSOR_FIELDS]


class GdnTensors(C.Structure):
    _fields_ = [(n, vp) for n in GDN_WEIGHT_FIELDS]


class QsaTensors(C.Structure):
    _fields_ = [(n, vp) for n in QSA_WEIGHT_FIELDS]


class QuantGeometry(C.Structure):
    _fields_ = [("type_id", u32), ("block_elements", u64), ("bytes_per_block", u64)]


class QuantBlockSpan(C.Structure):
    _fields_ = [("requested_element_offset", u64), ("requested_element_count", u64),
                ("first_block", u64), ("block_count", u64), ("physical_byte_offset", u64),
                ("physical_byte_length", u64), ("leading_elements", u64), ("trailing_elements", u64)]


class QsaSelection(C.Structure):
    _fields_ = [("token_index", u64), ("absolute_position", u64),
                ("candidate_block_ids", C.POINTER(u32)), ("candidate_scores", C.POINTER(f32)),
                ("candidate_count", u64), ("selected_block_ids", C.POINTER(u32)),
                ("selected_block_count", u64), ("selected_token_positions", C.POINTER(u32)),
                ("selected_token_count", u64), ("tail_count", u64)]


class GgufLayout(C.Structure):   # include/kq_b200.h kq_b200_gguf_layout
    _fields_ = [("gdn_key_heads", u32), ("gdn_value_repeat", u32), ("gdn_head_width", u32)]


class GdnCheckpoint(C.Structure):   # include/kq_gdn.h kq_gdn_checkpoint
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 4),
                ("values", C.POINTER(f32)), ("value_count", u64)]


class QsaCheckpoint(C.Structure):   # include/kq_qsa.h kq_qsa_checkpoint
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 3),
                ("values", C.POINTER(f32)), ("value_count", u64)]


class MoeRoute(C.Structure):   # include/kq_moe.h kq_moe_route
    _fields_ = [("token_index", u64), ("router_logits", C.POINTER(f32)), ("router_probabilities", C.POINTER(f32)),
                ("expert_count", u64), ("selected_expert_ids", C.POINTER(u32)), ("selected_weights", C.POINTER(f32)),
                ("selected_count", u32)]


class MoeCheckpoint(C.Structure):   # include/kq_moe.h kq_moe_checkpoint
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("expert_id", u32), ("top_k_position", u32),
                ("rank", u32), ("dimensions", u64 * 2), ("values", C.POINTER(f32)), ("value_count", u64)]


# int (*)(void *words, uint64_t count, void *cuda_stream, void *user)
EXCHANGE_FN = C.CFUNCTYPE(C.c_int, vp, u64, vp, vp)
SELECTION_OBSERVER = C.CFUNCTYPE(None, C.POINTER(QsaSelection), vp)
GDN_CHECKPOINT_OBSERVER = C.CFUNCTYPE(None, C.POINTER(GdnCheckpoint), vp)
QSA_CHECKPOINT_OBSERVER = C.CFUNCTYPE(None, C.POINTER(QsaCheckpoint), vp)
class LayerCheckpoint(C.Structure):   # include/kq_layer.h kq_layer_checkpoint
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 3),
                ("values", C.POINTER(f32)), ("value_count", u64)]


LAYER_CHECKPOINT_OBSERVER = C.CFUNCTYPE(None, C.POINTER(LayerCheckpoint), vp)
MOE_ROUTE_OBSERVER = C.CFUNCTYPE(None, C.POINTER(MoeRoute), vp)
MOE_CHECKPOINT_OBSERVER = C.CFUNCTYPE(None, C.POINTER(MoeCheckpoint), vp)


def checkpoint_collector():
    """(list, callback body): the body appends each checkpoint it sees as a
    dict (kind, token, rank, dims, values copied out of the library's buffer,
    which is valid only during the call)."""
    import numpy as np
    out = []

    def on_checkpoint(p, _user):
        c = p.contents
        vals = np.ctypeslib.as_array(c.values, (c.value_count,)).copy() if c.value_count else np.zeros(0, np.float32)
        out.append({"kind": int(c.kind), "token": int(c.token_index), "rank": int(c.rank),
                    "dims": tuple(int(c.dimensions[i]) for i in range(c.rank)), "values": vals})

    return out, on_checkpoint

_SIGNATURES = {
    "kq_status_string": (C.c_char_p, [C.c_int]),
    "kq_diagnostic_clear": (None, [vp]),
    "kq_quant_geometry_for_type": (C.c_int, [u32, C.POINTER(QuantGeometry), vp]),
    "kq_quant_packed_size": (C.c_int, [u32, u64, C.POINTER(u64), vp]),
    "kq_quant_element_to_block": (C.c_int, [u32, u64, u64, C.POINTER(u64), C.POINTER(u64), vp]),
    "kq_quant_range_to_blocks": (C.c_int, [u32, u64, u64, u64, C.POINTER(QuantBlockSpan), vp]),
    "kq_dequantize_blocks_f32": (C.c_int, [u32, vp, u64, vp, u64, C.POINTER(u64), vp]),
    "kq_quantized_row_dot_f32": (C.c_int, [u32, vp, u64, vp, u64, vp, vp]),
    "kq_b200_set_device": (C.c_int, [C.c_int, vp]),
    "kq_b200_set_stream": (C.c_int, [vp, vp]),
    "kq_b200_get_stream": (vp, []),
    "kq_b200_synchronize": (C.c_int, [vp]),
    "kq_b200_kernel_launch_count": (u64, []),
    "kq_b200_provider_create": (C.c_int, [C.c_int, C.POINTER(vp), vp]),
    "kq_weight_provider_close": (None, [vp]),
    "kq_weight_provider_open": (C.c_int, [vp, vp, u64, C.POINTER(vp), vp]),
    "kq_b200_provider_add_matrix": (C.c_int, [vp, C.c_char_p, C.c_int, u32, u64, u64, vp, u64,
                                              C.POINTER(vp), vp]),
    "kq_b200_provider_add_vector_f32": (C.c_int, [vp, C.c_char_p, C.c_int, vp, u64, C.POINTER(vp), vp]),
    "kq_b200_provider_add_gguf_matrix": (C.c_int, [vp, C.c_char_p, C.c_int, u32, u64, u64, vp, u64,
                                                   C.POINTER(GgufLayout), C.POINTER(vp), vp]),
    "kq_b200_provider_add_gguf_vector_f32": (C.c_int, [vp, C.c_char_p, C.c_int, vp, u64, C.POINTER(GgufLayout),
                                                       C.POINTER(vp), vp]),
    "kq_b200_provider_add_index_qk": (C.c_int, [vp, C.c_char_p, u32, u64, u64, u64, vp, u64, vp, u64,
                                                C.POINTER(vp), vp]),
    "kq_weight_provider_linear_f32": (C.c_int, [vp, vp, C.c_int, u32, u64, u64, vp, vp, u64, vp, u64, vp]),
    "kq_weight_provider_vector_f32": (C.c_int, [vp, vp, u64, vp, u64, vp, u64, vp]),
    "kq_b200_provider_linear_batch_f32": (C.c_int, [vp, vp, u64, u64, vp, u32, vp, vp]),
    "kq_b200_provider_linear_batch_f32_static": (C.c_int, [vp, vp, u64, u64, vp, u32, vp, vp, vp]),
    "kq_b200_profile_kernel": (None, [C.c_char_p]),
    "kq_b200_profile_read": (None, [C.POINTER(u64), C.POINTER(C.c_double)]),
    "kq_gdn_test_config_create": (C.c_int, [C.POINTER(GdnDimensions), C.POINTER(vp), vp]),
    "kq_gdn_config_create": (C.c_int, [vp, u32, C.POINTER(vp), vp]),
    "kq_gdn_config_close": (None, [vp]),
    "kq_b200_gdn_config_bind": (C.c_int, [vp, vp, C.POINTER(GdnTensors), vp]),
    "kq_gdn_config_scratch_bytes": (u64, [vp]),
    "kq_gdn_config_token_scratch_bytes": (u64, [vp]),
    "kq_gdn_config_dequant_scratch_bytes": (u64, [vp]),
    "kq_gdn_config_recurrent_element_count": (u64, [vp]),
    "kq_gdn_config_conv_state_element_count": (u64, [vp]),
    "kq_gdn_config_conv_channel_count": (u32, [vp]),
    "kq_gdn_config_hidden_size": (u32, [vp]),
    "kq_gdn_state_create": (C.c_int, [vp, C.POINTER(vp), vp]),
    "kq_gdn_state_close": (None, [vp]),
    "kq_gdn_state_reset": (C.c_int, [vp, vp]),
    "kq_gdn_state_export_f32": (C.c_int, [vp, vp, u64, vp, u64, C.POINTER(C.c_int), vp]),
    "kq_gdn_state_import_f32": (C.c_int, [vp, vp, u64, vp, u64, C.c_int, vp]),
    "kq_gdn_prefill_f32": (C.c_int, [vp, C.POINTER(GdnWeightsF32), vp, u64, vp, vp, u64, vp, vp, u64,
                                     vp, vp, vp]),
    "kq_gdn_decode_f32": (C.c_int, [vp, C.POINTER(GdnWeightsF32), vp, vp, u64, vp, vp, u64, vp, vp, vp]),
    "kq_gdn_execute_quantized": (C.c_int, [vp, vp, vp, u64, vp, vp, u64, vp, vp, u64, vp, u64, vp, vp, vp]),
    "kq_b200_gdn_decode_batch": (C.c_int, [vp, C.POINTER(vp), u32, vp, vp, vp]),
    "kq_qsa_test_config_create": (C.c_int, [C.POINTER(QsaDimensions), C.POINTER(vp), vp]),
    "kq_qsa_config_close": (None, [vp]),
    "kq_b200_qsa_config_bind": (C.c_int, [vp, vp, C.POINTER(QsaTensors), vp]),
    "kq_qsa_config_block_selection_limit": (u32, [vp]),
    "kq_qsa_config_semantic_state_bytes_per_token": (u64, [vp]),
    "kq_qsa_state_create": (C.c_int, [vp, u64, C.POINTER(vp), vp]),
    "kq_qsa_state_close": (None, [vp]),
    "kq_qsa_state_reset": (C.c_int, [vp, vp]),
    "kq_qsa_state_length": (u64, [vp]),
    "kq_qsa_state_capacity": (u64, [vp]),
    "kq_qsa_state_export_f32": (C.c_int, [vp, vp, u64, vp, u64, vp, u64, C.POINTER(u64), vp]),
    "kq_qsa_state_import_f32": (C.c_int, [vp, vp, u64, vp, u64, vp, u64, u64, vp]),
    "kq_qsa_required_scratch_bytes": (C.c_int, [vp, vp, u64, C.POINTER(u64), vp]),
    "kq_qsa_select_blocks_f32": (C.c_int, [vp, u64, u64, vp, u64, C.POINTER(u64), vp]),
    "kq_qsa_prefill_f32": (C.c_int, [vp, C.POINTER(QsaWeightsF32), vp, u64, vp, u64, vp, vp, u64,
                                     SELECTION_OBSERVER, vp, vp, vp]),
    "kq_qsa_decode_f32": (C.c_int, [vp, C.POINTER(QsaWeightsF32), vp, vp, u64, vp, vp, u64,
                                    SELECTION_OBSERVER, vp, vp, vp]),
    "kq_qsa_execute_quantized": (C.c_int, [vp, vp, vp, u64, vp, u64, vp, vp, u64, vp, u64,
                                           SELECTION_OBSERVER, vp, vp, vp]),
    "kq_b200_qsa_decode_batch": (C.c_int, [vp, C.POINTER(vp), u32, vp, vp, vp]),
    "kq_b200_gdn_prefill_async": (C.c_int, [vp, vp, vp, u64, vp, vp]),
    "kq_b200_qsa_prefill_async": (C.c_int, [vp, vp, vp, u64, vp, vp]),
    "kq_b200_qsa_prefill_sharded_async": (C.c_int, [vp, vp, vp, u64, vp, u32, u32, vp, vp, vp]),
    "kq_b200_qsa_prefill_split_async": (C.c_int, [vp, vp, vp, u64, vp, u32, u32, u32, u32, vp, vp, vp]),
    "kq_b200_provider_add_expert_stack": (C.c_int, [vp, C.c_char_p, C.c_int, u32, u32, u64, u64, vp, u64,
                                                    C.POINTER(vp), vp]),
    "kq_b200_provider_add_expert_gate_up": (C.c_int, [vp, C.c_char_p, u32, u32, u64, u64, vp, u64, vp, u64,
                                                      C.POINTER(vp), vp]),
    "kq_moe_test_config_create": (C.c_int, [C.POINTER(MoeDimensions), C.POINTER(vp), vp]),
    "kq_moe_config_create": (C.c_int, [vp, u32, C.POINTER(vp), vp]),
    "kq_moe_config_close": (None, [vp]),
    "kq_b200_moe_config_bind": (C.c_int, [vp, vp, C.POINTER(MoeTensors), vp]),
    "kq_moe_config_scratch_bytes": (u64, [vp]),
    "kq_moe_config_one_expert_workspace_bytes": (u64, [vp]),
    "kq_moe_config_router_workspace_bytes": (u64, [vp]),
    "kq_moe_config_top_k_workspace_bytes": (u64, [vp]),
    "kq_moe_config_routed_accumulation_workspace_bytes": (u64, [vp]),
    "kq_moe_config_shared_workspace_bytes": (u64, [vp]),
    "kq_moe_config_owned_bytes": (u64, [vp]),
    "kq_moe_config_layer_id": (u32, [vp]),
    "kq_moe_config_top_k": (u32, [vp]),
    "kq_moe_config_expert_count": (u32, [vp]),
    "kq_moe_config_activation_dtype": (C.c_int, [vp]),
    "kq_moe_route_f32": (C.c_int, [vp, vp, u64, vp, vp, u64, vp, u64, vp, u64, vp, u64, vp]),
    "kq_moe_execute_routed_expert_f32": (C.c_int, [vp, C.POINTER(MoeExpertWeightsF32), u32, vp, vp, u64, vp, u64,
                                                   vp]),
    "kq_moe_execute_f32": (C.c_int, [vp, C.POINTER(MoeWeightsF32), vp, u64, vp, u64, vp, u64, MOE_ROUTE_OBSERVER,
                                     MOE_CHECKPOINT_OBSERVER, vp, vp]),
    "kq_moe_execute_quantized": (C.c_int, [vp, vp, vp, u64, vp, u64, vp, u64, vp, u64, MOE_ROUTE_OBSERVER,
                                           MOE_CHECKPOINT_OBSERVER, vp, vp]),
    "kq_b200_moe_execute_async": (C.c_int, [vp, vp, u64, vp, vp]),
    "kq_moe_checkpoint_kind_name": (C.c_char_p, [C.c_int]),
    "kq_layer_test_config_create": (C.c_int, [C.POINTER(LayerDimensions), vp, vp, vp, vp, vp, C.POINTER(vp), vp]),
    "kq_layer_config_create": (C.c_int, [vp, u32, C.POINTER(vp), vp]),
    "kq_layer_config_close": (None, [vp]),
    "kq_layer_config_family": (C.c_int, [vp]),
    "kq_layer_config_gr_workspace_bytes": (u64, [vp]),
    "kq_layer_config_persistent_semantic_bytes": (u64, [vp, u64]),
    "kq_layer_config_owned_bytes": (u64, [vp]),
    "kq_b200_layer_config_bind": (C.c_int, [vp, vp, C.POINTER(LayerTensors), vp]),
    "kq_layer_state_create": (C.c_int, [vp, u64, C.POINTER(vp), vp]),
    "kq_layer_state_close": (None, [vp]),
    "kq_layer_state_reset": (C.c_int, [vp, vp]),
    "kq_layer_state_position": (u64, [vp]),
    "kq_layer_state_owned_bytes": (u64, [vp]),
    "kq_layer_state_rollback_last": (C.c_int, [vp, u64, vp]),
    "kq_layer_required_scratch_bytes": (C.c_int, [vp, vp, u64, C.POINTER(u64), vp]),
    "kq_layer_required_quantized_scratch_bytes": (C.c_int, [vp, vp, u64, C.POINTER(u64), vp]),
    "kq_layer_prefill_f32": (C.c_int, [vp, C.POINTER(LayerWeightsF32), vp, vp, u64, vp, vp, u64, vp, vp, u64,
                                       LAYER_CHECKPOINT_OBSERVER, vp, vp, vp]),
    "kq_layer_decode_f32": (C.c_int, [vp, C.POINTER(LayerWeightsF32), vp, u32, vp, u64, vp, vp, u64,
                                      LAYER_CHECKPOINT_OBSERVER, vp, vp, vp]),
    "kq_layer_prefill_quantized_f32": (C.c_int, [vp, vp, vp, vp, u64, vp, vp, u64, vp, vp, u64,
                                                 LAYER_CHECKPOINT_OBSERVER, vp, vp, vp]),
    "kq_layer_decode_quantized_f32": (C.c_int, [vp, vp, vp, u32, vp, u64, vp, vp, u64, LAYER_CHECKPOINT_OBSERVER,
                                                vp, vp, vp]),
    "kq_b200_layer_decode_batch": (C.c_int, [vp, C.POINTER(vp), u32, vp, vp, vp]),
    "kq_b200_layer_prefill_async": (C.c_int, [vp, vp, vp, u64, vp, vp]),
    "kq_layer_family_name": (C.c_char_p, [C.c_int]),
    "kq_layer_checkpoint_kind_name": (C.c_char_p, [C.c_int]),
    "kq_gdn_checkpoint_kind_name": (C.c_char_p, [C.c_int]),
    "kq_qsa_checkpoint_kind_name": (C.c_char_p, [C.c_int]),
}

_lib = None


def lib() -> C.CDLL:
    """Loads the library (raises if it was not built: there is no fallback)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run kestrel-q_b200/build.py "
                               "(the B200 operators have no CPU fallback)")
        handle = C.CDLL(str(LIB_PATH))
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(handle, name)
            fn.restype = res
            fn.argtypes = args
        _lib = handle
    return _lib


class KQError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(f"kq status {status}: {message}")
        self.status = status
        self.message = message


def check(status: int, diag: Diagnostic) -> None:
    if status != OK:
        raise KQError(status, diag.text())
