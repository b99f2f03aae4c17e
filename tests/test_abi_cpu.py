"""C-ABI library checks that need no GPU: it loads, exports every entry point
the headers in include/ declare, and its host-only entry points (status text,
block geometry, argument validation) behave like the reference's
(tests/numeric_test.c, tests/tensor_view_test.c of Kestrel-Q)."""
import ctypes as C
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in sorted((REPO / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"typedef[^;]*;", "", text)
        for m in re.finditer(r"\b(kq_\w+)\s*\(", text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_function(kq):
    lib = kq.lib()
    names = declared_functions()
    assert len(names) > 80
    missing = [n for n in sorted(names) if not hasattr(lib, n)]
    assert not missing, missing


def test_only_abi_symbols_are_exported(kq):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(kq.abi.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = [l.split()[-1] for l in out.splitlines() if " T " in l]
    assert exported and all(e.startswith("kq_") for e in exported)


def test_status_strings(kq):
    lib = kq.lib()
    assert lib.kq_status_string(0) == b"ok"
    assert lib.kq_status_string(39) == b"invalid numeric domain"
    assert lib.kq_status_string(32) == b"output buffer too small"
    assert lib.kq_status_string(9999) == b"unknown status"


@pytest.mark.parametrize("type_id,elems,nbytes", [(0, 1, 4), (30, 1, 2), (8, 32, 34), (12, 256, 144),
                                                   (14, 256, 210), (13, 256, 176), (7, 32, 24), (20, 32, 18)])
def test_quant_geometry(kq, type_id, elems, nbytes):
    g = kq.abi.QuantGeometry()
    d = kq.abi.Diagnostic()
    assert kq.lib().kq_quant_geometry_for_type(type_id, C.byref(g), C.byref(d)) == 0
    assert (g.type_id, g.block_elements, g.bytes_per_block) == (type_id, elems, nbytes)


def test_quant_geometry_rejects_unknown(kq):
    g = kq.abi.QuantGeometry()
    d = kq.abi.Diagnostic()
    assert kq.lib().kq_quant_geometry_for_type(3, C.byref(g), C.byref(d)) == kq.abi.UNSUPPORTED_TENSOR_TYPE
    assert kq.lib().kq_quant_geometry_for_type(0, None, C.byref(d)) == kq.abi.INVALID_ARGUMENT


def test_packed_size_and_spans(kq):
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    out = C.c_uint64()
    assert lib.kq_quant_packed_size(14, 2048, C.byref(out), C.byref(d)) == 0 and out.value == 8 * 210
    assert lib.kq_quant_packed_size(12, 100, C.byref(out), C.byref(d)) == abi.INVALID_QUANTIZED_GEOMETRY
    b, e = C.c_uint64(), C.c_uint64()
    assert lib.kq_quant_element_to_block(8, 128, 70, C.byref(b), C.byref(e), C.byref(d)) == 0
    assert (b.value, e.value) == (2, 6)
    assert lib.kq_quant_element_to_block(8, 128, 128, C.byref(b), C.byref(e), C.byref(d)) == abi.SPAN_OUT_OF_RANGE
    span = abi.QuantBlockSpan()
    assert lib.kq_quant_range_to_blocks(12, 1024, 300, 300, C.byref(span), C.byref(d)) == 0
    assert (span.first_block, span.block_count, span.physical_byte_offset, span.physical_byte_length,
            span.leading_elements, span.trailing_elements) == (1, 2, 144, 288, 44, 168)
    assert lib.kq_quant_range_to_blocks(12, 1024, 1000, 100, C.byref(span), C.byref(d)) == abi.SPAN_OUT_OF_RANGE


def test_model_entry_points_report_unsupported(kq):
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    out = C.c_void_p(1)
    assert lib.kq_gdn_config_create(None, 0, C.byref(out), C.byref(d)) == abi.UNSUPPORTED_MODEL
    assert out.value is None
    assert lib.kq_weight_provider_open(None, None, 0, C.byref(out), C.byref(d)) == abi.UNSUPPORTED_MODEL


def test_gdn_config_geometry_matches_reference_accounting(kq):
    """Config sizes of tests/gdn_test.c:336-338 (target geometry) and the
    scratch formula of src/kq_gdn.c:184-219."""
    lib, abi = kq.lib(), kq.abi
    dims = abi.GdnDimensions(2560, 16, 48, 128, 128, 4, 1e-6, 0)
    cfg = C.c_void_p()
    d = abi.Diagnostic()
    assert lib.kq_gdn_test_config_create(C.byref(dims), C.byref(cfg), C.byref(d)) == 0
    try:
        assert lib.kq_gdn_config_recurrent_element_count(cfg) == 786432
        assert lib.kq_gdn_config_conv_state_element_count(cfg) == 40960
        C_, V, Hv, H, rk = 10240, 6144, 48, 2560, 48 * 128
        tok = H + C_ + V + Hv + Hv + C_ + rk + rk + V + Hv + Hv + V + V + V + V + H
        assert lib.kq_gdn_config_token_scratch_bytes(cfg) == tok * 4
        assert lib.kq_gdn_config_scratch_bytes(cfg) == (tok + 786432 + 40960) * 4
        assert lib.kq_gdn_config_dequant_scratch_bytes(cfg) == 1024
    finally:
        lib.kq_gdn_config_close(cfg)
    bad = abi.GdnDimensions(8, 2, 3, 4, 4, 4, 1e-6, 0)   # value heads not a multiple of key heads
    assert lib.kq_gdn_test_config_create(C.byref(bad), C.byref(cfg), C.byref(d)) == abi.INCOMPATIBLE_GDN
    bad = abi.GdnDimensions(8, 2, 4, 4, 4, 3, 1e-6, 0)   # kernel must be 4
    assert lib.kq_gdn_test_config_create(C.byref(bad), C.byref(cfg), C.byref(d)) == abi.INCOMPATIBLE_GDN


def test_qsa_config_geometry(kq):
    lib, abi = kq.lib(), kq.abi
    dims = abi.QsaDimensions(2048, 16, 2, 256, 4, 128, 4, 2048, 262144, 64, 1e-6, 1e7, 0)
    cfg = C.c_void_p()
    d = abi.Diagnostic()
    assert lib.kq_qsa_test_config_create(C.byref(dims), C.byref(cfg), C.byref(d)) == 0
    try:
        assert lib.kq_qsa_config_block_selection_limit(cfg) == 512
        # (2 * 2 * 256 + 128) * 4 bytes per token (F32 descriptor)
        assert lib.kq_qsa_config_semantic_state_bytes_per_token(cfg) == (1024 + 128) * 4
    finally:
        lib.kq_qsa_config_close(cfg)
    bad = abi.QsaDimensions(8, 2, 1, 4, 2, 4, 4, 6, 16, 2, 1e-6, 1e7, 0)   # budget % block != 0
    assert lib.kq_qsa_test_config_create(C.byref(bad), C.byref(cfg), C.byref(d)) == abi.INCOMPATIBLE_QSA


def test_selection_helper_tie_order(kq):
    """kq_qsa_select_blocks_f32: (score desc, id asc), tests/qsa_test.c:203-209."""
    import numpy as np
    lib, abi = kq.lib(), kq.abi
    s = np.array([0.5, 1.0, 1.0, -0.0, 0.0, 2.0], np.float32)
    out = np.zeros(4, np.uint32)
    n = C.c_uint64()
    d = abi.Diagnostic()
    assert lib.kq_qsa_select_blocks_f32(s.ctypes.data, s.size, 4, out.ctypes.data, 4, C.byref(n), C.byref(d)) == 0
    assert n.value == 4 and list(out) == [5, 1, 2, 0]
    assert lib.kq_qsa_select_blocks_f32(s.ctypes.data, s.size, 4, out.ctypes.data, 3, C.byref(n),
                                        C.byref(d)) == abi.BUFFER_TOO_SMALL
    s[2] = np.nan
    assert lib.kq_qsa_select_blocks_f32(s.ctypes.data, s.size, 4, out.ctypes.data, 4, C.byref(n),
                                        C.byref(d)) == abi.NUMERIC_DOMAIN


def test_compute_entry_points_fail_loudly_without_gpu(kq):
    from conftest import HAS_GPU
    if HAS_GPU:
        pytest.skip("GPU present")
    lib, abi = kq.lib(), kq.abi
    p = C.c_void_p()
    d = abi.Diagnostic()
    st = lib.kq_b200_provider_create(0, C.byref(p), C.byref(d))
    assert st != 0 and p.value is None


def test_prefill_entry_points_validate_before_any_device_work(kq):
    """The device prefill entry points reject bad arguments on the host, with
    the reference's status codes, before touching a device."""
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    exch = abi.EXCHANGE_FN(lambda p, n, s, u: 0)
    # no config / state
    assert lib.kq_b200_gdn_prefill_async(None, None, None, 16, None, C.byref(d)) == abi.INVALID_ARGUMENT
    assert lib.kq_b200_qsa_prefill_async(None, None, None, 16, None, C.byref(d)) == abi.INVALID_ARGUMENT
    # rank outside the world, a world without an exchange, a token part outside its parts
    assert lib.kq_b200_qsa_prefill_split_async(None, None, None, 16, None, 2, 2, 0, 1, exch, None,
                                               C.byref(d)) == abi.INVALID_ARGUMENT
    assert lib.kq_b200_qsa_prefill_split_async(None, None, None, 16, None, 0, 2, 0, 1, None, None,
                                               C.byref(d)) == abi.INVALID_ARGUMENT
    assert lib.kq_b200_qsa_prefill_split_async(None, None, None, 16, None, 0, 2, 2, 2, exch, None,
                                               C.byref(d)) == abi.INVALID_ARGUMENT
    assert lib.kq_b200_qsa_prefill_split_async(None, None, None, 16, None, 0, 1, 0, 2, exch, None,
                                               C.byref(d)) == abi.INVALID_ARGUMENT
    assert b"token_part" in d.message or b"rank" in d.message or b"valid" in d.message


def test_moe_config_matches_reference_accounting(kq, oracle):
    """MoE config sizes and validation against the compiled reference
    (kq_moe_workspace_sizes, src/kq_moe.c:83-140): the target geometry, the
    golden tier configs, and rejected dimensions with the same status."""
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    getters = ["scratch_bytes", "one_expert_workspace_bytes", "router_workspace_bytes", "top_k_workspace_bytes",
               "routed_accumulation_workspace_bytes", "shared_workspace_bytes"]
    cases = [(2560, 512, 10, 640, 640, 0), (6, 4, 2, 4, 4, 0), (4, 512, 10, 2, 2, 0), (2560, 512, 10, 640, 640, 1)]
    have_ref = oracle.ref_available()
    for dims in cases:
        cfg = C.c_void_p()
        assert lib.kq_moe_test_config_create(C.byref(abi.MoeDimensions(*dims)), C.byref(cfg), C.byref(d)) == 0
        try:
            assert lib.kq_moe_config_top_k(cfg) == dims[2]
            assert lib.kq_moe_config_activation_dtype(cfg) == dims[5]
            assert lib.kq_moe_config_layer_id(cfg) == 0xFFFFFFFF
            mine = [getattr(lib, "kq_moe_config_" + g)(cfg) for g in getters]
        finally:
            lib.kq_moe_config_close(cfg)
        if have_ref:
            L = oracle.ref()
            rc = C.c_void_p()
            assert L.kq_moe_test_config_create(C.byref(oracle._RefMoeDims(*dims)), C.byref(rc), C.byref(d)) == 0
            try:
                for g in getters:
                    getattr(L, "kq_moe_config_" + g).restype = C.c_uint64
                ref = [getattr(L, "kq_moe_config_" + g)(rc) for g in getters]
            finally:
                L.kq_moe_config_close(rc)
            assert mine == ref, dims
    cfg = C.c_void_p()
    for bad in [(0, 4, 2, 4, 4, 0), (6, 4, 5, 4, 4, 0), (6, 4, 0, 4, 4, 0), (6, 4, 2, 0, 4, 0), (6, 4, 2, 4, 0, 0),
                (6, 4, 2, 4, 4, 7)]:
        assert lib.kq_moe_test_config_create(C.byref(abi.MoeDimensions(*bad)), C.byref(cfg),
                                             C.byref(d)) == abi.INCOMPATIBLE_MOE, bad
    # B200 limits
    assert lib.kq_moe_test_config_create(C.byref(abi.MoeDimensions(8, 64, 33, 4, 4, 0)), C.byref(cfg),
                                         C.byref(d)) == abi.INCOMPATIBLE_MOE
    assert lib.kq_moe_config_create(None, 0, C.byref(cfg), C.byref(d)) == abi.UNSUPPORTED_MODEL


def test_moe_entry_points_validate_before_any_device_work(kq):
    """kq_moe_execute_* status codes of src/kq_moe_qwen38.c:619-660,882-899
    for arguments the host rejects."""
    import numpy as np
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    cfg = C.c_void_p()
    assert lib.kq_moe_test_config_create(C.byref(abi.MoeDimensions(6, 4, 2, 4, 4, 0)), C.byref(cfg), C.byref(d)) == 0
    bf = C.c_void_p()
    assert lib.kq_moe_test_config_create(C.byref(abi.MoeDimensions(6, 4, 2, 4, 4, 1)), C.byref(bf), C.byref(d)) == 0
    try:
        x = np.zeros((2, 6), np.float32)
        y = np.zeros((2, 6), np.float32)
        sb = lib.kq_moe_config_scratch_bytes(cfg)
        scratch = np.zeros(sb // 4 + 1, np.float32)
        w = abi.MoeWeightsF32()
        none_r, none_c = abi.MOE_ROUTE_OBSERVER(), abi.MOE_CHECKPOINT_OBSERVER()
        args = lambda c, wt, T, cap, sbytes: (c, wt, x.ctypes.data, T, y.ctypes.data, cap, scratch.ctypes.data, sbytes,
                                              none_r, none_c, None, C.byref(d))
        assert lib.kq_moe_execute_f32(*args(cfg, None, 2, 12, sb)) == abi.INVALID_ARGUMENT
        assert lib.kq_moe_execute_f32(*args(bf, C.byref(w), 2, 12, sb)) == abi.INCOMPATIBLE_MOE
        assert lib.kq_moe_execute_f32(*args(cfg, C.byref(w), 0, 12, sb)) == abi.LIMIT_EXCEEDED
        assert lib.kq_moe_execute_f32(*args(cfg, C.byref(w), 2, 11, sb)) == abi.BUFFER_TOO_SMALL
        assert lib.kq_moe_execute_f32(*args(cfg, C.byref(w), 2, 12, sb - 1)) == abi.BUFFER_TOO_SMALL
        assert lib.kq_moe_execute_f32(*args(cfg, C.byref(w), 2, 12, sb)) == abi.DIMENSION_MISMATCH
        x[1, 3] = np.inf
        assert lib.kq_moe_execute_f32(*args(cfg, C.byref(w), 2, 12, sb)) == abi.NUMERIC_DOMAIN
        ws = np.zeros(100, np.float32)
        assert lib.kq_moe_execute_quantized(cfg, None, x.ctypes.data, 2, y.ctypes.data, 12, scratch.ctypes.data, sb,
                                            ws.ctypes.data, ws.nbytes, none_r, none_c, None,
                                            C.byref(d)) == abi.BUFFER_TOO_SMALL
    finally:
        lib.kq_moe_config_close(cfg)
        lib.kq_moe_config_close(bf)


def test_layer_config_matches_reference_accounting(kq, oracle):
    """kq_layer_test_config_create checks and sizes against the compiled
    reference (src/kq_layer.c:220-262,294-318): the gated-residual workspace
    and persistent-state bytes of the reference's reduced fixture, argument
    and geometry failures, and the PLE_GDN family refused."""
    import ctypes as Cx
    lib, abi = kq.lib(), kq.abi
    d = abi.Diagnostic()
    gdn, moe, lay = Cx.c_void_p(), Cx.c_void_p(), Cx.c_void_p()
    assert lib.kq_gdn_test_config_create(Cx.byref(abi.GdnDimensions(8, 2, 4, 4, 4, 4, 1e-6, 0)), Cx.byref(gdn),
                                         Cx.byref(d)) == 0
    assert lib.kq_moe_test_config_create(Cx.byref(abi.MoeDimensions(8, 4, 2, 4, 4, 0)), Cx.byref(moe),
                                         Cx.byref(d)) == 0
    try:
        ld = abi.LayerDimensions(0, 8, 4, 4, 1e-6, 1)
        assert lib.kq_layer_test_config_create(Cx.byref(ld), gdn, None, moe, None, None, Cx.byref(lay),
                                               Cx.byref(d)) == 0
        mine = (lib.kq_layer_config_gr_workspace_bytes(lay), lib.kq_layer_config_persistent_semantic_bytes(lay, 16))
        assert lib.kq_layer_config_family(lay) == 1
        lib.kq_layer_config_close(lay)
        if oracle.ref_available():
            L = oracle.ref()
            rg, rm, rl = Cx.c_void_p(), Cx.c_void_p(), Cx.c_void_p()
            assert L.kq_gdn_test_config_create(Cx.byref(oracle._RefGdnDims(8, 2, 4, 4, 4, 4, 1e-6, 0)),
                                               Cx.byref(rg), Cx.byref(d)) == 0
            assert L.kq_moe_test_config_create(Cx.byref(oracle._RefMoeDims(8, 4, 2, 4, 4, 0)), Cx.byref(rm),
                                               Cx.byref(d)) == 0
            assert L.kq_layer_test_config_create(Cx.byref(oracle._RefLayerDims(0, 8, 4, 4, 1e-6, 1)), rg, None, rm,
                                                 None, None, Cx.byref(rl), Cx.byref(d)) == 0
            L.kq_layer_config_gr_workspace_bytes.restype = Cx.c_uint64
            L.kq_layer_config_persistent_semantic_bytes.restype = Cx.c_uint64
            ref = (L.kq_layer_config_gr_workspace_bytes(rl),
                   L.kq_layer_config_persistent_semantic_bytes(rl, Cx.c_uint64(16)))
            L.kq_layer_config_close(rl)
            L.kq_moe_config_close(rm)
            L.kq_gdn_config_close(rg)
            assert mine == ref
        bad = abi.LayerDimensions(0, 0, 4, 4, 1e-6, 1)
        assert lib.kq_layer_test_config_create(Cx.byref(bad), gdn, None, moe, None, None, Cx.byref(lay),
                                               Cx.byref(d)) == abi.INVALID_ARGUMENT
        wrong = abi.LayerDimensions(0, 16, 4, 4, 1e-6, 1)   # sub-configs of hidden 8
        assert lib.kq_layer_test_config_create(Cx.byref(wrong), gdn, None, moe, None, None, Cx.byref(lay),
                                               Cx.byref(d)) == abi.INCOMPATIBLE_LAYER
        ple = abi.LayerDimensions(1, 8, 4, 4, 1e-6, 3)
        assert lib.kq_layer_test_config_create(Cx.byref(ple), gdn, None, moe, None, None, Cx.byref(lay),
                                               Cx.byref(d)) == abi.INCOMPATIBLE_LAYER
        assert lib.kq_layer_config_create(None, 0, Cx.byref(lay), Cx.byref(d)) == abi.UNSUPPORTED_MODEL
        assert lib.kq_layer_family_name(3) == b"PLE_GDN"
    finally:
        lib.kq_moe_config_close(moe)
        lib.kq_gdn_config_close(gdn)
