"""BF16 activation descriptors: the B200 library against the compiled
reference on the same calls.

The reference accepts activation dtype BF16 in both configs
(src/kq_gdn.c:109-122, src/kq_qsa.c:80-93), stores the GDN convolution
history and the QSA key/value/raw caches as BF16 (round to nearest even on
import, widening on export; src/kq_gdn.c:599-701, src/kq_qsa.c:513-620),
keeps the GDN recurrent state in F32, and refuses F32 execution on a BF16
config (src/kq_gdn_qwen38.c:393-397, src/kq_qsa_qwen38.c:415-418).  Every
exported bit and every status must match.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

KQ_STATUS_INCOMPATIBLE_GDN = 42


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def state_values(rng, n):
    """Random F32 values plus exact BF16 ties (odd and even upper halves) so
    that round-to-nearest-even is exercised in both directions."""
    v = rng.standard_normal(n).astype(np.float32) * 3
    u = v.view(np.uint32).copy()
    u[::7] = (u[::7] & 0xFFFF0000) | 0x8000
    return u.view(np.float32)


@pytest.mark.parametrize("dtype", [0, 1])
def test_gdn_state_descriptor_matches_reference(kq, oracle, dtype):
    from test_oracle_pin import gdn_dims, gdn_golden, gdn_weights
    from test_gpu_parity import _gdn_f32_call
    meta, arr = gdn_golden()
    dims = gdn_dims(meta)
    w = gdn_weights(arr)
    rng = np.random.default_rng(11 + dtype)
    layer = kq.GdnLayer(dims, activation_dtype=dtype)
    try:
        assert kq.lib().kq_gdn_config_activation_dtype(layer.handle) == dtype
        nc = kq.lib().kq_gdn_config_conv_state_element_count(layer.handle)
        nr = kq.lib().kq_gdn_config_recurrent_element_count(layer.handle)
        conv, rec = state_values(rng, nc), state_values(rng, nr)
        x = rng.standard_normal((3, dims.hidden)).astype(np.float32)
        st_ref, conv_ref, rec_ref, exec_ref = oracle.gdn_state_roundtrip_ref(dims, dtype, conv, rec, x, w)
        assert st_ref == 0
        s = kq.GdnState(layer)
        try:
            s.load(conv, rec, 1)
            c2, r2, init = s.save()
            assert init == 1
            assert np.array_equal(bits(c2), bits(conv_ref)), "conv history bits differ from the reference"
            assert np.array_equal(bits(r2), bits(rec_ref)), "recurrent state bits differ from the reference"
            st, _, d = _gdn_f32_call(kq, layer.handle, dims, w, x, s)
            assert st == exec_ref, d.text()
            if dtype == 1:
                assert st == KQ_STATUS_INCOMPATIBLE_GDN
                c3, r3, _ = s.save()      # a refused call leaves the state as it was
                assert np.array_equal(bits(c3), bits(c2)) and np.array_equal(bits(r3), bits(r2))
        finally:
            s.close()
    finally:
        layer.close()


@pytest.mark.parametrize("dtype", [0, 1])
def test_qsa_cache_descriptor_matches_reference(kq, oracle, dtype):
    from test_oracle_pin import QSA_W, qsa_dims, qsa_golden
    meta, arr = qsa_golden()
    dims = qsa_dims(meta)
    w = {k: np.ascontiguousarray(arr[f"w_{k}"]) for k in QSA_W}
    rng = np.random.default_rng(23 + dtype)
    length, capacity = 10, 32
    key = state_values(rng, length * dims.kv_width).reshape(length, dims.kv_width)
    value = state_values(rng, length * dims.kv_width).reshape(length, dims.kv_width)
    raw = state_values(rng, length * dims.index_dim).reshape(length, dims.index_dim)
    x = rng.standard_normal((2, dims.hidden)).astype(np.float32)
    st_ref, k_ref, v_ref, r_ref, n_ref, exec_ref = oracle.qsa_state_roundtrip_ref(dims, dtype, key, value, raw,
                                                                                  length, capacity, x, w)
    assert st_ref == 0 and n_ref == length
    lib, abi = kq.lib(), kq.abi
    layer = kq.QsaLayer(dims, activation_dtype=dtype)
    try:
        assert lib.kq_qsa_config_activation_dtype(layer.handle) == dtype
        s = kq.QsaState(layer, capacity)
        try:
            s.load(key, value, raw)
            assert s.length == length
            k2, v2, r2 = s.save()
            assert np.array_equal(bits(k2), bits(k_ref)), "key cache bits differ from the reference"
            assert np.array_equal(bits(v2), bits(v_ref)), "value cache bits differ from the reference"
            assert np.array_equal(bits(r2), bits(r_ref)), "raw index cache bits differ from the reference"
            qw = abi.QsaWeightsF32()
            for k in QSA_W:
                setattr(qw, k, w[k].ctypes.data)
                setattr(qw, k + "_count", w[k].size)
            need = C.c_uint64()
            d = abi.Diagnostic()
            assert lib.kq_qsa_required_scratch_bytes(layer.handle, s.handle, x.shape[0], C.byref(need),
                                                     C.byref(d)) == 0
            scratch = np.zeros(need.value // 4 + 1, np.float32)
            y = np.zeros((x.shape[0], dims.hidden), np.float32)
            st = lib.kq_qsa_prefill_f32(layer.handle, C.byref(qw), x.ctypes.data, x.shape[0], y.ctypes.data, y.size,
                                        s.handle, scratch.ctypes.data, need.value, abi.SELECTION_OBSERVER(), None,
                                        None, C.byref(d))
            assert st == exec_ref, d.text()
            if dtype == 1:
                assert st != 0 and s.length == length
        finally:
            s.close()
    finally:
        layer.close()
