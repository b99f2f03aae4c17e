"""Checkpoint observers on the GPU path.

With an observer attached, the reference-shaped entry points run token by
token and hand the observer every checkpoint the reference's operators emit:
the 21 GDN kinds of include/kq_gdn.h (src/kq_gdn_qwen38.c:554-838) and the
12 QSA kinds of include/kq_qsa.h (src/kq_qsa_qwen38.c:687-815), in the same
order, with the same ranks and dimensions.  Each test compares the whole
stream with the CPU oracle's (whose checkpoints test_oracle_pin.py pins to
the reference's bit for bit) at the parity tolerance, and the state the call
leaves with the oracle's.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3
GDN_KINDS = 21
QSA_KINDS = 12


def assert_close(gpu, cpu, what):
    gpu = np.asarray(gpu, np.float64).reshape(-1)
    cpu = np.asarray(cpu, np.float64).reshape(-1)
    assert gpu.shape == cpu.shape, f"{what}: {gpu.shape} values against {cpu.shape}"
    err = np.abs(gpu - cpu)
    bad = np.nonzero(err > ATOL + RTOL * np.abs(cpu))[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance, worst {err.max():.3e}"


def compare_streams(gpu, cpu, kinds, names):
    assert len(gpu) == len(cpu), f"{len(gpu)} checkpoints against {len(cpu)}"
    for g, c in zip(gpu, cpu):
        key = (c["kind"], c["token"], c["rank"], c["dims"])
        assert (g["kind"], g["token"], g["rank"], g["dims"]) == key, (names(g["kind"]), key)
        assert_close(g["values"], c["values"], f"{names(c['kind'])} token {c['token']}")
    assert {c["kind"] for c in gpu} == set(range(kinds))


def gdn_names(kq):
    return lambda k: kq.lib().kq_gdn_checkpoint_kind_name(k).decode()


def qsa_names(kq):
    return lambda k: kq.lib().kq_qsa_checkpoint_kind_name(k).decode()


def test_gdn_checkpoints_golden_config_f32_api(kq, oracle):
    """Every golden GDN case of the reference's reduced configuration through
    kq_gdn_prefill_f32 with an observer: the stream against the oracle's, and
    the end state."""
    from test_oracle_pin import gdn_dims, gdn_golden, gdn_weights
    meta, arr = gdn_golden()
    dims = gdn_dims(meta)
    w = {k: np.ascontiguousarray(v, np.float32) for k, v in gdn_weights(arr).items()}
    lib, abi = kq.lib(), kq.abi
    layer = kq.GdnLayer(dims)
    try:
        for i, c in enumerate(meta["cases"]):
            x = np.ascontiguousarray(arr[f"c{i}_input"], np.float32)
            T = x.shape[0]
            s = kq.GdnState(layer)
            s.load(arr[f"c{i}_conv0"], arr[f"c{i}_rec0"], int(c["initialized"]))
            gw = abi.GdnWeightsF32()
            for k in abi.GDN_WEIGHT_FIELDS:
                setattr(gw, k, w[k].ctypes.data)
                setattr(gw, k + "_count", w[k].size)
            mask = None if c["mask"] is None else np.ascontiguousarray(c["mask"], np.uint8)
            y = np.zeros((T, dims.hidden), np.float32)
            scratch = np.zeros(lib.kq_gdn_config_scratch_bytes(layer.handle) // 4 + 1, np.float32)
            got, body = abi.checkpoint_collector()
            cb = abi.GDN_CHECKPOINT_OBSERVER(body)
            d = abi.Diagnostic()
            st = lib.kq_gdn_prefill_f32(layer.handle, C.byref(gw), x.ctypes.data, T,
                                        None if mask is None else mask.ctypes.data, y.ctypes.data, y.size, s.handle,
                                        scratch.ctypes.data, scratch.nbytes, C.cast(cb, C.c_void_p), None,
                                        C.byref(d))
            assert st == 0, (c["id"], d.text())
            so, want = oracle.gdn_checkpoints(dims, w, x, arr[f"c{i}_conv0"], arr[f"c{i}_rec0"], mask)
            assert so == 0 and len(got) == GDN_KINDS * T
            compare_streams(got, want, GDN_KINDS, gdn_names(kq))
            _, yo, convo, reco = oracle.gdn_run(dims, w, x, arr[f"c{i}_conv0"], arr[f"c{i}_rec0"], mask)
            assert_close(y, yo, f"{c['id']} output")
            conv, rec, _ = s.save()
            assert_close(rec, reco, f"{c['id']} recurrent state")
            assert_close(conv, convo, f"{c['id']} conv state")
            s.close()
    finally:
        layer.close()


def test_gdn_checkpoints_quantized_provider_path(kq, oracle):
    """kq_gdn_execute_quantized with an observer: Q4_K in-projections, Q6_K
    out-projection, 128-wide heads, a padding mask and a non-zero state."""
    from kqb200 import synth
    dims = synth.GdnDims(hidden=512, key_heads=2, value_heads=4)
    weights = synth.gdn_layer(41, dims, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    w = oracle.gdn_weights_f32(weights)
    prov = kq.Provider(0)
    layer = kq.GdnLayer(dims, weights, prov)
    lib, abi = kq.lib(), kq.abi
    try:
        s = kq.GdnState(layer)
        conv0, rec0 = synth.gdn_state(42, dims)
        s.load(conv0, rec0)
        T = 4
        x = synth.hidden(43, T, dims.hidden)
        mask = np.array([1, 0, 1, 1], np.uint8)
        y = np.zeros((T, dims.hidden), np.float32)
        scratch = np.zeros(layer.scratch_bytes // 4 + 1, np.float32)
        wscratch = np.zeros(s._weight_scratch_floats(), np.float32)
        got, body = abi.checkpoint_collector()
        cb = abi.GDN_CHECKPOINT_OBSERVER(body)
        d = abi.Diagnostic()
        st = lib.kq_gdn_execute_quantized(layer.handle, prov.handle, x.ctypes.data, T, mask.ctypes.data,
                                          y.ctypes.data, y.size, s.handle, scratch.ctypes.data, scratch.nbytes,
                                          wscratch.ctypes.data, wscratch.nbytes, C.cast(cb, C.c_void_p), None,
                                          C.byref(d))
        assert st == 0, d.text()
        so, want = oracle.gdn_checkpoints(dims, w, x, conv0, rec0, mask)
        assert so == 0
        compare_streams(got, want, GDN_KINDS, gdn_names(kq))
        _, yo, _, reco = oracle.gdn_run(dims, w, x, conv0, rec0, mask)
        assert_close(y, yo, "output")
        assert_close(s.save()[1], reco, "recurrent state")
        s.close()
    finally:
        layer.close()
        prov.close()


def test_qsa_checkpoints_golden_config_f32_api(kq, oracle):
    """Every golden QSA case of the reference's reduced configuration through
    kq_qsa_prefill_f32 with both observers: the checkpoint stream against the
    oracle's, the selections in order, the output and the cache."""
    from test_oracle_pin import QSA_W, qsa_dims, qsa_golden
    meta, arr = qsa_golden()
    dims = qsa_dims(meta)
    w = {k: np.ascontiguousarray(arr[f"w_{k}"], np.float32) for k in QSA_W}
    lib, abi = kq.lib(), kq.abi
    layer = kq.QsaLayer(dims)
    try:
        for i, c in enumerate(meta["cases"]):
            x = np.ascontiguousarray(arr[f"c{i}_input"], np.float32)
            T = x.shape[0]
            cap = max(16, T)
            s = kq.QsaState(layer, cap)
            qw = abi.QsaWeightsF32()
            for k in QSA_W:
                setattr(qw, k, w[k].ctypes.data)
                setattr(qw, k + "_count", w[k].size)
            need = C.c_uint64()
            d = abi.Diagnostic()
            assert lib.kq_qsa_required_scratch_bytes(layer.handle, s.handle, T, C.byref(need), C.byref(d)) == 0
            scratch = np.zeros(need.value // 4 + 1, np.float32)
            y = np.zeros((T, dims.hidden), np.float32)
            sels, order = [], []
            got, body = abi.checkpoint_collector()

            def on_sel(p, _u):
                sv = p.contents
                order.append(("selection", int(sv.token_index)))
                sels.append([sv.selected_block_ids[j] for j in range(sv.selected_block_count)])

            def on_ck(p, u):
                if p.contents.kind == 0:
                    order.append(("checkpoints", int(p.contents.token_index)))
                body(p, u)

            scb = abi.SELECTION_OBSERVER(on_sel)
            ccb = abi.QSA_CHECKPOINT_OBSERVER(on_ck)
            st = lib.kq_qsa_prefill_f32(layer.handle, C.byref(qw), x.ctypes.data, T, y.ctypes.data, y.size,
                                        s.handle, scratch.ctypes.data, scratch.nbytes, scb, C.cast(ccb, C.c_void_p),
                                        None, C.byref(d))
            assert st == 0, (c["id"], d.text())
            z = np.zeros((0, dims.kv_width), np.float32)
            zr = np.zeros((0, dims.index_dim), np.float32)
            so, want = oracle.qsa_checkpoints(dims, w, x, z, z, zr, 0, cap)
            assert so == 0 and len(got) == QSA_KINDS * T
            compare_streams(got, want, QSA_KINDS, qsa_names(kq))
            # the reference calls the selection observer before each token's checkpoints
            assert order == [(kind, t) for t in range(T) for kind in ("selection", "checkpoints")]
            _, yo, ko, vo, ro, n, osel = oracle.qsa_run(dims, w, x, z, z, zr, 0, cap)
            assert [list(o["selected"]) for o in osel] == sels
            assert_close(y, yo, f"{c['id']} output")
            k1, v1, r1 = s.save()
            assert_close(k1, ko, f"{c['id']} key cache")
            assert_close(v1, vo, f"{c['id']} value cache")
            s.close()
    finally:
        layer.close()


def test_qsa_checkpoints_quantized_provider_path(kq, oracle):
    """kq_qsa_execute_quantized with a checkpoint observer on a cache of 299
    prior tokens (74 complete blocks) and a budget of 64 tokens, so that the
    top-k selects among candidates: block keys, scores, logits and
    probabilities over the selected tokens against the oracle's."""
    from kqb200 import synth
    dims = synth.QsaDims(hidden=512, query_heads=8, kv_heads=2, head_dim=256, index_heads=4, index_dim=128,
                         block=4, budget=64, max_context=1024, rotary=64)
    weights = synth.qsa_layer(44, dims, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_BF16)
    w = oracle.qsa_weights_f32(weights)
    prov = kq.Provider(0)
    layer = kq.QsaLayer(dims, weights, prov)
    lib, abi = kq.lib(), kq.abi
    try:
        L0, T = 299, 3
        s = kq.QsaState(layer, 512)
        k0, v0, r0 = synth.qsa_cache(45, dims, L0)
        s.load(k0, v0, r0)
        x = synth.hidden(46, T, dims.hidden)
        y = np.zeros((T, dims.hidden), np.float32)
        need = C.c_uint64()
        d = abi.Diagnostic()
        assert lib.kq_qsa_required_scratch_bytes(layer.handle, s.handle, T, C.byref(need), C.byref(d)) == 0
        scratch = np.zeros(need.value // 4 + 1, np.float32)
        wscratch = np.zeros((65536 + 8 * (dims.head_dim + dims.index_dim) * 4) // 4 + 64, np.float32)
        got, body = abi.checkpoint_collector()
        ccb = abi.QSA_CHECKPOINT_OBSERVER(body)
        st = lib.kq_qsa_execute_quantized(layer.handle, prov.handle, x.ctypes.data, T, y.ctypes.data, y.size,
                                          s.handle, scratch.ctypes.data, scratch.nbytes, wscratch.ctypes.data,
                                          wscratch.nbytes, abi.SELECTION_OBSERVER(), C.cast(ccb, C.c_void_p), None,
                                          C.byref(d))
        assert st == 0, d.text()
        so, want = oracle.qsa_checkpoints(dims, w, x, k0, v0, r0, L0, 512)
        assert so == 0
        compare_streams(got, want, QSA_KINDS, qsa_names(kq))
        _, yo, *_ = oracle.qsa_run(dims, w, x, k0, v0, r0, L0, 512)
        assert_close(y, yo, "output")
        assert s.length == L0 + T
        s.close()
    finally:
        layer.close()
        prov.close()
