"""GPU parity: the B200 library, called through its C-ABI, against the CPU
oracle (pinned to the reference by test_oracle_pin.py) on identical seeded
inputs.

Bars: dequantised weights and index-path values are
bit-exact; operator outputs and recurrent states are within
|gpu - cpu| <= ATOL + RTOL * |cpu| with ATOL = 2e-3, RTOL = 1e-3.
"""
import ctypes as C
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3
GOLD = Path(__file__).resolve().parent / "golden"


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def assert_close(gpu, cpu, what=""):
    gpu = np.asarray(gpu, np.float32).reshape(-1)
    cpu = np.asarray(cpu, np.float32).reshape(-1)
    err = np.abs(gpu.astype(np.float64) - cpu.astype(np.float64))
    lim = ATOL + RTOL * np.abs(cpu.astype(np.float64))
    bad = np.nonzero(err > lim)[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance, worst {err.max():.3e} at {bad[:5]}"


# ------------------------------------------------------------------ numerics

@pytest.mark.parametrize("type_id", [0, 30, 8, 12, 14])
def test_dequant_bit_exact(kq, oracle, type_id):
    from kqb200 import synth
    rng = np.random.default_rng(100 + type_id)
    q = synth.pack(type_id, rng, 37, 1024)
    n = q.rows * q.cols
    out = np.empty(n, np.float32)
    cnt = C.c_uint64()
    d = kq.abi.Diagnostic()
    st = kq.lib().kq_dequantize_blocks_f32(type_id, q.data.ctypes.data, q.data.size, out.ctypes.data, n,
                                           C.byref(cnt), C.byref(d))
    assert st == 0, d.text()
    assert cnt.value == n
    assert np.array_equal(bits(out), bits(oracle.dequantize(type_id, q.data)))


def test_dequant_golden_vectors_on_gpu(kq):
    meta = json.loads((GOLD / "dequant_golden.json").read_text())
    tid = {"F32": 0, "BF16": 30, "Q8_0": 8, "Q4_K": 12}
    for c in meta["cases"]:
        packed = np.frombuffer(bytes.fromhex(c["packed_hex"]), np.uint8).copy()
        want = np.array([int(h, 16) for h in c["expected_f32_bits"]], np.uint32)
        out = np.empty(want.size, np.float32)
        cnt = C.c_uint64()
        d = kq.abi.Diagnostic()
        st = kq.lib().kq_dequantize_blocks_f32(tid[c["type"]], packed.ctypes.data, packed.size, out.ctypes.data,
                                               out.size, C.byref(cnt), C.byref(d))
        if c["type"] == "F32" and not np.isfinite(out).all() and st != 0:
            continue
        assert st == 0, (c["id"], d.text())
        assert np.array_equal(bits(out), want), c["id"]


@pytest.mark.parametrize("type_id", [8, 12, 14, 30])
def test_row_dot_bit_exact(kq, oracle, type_id):
    from kqb200 import synth
    rng = np.random.default_rng(7 + type_id)
    q = synth.pack(type_id, rng, 1, 2048)
    x = rng.normal(size=2048).astype(np.float32)
    out = C.c_float()
    d = kq.abi.Diagnostic()
    st = kq.lib().kq_quantized_row_dot_f32(type_id, q.data.ctypes.data, q.data.size, x.ctypes.data, x.size,
                                           C.byref(out), C.byref(d))
    assert st == 0, d.text()
    assert bits(np.float32(out.value)) == bits(oracle.matvec(type_id, q.data, 1, 2048, x))[0, 0]


@pytest.mark.parametrize("type_id", [8, 12, 14])
def test_provider_linear(kq, oracle, type_id):
    from kqb200 import synth
    rng = np.random.default_rng(3)
    q = synth.pack(type_id, rng, 512, 2048)
    p = kq.Provider(0)
    try:
        h = p.add_matrix("m", 11, q)
        x = rng.normal(size=2048).astype(np.float32)
        y = p.linear(h, 512, 2048, x)
        assert_close(y, oracle.matvec(type_id, q.data, 512, 2048, x)[0], "linear")
        with pytest.raises(kq.KQError) as e:
            p.linear(h, 511, 2048, x)
        assert e.value.status == kq.abi.DIMENSION_MISMATCH
    finally:
        p.close()


@pytest.mark.parametrize("type_id,rows,cols,batch,wide", [
    (12, 520, 2048, 64, None), (14, 2048, 4096, 64, None), (8, 300, 2048, 9, None), (30, 640, 2048, 100, None),
    (0, 200, 512, 33, None), (12, 12352, 2048, 64, None), (14, 130, 256, 129, None),
    # the 256-row activation tile of prefill batches, forced on and off
    (12, 12352, 2048, 600, "1"), (12, 12352, 2048, 600, "0"), (14, 2048, 4096, 513, "1"),
    (8, 300, 2048, 257, "1"), (30, 640, 2048, 300, "1"), (14, 130, 256, 65, "1")])
def test_tensor_core_projection(kq, oracle, type_id, rows, cols, batch, wide, monkeypatch):
    """Dequant-fused tcgen05 GEMM (three-term BF16 split) against the
    reference's sequential F32 row dots: ragged rows, batches and K."""
    import torch
    from kqb200 import synth
    if wide is not None:
        monkeypatch.setenv("KQ_B200_PROJ_WIDE", wide)
    rng = np.random.default_rng(rows + cols + batch)
    q = synth.pack(type_id, rng, rows, cols)
    p = kq.Provider(0)
    try:
        h = p.add_matrix("m", 11, q)
        x = rng.normal(size=(batch, cols)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.full((batch, rows), float("nan"), device="cuda")
        torch.cuda.synchronize()
        d = kq.abi.Diagnostic()
        st = kq.lib().kq_b200_provider_linear_batch_f32(p.handle, h, rows, cols, xd.data_ptr(), batch,
                                                        yd.data_ptr(), C.byref(d))
        assert st == 0, d.text()
        kq.synchronize()
        y = yd.cpu().numpy()
        want = oracle.matvec(type_id, q.data, rows, cols, x)
        assert_close(y, want, f"type {type_id}")
    finally:
        p.close()


@pytest.mark.parametrize("type_id,rows,cols,batch,mean", [
    (12, 520, 2048, 64, 0.0), (12, 12352, 2048, 64, 1.5), (12, 640, 4096, 130, -2.0), (12, 96, 256, 17, 0.0),
    (14, 2048, 4096, 64, 0.0), (14, 2048, 4096, 64, 1.5), (14, 300, 1024, 100, 0.5), (14, 130, 256, 9, 0.0)])
def test_factored_projection(kq, oracle, type_id, rows, cols, batch, mean, monkeypatch):
    """The factored-scale Q4_K / Q6_K kernel (integer A operand, per
    super-block d in the epilogue, Q4_K minimum term as a second product) and
    the two-term kernel both against the reference's sequential row dots,
    including activations with a large common mode, where the Q4_K minimum
    term and the scaled main term nearly cancel."""
    import torch
    from kqb200 import synth
    rng = np.random.default_rng(rows * 3 + cols + batch)
    q = synth.pack(type_id, rng, rows, cols)
    x = (rng.normal(size=(batch, cols)) + mean).astype(np.float32)
    want = oracle.matvec(type_id, q.data, rows, cols, x)
    p = kq.Provider(0)
    try:
        h = p.add_matrix("m", 11, q)
        xd = torch.from_numpy(x).cuda()
        for fact in ("1", "0"):
            monkeypatch.setenv("KQ_B200_PROJ_FACT", fact)
            yd = torch.full((batch, rows), float("nan"), device="cuda")
            torch.cuda.synchronize()
            d = kq.abi.Diagnostic()
            st = kq.lib().kq_b200_provider_linear_batch_f32(p.handle, h, rows, cols, xd.data_ptr(), batch,
                                                            yd.data_ptr(), C.byref(d))
            assert st == 0, d.text()
            kq.synchronize()
            assert_close(yd.cpu().numpy(), want, f"type {type_id} factored={fact}")
    finally:
        p.close()


# ------------------------------------------------------------------ GDN

def _gdn_f32_call(kq, layer_handle, dims, w, x, state, mask=None):
    lib, abi = kq.lib(), kq.abi
    ws = {k: np.ascontiguousarray(w[k], np.float32) for k in abi.GDN_WEIGHT_FIELDS}
    gw = abi.GdnWeightsF32()
    for k in abi.GDN_WEIGHT_FIELDS:
        setattr(gw, k, ws[k].ctypes.data)
        setattr(gw, k + "_count", ws[k].size)
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    y = np.zeros((T, dims.hidden), np.float32)
    scratch = np.zeros(lib.kq_gdn_config_scratch_bytes(layer_handle) // 4 + 1, np.float32)
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    d = abi.Diagnostic()
    st = lib.kq_gdn_prefill_f32(layer_handle, C.byref(gw), x.ctypes.data, T, None if m is None else m.ctypes.data,
                                y.ctypes.data, y.size, state.handle, scratch.ctypes.data, scratch.nbytes, None,
                                None, C.byref(d))
    return st, y, d


def test_gdn_golden_cases_f32_api(kq, oracle):
    from test_oracle_pin import accepts, gdn_dims, gdn_golden, gdn_weights
    meta, arr = gdn_golden()
    dims = gdn_dims(meta)
    w = gdn_weights(arr)
    layer = kq.GdnLayer(dims)
    try:
        for i, c in enumerate(meta["cases"]):
            s = kq.GdnState(layer)
            s.load(arr[f"c{i}_conv0"], arr[f"c{i}_rec0"], int(c["initialized"]))
            st, y, d = _gdn_f32_call(kq, layer.handle, dims, w, arr[f"c{i}_input"], s, c["mask"])
            assert st == 0, (c["id"], d.text())
            conv, rec, init = s.save()
            assert init == 1
            _, yo, convo, reco = oracle.gdn_run(dims, w, arr[f"c{i}_input"], arr[f"c{i}_conv0"], arr[f"c{i}_rec0"],
                                                c["mask"])
            assert_close(y, yo, c["id"])
            assert_close(rec, reco, c["id"])
            assert_close(conv, convo, c["id"])   # history of projected (tolerance-level) values
            # the reference's golden expectations, at the north-star bar
            assert_close(y, arr[f"c{i}_output"], c["id"] + " vs golden")
            assert_close(conv, arr[f"c{i}_conv"], c["id"] + " vs golden")
            assert_close(rec, arr[f"c{i}_rec"], c["id"] + " vs golden")
            s.close()
    finally:
        layer.close()


def test_f32_api_reuses_uploaded_weights_until_they_change(kq, oracle):
    """The F32 entry point keeps host weight arrays it has uploaded on the
    device for later calls; an array changed in place (same address, new
    contents) must be uploaded again, so every call matches the oracle on
    the weights as they are at that call."""
    from kqb200 import synth
    dims = synth.GdnDims(hidden=256, key_heads=2, value_heads=4)
    weights = synth.gdn_layer(31, dims, synth.TYPE_Q8_0, synth.TYPE_Q8_0, synth.TYPE_F32)
    w = {k: np.ascontiguousarray(v, np.float32) for k, v in oracle.gdn_weights_f32(weights).items()}
    addresses = {k: v.ctypes.data for k, v in w.items()}
    layer = kq.GdnLayer(dims)
    try:
        for call in range(3):
            if call == 2:
                w["qkv"] *= 1.5
                w["output"][0, :] += 0.01
                w["a_log"][1] -= 0.25
            assert all(v.ctypes.data == addresses[k] for k, v in w.items())
            s = kq.GdnState(layer)
            c0, r0 = synth.gdn_state(32, dims)
            s.load(c0, r0)
            x = synth.hidden(33 + call, 3, dims.hidden)
            st, y, d = _gdn_f32_call(kq, layer.handle, dims, w, x, s)
            assert st == 0, d.text()
            _, yo, _, reco = oracle.gdn_run(dims, w, x, c0, r0)
            assert_close(y, yo, f"call {call} output")
            assert_close(s.save()[1], reco, f"call {call} state")
            s.close()
    finally:
        layer.close()


def _gdn_setup(kq, oracle, dims, seed, in_type, out_type, gate_type):
    from kqb200 import synth
    weights = synth.gdn_layer(seed, dims, in_type, out_type, gate_type)
    prov = kq.Provider(0)
    layer = kq.GdnLayer(dims, weights, prov)
    return weights, prov, layer, oracle.gdn_weights_f32(weights)


@pytest.mark.parametrize("hidden,kh,vh,T,seed", [(512, 16, 32, 300, 61), (256, 2, 4, 2100, 62)])
def test_gdn_chunked_prefill(kq, oracle, hidden, kh, vh, T, seed):
    """Prefill long enough for the chunked (WY-form) recurrence: 64-token
    chunks with a partial last chunk, a padding mask, a non-zero initial
    state, and (T = 2100) two device passes; outputs and both states against
    the reference's token-by-token recurrence."""
    from kqb200 import synth
    dims = synth.GdnDims(hidden=hidden, key_heads=kh, value_heads=vh)
    weights, prov, layer, w = _gdn_setup(kq, oracle, dims, seed, synth.TYPE_Q6_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    try:
        conv0, rec0 = synth.gdn_state(seed + 1, dims)
        x = synth.hidden(seed + 2, T, dims.hidden)
        mask = np.ones(T, np.uint8)
        mask[5:9] = 0
        mask[T - 3:] = 0
        s = kq.GdnState(layer)
        s.load(conv0, rec0)
        y = s.execute_quantized(x, mask)
        conv, rec, _ = s.save()
        st, yo, convo, reco = oracle.gdn_run(dims, w, x, conv0, rec0, mask)
        assert st == 0
        assert_close(y, yo, "output")
        assert_close(rec, reco, "recurrent state")
        assert_close(conv, convo, "conv state")
        s.close()
    finally:
        layer.close()
        prov.close()


def test_gdn_config0_decode_quantized(kq, oracle):
    """one decode step, hidden 2048, 16x128 key heads,
    32x128 value heads, Q8_0 qkv/z/out, F32 alpha/beta, N(0,1) conv state,
    N(0,0.02) recurrent state."""
    from kqb200 import synth
    dims = synth.GdnDims()
    weights, prov, layer, w = _gdn_setup(kq, oracle, dims, 0, synth.TYPE_Q8_0, synth.TYPE_Q8_0, synth.TYPE_F32)
    try:
        conv0, rec0 = synth.gdn_state(1, dims)
        x = synth.hidden(2, 1, dims.hidden)
        s = kq.GdnState(layer)
        s.load(conv0, rec0)
        y = s.execute_quantized(x)
        conv, rec, _ = s.save()
        st, yo, convo, reco = oracle.gdn_run(dims, w, x, conv0, rec0)
        assert st == 0
        assert_close(y, yo, "output")
        assert_close(rec, reco, "recurrent state")
        assert_close(conv, convo, "conv state")
        s.close()
    finally:
        layer.close()
        prov.close()


def test_gdn_prefill_quantized_q6k_with_mask(kq, oracle):
    """Multi-token path (config-2 style: Q6_K projections, zero initial state)
    on a short sequence with padding, then a decode continuation."""
    from kqb200 import synth
    dims = synth.GdnDims(hidden=512, key_heads=4, value_heads=8, key_dim=128, value_dim=128)
    weights, prov, layer, w = _gdn_setup(kq, oracle, dims, 4, synth.TYPE_Q6_K, synth.TYPE_Q6_K, synth.TYPE_Q6_K)
    try:
        T = 24
        x = synth.hidden(5, T, dims.hidden)
        mask = (np.arange(T) % 7 != 3).astype(np.uint8)
        s = kq.GdnState(layer)
        y = s.execute_quantized(x, mask)
        conv, rec, init = s.save()
        conv0, rec0 = synth.gdn_state(0, dims, zero=True)
        st, yo, convo, reco = oracle.gdn_run(dims, w, x, conv0, rec0, mask)
        assert st == 0 and init == 1
        assert_close(y, yo, "prefill output")
        assert_close(rec, reco, "prefill state")
        x2 = synth.hidden(6, 1, dims.hidden)
        y2 = s.execute_quantized(x2)
        st, yo2, _, reco2 = oracle.gdn_run(dims, w, x2, convo, reco)
        assert_close(y2, yo2, "decode after prefill")
        assert_close(s.save()[1], reco2, "state after decode")
        s.close()
    finally:
        layer.close()
        prov.close()


def test_gdn_decode_batch_matches_per_sequence_oracle(kq, oracle):
    import torch
    from kqb200 import synth
    dims = synth.GdnDims(hidden=1024, key_heads=4, value_heads=8, key_dim=128, value_dim=128)
    weights, prov, layer, w = _gdn_setup(kq, oracle, dims, 9, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    try:
        B = 70   # > one 64-sequence launch group
        states, init = [], []
        for b in range(B):
            s = kq.GdnState(layer)
            c0, r0 = synth.gdn_state(100 + b, dims)
            s.load(c0, r0)
            states.append(s)
            init.append((c0, r0))
        x = synth.hidden(11, B, dims.hidden)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        torch.cuda.synchronize()
        kq.gdn_decode_batch(layer, states, xd.data_ptr(), yd.data_ptr())
        kq.synchronize()
        y = yd.cpu().numpy()
        for b in (0, 1, 33, 63, 64, 69):
            st, yo, convo, reco = oracle.gdn_run(dims, w, x[b:b + 1], *init[b])
            assert_close(y[b], yo, f"seq {b}")
            assert_close(states[b].save()[1], reco, f"state {b}")
        for s in states:
            s.close()
    finally:
        layer.close()
        prov.close()


@pytest.mark.parametrize("B", [5, 40])
def test_decode_batch_rejects_non_finite_input(kq, oracle, B):
    """A NaN in one sequence's hidden state makes the batched decode of both
    operators fail with NUMERIC_DOMAIN and roll every state back; B = 40 runs
    the tensor-core projections (input check fused into their activation
    staging), B = 5 the warp GEMV (separate check)."""
    import torch
    from kqb200 import synth
    gdims = synth.GdnDims(hidden=512, key_heads=2, value_heads=4, key_dim=128, value_dim=128)
    _, gprov, glayer, _ = _gdn_setup(kq, oracle, gdims, 21, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    qdims = synth.QsaDims(hidden=512, query_heads=8, kv_heads=2, head_dim=256, index_heads=4, index_dim=128,
                          block=4, budget=256, max_context=4096, rotary=64)
    _, qprov, qlayer, _ = _qsa_setup(kq, oracle, qdims, 22)
    try:
        gstates, qstates, g0, q0 = [], [], [], []
        for b in range(B):
            s = kq.GdnState(glayer)
            c0, r0 = synth.gdn_state(300 + b, gdims)
            s.load(c0, r0)
            gstates.append(s)
            g0.append((c0, r0))
            q = kq.QsaState(qlayer, 64)
            k, v, r = synth.qsa_cache(400 + b, qdims, 9)
            q.load(k, v, r)
            qstates.append(q)
            q0.append(len(k))
        x = synth.hidden(23, B, 512)
        x[B // 2, 7] = np.nan
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        torch.cuda.synchronize()
        for call in (lambda: kq.gdn_decode_batch(glayer, gstates, xd.data_ptr(), yd.data_ptr()),
                     lambda: kq.qsa_decode_batch(qlayer, qstates, xd.data_ptr(), yd.data_ptr())):
            call()
            with pytest.raises(kq.KQError) as e:
                kq.synchronize()
            assert e.value.status == kq.abi.NUMERIC_DOMAIN
        for b in (0, B // 2, B - 1):
            c1, r1, _ = gstates[b].save()
            assert np.array_equal(bits(c1), bits(g0[b][0])) and np.array_equal(bits(r1), bits(g0[b][1]))
            assert kq.lib().kq_qsa_state_length(qstates[b].handle) == q0[b]
        for s in gstates + qstates:
            s.close()
    finally:
        glayer.close()
        qlayer.close()
        gprov.close()
        qprov.close()


def test_decode_batch_rejects_activation_beyond_fp16_range(kq, oracle):
    """The tensor-core projection carries activations as fp16 hi/lo parts of
    x / 4, so |x| must stay below 2^18: a batch (B = 40, tensor-core path)
    with one such value fails with NUMERIC_DOMAIN naming the range, and every
    GDN state rolls back; a value just below the limit decodes normally."""
    import torch
    from kqb200 import synth
    gdims = synth.GdnDims(hidden=512, key_heads=2, value_heads=4, key_dim=128, value_dim=128)
    _, gprov, glayer, w = _gdn_setup(kq, oracle, gdims, 24, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    try:
        B = 40
        states, init = [], []
        for b in range(B):
            s = kq.GdnState(glayer)
            c0, r0 = synth.gdn_state(500 + b, gdims)
            s.load(c0, r0)
            states.append(s)
            init.append((c0, r0))
        x = synth.hidden(25, B, 512)
        x[3, 100] = 3.0e5
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        torch.cuda.synchronize()
        kq.gdn_decode_batch(glayer, states, xd.data_ptr(), yd.data_ptr())
        with pytest.raises(kq.KQError) as e:
            kq.synchronize()
        assert e.value.status == kq.abi.NUMERIC_DOMAIN and "range" in str(e.value)
        for b in (0, 3, B - 1):
            c1, r1, _ = states[b].save()
            assert np.array_equal(bits(c1), bits(init[b][0])) and np.array_equal(bits(r1), bits(init[b][1]))
        x[3, 100] = 2.5e5   # inside the range
        xd.copy_(torch.from_numpy(x))
        torch.cuda.synchronize()
        kq.gdn_decode_batch(glayer, states, xd.data_ptr(), yd.data_ptr())
        kq.synchronize()
        st, yo, _, reco = oracle.gdn_run(gdims, w, x[3:4], *init[3])
        assert st == 0
        assert_close(yd.cpu().numpy()[3], yo, "decode with a large activation")
        assert_close(states[3].save()[1], reco, "state after a large activation")
        for s in states:
            s.close()
    finally:
        glayer.close()
        gprov.close()


def test_gdn_failure_leaves_state_unchanged(kq, oracle):
    from kqb200 import synth
    dims = synth.GdnDims(hidden=256, key_heads=2, value_heads=4, key_dim=128, value_dim=128)
    weights, prov, layer, w = _gdn_setup(kq, oracle, dims, 2, synth.TYPE_Q8_0, synth.TYPE_Q8_0, synth.TYPE_F32)
    try:
        s = kq.GdnState(layer)
        c0, r0 = synth.gdn_state(3, dims)
        s.load(c0, r0)
        x = synth.hidden(4, 3, dims.hidden)
        x[1, 5] = np.nan
        with pytest.raises(kq.KQError) as e:
            s.execute_quantized(x)
        assert e.value.status == kq.abi.NUMERIC_DOMAIN
        c1, r1, init = s.save()
        assert np.array_equal(bits(c1), bits(c0)) and np.array_equal(bits(r1), bits(r0)) and init == 1
        # a state that overflows inside the recurrence is also rejected and rolled back
        x = synth.hidden(5, 1, dims.hidden)
        big = np.full_like(r0, 3.0e38)
        s.load(c0, big)
        with pytest.raises(kq.KQError) as e:
            s.execute_quantized(x)
        assert e.value.status == kq.abi.NUMERIC_DOMAIN
        assert np.array_equal(bits(s.save()[1]), bits(big))
        # the library keeps working after the error
        s.load(c0, r0)
        y = s.execute_quantized(x)
        _, yo, _, _ = oracle.gdn_run(dims, w, x, c0, r0)
        assert_close(y, yo, "after error")
        s.close()
    finally:
        layer.close()
        prov.close()


# ------------------------------------------------------------------ QSA

def test_qsa_golden_cases_f32_api(kq, oracle):
    from test_oracle_pin import QSA_W, qsa_dims, qsa_golden, within
    meta, arr = qsa_golden()
    dims = qsa_dims(meta)
    w = {k: np.ascontiguousarray(arr[f"w_{k}"]) for k in QSA_W}
    lib, abi = kq.lib(), kq.abi
    layer = kq.QsaLayer(dims)
    try:
        for i, c in enumerate(meta["cases"]):
            x = arr[f"c{i}_input"]
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
            sels = []

            def on_sel(p, _u):
                sv = p.contents
                sels.append([sv.selected_block_ids[j] for j in range(sv.selected_block_count)])

            cb = abi.SELECTION_OBSERVER(on_sel)
            st = lib.kq_qsa_prefill_f32(layer.handle, C.byref(qw), x.ctypes.data, T, y.ctypes.data, y.size,
                                        s.handle, scratch.ctypes.data, scratch.nbytes, cb, None, None, C.byref(d))
            assert st == 0, (c["id"], d.text())
            z = np.zeros((cap, dims.kv_width), np.float32)
            zr = np.zeros((cap, dims.index_dim), np.float32)
            _, yo, ko, vo, ro, n, osel = oracle.qsa_run(dims, w, x, z, z, zr, 0, cap)
            assert s.length == n == c["length"]
            assert_close(y, yo, c["id"])
            k, v, r = s.save()
            assert np.array_equal(bits(r), bits(ro)), c["id"]          # exact index path
            assert_close(k, ko, c["id"])
            for j, sel in enumerate(c["selection"]):
                assert sels[j] == sel["selected_block_ids"], (c["id"], j)
                assert sels[j] == list(osel[j]["selected"])
            s.close()
    finally:
        layer.close()


def _qsa_setup(kq, oracle, dims, seed, proj_type=12, index_type=30):
    from kqb200 import synth
    weights = synth.qsa_layer(seed, dims, proj_type, index_type=index_type)
    prov = kq.Provider(0)
    layer = kq.QsaLayer(dims, weights, prov)
    return weights, prov, layer, oracle.qsa_weights_f32(weights)


@pytest.mark.parametrize("simt", ["0", "1"])
def test_qsa_config1_decode_context_4096(kq, oracle, simt, monkeypatch):
    """decode at context 4096 (4095 prior positions),
    hidden 2048, 16 q heads / 2 KV heads of 256, partial RoPE 64, theta 1e7,
    Q4_K q/k/v/o, BF16 index projections, N(0,1) caches.  Block selection
    (512 of 1024 blocks) must match the reference exactly.  The attention
    runs on the tensor cores (bf16 hi / lo cache copies) and, with
    KQ_B200_SIMT_ATTENTION=1, on the F32 CUDA-core kernel."""
    from kqb200 import synth
    monkeypatch.setenv("KQ_B200_SIMT_ATTENTION", simt)
    dims = synth.QsaDims(max_context=8192)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, 21)
    try:
        L0 = 4095
        k0, v0, r0 = synth.qsa_cache(22, dims, L0)
        s = kq.QsaState(layer, 4096)
        s.load(k0, v0, r0)
        x = synth.hidden(23, 1, dims.hidden)
        y, sels = s.execute_quantized(x, want_selection=True)
        st, yo, ko, vo, ro, n, osel = oracle.qsa_run(dims, w, x, k0, v0, r0, L0, 4096)
        assert st == 0 and s.length == n == 4096
        assert np.array_equal(bits(sels[0]["scores"]), bits(osel[0]["scores"]))
        assert np.array_equal(sels[0]["selected"], osel[0]["selected"])
        assert_close(y, yo, "output")
        k, v, r = s.save()
        assert np.array_equal(bits(r), bits(ro))
        assert_close(k[-1], ko[-1], "appended key")
        assert np.array_equal(bits(v[:-1]), bits(v0))
        s.close()
    finally:
        layer.close()
        prov.close()


def test_qsa_prefill_then_decode_selection_exact(kq, oracle):
    from kqb200 import synth
    dims = synth.QsaDims(hidden=512, query_heads=8, kv_heads=2, head_dim=128, index_heads=4, index_dim=128,
                         block=4, budget=64, max_context=1024, rotary=64)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, 31, proj_type=8)
    try:
        T = 70
        x = synth.hidden(32, T, dims.hidden)
        s = kq.QsaState(layer, 256)
        y, sels = s.execute_quantized(x, want_selection=True)
        z = np.zeros((256, dims.kv_width), np.float32)
        zr = np.zeros((256, dims.index_dim), np.float32)
        st, yo, ko, vo, ro, n, osel = oracle.qsa_run(dims, w, x, z, z, zr, 0, 256)
        assert st == 0 and n == T
        for t in range(T):
            assert np.array_equal(bits(sels[t]["scores"]), bits(osel[t]["scores"])), t
            assert np.array_equal(sels[t]["selected"], osel[t]["selected"]), t
        assert_close(y, yo, "prefill")
        x2 = synth.hidden(33, 3, dims.hidden)
        y2 = np.concatenate([s.execute_quantized(x2[i:i + 1]) for i in range(3)])
        st, yo2, *_ = oracle.qsa_run(dims, w, x2, ko, vo, ro, n, 256)
        assert_close(y2, yo2, "decode after prefill")
        s.close()
    finally:
        layer.close()
        prov.close()


@pytest.mark.parametrize("hidden,qh,hd,budget,L0,T,seed,shared", [
    (512, 8, 128, 64, 37, 150, 71, "0"),       # three chunks (64, 64, 22), prior context mid-block
    (2048, 16, 256, 512, 1001, 130, 72, "0"),  # config-1 head geometry, head-blocked attention
    (2048, 16, 256, 512, 1001, 130, 73, "1"),  # scores of four entries per key load
    (512, 8, 128, 64, 5, 1100, 74, "1"),       # >= 1024 tokens: 32-row tiles of the exact index projection
])
def test_qsa_chunked_prefill(kq, oracle, hidden, qh, hd, budget, L0, T, seed, shared, monkeypatch):
    """A prefill without a selection observer runs 64 tokens per launch
    sequence as batch entries over one cache; its outputs, caches and the
    block keys it writes (checked through the bit-exact scores of the next
    decode token) must match the per-token reference."""
    from kqb200 import synth
    monkeypatch.setenv("KQ_B200_SCORE_SHARED", shared)
    dims = synth.QsaDims(hidden=hidden, query_heads=qh, kv_heads=2, head_dim=hd, index_heads=4, index_dim=128,
                         block=4, budget=budget, max_context=4096, rotary=64)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, seed, proj_type=8)
    try:
        cap = 2048
        k0, v0, r0 = synth.qsa_cache(seed + 100, dims, L0)
        s = kq.QsaState(layer, cap)
        s.load(k0, v0, r0)
        x = synth.hidden(seed + 200, T + 1, dims.hidden)
        y = s.execute_quantized(x[:T])
        st, yo, ko, vo, ro, n, _ = oracle.qsa_run(dims, w, x[:T], k0, v0, r0, L0, cap)
        assert st == 0 and s.length == n == L0 + T
        assert_close(y, yo, "chunked prefill")
        k, v, r = s.save()
        assert np.array_equal(bits(r), bits(ro[:n]))
        assert_close(k, ko[:n], "keys")
        y1, sels = s.execute_quantized(x[T:], want_selection=True)
        st, yo1, *_, osel = oracle.qsa_run(dims, w, x[T:], ko, vo, ro, n, cap)
        assert st == 0
        assert np.array_equal(bits(sels[0]["scores"]), bits(osel[0]["scores"]))
        assert np.array_equal(sels[0]["selected"], osel[0]["selected"])
        assert_close(y1, yo1, "decode after chunked prefill")
        s.close()
    finally:
        layer.close()
        prov.close()


def test_qsa_paired_scores_select_like_single_entry_scores(kq, oracle, monkeypatch):
    """The eight-entry score kernel (f32x2 products and sums, each lane
    rounded like the scalar ones) gives bit-identical block scores to the
    one-entry kernel: a chunked prefill run with either produces the same
    outputs and caches bit for bit."""
    from kqb200 import synth
    dims = synth.QsaDims(hidden=2048, query_heads=16, kv_heads=2, head_dim=256, index_heads=4, index_dim=128,
                         block=4, budget=512, max_context=4096, rotary=64)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, 77, proj_type=8)
    try:
        k0, v0, r0 = synth.qsa_cache(177, dims, 1500)
        x = synth.hidden(277, 200, dims.hidden)
        runs = []
        for shared in ("0", "1"):
            monkeypatch.setenv("KQ_B200_SCORE_SHARED", shared)
            s = kq.QsaState(layer, 2048)
            s.load(k0, v0, r0)
            y = s.execute_quantized(x)
            runs.append((y, *s.save()))
            s.close()
        for a, b in zip(*runs):
            assert np.array_equal(bits(a), bits(b))
    finally:
        layer.close()
        prov.close()


def test_qsa_decode_batch_ragged_contexts(kq, oracle):
    import torch
    from kqb200 import synth
    dims = synth.QsaDims(hidden=1024, query_heads=8, kv_heads=2, head_dim=256, index_heads=4, index_dim=128,
                         block=4, budget=256, max_context=4096, rotary=64)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, 41)
    try:
        lengths = [0, 1, 3, 4, 63, 64, 255, 256, 257, 1000, 2047]
        states, caches = [], []
        for i, L in enumerate(lengths):
            s = kq.QsaState(layer, 2048)
            k0, v0, r0 = synth.qsa_cache(50 + i, dims, L)
            if L:
                s.load(k0, v0, r0)
            states.append(s)
            caches.append((k0, v0, r0))
        B = len(lengths)
        x = synth.hidden(42, B, dims.hidden)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        torch.cuda.synchronize()
        kq.qsa_decode_batch(layer, states, xd.data_ptr(), yd.data_ptr())
        kq.synchronize()
        y = yd.cpu().numpy()
        for b, L in enumerate(lengths):
            st, yo, *_ = oracle.qsa_run(dims, w, x[b:b + 1], *caches[b], L, 2048)
            assert st == 0 and states[b].length == L + 1
            assert_close(y[b], yo, f"seq {b} (context {L})")
        for s in states:
            s.close()
    finally:
        layer.close()
        prov.close()


def test_qsa_failure_leaves_state_and_output_untouched(kq, oracle):
    from kqb200 import synth
    dims = synth.QsaDims(hidden=256, query_heads=4, kv_heads=2, head_dim=64, index_heads=2, index_dim=64,
                         block=4, budget=32, max_context=256, rotary=32)
    weights, prov, layer, w = _qsa_setup(kq, oracle, dims, 61, proj_type=8)
    try:
        s = kq.QsaState(layer, 64)
        x = synth.hidden(62, 5, dims.hidden)
        s.execute_quantized(x)
        k0, v0, r0 = s.save()
        bad = synth.hidden(63, 2, dims.hidden)
        bad[1, 0] = np.inf
        with pytest.raises(kq.KQError) as e:
            s.execute_quantized(bad)
        assert e.value.status == kq.abi.NUMERIC_DOMAIN
        assert s.length == 5
        k1, v1, r1 = s.save()
        assert np.array_equal(bits(k1), bits(k0)) and np.array_equal(bits(r1), bits(r0))
        with pytest.raises(kq.KQError) as e:   # capacity
            s.execute_quantized(synth.hidden(64, 60, dims.hidden))
        assert e.value.status == kq.abi.LIMIT_EXCEEDED
        s.close()
    finally:
        layer.close()
        prov.close()
