"""Weights uploaded as the model's GGUF stores them (kq_b200_provider_add_gguf_*,
kq_b200_provider_add_index_qk).

The converter that wrote the model's GGUF reordered GDN value heads from
grouped to tiled order in the qkv / gate / alpha / beta rows, the conv
channels, A_log and dt_bias and the out-projection columns, stored A_log as
-exp(A_log) and the QSA q/k and index q/k norms as 1 + delta, and split the
index projection into a query and a key tensor (Kestrel-Q's
docs/MODEL-GGUF-MAPPING.md; undone by src/kq_weight_provider.c:205-248,
438-451, 680-717).  `stored_*` below play that converter on synthetic
canonical layers; the library must present the canonical layer again, so
the operators match the oracle run on the canonical weights (and the
vectors come back canonical).  The reference's own provider needs the real
model's verified tensor registry, which is not available, so these layouts
are checked against the restated transforms, not against the reference.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3
HK, R, W = 2, 3, 128   # key heads, value heads per key head, head width


def assert_close(gpu, cpu, what):
    gpu = np.asarray(gpu, np.float64).reshape(-1)
    cpu = np.asarray(cpu, np.float64).reshape(-1)
    err = np.abs(gpu - cpu)
    bad = np.nonzero(err > ATOL + RTOL * np.abs(cpu))[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance, worst {err.max():.3e}"


def tiled(i, width):
    """Position in the stored (tiled) order of canonical value-head-major
    element i: canonical head g * R + r is stored as head r * HK + g."""
    group, within = divmod(i, R * width)
    rep, feature = divmod(within, width)
    return (rep * HK + group) * width + feature


def stored_rows(t, phys):
    """The GGUF rows of a canonical matrix whose canonical row r is stored
    at row phys(r)."""
    from kqb200.synth import QTensor
    rows = t.data.reshape(t.rows, t.row_bytes)
    out = np.empty_like(rows)
    for r in range(t.rows):
        out[phys(r)] = rows[r]
    return QTensor(t.type_id, t.rows, t.cols, out.reshape(-1))


def _desc(kq, fn, *args):
    out = C.c_void_p()
    d = kq.abi.Diagnostic()
    kq.abi.check(fn(*args, C.byref(out), C.byref(d)), d)
    return out.value


def test_gdn_layer_from_gguf_layout(kq, oracle):
    """A GDN layer (2 key heads x 3 value heads of 128) uploaded in the
    stored layout: vectors read back canonical, the out-projection's linear
    seam (host and batched, which permute their canonical input) and the
    operator (decode, chunked prefill, batched decode, checkpoint path) match
    the oracle on the canonical layer."""
    import torch
    from kqb200 import synth
    dims = synth.GdnDims(hidden=512, key_heads=HK, value_heads=HK * R)
    w = synth.gdn_layer(61, dims, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K)
    lib, abi = kq.lib(), kq.abi
    qk, Hv = 2 * HK * W, HK * R
    # canonical F32 weights for the oracle; the out-projection is generated in
    # its stored (tiled-column) form and its canonical columns derived from it
    wf = oracle.gdn_weights_f32(w)
    out_stored = w.output
    dq = oracle.dequantize(out_stored.type_id, out_stored.data).reshape(out_stored.rows, out_stored.cols)
    wf["output"] = np.ascontiguousarray(dq[:, [tiled(c, W) for c in range(Hv * W)]])
    a_log_stored = np.empty(Hv, np.float32)
    dt_stored = np.empty(Hv, np.float32)
    for i in range(Hv):
        a_log_stored[tiled(i, 1)] = -np.exp(w.a_log[i].astype(np.float32))
        dt_stored[tiled(i, 1)] = w.dt_bias[i]
    wf["a_log"] = np.log(-a_log_stored[[tiled(i, 1) for i in range(Hv)]]).astype(np.float32)
    conv = w.conv.reshape(-1, 4)
    conv_stored = conv.copy()
    for c in range(qk, conv.shape[0]):
        conv_stored[qk + tiled(c - qk, W)] = conv[c]
    layout = abi.GgufLayout(HK, R, W)
    prov = kq.Provider(0)
    try:
        def mat(name, role, t, phys=None):
            st = stored_rows(t, phys) if phys else t
            data = np.ascontiguousarray(st.data)
            return _desc(kq, lib.kq_b200_provider_add_gguf_matrix, prov.handle, name.encode(), role, st.type_id,
                         st.rows, st.cols, data.ctypes.data, data.size, C.byref(layout))

        def vec(name, role, v):
            v = np.ascontiguousarray(v, np.float32)
            return _desc(kq, lib.kq_b200_provider_add_gguf_vector_f32, prov.handle, name.encode(), role,
                         v.ctypes.data, v.size, C.byref(layout))

        ROLE = kq.ROLE
        t = abi.GdnTensors(
            a_log=vec("a_log", ROLE["a_log"], a_log_stored),
            conv=vec("conv", ROLE["conv"], conv_stored.reshape(-1)),
            dt_bias=vec("dt_bias", ROLE["dt_bias"], dt_stored),
            alpha=mat("alpha", ROLE["alpha"], w.alpha, lambda r: tiled(r, 1)),
            beta=mat("beta", ROLE["beta"], w.beta, lambda r: tiled(r, 1)),
            qkv=mat("qkv", ROLE["qkv"], w.qkv, lambda r: r if r < qk else qk + tiled(r - qk, W)),
            gate=mat("gate", ROLE["gate"], w.gate, lambda r: tiled(r, W)),
            norm=vec("norm", ROLE["norm"], w.norm),
            output=mat("out", ROLE["out"], out_stored))
        # vectors read back canonical
        for name, want in (("a_log", wf["a_log"]), ("conv", w.conv), ("dt_bias", w.dt_bias)):
            got = np.empty(want.size, np.float32)
            d = abi.Diagnostic()
            abi.check(lib.kq_weight_provider_vector_f32(prov.handle, getattr(t, name), want.size, got.ctypes.data,
                                                        want.size, None, 0, C.byref(d)), d)
            assert_close(got, want, f"{name} read back")
        # the out-projection's linear seam takes canonical input
        x = np.random.default_rng(62).normal(size=(40, Hv * W)).astype(np.float32)
        y1 = prov.linear(t.output, dims.hidden, Hv * W, x[0])
        assert_close(y1, oracle.matvec(0, wf["output"].reshape(-1).view(np.uint8), dims.hidden, Hv * W, x[0])[0],
                     "host linear seam")
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty(40, dims.hidden, device="cuda")
        torch.cuda.synchronize()
        d = abi.Diagnostic()
        abi.check(lib.kq_b200_provider_linear_batch_f32(prov.handle, t.output, dims.hidden, Hv * W, xd.data_ptr(),
                                                        40, yd.data_ptr(), C.byref(d)), d)
        kq.synchronize()
        assert_close(yd.cpu().numpy(), x @ wf["output"].T.astype(np.float64), "batched linear seam")
        st = lib.kq_b200_provider_linear_batch_f32_static(prov.handle, t.output, dims.hidden, Hv * W,
                                                          xd.data_ptr(), 40, yd.data_ptr(), None, C.byref(d))
        assert st == abi.TENSOR_LAYOUT_MISMATCH

        layer = kq.GdnLayer(dims)
        layer.provider = prov
        d = abi.Diagnostic()
        abi.check(lib.kq_b200_gdn_config_bind(layer.handle, prov.handle, C.byref(t), C.byref(d)), d)
        try:
            c0, r0 = synth.gdn_state(63, dims)
            # decode, then a chunked prefill (>= 32 tokens) continuing it
            s = kq.GdnState(layer)
            s.load(c0, r0)
            x1 = synth.hidden(64, 1, dims.hidden)
            x2 = synth.hidden(65, 70, dims.hidden)
            y1 = s.execute_quantized(x1)
            y2 = s.execute_quantized(x2)
            _, o1, c1, r1 = oracle.gdn_run(dims, wf, x1, c0, r0)
            _, o2, c2, r2 = oracle.gdn_run(dims, wf, x2, c1, r1)
            assert_close(y1, o1, "decode")
            assert_close(y2, o2, "chunked prefill")
            assert_close(s.save()[1], r2, "state")
            s.close()
            # batched decode (fused kernel)
            states = []
            for b in range(3):
                sb = kq.GdnState(layer)
                sb.load(c0, r0)
                states.append(sb)
            xb = torch.from_numpy(synth.hidden(66, 3, dims.hidden)).cuda()
            yb = torch.empty_like(xb)
            torch.cuda.synchronize()
            kq.gdn_decode_batch(layer, states, xb.data_ptr(), yb.data_ptr())
            kq.synchronize()
            ybn = yb.cpu().numpy()
            for b in range(3):
                _, ob, _, _ = oracle.gdn_run(dims, wf, xb.cpu().numpy()[b:b + 1], c0, r0)
                assert_close(ybn[b], ob, f"batched decode {b}")
                states[b].close()
            # checkpoint path: canonical checkpoints, output through the tiled columns
            s = kq.GdnState(layer)
            s.load(c0, r0)
            got, body = abi.checkpoint_collector()
            cb = abi.GDN_CHECKPOINT_OBSERVER(body)
            x3 = synth.hidden(67, 2, dims.hidden)
            y3 = np.zeros((2, dims.hidden), np.float32)
            scratch = np.zeros(layer.scratch_bytes // 4 + 1, np.float32)
            wscratch = np.zeros(s._weight_scratch_floats(), np.float32)
            abi.check(lib.kq_gdn_execute_quantized(layer.handle, prov.handle, x3.ctypes.data, 2, None, y3.ctypes.data,
                                                   y3.size, s.handle, scratch.ctypes.data, scratch.nbytes,
                                                   wscratch.ctypes.data, wscratch.nbytes, C.cast(cb, C.c_void_p),
                                                   None, C.byref(d)), d)
            _, want = oracle.gdn_checkpoints(dims, wf, x3, c0, r0)
            assert len(got) == len(want)
            for g, c in zip(got, want):
                assert (g["kind"], g["token"], g["dims"]) == (c["kind"], c["token"], c["dims"])
                assert_close(g["values"], c["values"], f"checkpoint {c['kind']} token {c['token']}")
            s.close()
        finally:
            layer.close()
    finally:
        prov.close()


def test_qsa_layer_from_gguf_layout(kq, oracle):
    """A QSA layer whose q/k and index q/k norms are stored as 1 + delta and
    whose index projection is one split semantic (INDEX_QUERY and INDEX_KEY
    parts): the parts through the linear seam, and the operator's outputs and
    selections on a cache past the token budget against the oracle on the
    canonical layer."""
    from kqb200 import synth
    dims = synth.QsaDims(hidden=512, query_heads=8, kv_heads=2, head_dim=256, index_heads=4, index_dim=128,
                         block=4, budget=64, max_context=1024, rotary=64)
    w = synth.qsa_layer(71, dims, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_BF16)
    wf = oracle.qsa_weights_f32(w)
    lib, abi = kq.lib(), kq.abi
    layout = abi.GgufLayout(HK, R, W)
    prov = kq.Provider(0)
    try:
        ROLE = kq.ROLE

        def vec(name, role, v):
            v = np.ascontiguousarray(v, np.float32)
            return _desc(kq, lib.kq_b200_provider_add_gguf_vector_f32, prov.handle, name.encode(), role,
                         v.ctypes.data, v.size, C.byref(layout))

        iq, ik = np.ascontiguousarray(w.index_query.data), np.ascontiguousarray(w.index_key.data)
        qk = _desc(kq, lib.kq_b200_provider_add_index_qk, prov.handle, b"index_qk", w.index_query.type_id,
                   w.index_query.rows, w.index_key.rows, dims.hidden, iq.ctypes.data, iq.size, ik.ctypes.data,
                   ik.size)
        t = abi.QsaTensors(
            query=prov.add_matrix("q", ROLE["q"], w.query), key=prov.add_matrix("k", ROLE["k"], w.key),
            value=prov.add_matrix("v", ROLE["v"], w.value), output=prov.add_matrix("o", ROLE["o"], w.output),
            query_norm=vec("qn", ROLE["q_norm"], 1.0 + w.query_norm),
            key_norm=vec("kn", ROLE["k_norm"], 1.0 + w.key_norm),
            index_query=qk, index_key=qk,
            index_query_norm=vec("iqn", ROLE["index_q_norm"], 1.0 + w.index_query_norm),
            index_key_norm=vec("ikn", ROLE["index_k_norm"], 1.0 + w.index_key_norm))
        x = np.random.default_rng(72).normal(size=dims.hidden).astype(np.float32)
        for part, want in ((3, "index_query"), (4, "index_key")):   # KQ_BINDING_PART_INDEX_QUERY / _KEY
            m = wf[want]
            y = np.empty(m.shape[0], np.float32)
            d = abi.Diagnostic()
            abi.check(lib.kq_weight_provider_linear_f32(prov.handle, qk, part, 0xFFFFFFFF, m.shape[0], m.shape[1],
                                                        x.ctypes.data, y.ctypes.data, y.size, None, 0, C.byref(d)), d)
            assert_close(y, m.astype(np.float64) @ x, f"{want} part")
        d = abi.Diagnostic()
        y = np.empty(640, np.float32)
        assert lib.kq_weight_provider_linear_f32(prov.handle, qk, 0, 0xFFFFFFFF, 640, dims.hidden, x.ctypes.data,
                                                 y.ctypes.data, 640, None, 0, C.byref(d)) == abi.TENSOR_LAYOUT_MISMATCH

        layer = kq.QsaLayer(dims)
        layer.provider = prov
        abi.check(lib.kq_b200_qsa_config_bind(layer.handle, prov.handle, C.byref(t), C.byref(d)), d)
        try:
            L0 = 299
            s = kq.QsaState(layer, 512)
            k0, v0, r0 = synth.qsa_cache(73, dims, L0)
            s.load(k0, v0, r0)
            xs = synth.hidden(74, 3, dims.hidden)
            y, sel = s.execute_quantized(xs, want_selection=True)
            st, yo, *_rest, osel = oracle.qsa_run(dims, wf, xs, k0, v0, r0, L0, 512)
            assert st == 0
            assert_close(y, yo, "QSA output")
            assert [list(a["selected"]) for a in sel] == [list(b["selected"]) for b in osel]
            s.close()
        finally:
            layer.close()
    finally:
        prov.close()
