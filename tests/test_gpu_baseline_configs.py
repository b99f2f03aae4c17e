"""GPU parity at the sizes the benchmark runs (3 and 4).

The CUDA path is called through the C-ABI and compared with the CPU oracle
(pinned to the reference by test_oracle_pin.py) on the same seeded inputs, at
the north-star tolerance |gpu - cpu| <= 2e-3 + 1e-3 |cpu|, with block
selections exact.  Sequences too long for the scalar oracle are checked on
windows spliced from the GPU's own exported states (the reference's
kq_gdn_state_import_f32 / kq_qsa_state_import_f32, src/kq_gdn.c:599-701,
src/kq_qsa.c:532-620): the oracle starts from the state the GPU reached at
token t0 and must reproduce the GPU's outputs over [t0, t0 + W) and its
state at t0 + W.  The 8192-token GDN prefill is also compared over its whole
length with a float64 restatement of the layer, which bounds the drift of
the chunked (WY-form) recurrence over its 128 chunks.

Oracle windows run on host threads (the oracle's ctypes calls release the
GIL and share no state).
"""
import concurrent.futures as cf
import ctypes as C

import numpy as np
import pytest

ATOL, RTOL = 2e-3, 1e-3


def assert_close(gpu, cpu, what):
    gpu = np.asarray(gpu, np.float64).reshape(-1)
    cpu = np.asarray(cpu, np.float64).reshape(-1)
    err = np.abs(gpu - cpu)
    ratio = err / (ATOL + RTOL * np.abs(cpu))
    print(f"{what}: worst |error| / tolerance = {ratio.max():.3f} (max |error| {err.max():.3e})")
    bad = np.nonzero(ratio > 1.0)[0]
    assert bad.size == 0, f"{what}: {bad.size} of {cpu.size} values out of tolerance, worst {err.max():.3e}"


def pool_map(fn, items):
    with cf.ThreadPoolExecutor(max_workers=max(1, len(items))) as ex:
        return list(ex.map(fn, items))


# ----------------------------------------------------------------- config 2

def gdn_layer_f64(dims, w, x, chunk=64):
    """The GDN layer (src/kq_gdn_qwen38.c:545-840) in float64 from a zero
    state: projections, causal conv + SiLU, L2-normalised q/k, gates, the
    delta rule in chunked form (exact algebra, every decay factor
    exp(G_i - G_j) <= 1), gated RMSNorm and the out-projection.
    Returns (y [T][H], recurrent state [Hv][dk][dv])."""
    T, H = x.shape
    Hk, Hv, dk, dv, K = dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim, dims.conv_kernel
    C, Vd, kw = dims.conv_channels, dims.value_width, Hk * dk
    xd = x.astype(np.float64)
    mixed = xd @ w["qkv"].astype(np.float64).T
    z = xd @ w["gate"].astype(np.float64).T
    b = xd @ w["beta"].astype(np.float64).T
    a = xd @ w["alpha"].astype(np.float64).T
    taps = w["conv"].astype(np.float64).reshape(C, K)
    pad = np.concatenate([np.zeros((K - 1, C)), mixed])
    conv = sum(pad[j:j + T] * taps[:, j] for j in range(K))
    conv = conv / (1.0 + np.exp(-conv))
    q = conv[:, :kw].reshape(T, Hk, dk)
    k = conv[:, kw:2 * kw].reshape(T, Hk, dk)
    v = conv[:, 2 * kw:].reshape(T, Hv, dv)
    rep = Hv // Hk
    q = np.repeat(q, rep, axis=1)
    k = np.repeat(k, rep, axis=1)
    q = q / np.sqrt((q * q).sum(-1, keepdims=True) + 1e-6) / np.sqrt(dk)
    k = k / np.sqrt((k * k).sum(-1, keepdims=True) + 1e-6)
    beta = 1.0 / (1.0 + np.exp(-b))
    sp = a + w["dt_bias"].astype(np.float64)
    sp = np.where(sp > 20.0, sp, np.log1p(np.exp(np.minimum(sp, 20.0))))
    g = -np.exp(w["a_log"].astype(np.float64)) * sp          # [T][Hv]
    S = np.zeros((Hv, dk, dv))
    out = np.zeros((T, Hv, dv))
    for c0 in range(0, T, chunk):
        c1 = min(T, c0 + chunk)
        n = c1 - c0
        kc = k[c0:c1].transpose(1, 0, 2)                     # [Hv][n][dk]
        qc = q[c0:c1].transpose(1, 0, 2)
        vc = v[c0:c1].transpose(1, 0, 2)                     # [Hv][n][dv]
        bc = beta[c0:c1].T                                   # [Hv][n]
        G = np.cumsum(g[c0:c1].T, axis=1)                    # [Hv][n]
        D = np.exp(np.minimum(G[:, :, None] - G[:, None, :], 0.0))
        low = np.tril(np.ones((n, n)), -1)
        L = (kc @ kc.transpose(0, 2, 1)) * D * low
        A = np.eye(n)[None] + bc[:, :, None] * L
        U = np.linalg.solve(A, bc[:, :, None] * vc)
        Wm = np.linalg.solve(A, (bc * np.exp(G))[:, :, None] * kc)
        delta = U - Wm @ S
        P = (qc @ kc.transpose(0, 2, 1)) * D * np.tril(np.ones((n, n)))
        O = np.exp(G)[:, :, None] * (qc @ S) + P @ delta
        out[c0:c1] = O.transpose(1, 0, 2)
        gl = G[:, -1]
        S = np.exp(gl)[:, None, None] * S + (np.exp(gl[:, None] - G)[:, :, None] * kc).transpose(0, 2, 1) @ delta
    rms = np.sqrt((out * out).mean(-1, keepdims=True) + dims.eps)
    gate = 1.0 / (1.0 + np.exp(-z.reshape(T, Hv, dv)))
    gated = (w["norm"].astype(np.float64) * (out / rms) * gate).reshape(T, Vd)
    y = gated @ w["output"].astype(np.float64).T
    return y, S


def test_f64_restatement_matches_oracle(oracle):
    """CPU check of the float64 restatement used for the 8192-token drift
    bound: on a small layer (300 tokens, five chunks with a partial last one)
    it agrees with the oracle's F32 token recurrence at the parity tolerance."""
    from kqb200 import synth
    dims = synth.GdnDims(hidden=256, key_heads=2, value_heads=4)
    weights = synth.gdn_layer(77, dims, synth.TYPE_Q6_K, synth.TYPE_Q6_K, synth.TYPE_Q6_K)
    w = oracle.gdn_weights_f32(weights)
    x = synth.hidden(78, 300, dims.hidden)
    st, yo, _, reco = oracle.gdn_run(dims, w, x, *synth.gdn_state(0, dims, zero=True))
    assert st == 0
    y64, S64 = gdn_layer_f64(dims, w, x)
    assert_close(y64, yo, "float64 restatement outputs")
    assert_close(S64, reco, "float64 restatement state")


@pytest.mark.gpu
def test_config2_gdn_prefill_8192_full_dims(kq, oracle):
    """one GDN layer (hidden 2048, 16 x 128 key heads,
    32 x 128 value heads, Q6_K projections, zero initial state) prefills 8192
    tokens in one call (128 chunks of 64).  Checked against the oracle on
    128-token windows at t0 = 0, 4096 and 8064, each started from the state a
    GPU prefill of the first t0 tokens exported: outputs of the full call
    over the window, and the state at t0 + 128 (a GPU prefill of t0 + 128
    tokens, or the full call's end state).  The full call's outputs and end
    state are also compared with the float64 restatement over all 8192
    tokens."""
    import torch
    from kqb200 import synth
    dims = synth.GdnDims()
    weights = synth.gdn_layer(202, dims, synth.TYPE_Q6_K, synth.TYPE_Q6_K, synth.TYPE_Q6_K)
    w = oracle.gdn_weights_f32(weights)
    T, W = 8192, 128
    x = synth.hidden(203, T, dims.hidden)
    prov = kq.Provider(0)
    layer = kq.GdnLayer(dims, weights, prov)
    try:
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        scratch = torch.empty_like(xd)
        torch.cuda.synchronize()
        s = kq.GdnState(layer)
        kq.gdn_prefill_async(s, xd.data_ptr(), T, yd.data_ptr())
        kq.synchronize()
        y_full = yd.cpu().numpy()
        conv_T, rec_T, init = s.save()
        s.close()
        assert init == 1 and np.isfinite(y_full).all()

        def prefix_state(n):
            st = kq.GdnState(layer)
            kq.gdn_prefill_async(st, xd.data_ptr(), n, scratch.data_ptr())
            kq.synchronize()
            c, r, _ = st.save()
            st.close()
            return c, r

        zero = synth.gdn_state(0, dims, zero=True)
        starts = [0, 4096, T - W]
        start_state = {t0: (zero if t0 == 0 else prefix_state(t0)) for t0 in starts}
        end_state = {t0: ((conv_T, rec_T) if t0 + W == T else prefix_state(t0 + W)) for t0 in starts}
        runs = pool_map(lambda t0: oracle.gdn_run(dims, w, x[t0:t0 + W], *start_state[t0]), starts)
        for t0, (st, yo, convo, reco) in zip(starts, runs):
            assert st == 0
            assert_close(y_full[t0:t0 + W], yo, f"outputs [{t0}, {t0 + W})")
            assert_close(end_state[t0][1], reco, f"recurrent state at {t0 + W}")
            assert_close(end_state[t0][0], convo, f"conv state at {t0 + W}")

        y64, S64 = gdn_layer_f64(dims, w, x)
        assert_close(y_full, y64, "8192-token outputs against float64")
        assert_close(rec_T, S64, "end state against float64")
    finally:
        layer.close()
        prov.close()


# ----------------------------------------------------------------- config 3

@pytest.mark.gpu
def test_config3_block_decode_as_benched(kq, oracle):
    """BASELINE config 3 as bench.py runs it: the 4-layer block (3 GDN
    layers with Q4_K in-projections and Q6_K out-projections, then a QSA
    layer with Q4_K q/k/v, Q6_K o and BF16 index projections; hidden 2048,
    16/32 x 128 GDN heads, 16/2 x 256 QSA heads, budget 2048) decodes one
    token for 64 sequences whose contexts are drawn from U[1k, 32k] (seed 0),
    through the batched entry points.  Four sequences (the longest, the
    shortest and two more above 16k) are checked layer by layer against the
    oracle, each layer on the GPU's input to it: outputs and GDN states
    within tolerance, the QSA block selection exactly (read through the
    reference-shaped entry point on a copy of the sequence's cache)."""
    import torch
    from kqb200 import synth
    gd, qd = synth.GdnDims(), synth.QsaDims()
    gdn_w = [synth.gdn_layer(l, gd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K) for l in range(3)]
    qsa_w = synth.qsa_layer(7, qd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_BF16)
    B = 64
    ctx = np.random.default_rng(0).integers(1024, 32768 + 1, size=B)
    order = np.argsort(ctx)
    long_ones = [int(b) for b in order[::-1] if ctx[b] > 16384]
    pick = sorted({int(order[-1]), int(order[0]), long_ones[1], long_ones[len(long_ones) // 2]})
    prov = kq.Provider(0)
    glayers = [kq.GdnLayer(gd, w, prov, layer=l) for l, w in enumerate(gdn_w)]
    qlayer = kq.QsaLayer(qd, qsa_w, prov, layer=3)
    gstates, qstates = [], []
    try:
        gen = torch.Generator(device="cuda")
        gen.manual_seed(1234)
        lib = kq.lib()
        for layer in glayers:
            row = []
            for _ in range(B):
                s = kq.GdnState(layer)
                conv = torch.randn(gd.conv_channels * 4, device="cuda", generator=gen)
                rec = torch.randn(gd.value_heads * gd.key_dim * gd.value_dim, device="cuda", generator=gen) * 0.02
                torch.cuda.synchronize()
                d = kq.abi.Diagnostic()
                kq.abi.check(lib.kq_gdn_state_import_f32(s.handle, conv.data_ptr(), conv.numel(), rec.data_ptr(),
                                                         rec.numel(), 1, C.byref(d)), d)
                row.append(s)
            gstates.append(row)
        for b in range(B):
            L = int(ctx[b])
            s = kq.QsaState(qlayer, L + 1)
            k = torch.randn(L, qd.kv_width, device="cuda", generator=gen)
            v = torch.randn(L, qd.kv_width, device="cuda", generator=gen)
            r = torch.randn(L, qd.index_dim, device="cuda", generator=gen)
            torch.cuda.synchronize()
            d = kq.abi.Diagnostic()
            kq.abi.check(lib.kq_qsa_state_import_f32(s.handle, k.data_ptr(), k.numel(), v.data_ptr(), v.numel(),
                                                     r.data_ptr(), r.numel(), L, C.byref(d)), d)
            qstates.append(s)
        pre_g = {b: [gstates[l][b].save()[:2] for l in range(3)] for b in pick}
        pre_q = {b: qstates[b].save() for b in pick}

        h = [torch.randn(B, gd.hidden, device="cuda", generator=gen)]
        torch.cuda.synchronize()   # the library's stream does not wait for torch's
        for l in range(3):
            h.append(torch.empty_like(h[0]))
            kq.gdn_decode_batch(glayers[l], gstates[l], h[l].data_ptr(), h[l + 1].data_ptr())
        y = torch.empty_like(h[0])
        kq.qsa_decode_batch(qlayer, qstates, h[3].data_ptr(), y.data_ptr())
        kq.synchronize()
        hs = [t.cpu().numpy() for t in h]
        yb = y.cpu().numpy()
        post_g = {b: [gstates[l][b].save()[:2] for l in range(3)] for b in pick}
        assert all(qstates[b].length == ctx[b] + 1 for b in range(B))

        # the GPU's selection for each picked sequence, through the
        # reference-shaped entry point on a copy of its pre-step cache
        single = {}
        for b in pick:
            s = kq.QsaState(qlayer, int(ctx[b]) + 1)
            s.load(*pre_q[b])
            single[b] = s.execute_quantized(hs[3][b:b + 1], want_selection=True)
            s.close()

        gw = [oracle.gdn_weights_f32(w) for w in gdn_w]
        qw = oracle.qsa_weights_f32(qsa_w)
        jobs = [("g", b, l) for b in pick for l in range(3)] + [("q", b, 3) for b in pick]

        def run(job):
            kind, b, l = job
            if kind == "g":
                return oracle.gdn_run(gd, gw[l], hs[l][b:b + 1], *pre_g[b][l])
            L = int(ctx[b])
            return oracle.qsa_run(qd, qw, hs[3][b:b + 1], *pre_q[b], L, L + 1)

        for (kind, b, l), res in zip(jobs, pool_map(run, jobs)):
            assert res[0] == 0
            if kind == "g":
                _, yo, convo, reco = res
                assert_close(hs[l + 1][b], yo, f"seq {b} (ctx {ctx[b]}) GDN layer {l} output")
                assert_close(post_g[b][l][1], reco, f"seq {b} GDN layer {l} recurrent state")
                assert_close(post_g[b][l][0], convo, f"seq {b} GDN layer {l} conv state")
            else:
                yo, sels = res[1], res[6]
                y1, gsel = single[b]
                assert np.array_equal(gsel[0]["selected"], sels[0]["selected"]), f"seq {b} selection"
                assert_close(yb[b], yo, f"seq {b} (ctx {ctx[b]}) QSA output, batched")
                assert_close(y1, yo, f"seq {b} QSA output, single")
    finally:
        for row in gstates:
            for s in row:
                s.close()
        for s in qstates:
            s.close()
        for layer in glayers:
            layer.close()
        qlayer.close()
        prov.close()


# ----------------------------------------------------------------- config 4

def _assemble_gdn_state(tp, dims, shards, world):
    conv = np.zeros((dims.conv_channels, dims.conv_kernel), np.float32)
    rec = np.zeros((dims.value_heads, dims.key_dim * dims.value_dim), np.float32)
    for r, (c, s) in enumerate(shards):
        _, _, v0, nv = tp.gdn_head_range(dims, r, world)
        conv[tp.gdn_channels(dims, r, world)] = c.reshape(-1, dims.conv_kernel)
        rec[v0:v0 + nv] = s.reshape(nv, -1)
    return conv.reshape(-1), rec.reshape(-1)


def _assemble_qsa_state(tp, dims, shards, world):
    n = shards[0][0].shape[0]
    hd = dims.head_dim
    k = np.zeros((n, dims.kv_width), np.float32)
    v = np.zeros_like(k)
    for r, (ks, vs, rs) in enumerate(shards):
        _, _, kv0, nkv = tp.qsa_head_range(dims, r, world)
        k[:, kv0 * hd:(kv0 + nkv) * hd] = ks
        v[:, kv0 * hd:(kv0 + nkv) * hd] = vs
        assert np.array_equal(rs, shards[0][2]), "every shard holds the same raw index keys"
    return k, v, shards[0][2]


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_config4_head_group_shards_full_dims(kq, oracle, world):
    """BASELINE config 4 geometry (hidden 2048, 3 GDN layers of 16/32 x 128
    heads + 1 QSA layer of 16/2 x 256 heads, budget 2048, all projections
    Q4_K, index BF16) split into `world` head-group shards, every shard run
    on this GPU and the partial outputs summed per layer (what the
    all-reduce does).  An 8192-token prefill is followed by a 64-token
    window; each layer's window is compared with the oracle started from the
    full-layer state assembled from the shards' exported states, on the
    summed GPU input to that layer: outputs, and the GDN end states."""
    import torch
    from kqb200 import synth, tp
    gd, qd = synth.GdnDims(), synth.QsaDims()
    gdn_w = [synth.gdn_layer(20 + l, gd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K) for l in range(3)]
    qsa_w = synth.qsa_layer(27, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
    T0, W = 8192, 64
    T = T0 + W
    provs = [kq.Provider(0) for _ in range(world)]
    blocks = [tp.TensorParallelBlock(kq, provs[r], gdn_w, [qsa_w], r, world, capacity=T) for r in range(world)]
    try:
        x = torch.from_numpy(synth.hidden(4321, T, gd.hidden)).cuda()
        part = [[torch.zeros_like(x) for _ in range(4)] for _ in range(world)]
        sums = [torch.zeros_like(x) for _ in range(4)]

        def run(t0, n):
            src = x
            for layer in range(4):
                for r in range(world):
                    blocks[r].run_layer(layer, src[t0:t0 + n].data_ptr(), n, part[r][layer][t0:t0 + n].data_ptr())
                kq.synchronize()
                sums[layer][t0:t0 + n] = sum(part[r][layer][t0:t0 + n] for r in range(world))
                # the sum runs on torch's stream; the library's stream does not
                # wait for it
                torch.cuda.synchronize()
                src = sums[layer]

        def states():
            g = [_assemble_gdn_state(tp, gd, [blocks[r].gdn_states[l].save()[:2] for r in range(world)], world)
                 for l in range(3)]
            q = _assemble_qsa_state(tp, qd, [blocks[r].qsa_states[0].save() for r in range(world)], world)
            return g, q

        run(0, T0)
        g0, q0 = states()
        run(T0, W)
        g1, _ = states()
        ins = [x.cpu().numpy()[T0:]] + [s.cpu().numpy()[T0:] for s in sums[:3]]
        outs = [s.cpu().numpy()[T0:] for s in sums]
        gw = [oracle.gdn_weights_f32(w) for w in gdn_w]
        qw = oracle.qsa_weights_f32(qsa_w)

        def ref(layer):
            if layer < 3:
                return oracle.gdn_run(gd, gw[layer], ins[layer], *g0[layer])
            return oracle.qsa_run(qd, qw, ins[3], *q0, T0, T)

        for layer, res in enumerate(pool_map(ref, list(range(4)))):
            assert res[0] == 0
            assert_close(outs[layer], res[1], f"layer {layer} window outputs, {world} shards")
            if layer < 3:
                assert_close(g1[layer][1], res[3], f"layer {layer} recurrent state at {T}, {world} shards")
                assert_close(g1[layer][0], res[2], f"layer {layer} conv state at {T}, {world} shards")
    finally:
        for b in blocks:
            b.close()
        for p in provs:
            p.close()
