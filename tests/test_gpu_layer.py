"""GPU parity of the decoder layer (api_layer.cpp, kernels_layer.cu: gated
residual, GDN or QSA mixer, gated residual, MoE) through the C-ABI, against
the CPU oracle's layer (pinned bit for bit to the compiled reference's
kq_layer_prefill_f32 and to the reference's golden layer cases by
test_oracle_pin.py).

Bar: every output and checkpoint within |gpu - cpu| <= 2e-3 + 1e-3 * |cpu|;
checkpoint kinds, tokens, ranks and dimensions in the reference's order.
"""
import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3
GOLD = Path(__file__).resolve().parent / "golden"


def assert_close(gpu, cpu, what=""):
    gpu = np.asarray(gpu, np.float32).reshape(-1).astype(np.float64)
    cpu = np.asarray(cpu, np.float32).reshape(-1).astype(np.float64)
    assert gpu.shape == cpu.shape, what
    err = np.abs(gpu - cpu)
    bad = np.nonzero(err > ATOL + RTOL * np.abs(cpu))[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance, worst {err.max():.3e} at {bad[:5]}"


def same_checkpoints(gpu, cpu):
    assert len(gpu) == len(cpu)
    for g, c in zip(gpu, cpu):
        assert g[:4] == c[:4], (g[:4], c[:4])
        assert_close(g[4], c[4], f"checkpoint {g[:4]}")


def golden():
    meta = json.loads((GOLD / "layer_golden.json").read_text())
    return meta, np.load(GOLD / "layer_golden.npz")


def golden_layer(kq, oracle, meta, arr, i):
    """GPU layer (F32 test configs) and the oracle's arguments for golden
    case i (the reduced geometry of the reference's layer fixture)."""
    from test_oracle_pin import layer_case
    ld, gr, md, mw, moe_d, moe_w = layer_case(oracle, meta, arr, i)
    fam = ld[4]
    mixer = kq.GdnLayer(md) if fam == 1 else kq.QsaLayer(md)
    moe = kq.MoeLayer(moe_d)
    layer = kq.DecoderLayer(fam, 8, 4, 4, 1e-6, mixer, moe)
    weights = {"attn": gr["attn"], "moe_gr": gr["moe"], "mixer": mw, "moe": moe_w}
    return layer, mixer, moe, weights, (ld, gr, md, mw, moe_d, moe_w)


@pytest.mark.parametrize("case", [0, 1, 2, 3])
def test_layer_golden_cases_f32_api(kq, oracle, case):
    """The reference's golden GDN / QSA layer cases through
    kq_layer_prefill_f32 (a 4-token prefill from a zero state, every
    checkpoint observed), then two one-token calls on the same state."""
    meta, arr = golden()
    layer, mixer, moe, weights, args = golden_layer(kq, oracle, meta, arr, case)
    ld, gr, md, mw, moe_d, moe_w = args
    state = layer.state(16)
    try:
        x = arr[f"c{case}_input"]
        st, y, cps, met, d = state.run_f32(weights, x, checkpoints=True)
        assert st == 0, d.text()
        assert_close(y, arr[f"c{case}_output"], "vs golden")
        rng = np.random.default_rng(case)
        steps = [rng.normal(0, 0.3, (1, 32)).astype(np.float32) for _ in range(2)]
        ref = oracle.layer_sequence("port", ld, gr, md, mw, moe_d, moe_w, [x] + steps, capacity=16,
                                    checkpoints=True)
        assert ref[0][0] == 0
        assert_close(y, ref[0][1], "prefill vs oracle")
        same_checkpoints(cps, ref[0][2])
        assert met.tokens_processed == 4 and state.position == 4
        for j, xs in enumerate(steps):
            st, y, cps, _, d = state.run_f32(weights, xs, checkpoints=True)
            assert st == 0, d.text()
            assert_close(y, ref[1 + j][1], f"step {j}")
            same_checkpoints(cps, ref[1 + j][2])
        assert state.position == 6
    finally:
        state.close()
        layer.close()
        mixer.close()
        moe.close()


def quantized_layer(kq, oracle, family, seed):
    """A provider-bound layer (hidden 256, 4 branches, rank 32; Q8_0 mixer
    projections, Q4_K / Q8_0 MoE with 8 experts top-2, BF16 gated residual)
    and the oracle's F32 arguments (dequantised weights)."""
    s = kq.synth
    p = kq.Provider()
    if family == 1:
        md = s.GdnDims(hidden=256, key_heads=1, value_heads=2, key_dim=128, value_dim=128, conv_kernel=4, eps=1e-6)
        mwq = s.gdn_layer(seed, md, s.TYPE_Q8_0, s.TYPE_Q8_0, s.TYPE_F32)
        mixer = kq.GdnLayer(md, mwq, p, layer=0)
        mw = oracle.gdn_weights_f32(mwq)
    else:
        md = s.QsaDims(hidden=256, query_heads=2, kv_heads=1, head_dim=64, index_heads=2, index_dim=64, block=4,
                       budget=16, max_context=64, rotary=32, eps=1e-6, theta=1e7)
        mwq = s.qsa_layer(seed, md, s.TYPE_Q8_0, s.TYPE_Q8_0, s.TYPE_BF16)
        mixer = kq.QsaLayer(md, mwq, p, layer=0)
        mw = oracle.qsa_weights_f32(mwq)
    moe_d = s.MoeDims(hidden=256, experts=8, top_k=2, routed=64, shared=64)
    moe_q = s.moe_layer(seed + 1, moe_d)
    moe = kq.MoeLayer(moe_d, moe_q, p, layer=0)
    grq = {"attn": s.gr_weights(seed + 2, 256, 4, 32), "moe": s.gr_weights(seed + 3, 256, 4, 32)}
    layer = kq.DecoderLayer(family, 256, 4, 32, 1e-6, mixer, moe, grq, p)

    def deq(t):
        return oracle.dequantize(t.type_id, t.data).reshape(-1)

    gr = {k: {"norm": g.norm, "down": deq(g.down), "up": deq(g.up), "inject": deq(g.inject)} for k, g in grq.items()}
    args = ((256, 4, 32, 1e-6, family), gr, md, mw, moe_d, oracle.moe_weights_f32(moe_q))
    return p, layer, mixer, moe, args


@pytest.mark.parametrize("family", [1, 2])
def test_layer_quantized_prefill_then_decode_batch(kq, oracle, family):
    """Provider mode: three sequences prefilled through
    kq_layer_prefill_quantized_f32 (5, 3 and 7 tokens), then one token of
    each through the batched device entry point kq_b200_layer_decode_batch;
    every output against the oracle's layer run of that sequence."""
    import torch
    p, layer, mixer, moe, args = quantized_layer(kq, oracle, family, 20 + family)
    states = [layer.state(64) for _ in range(3)]
    try:
        rng = np.random.default_rng(family)
        pre = [rng.normal(0, 1, (n, 1024)).astype(np.float32) for n in (5, 3, 7)]
        dec = rng.normal(0, 1, (3, 1024)).astype(np.float32)
        ys = []
        for s_, x in zip(states, pre):
            st, y, _, _, d = s_.run_quantized(x)
            assert st == 0, d.text()
            ys.append(y)
        xd = torch.from_numpy(dec).cuda()
        yd = torch.empty_like(xd)
        kq.layer_decode_batch(layer, states, xd.data_ptr(), yd.data_ptr())
        kq.synchronize()
        yb = yd.cpu().numpy()
        for i in range(3):
            ref = oracle.layer_sequence("port", *args, [pre[i], dec[i:i + 1]], capacity=64)
            assert ref[0][0] == 0 and ref[1][0] == 0
            assert_close(ys[i], ref[0][1], f"prefill {i}")
            assert_close(yb[i], ref[1][1], f"decode {i}")
            assert states[i].position == pre[i].shape[0] + 1
    finally:
        for s_ in states:
            s_.close()
        layer.close()
        mixer.close()
        moe.close()
        p.close()


@pytest.mark.parametrize("family", [1, 2])
def test_layer_rollback_and_failed_call(kq, oracle, family):
    """kq_layer_state_rollback_last undoes the last call once; a call with a
    non-finite token fails with NUMERIC_DOMAIN and leaves the state as it
    was; the following calls continue from the committed state."""
    p, layer, mixer, moe, args = quantized_layer(kq, oracle, family, 40 + family)
    state = layer.state(64)
    try:
        rng = np.random.default_rng(7)
        x0 = rng.normal(0, 1, (4, 1024)).astype(np.float32)
        x1, x2, x3 = (rng.normal(0, 1, (1, 1024)).astype(np.float32) for _ in range(3))
        assert state.run_quantized(x0)[0] == 0
        assert state.run_quantized(x1)[0] == 0
        assert state.position == 5
        assert state.rollback_last(1) == 0
        assert state.position == 4
        assert state.rollback_last(1) == kq.abi.INVALID_LAYER_STATE   # once per commit
        st, y2, *_ = state.run_quantized(x2)
        assert st == 0
        bad = x3.copy()
        bad[0, 17] = np.inf
        st, *_ = state.run_quantized(bad)
        assert st == kq.abi.NUMERIC_DOMAIN
        assert state.position == 5
        st, y3, *_ = state.run_quantized(x3)
        assert st == 0
        ref = oracle.layer_sequence("port", *args, [x0, x2, x3], capacity=64)
        assert all(r[0] == 0 for r in ref)
        assert_close(y2, ref[1][1], "after rollback")
        assert_close(y3, ref[2][1], "after the failed call")
    finally:
        state.close()
        layer.close()
        mixer.close()
        moe.close()
        p.close()
