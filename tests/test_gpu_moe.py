"""GPU parity of the routed-expert MoE (kernels_moe.cu) through the C-ABI,
against the CPU oracle (pinned bit for bit to the compiled reference and to
the reference's golden vectors by test_oracle_pin.py).

Bars: expert selections EXACT (the router logits are an exact F32 product;
routing is EXACT_DISCRETE in the reference's own validation); router logits
bit-exact; probabilities within one F32 ulp (the softmax exponential is
correctly rounded here, the host libm's expf is not always); every other
value within |gpu - cpu| <= 2e-3 + 1e-3 * |cpu|.
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
    gpu = np.asarray(gpu, np.float32).reshape(-1).astype(np.float64)
    cpu = np.asarray(cpu, np.float32).reshape(-1).astype(np.float64)
    assert gpu.shape == cpu.shape, what
    err = np.abs(gpu - cpu)
    bad = np.nonzero(err > ATOL + RTOL * np.abs(cpu))[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance, worst {err.max():.3e} at {bad[:5]}"


def ulps(a, b):
    ia = bits(a).astype(np.int64)
    ib = bits(b).astype(np.int64)
    ia = np.where(ia & 0x80000000, -(ia & 0x7FFFFFFF), ia)
    ib = np.where(ib & 0x80000000, -(ib & 0x7FFFFFFF), ib)
    return np.abs(ia - ib)


def golden():
    meta = json.loads((GOLD / "moe_golden.json").read_text())
    return meta, np.load(GOLD / "moe_golden.npz")


def dims_of(kq, cfg):
    return kq.synth.MoeDims(hidden=cfg["hidden_size"], experts=cfg["expert_count"], top_k=cfg["top_k"],
                            routed=cfg["routed_intermediate_size"], shared=cfg["shared_intermediate_size"])


def same_checkpoints(gpu, cpu, K):
    """Same kinds, tokens, experts and positions in the same order; values
    within tolerance (logits bit-exact, probabilities within one ulp)."""
    assert len(gpu) == len(cpu)
    for g, c in zip(gpu, cpu):
        assert g[:4] == c[:4], (g[:4], c[:4])
        if g[0] == 0:
            assert np.array_equal(bits(g[4]), bits(c[4]))
        elif g[0] in (1, 2):
            assert ulps(g[4], c[4]).max() <= 1, g[:4]
        else:
            assert_close(g[4], c[4], f"checkpoint {g[:4]}")


def test_moe_golden_cases_f32_api(kq, oracle):
    """The reference's tier-A cases through kq_moe_execute_f32: selections
    exact, outputs and all 12 + 5k checkpoints per token against the oracle,
    and the final output against the golden value at the north-star bar."""
    meta, arr = golden()
    dims = dims_of(kq, meta["tier_a_config"])
    w = {k: arr[f"w_{k}"] for k in kq.abi.MOE_WEIGHT_FIELDS}
    layer = kq.MoeLayer(dims)
    try:
        for i, c in enumerate(meta["cases"]):
            x = arr[f"c{i}_input"]
            st, y, routes, cps, d = layer.execute_f32(w, x, route=True, checkpoints=True)
            assert st == 0, (c["id"], d.text())
            assert [r["ids"].tolist() for r in routes] == c["selected_expert_ids"], c["id"]
            so, yo, ro, co = oracle.moe_run(dims, w, x, "port", checkpoints=True)
            assert so == 0
            assert_close(y, yo, c["id"])
            assert_close(y, arr[f"c{i}_final_output"], c["id"] + " vs golden")
            for t, r in enumerate(routes):
                assert np.array_equal(bits(r["logits"]), bits(ro["logits"][t]))
                assert ulps(r["probabilities"], ro["probabilities"][t]).max() <= 1
                assert_close(r["weights"], ro["weights"][t], "selected weights")
            same_checkpoints(cps, co, dims.top_k)
    finally:
        layer.close()


def test_moe_routing_vectors_on_gpu(kq, oracle):
    """Tier-B routing vectors (512 experts, top-10: all-equal, k-th boundary
    tie, near ties, one dominant, ...) through kq_moe_route_f32: the selected
    ids of the reference's golden vectors, exactly."""
    meta, arr = golden()
    dims = dims_of(kq, meta["tier_b_config"])
    lib, abi = kq.lib(), kq.abi
    layer = kq.MoeLayer(dims)
    try:
        E, K = dims.experts, dims.top_k
        for j, c in enumerate(meta["routing_cases"]):
            router = np.ascontiguousarray(arr[f"r{j}_router"], np.float32)
            xs = arr[f"r{j}_input"]
            for t in range(xs.shape[0]):
                x = np.ascontiguousarray(xs[t], np.float32)
                lg, pr = np.zeros(E, np.float32), np.zeros(E, np.float32)
                ids, wt = np.zeros(K, np.uint32), np.zeros(K, np.float32)
                d = abi.Diagnostic()
                st = lib.kq_moe_route_f32(layer.handle, router.ctypes.data, router.size, x.ctypes.data,
                                          lg.ctypes.data, E, pr.ctypes.data, E, ids.ctypes.data, K, wt.ctypes.data, K,
                                          C.byref(d))
                assert st == 0, d.text()
                assert ids.tolist() == c["selected_expert_ids"][t], c["id"]
                assert np.allclose(pr, arr[f"r{j}_router_probabilities"][t], rtol=1e-4, atol=1e-7)
    finally:
        layer.close()


def _quantized_setup(kq, oracle, dims, seed):
    p = kq.Provider()
    weights = kq.synth.moe_layer(seed, dims)
    layer = kq.MoeLayer(dims, weights, p)
    return p, layer, oracle.moe_weights_f32(weights), weights


@pytest.mark.parametrize("T", [1, 3, 24, 64])
def test_moe_quantized_full_width(kq, oracle, T):
    """Full-width experts (hidden 2560, intermediate 640, top-10) in the
    target's GGUF types (gate/up Q4_K, down Q8_0, shared Q8_0, F32 router) on
    64 experts: a 64-token decode batch puts ~10 tokens on each expert (two
    token groups per weight pass); batches above 8 run the shared expert on
    the tensor-core projection."""
    dims = kq.synth.MoeDims(hidden=2560, experts=64, top_k=10, routed=640, shared=640)
    p, layer, w, _ = _quantized_setup(kq, oracle, dims, 41)
    try:
        x = kq.synth.hidden(100 + T, T, dims.hidden)
        st, y, routes, _, d = layer.execute_quantized(x, route=True)
        assert st == 0, d.text()
        so, yo, ro, _ = oracle.moe_run(dims, w, x, "port")
        assert so == 0
        for t, r in enumerate(routes):
            assert r["ids"].tolist() == ro["ids"][t].tolist(), t
            assert np.array_equal(bits(r["logits"]), bits(ro["logits"][t]))
        assert_close(y, yo, f"T={T}")
    finally:
        layer.close()
        p.close()


def test_moe_quantized_checkpoints(kq, oracle):
    """Provider mode with a checkpoint observer: the reference's 17 kinds in
    its order for every token and selected expert."""
    dims = kq.synth.MoeDims(hidden=512, experts=16, top_k=4, routed=128, shared=96)
    p, layer, w, _ = _quantized_setup(kq, oracle, dims, 7)
    try:
        x = kq.synth.hidden(8, 5, dims.hidden)
        st, y, _, cps, d = layer.execute_quantized(x, checkpoints=True)
        assert st == 0, d.text()
        so, yo, _, co = oracle.moe_run(dims, w, x, "port", checkpoints=True)
        assert so == 0
        assert len(cps) == 5 * (12 + 5 * dims.top_k)
        same_checkpoints(cps, co, dims.top_k)
        assert_close(y, yo)
    finally:
        layer.close()
        p.close()


def test_moe_async_batch_matches_sync(kq, oracle):
    """kq_b200_moe_execute_async on device arrays (the serving path) gives the
    synchronous call's output; a token chunk boundary (2048) is crossed."""
    import torch
    dims = kq.synth.MoeDims(hidden=256, experts=32, top_k=6, routed=64, shared=64)
    p, layer, w, _ = _quantized_setup(kq, oracle, dims, 3)
    try:
        T = 2100
        x = kq.synth.hidden(5, T, dims.hidden)
        st, y, _, _, d = layer.execute_quantized(x)
        assert st == 0, d.text()
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty_like(xd)
        kq.moe_execute_async(layer, xd.data_ptr(), T, yd.data_ptr())
        kq.synchronize()
        assert np.array_equal(bits(yd.cpu().numpy()), bits(y))
        so, yo, _, _ = oracle.moe_run(dims, w, x[:300], "port")
        assert so == 0
        assert_close(y[:300], yo)
    finally:
        layer.close()
        p.close()


def test_moe_routed_expert_and_provider_expert_linear(kq, oracle):
    """kq_moe_execute_routed_expert_f32 against the compiled reference's, and
    kq_weight_provider_linear_f32 reading one expert of a stack by id."""
    lib, abi = kq.lib(), kq.abi
    dims = kq.synth.MoeDims(hidden=256, experts=8, top_k=2, routed=64, shared=32)
    p, layer, w, weights = _quantized_setup(kq, oracle, dims, 11)
    try:
        H, I, e = dims.hidden, dims.routed, 5
        gate = np.ascontiguousarray(w["routed_gate"].reshape(dims.experts, I, H)[e])
        up = np.ascontiguousarray(w["routed_up"].reshape(dims.experts, I, H)[e])
        down = np.ascontiguousarray(w["routed_down"].reshape(dims.experts, H, I)[e])
        x = kq.synth.hidden(2, 1, H)[0]
        ew = abi.MoeExpertWeightsF32(gate.ctypes.data, gate.size, up.ctypes.data, up.size, down.ctypes.data,
                                     down.size)
        out = np.zeros(H, np.float32)
        scratch = np.zeros(lib.kq_moe_config_one_expert_workspace_bytes(layer.handle) // 4 + 1, np.float32)
        d = abi.Diagnostic()
        st = lib.kq_moe_execute_routed_expert_f32(layer.handle, C.byref(ew), e, x.ctypes.data, out.ctypes.data, H,
                                                  scratch.ctypes.data, scratch.nbytes, C.byref(d))
        assert st == 0, d.text()
        want = oracle.matvec(0, down.view(np.uint8).reshape(-1), H, I,
                             _swiglu(oracle.matvec(0, gate.view(np.uint8).reshape(-1), I, H, x)[0],
                                     oracle.matvec(0, up.view(np.uint8).reshape(-1), I, H, x)[0]))[0]
        assert_close(out, want, "routed expert")
        # provider: expert e of the gate part of the split gate/up semantic
        y = np.zeros(I, np.float32)
        ws = np.zeros(4096, np.float32)
        st = lib.kq_weight_provider_linear_f32(p.handle, layer.tensors.routed_gate_up, 1, e, I, H, x.ctypes.data,
                                               y.ctypes.data, I, ws.ctypes.data, ws.nbytes, C.byref(d))
        assert st == 0, d.text()
        assert_close(y, gate @ x, "provider expert linear")
        st = lib.kq_weight_provider_linear_f32(p.handle, layer.tensors.routed_gate_up, 1, dims.experts, I, H,
                                               x.ctypes.data, y.ctypes.data, I, ws.ctypes.data, ws.nbytes, C.byref(d))
        assert st == abi.INVALID_ARGUMENT
        st = lib.kq_weight_provider_linear_f32(p.handle, layer.tensors.routed_down, 0, 0xFFFFFFFF, H, I,
                                               x.ctypes.data, y.ctypes.data, H, ws.ctypes.data, ws.nbytes, C.byref(d))
        assert st == abi.TENSOR_LAYOUT_MISMATCH
    finally:
        layer.close()
        p.close()


def _swiglu(g, u):
    g = g.astype(np.float64)
    return (g / (1.0 + np.exp(-g)) * u).astype(np.float32)


def test_moe_non_finite_input_leaves_output_untouched(kq, oracle):
    """A non-finite token staged from device memory is reported as
    NUMERIC_DOMAIN by the device check, and the output is not written."""
    import torch
    dims = kq.synth.MoeDims(hidden=256, experts=8, top_k=2, routed=64, shared=32)
    p, layer, _, _ = _quantized_setup(kq, oracle, dims, 13)
    try:
        lib, abi = kq.lib(), kq.abi
        x = kq.synth.hidden(4, 3, dims.hidden)
        x[2, 7] = np.nan
        xd = torch.from_numpy(x).cuda()
        y = np.full((3, dims.hidden), 7.0, np.float32)
        scratch = np.zeros(layer.scratch_bytes // 4 + 1, np.float32)
        ws = np.zeros(16385, np.float32)
        d = abi.Diagnostic()
        st = lib.kq_moe_execute_quantized(layer.handle, p.handle, xd.data_ptr(), 3, y.ctypes.data, y.size,
                                          scratch.ctypes.data, scratch.nbytes, ws.ctypes.data, ws.nbytes,
                                          abi.MOE_ROUTE_OBSERVER(), abi.MOE_CHECKPOINT_OBSERVER(), None, C.byref(d))
        assert st == abi.NUMERIC_DOMAIN
        assert np.all(y == 7.0)
    finally:
        layer.close()
        p.close()
