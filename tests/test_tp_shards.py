"""Head-group sharding of the tensor-parallel prefill, on CPU.

Each shard of a GDN or QSA layer (kqb200.tp) is run through the CPU oracle
as a layer of its own; the shards' outputs are partial sums of the
out-projection, so they must add up to the full layer's output, and each
shard's end state must be the matching slice of the full layer's end state
(bit for bit: the per-head work is the same arithmetic in the same order).
The two-rank test adds the partial outputs with a gloo all-reduce, the same
exchange the benchmark makes over NCCL.
"""
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def close(a, b, atol=2e-3, rtol=1e-3):
    """max-abs 2e-3 / relative 1e-3 (elementwise |a-b| <= atol + rtol*|b|)."""
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return bool(np.all(np.abs(a - b) <= atol + rtol * np.abs(b)))


def _gdn_case(seed=3):
    from kqb200 import synth
    dims = synth.GdnDims(hidden=128, key_heads=4, value_heads=8, key_dim=32, value_dim=32)
    layer = synth.gdn_layer(seed, dims, synth.TYPE_Q8_0, synth.TYPE_Q8_0, synth.TYPE_F32)
    conv, rec = synth.gdn_state(seed + 10, dims)
    x = synth.hidden(seed + 20, 6, dims.hidden)
    return dims, layer, conv, rec, x


def _qsa_case(seed=4, L0=41):
    from kqb200 import synth
    dims = synth.QsaDims(hidden=128, query_heads=8, kv_heads=2, head_dim=32, index_heads=2, index_dim=32,
                         block=4, budget=32, max_context=256, rotary=16)
    layer = synth.qsa_layer(seed, dims, synth.TYPE_Q8_0, index_type=synth.TYPE_BF16)
    k, v, r = synth.qsa_cache(seed + 5, dims, L0)
    x = synth.hidden(seed + 7, 5, dims.hidden)
    return dims, layer, (k, v, r), L0, x


def _gdn_shard_out(oracle, dims, layer, conv, rec, x, rank, world):
    from kqb200 import tp
    sw = tp.shard_gdn(layer, rank, world)
    c, r = tp.shard_gdn_state(dims, conv, rec, rank, world)
    return oracle.gdn_run(sw.dims, oracle.gdn_weights_f32(sw), x, c, r)


def _qsa_shard_out(oracle, dims, layer, cache, L0, x, rank, world, cap=128):
    from kqb200 import tp
    sw = tp.shard_qsa(layer, rank, world)
    k, v, r = tp.shard_qsa_cache(dims, *cache, rank, world)
    return oracle.qsa_run(sw.dims, oracle.qsa_weights_f32(sw), x, k, v, r, L0, cap)


@pytest.mark.parametrize("world", [1, 2, 4])
def test_gdn_shards_sum_to_the_full_layer(oracle, world):
    from kqb200 import tp
    dims, layer, conv, rec, x = _gdn_case()
    st, y, conv_full, rec_full = oracle.gdn_run(dims, oracle.gdn_weights_f32(layer), x, conv, rec)
    assert st == 0
    total = np.zeros_like(y, np.float64)
    for rank in range(world):
        st, yr, cr, rr = _gdn_shard_out(oracle, dims, layer, conv, rec, x, rank, world)
        assert st == 0
        total += yr
        c_want, r_want = tp.shard_gdn_state(dims, conv_full, rec_full, rank, world)
        assert np.array_equal(bits(cr), bits(c_want)), rank
        assert np.array_equal(bits(rr), bits(r_want)), rank
    if world == 1:
        assert np.array_equal(bits(total.astype(np.float32)), bits(y))
    assert close(total, y)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_qsa_shards_sum_to_the_full_layer(oracle, world):
    from kqb200 import tp
    dims, layer, cache, L0, x = _qsa_case()
    st, y, k_full, v_full, r_full, n, sels = oracle.qsa_run(dims, oracle.qsa_weights_f32(layer), x, *cache, L0, 128)
    assert st == 0
    total = np.zeros_like(y, np.float64)
    for rank in range(world):
        st, yr, kr, vr, rr, nr, selr = _qsa_shard_out(oracle, dims, layer, cache, L0, x, rank, world)
        assert st == 0 and nr == n
        total += yr
        k_want, v_want, r_want = tp.shard_qsa_cache(dims, k_full, v_full, r_full, rank, world)
        assert np.array_equal(bits(kr), bits(k_want)) and np.array_equal(bits(vr), bits(v_want))
        assert np.array_equal(bits(rr), bits(r_want))
        # the replicated indexer selects the same blocks on every rank
        for a, b in zip(selr, sels):
            assert np.array_equal(a["selected"], b["selected"])
    assert close(total, y)


def test_shard_geometry_and_rejections():
    from kqb200 import synth, tp
    g = synth.GdnDims()
    assert tp.gdn_head_range(g, 3, 8) == (6, 2, 12, 4)
    ch = tp.gdn_channels(g, 1, 8)
    assert len(ch) == 2 * 2 * 128 + 4 * 128 and ch[0] == 256 and ch[256] == 2048 + 256 and ch[512] == 4096 + 512
    q = synth.QsaDims()
    assert tp.qsa_head_range(q, 0, 1) == (0, 16, 0, 2)
    assert tp.qsa_head_range(q, 1, 2) == (8, 8, 1, 1)
    assert tp.qsa_head_range(q, 5, 8) == (10, 2, 1, 1)
    with pytest.raises(ValueError):
        tp.gdn_head_range(g, 0, 3)
    with pytest.raises(ValueError):
        tp.qsa_head_range(q, 0, 32)
    rng = np.random.default_rng(0)
    t = synth.pack_q4_k(rng, 4, 1024)
    part = tp.cols(t, 256, 768)
    assert part.cols == 512 and part.data.size == 4 * 2 * 144
    assert np.array_equal(part.data.reshape(4, -1), t.data.reshape(4, -1)[:, 144:432])
    with pytest.raises(ValueError):
        tp.cols(t, 128, 512)
    # more ranks than key/value heads: ranks split the tokens within a head group
    assert tp.qsa_token_part(q, 5, 8) == (1, 1, 4)
    assert tp.qsa_token_part(q, 1, 2) is None


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    for p in (REPO, REPO / "kestrel-q_b200"):
        sys.path.insert(0, str(p))
    import torch
    import torch.distributed as dist
    from oracle import oracle
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    dims, layer, conv, rec, x = _gdn_case()
    _, y, _, _ = _gdn_shard_out(oracle, dims, layer, conv, rec, x, rank, world)
    gdn = torch.from_numpy(np.ascontiguousarray(y))
    dist.all_reduce(gdn)
    qd, ql, cache, L0, xq = _qsa_case()
    _, yq, *_ = _qsa_shard_out(oracle, qd, ql, cache, L0, xq, rank, world)
    qsa = torch.from_numpy(np.ascontiguousarray(yq))
    dist.all_reduce(qsa)
    np.save(Path(out_dir) / f"gdn{rank}.npy", gdn.numpy())
    np.save(Path(out_dir) / f"qsa{rank}.npy", qsa.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_all_reduce_of_partial_outputs(oracle, tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    dims, layer, conv, rec, x = _gdn_case()
    _, y, _, _ = oracle.gdn_run(dims, oracle.gdn_weights_f32(layer), x, conv, rec)
    qd, ql, cache, L0, xq = _qsa_case()
    _, yq, *_ = oracle.qsa_run(qd, oracle.qsa_weights_f32(ql), xq, *cache, L0, 128)
    for r in range(2):
        g = np.load(tmp_path / f"gdn{r}.npy")
        q = np.load(tmp_path / f"qsa{r}.npy")
        assert close(g, y) and close(q, yq)
    # every rank holds the same reduced activations
    assert np.array_equal(np.load(tmp_path / "gdn0.npy"), np.load(tmp_path / "gdn1.npy"))
