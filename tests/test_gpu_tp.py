"""Tensor-parallel prefill on the GPU.

`test_head_group_shards_on_one_gpu` runs every rank's shards of a small
block (2 GDN layers + 1 QSA layer) through the library on one GPU, sums the
partial outputs after each layer (what the all-reduce does) and compares
each layer with the oracle run on the same input.  The two-GPU test runs the
benchmark's NCCL path (bench.py --workload prefill) on a small prefill and
needs two devices.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

REPO = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu


def assert_close(a, b, what, atol=2e-3, rtol=1e-3):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    err = np.abs(a - b) - (atol + rtol * np.abs(b))
    assert np.all(err <= 0), f"{what}: worst excess {err.max():.3g}"


@pytest.mark.parametrize("world", [2, 4])
def test_head_group_shards_on_one_gpu(kq, oracle, world):
    import torch
    from kqb200 import synth, tp
    gd = synth.GdnDims(hidden=512, key_heads=4, value_heads=8, key_dim=128, value_dim=128)
    qd = synth.QsaDims(hidden=512, query_heads=8, kv_heads=2, head_dim=128, index_heads=4, index_dim=128,
                       block=4, budget=64, max_context=1024, rotary=64)
    gdn_w = [synth.gdn_layer(80 + l, gd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K) for l in range(2)]
    qsa_w = synth.qsa_layer(85, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
    T = 150
    provs = [kq.Provider(0) for _ in range(world)]
    blocks = [tp.TensorParallelBlock(kq, provs[r], gdn_w, [qsa_w], r, world, capacity=256) for r in range(world)]
    try:
        x = torch.from_numpy(synth.hidden(86, T, gd.hidden)).cuda()
        bufs = [[torch.empty_like(x) for _ in range(3)] for _ in range(world)]
        src = x
        conv = np.zeros(gd.conv_channels * gd.conv_kernel, np.float32)
        rec = np.zeros(gd.value_heads * gd.key_dim * gd.value_dim, np.float32)
        for layer in range(3):
            for r in range(world):
                blocks[r].run_layer(layer, src.data_ptr(), T, bufs[r][layer].data_ptr())
            kq.synchronize()
            total = sum(bufs[r][layer] for r in range(world))
            xin = src.cpu().numpy()
            if layer < 2:
                st, yo, _, _ = oracle.gdn_run(gd, oracle.gdn_weights_f32(gdn_w[layer]), xin, conv, rec)
            else:
                z = np.zeros((256, qd.kv_width), np.float32)
                zr = np.zeros((256, qd.index_dim), np.float32)
                st, yo, *_ = oracle.qsa_run(qd, oracle.qsa_weights_f32(qsa_w), xin, z, z, zr, 0, 256)
            assert st == 0
            assert_close(total.cpu().numpy(), yo, f"layer {layer}, {world} shards")
            src = total
    finally:
        for b in blocks:
            b.close()
        for p in provs:
            p.close()


def test_two_gpu_nccl_prefill_runs():
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", "--master-port=29517", str(REPO / "bench.py"), "--gpus", "2",
           "--workload", "prefill", "--tokens", "4096", "--slice-tokens", "1024", "--steps", "2",
           "--warmup", "1", "--no-cpu-baseline"]
    out = subprocess.run(["timeout", "-k", "30", "600"] + cmd, capture_output=True, text=True, cwd=REPO)
    assert out.returncode == 0, out.stderr[-3000:]
    line = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][-1])
    assert line["n_gpus"] == 2 and line["value"] > 0 and line["scaling"] == "strong"


def _tp_worker(rank, world, port, out_dir, kv_heads):
    import os
    import sys
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    for p in (REPO, REPO / "kestrel-q_b200"):
        sys.path.insert(0, str(p))
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    import kqb200 as kq
    from kqb200 import synth, tp
    torch.cuda.set_device(rank)
    d = kq.abi.Diagnostic()
    kq.abi.check(kq.lib().kq_b200_set_device(rank, __import__("ctypes").byref(d)), d)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    gd, qd, gdn_w, qsa_w, T = _small_block(kv_heads)
    prov = kq.Provider(rank)
    stream = torch.cuda.ExternalStream(kq.lib().kq_b200_get_stream())
    block = tp.TensorParallelBlock(kq, prov, gdn_w, [qsa_w], rank, world, capacity=512,
                                   exchange=tp.torch_exchange(stream))
    x = torch.from_numpy(synth.hidden(96, T, gd.hidden)).cuda()
    bufs = [torch.empty_like(x) for _ in range(block.layer_count)]
    torch.cuda.synchronize()

    def all_reduce(t):
        return dist.all_reduce(t, async_op=True)

    with torch.cuda.stream(stream):
        block.prefill(x, bufs, T, all_reduce, slice_tokens=128)
    kq.synchronize()
    torch.cuda.synchronize()
    if rank == 0:
        for i, b in enumerate(bufs):
            np.save(Path(out_dir) / f"layer{i}.npy", b.cpu().numpy())
        np.save(Path(out_dir) / "x.npy", x.cpu().numpy())
    block.close()
    prov.close()
    dist.barrier()
    dist.destroy_process_group()


def _small_block(kv_heads=2):
    from kqb200 import synth
    gd = synth.GdnDims(hidden=512, key_heads=4, value_heads=8, key_dim=128, value_dim=128)
    qd = synth.QsaDims(hidden=512, query_heads=8, kv_heads=kv_heads, head_dim=256, index_heads=4, index_dim=128,
                       block=4, budget=128, max_context=1024, rotary=64)
    gdn_w = [synth.gdn_layer(90 + l, gd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K) for l in range(2)]
    qsa_w = synth.qsa_layer(95, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
    return gd, qd, gdn_w, qsa_w, 300


@pytest.mark.parametrize("kv_heads", [2, 1])
def test_two_gpu_tensor_parallel_block_with_sharded_indexer(oracle, tmp_path, kv_heads):
    """Two GPUs over NCCL: head-group shards, the QSA scores / top-k split by
    64-token chunk with one exchange of the selections, an all-reduce after
    every layer; each layer's reduced output against the oracle layer run on
    the same input.  With one key/value head the two ranks split the QSA
    attention by token instead of by query head."""
    import socket

    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_tp_worker, args=(2, port, str(tmp_path), kv_heads), nprocs=2, join=True)
    gd, qd, gdn_w, qsa_w, T = _small_block(kv_heads)
    src = np.load(tmp_path / "x.npy")
    conv = np.zeros(gd.conv_channels * gd.conv_kernel, np.float32)
    rec = np.zeros(gd.value_heads * gd.key_dim * gd.value_dim, np.float32)
    for layer in range(3):
        got = np.load(tmp_path / f"layer{layer}.npy")
        if layer < 2:
            st, yo, _, _ = oracle.gdn_run(gd, oracle.gdn_weights_f32(gdn_w[layer]), src, conv, rec)
        else:
            z = np.zeros((512, qd.kv_width), np.float32)
            zr = np.zeros((512, qd.index_dim), np.float32)
            st, yo, *_ = oracle.qsa_run(qd, oracle.qsa_weights_f32(qsa_w), src, z, z, zr, 0, 512)
        assert st == 0
        assert_close(got, yo, f"layer {layer}")
        src = got
