"""Multi-rank logic of bench.py on CPU: two gloo ranks on 127.0.0.1.

The decode benchmark shards sequences across ranks with no data-path
collective; the only exchange is the max-over-ranks of the device times.
These tests run that exchange and the sharding helpers with the gloo
backend (world size 2), no GPU involved.
"""
import json
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    sys.path.insert(0, str(REPO))
    import torch.distributed as dist
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    import bench
    per_rank = [(2.0, 4.0), (3.5, 3.0)][rank]          # (device ms, e2e ms) of this rank
    ms, e2e = bench.max_over_ranks(per_rank, world, "cpu")
    ctx = [int(c) for c in bench.contexts(rank)]
    out = {"ms": ms, "e2e": e2e, "value": bench.job_tokens_per_s(world, bench.BATCH, ms), "ctx": ctx}
    (Path(out_dir) / f"rank{rank}.json").write_text(json.dumps(out))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_times_reduce_to_the_slowest_rank(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    r0 = json.loads((tmp_path / "rank0.json").read_text())
    r1 = json.loads((tmp_path / "rank1.json").read_text())
    # every rank sees the max over ranks of each timer
    assert r0["ms"] == r1["ms"] == 3.5
    assert r0["e2e"] == r1["e2e"] == 4.0
    # whole-job throughput: both ranks' sequences over the slowest rank's time
    assert r0["value"] == pytest.approx(2 * 64 * 1000.0 / 3.5)
    # each rank serves its own sequences (different seeded contexts, same range)
    assert r0["ctx"] != r1["ctx"]
    assert all(1024 <= c <= 32768 for c in r0["ctx"] + r1["ctx"])
    assert len(r0["ctx"]) == len(r1["ctx"]) == 64


def test_single_rank_reduction_is_identity():
    sys.path.insert(0, str(REPO))
    import bench
    assert bench.max_over_ranks([1.25, 2.5], 1, "cpu") == [1.25, 2.5]
    assert bench.job_tokens_per_s(1, 64, 1.0) == pytest.approx(64000.0)


def test_reference_arm_runs_on_rank_zero_only():
    sys.path.insert(0, str(REPO))
    import bench
    # a non-zero rank returns at once, without touching the oracle
    assert bench.run_reference(None, rank=1, world=2) == 0


def test_reference_arm_prints_the_contract_line():
    """`bench.py --impl reference` times the reference's own CPU operators
    (oracle/_ref, else the restatement) on this host and prints one JSON
    line with the fields the driver reads."""
    import subprocess
    out = subprocess.run([sys.executable, str(REPO / "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, cwd=REPO, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["unit"] == "tok/s" and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 1 and line["n_gpus"] == 1
    assert line["value"] > 0 and line["config"]["workload"].startswith("config3")
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("reference", "port") and cb["cores"] >= 1
    assert line["e2e"] == {"value": line["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
