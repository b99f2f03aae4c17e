"""GDN+QSA layer-block decode benchmark on B200.

Workload per GPU: a 4-layer hybrid block (3 GDN layers + 1 QSA layer, hidden
2048, GDN 16x128 key / 32x128 value heads, QSA 16 query / 2 KV heads of 256,
block 4, budget 2048) decoding one token for each of 64 independent
sequences whose contexts are drawn uniformly from [1k, 32k] (seed 0 + rank).
In-projections Q4_K, out-projections Q6_K, index projections BF16; F32 state
and KV caches.  A step = one token through the whole block for all 64
sequences.  Multi-GPU: one process per GPU, each rank serves its own 64
sequences (sequence sharding, no data-path collective; weak scaling).

Inputs are synthetic and seeded (no dataset): weights and states are drawn
with the distributions BASELINE.json names.  The per-step working set
(≈1.6 GB of state, KV and weights) is larger than the 126 MB L2, so no L2
flush is needed between steps.

`--workload prefill` runs BASELINE config 4 instead: one 131072-token
prefill of the same block (all projections Q4_K, index BF16) with the layers
tensor-parallel over the ranks (GDN by value-head group, QSA by query-head
group, indexer replicated) and one NCCL all-reduce of the partial outputs
after every layer's out-projection (strong scaling).

Arms:
  default          the B200 library through its C-ABI (kestrel-q_b200)
  --impl reference the reference's own CPU operators (oracle/_ref, compiled
                   from Kestrel-Q's C sources) on the host cores, same
                   metric, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
for _p in (REPO, REPO / "kestrel-q_b200"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

METRIC = "GDN+QSA block tok/s (decode B=64, prefill 8k) at 1-8 B200; % HBM/TC roofline"
BATCH = 64
CTX_RANGE = (1024, 32768)
GDN_LAYERS = 3


def peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops_sustained"]), "measured (bf16, sustained)"
    return 1400.0, "fallback (bf16, sustained)"


def dims():
    from kqb200 import synth
    return synth.GdnDims(), synth.QsaDims()


def contexts(rank: int, n: int = BATCH, ctx_max: int = CTX_RANGE[1]):
    rng = np.random.default_rng(0 + rank)
    return rng.integers(CTX_RANGE[0], ctx_max + 1, size=n)


def layer_weights():
    """The block's weights: one model, replicated on every rank."""
    from kqb200 import synth
    gd, qd = dims()
    gdn = [synth.gdn_layer(l, gd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
           for l in range(GDN_LAYERS)]
    qsa = synth.qsa_layer(7, qd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_BF16)
    return gdn, qsa


PREFILL_TOKENS = 131072
PREFILL_SLICE = 16384


def prefill_weights():
    """Config 4: the block with every projection Q4_K (index projections BF16)."""
    from kqb200 import synth
    gd, qd = dims()
    gdn = [synth.gdn_layer(20 + l, gd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K)
           for l in range(GDN_LAYERS)]
    qsa = synth.qsa_layer(27, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
    return gdn, qsa


def wy_flops_per_chunk_head(C: int = 64, d: int = 128) -> int:
    """FLOPs of the chunked WY form for one head and one chunk of C tokens
    (dk = dv = d): K K^T and Q K^T (2 C^2 d each), the two triangular solves
    for W and U (C^2 d each), the causal P delta (C^2 d), and W S, Q S,
    K^T delta against the d x d state (2 C d^2 each)."""
    return 7 * C * C * d + 6 * C * d * d


def prefill_flops(T: int):
    """Algorithmic FLOPs of one T-token prefill of the whole block (all
    ranks together), by part."""
    gd, qd = dims()
    H, C, Vd, Hv = gd.hidden, gd.conv_channels, gd.value_width, gd.value_heads
    gdn_proj = GDN_LAYERS * (2 * T * H * (C + Vd + 2 * Hv) + 2 * T * Vd * H)
    chunks = (T + 63) // 64
    wy = GDN_LAYERS * Hv * chunks * wy_flops_per_chunk_head(64, gd.key_dim)
    qw, kvw = qd.q_width, qd.kv_width
    iw = qd.index_heads * qd.index_dim + qd.index_dim
    qsa_proj = 2 * T * H * (2 * qw + 2 * kvw) + 2 * T * qw * H + 2 * T * H * iw
    pos = np.arange(T, dtype=np.int64)
    nb = (pos + 1) // qd.block
    ntok = np.minimum(nb, qd.budget // qd.block) * qd.block + (pos + 1) % qd.block
    indexer = int(2 * qd.index_heads * qd.index_dim * nb.sum())
    attention = int(4 * qd.query_heads * qd.head_dim * ntok.sum())
    parts = {"gdn_proj": gdn_proj, "gdn_wy": wy, "qsa_proj": qsa_proj, "qsa_indexer": indexer,
             "qsa_attention": attention}
    return sum(parts.values()), parts


def rank_tensor_core_flops(block, T: int) -> int:
    """FLOPs of the projections this rank runs on the tensor cores (all but
    the index projections, which take the exact CUDA-core path)."""
    f = 0
    for L in block.gdn_layers:
        d = L.dims
        f += 2 * T * d.hidden * (d.conv_channels + 2 * d.value_width + 2 * d.value_heads)
    for L in block.qsa_layers:
        d = L.dims
        f += 2 * T * d.hidden * (3 * d.q_width + 2 * d.kv_width)
    return f


def max_over_ranks(values, world: int, device):
    """Per-rank device times -> their maximum over all ranks (every rank
    calls this, in the same order, with the same number of values)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t]


def job_tokens_per_s(world: int, batch_per_rank: int, ms_per_step: float) -> float:
    """Whole-job throughput: every rank decodes batch_per_rank tokens per step."""
    return world * batch_per_rank * 1000.0 / ms_per_step


def algorithmic_bytes(gdn, qsa, ctx, batch):
    """HBM bytes one step must move at minimum (per GPU): every weight once,
    GDN state and conv state read + written once, QSA K/V read only for the
    selected tokens, cached block keys once, new K/V/raw rows written, and
    the block's activations."""
    gd, qd = dims()
    w = sum(t.nbytes for L in gdn for t in (L.qkv, L.gate, L.beta, L.alpha, L.output))
    w += sum(t.nbytes for t in (qsa.query, qsa.key, qsa.value, qsa.output, qsa.index_query, qsa.index_key))
    rec = gd.value_heads * gd.key_dim * gd.value_dim * 4
    conv = gd.conv_channels * gd.conv_kernel * 4
    state = GDN_LAYERS * batch * 2 * (rec + conv)
    kv = 0
    for L in ctx:
        pos = int(L)  # position of the new token
        nb = (pos + 1) // qd.block
        ntok = min(nb, qd.budget // qd.block) * qd.block + (pos + 1) % qd.block
        kv += ntok * qd.kv_width * 4 * 2 + nb * qd.index_dim * 4
        kv += (2 * qd.kv_width + qd.index_dim) * 4
    act = (GDN_LAYERS + 1) * 2 * batch * gd.hidden * 4
    return w + state + kv + act, {"weights": w, "gdn_state": state, "qsa_kv_and_block_keys": kv,
                                  "activations": act}


def recurrence_bytes_per_launch(batch):
    """Algorithmic HBM bytes of one launch of the fused decode kernel
    (conv / gates + delta-rule recurrence + gated RMSNorm) for `batch`
    sequences: the recurrent state read and written, the conv state read and
    written, the projected row read (q | k | v | gate | beta | alpha) and the
    gated output written, each once."""
    gd, _ = dims()
    state = gd.value_heads * gd.key_dim * gd.value_dim * 4 * 2
    conv = gd.conv_channels * gd.conv_kernel * 4 * 2
    proj_row = (gd.conv_channels + gd.value_width + 2 * gd.value_heads) * 4
    out = gd.value_width * 4
    return batch * (state + conv + proj_row + out)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons during the timed region."""

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines = []

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            parts = [p.strip() for p in l.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[3:7]):
                if v.lower() in ("active", "1", "0x1"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU arm

def cpu_block_sample(n_seqs: int, threads: int, rank: int = 0):
    """The reference's own F32 operators (oracle/_ref when built, else the
    restatement) decoding one token of the 4-layer block for `n_seqs`
    sequences of the workload, `threads` sequences in parallel.
    Returns (tokens_per_second, kind, seconds)."""
    from kqb200 import synth
    from oracle import oracle as O
    impl = "reference" if O.ref_available() else "port"
    gd, qd = dims()
    gdn, qsa = layer_weights()
    gw = [O.gdn_weights_f32(L) for L in gdn]
    qw = O.qsa_weights_f32(qsa)
    ctx = contexts(rank)[:n_seqs]

    def one(i):
        rng = np.random.default_rng(10_000 + i)
        L = int(ctx[i])
        x = rng.normal(size=(1, gd.hidden)).astype(np.float32)
        states = [(rng.normal(0, 1, gd.conv_channels * 4).astype(np.float32),
                   rng.normal(0, 0.02, gd.value_heads * gd.key_dim * gd.value_dim).astype(np.float32))
                  for _ in range(GDN_LAYERS)]
        k = rng.standard_normal((L, qd.kv_width), np.float32)
        v = rng.standard_normal((L, qd.kv_width), np.float32)
        r = rng.standard_normal((L, qd.index_dim), np.float32)
        t0 = time.perf_counter()
        h = x
        for l in range(GDN_LAYERS):
            st, h, _, _ = O.gdn_run(gd, gw[l], h, *states[l], impl=impl)
            assert st == 0
        st, h, *_ = O.qsa_run(qd, qw, h, k, v, r, L, L + 1, impl=impl)
        assert st == 0
        return time.perf_counter() - t0

    t0 = time.perf_counter()
    with cf.ThreadPoolExecutor(max_workers=threads) as pool:
        list(pool.map(one, range(n_seqs)))
    elapsed = time.perf_counter() - t0
    return n_seqs / elapsed, impl, elapsed


def cpu_prefill_sample(tokens: int):
    """The reference's own F32 operators (oracle/_ref when built, else the
    restatement) prefilling the first `tokens` tokens of the config-4 block
    from empty states, one thread (the reference prefill of one sequence is
    sequential).  Returns (tokens_per_second, kind, seconds)."""
    from oracle import oracle as O
    impl = "reference" if O.ref_available() else "port"
    gd, qd = dims()
    gdn, qsa = prefill_weights()
    gw = [O.gdn_weights_f32(L) for L in gdn]
    qw = O.qsa_weights_f32(qsa)
    x = np.random.default_rng(99).normal(size=(tokens, gd.hidden)).astype(np.float32)
    conv = np.zeros(gd.conv_channels * gd.conv_kernel, np.float32)
    rec = np.zeros(gd.value_heads * gd.key_dim * gd.value_dim, np.float32)
    z = np.zeros((tokens, qd.kv_width), np.float32)
    zr = np.zeros((tokens, qd.index_dim), np.float32)
    t0 = time.perf_counter()
    h = x
    for l in range(GDN_LAYERS):
        st, h, _, _ = O.gdn_run(gd, gw[l], h, conv, rec, impl=impl)
        assert st == 0
    st, h, *_ = O.qsa_run(qd, qw, h, z, z, zr, 0, tokens, impl=impl)
    assert st == 0
    elapsed = time.perf_counter() - t0
    return tokens / elapsed, impl, elapsed


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference_prefill(args, rank, world):
    if rank != 0:
        return 0
    from oracle import oracle as O
    if not O.PORT_LIB.exists():
        O.build()
    n = args.cpu_tokens
    cpu_prefill_sample(2)
    vals, kind = [], "reference"
    t_all = time.perf_counter()
    for _ in range(args.steps):
        v, impl, _ = cpu_prefill_sample(n)
        kind = "reference" if impl == "reference" else "port"
        vals.append(v)
    elapsed = time.perf_counter() - t_all
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config4: 4-layer GDN+QSA block prefill, batch 1, Q4_K",
                   "sample": f"first {n} tokens of the prefill per step"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": 1, "kind": kind,
                         "sample": f"first {n} tokens of the 4-layer block prefill from empty states, 1 thread"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    if args.workload == "prefill":
        return run_reference_prefill(args, rank, world)
    threads = min(cpu_threads(), 16)
    n = threads
    from oracle import oracle as O
    if not O.PORT_LIB.exists():
        O.build()
    for _ in range(args.warmup if args.warmup < 1 else 1):
        cpu_block_sample(min(2, n), min(2, threads))
    vals = []
    kind = "reference"
    t_all = time.perf_counter()
    for _ in range(args.steps):
        v, impl, _ = cpu_block_sample(n, threads)
        kind = "reference" if impl == "reference" else "port"
        vals.append(v)
    elapsed = time.perf_counter() - t_all
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / max(1, args.steps),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config3: 4-layer GDN+QSA block decode, B=64, ctx U[1k,32k]",
                   "sample": f"{n} sequences x 1 token per step"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": kind,
                         "sample": f"{n} sequences x 1 token of the 4-layer block, {threads} threads"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- B200 arm

def run_b200(args, rank, world, local_rank):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import kqb200
    from kqb200 import synth

    torch.cuda.set_device(local_rank)
    d = kqb200.abi.Diagnostic()
    kqb200.abi.check(kqb200.lib().kq_b200_set_device(local_rank, C.byref(d)), d)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    gd, qd = dims()
    gdn_w, qsa_w = layer_weights()
    ctx = contexts(rank, ctx_max=args.ctx_max)
    B = BATCH
    steps_total = args.warmup + 2 * args.steps + 40
    prov = kqb200.Provider(local_rank)
    gdn_layers = [kqb200.GdnLayer(gd, w, prov, layer=l) for l, w in enumerate(gdn_w)]
    qsa_layer = kqb200.QsaLayer(qd, qsa_w, prov, layer=3)

    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234 + rank)
    gdn_states = []
    for layer in gdn_layers:
        row = []
        for b in range(B):
            s = kqb200.GdnState(layer)
            conv = torch.randn(gd.conv_channels * 4, device="cuda", generator=gen)
            rec = torch.randn(gd.value_heads * gd.key_dim * gd.value_dim, device="cuda", generator=gen) * 0.02
            torch.cuda.synchronize()
            dd = kqb200.abi.Diagnostic()
            kqb200.abi.check(kqb200.lib().kq_gdn_state_import_f32(s.handle, conv.data_ptr(), conv.numel(),
                                                                  rec.data_ptr(), rec.numel(), 1, C.byref(dd)), dd)
            row.append(s)
        gdn_states.append(row)
    qsa_states = []
    for b in range(B):
        L = int(ctx[b])
        s = kqb200.QsaState(qsa_layer, L + steps_total)
        k = torch.randn(L, qd.kv_width, device="cuda", generator=gen)
        v = torch.randn(L, qd.kv_width, device="cuda", generator=gen)
        r = torch.randn(L, qd.index_dim, device="cuda", generator=gen)
        torch.cuda.synchronize()
        dd = kqb200.abi.Diagnostic()
        kqb200.abi.check(kqb200.lib().kq_qsa_state_import_f32(s.handle, k.data_ptr(), k.numel(), v.data_ptr(),
                                                              v.numel(), r.data_ptr(), r.numel(), L, C.byref(dd)), dd)
        del k, v, r
        qsa_states.append(s)
    torch.cuda.synchronize()

    lib = kqb200.lib()
    stream = torch.cuda.ExternalStream(lib.kq_b200_get_stream())
    bufs = [torch.randn(B, gd.hidden, device="cuda", generator=gen) for _ in range(GDN_LAYERS + 2)]
    torch.cuda.synchronize()

    def step(x_ptr, y_ptr):
        h_in = x_ptr
        for l in range(GDN_LAYERS):
            kqb200.gdn_decode_batch(gdn_layers[l], gdn_states[l], h_in, bufs[l + 1].data_ptr())
            h_in = bufs[l + 1].data_ptr()
        kqb200.qsa_decode_batch(qsa_layer, qsa_states, h_in, y_ptr)

    x0, y0 = bufs[0].data_ptr(), bufs[GDN_LAYERS + 1].data_ptr()
    for _ in range(args.warmup):
        step(x0, y0)
    kqb200.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()

    # ---- device-resident timed region
    lib.kq_b200_profile_kernel(b"gdn_recurrence")
    launches0 = lib.kq_b200_kernel_launch_count()
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize()
        kqb200.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step(x0, y0)
        e1.record(stream)
        kqb200.synchronize()
        torch.cuda.synchronize()
        barrier()
    launches = lib.kq_b200_kernel_launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    rec_n, rec_ms = C.c_uint64(), C.c_double()
    lib.kq_b200_profile_read(C.byref(rec_n), C.byref(rec_ms))
    lib.kq_b200_profile_kernel(None)

    breakdown = {}
    if args.breakdown:
        for fam in ("proj", "proj_exact", "gdn_conv", "gdn_recurrence", "qsa_prepare", "qsa_score",
                    "qsa_select", "qsa_attend", "qsa_combine"):
            lib.kq_b200_profile_kernel(fam.encode())
            for _ in range(3):
                step(x0, y0)
            kqb200.synchronize()
            n_, t_ = C.c_uint64(), C.c_double()
            lib.kq_b200_profile_read(C.byref(n_), C.byref(t_))
            breakdown[fam] = {"ms_per_step": t_.value / 3, "launches_per_step": n_.value / 3}
        lib.kq_b200_profile_kernel(None)

    # ---- end-to-end: pinned host input -> block -> host result, every step
    xh = torch.randn(B, gd.hidden, generator=torch.Generator().manual_seed(5)).pin_memory()
    yh = torch.empty(B, gd.hidden).pin_memory()
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            bufs[0].copy_(xh, non_blocking=True)
            step(x0, y0)
            yh.copy_(bufs[GDN_LAYERS + 1], non_blocking=True)
    f1.record(stream)
    kqb200.synchronize()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    assert torch.isfinite(yh).all(), "non-finite block output"

    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world, torch.device("cuda", local_rank))

    step_bytes, parts = algorithmic_bytes(gdn_w, qsa_w, ctx, B)
    hbm, peak_kind = peaks()
    rec_avg_ms = rec_ms.value / max(1, rec_n.value)
    rec_bytes = recurrence_bytes_per_launch(B)
    achieved = rec_bytes / (rec_avg_ms * 1e-3) / 1e9
    traffic = None
    tf = REPO / "profiles" / "gdn_recurrence_traffic.json"
    if tf.exists():
        traffic = json.loads(tf.read_text()).get("bytes_per_launch_b64")
    line = {
        "metric": METRIC,
        "value": job_tokens_per_s(world, B, ms),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": f"config3: 4-layer block (3 GDN + 1 QSA) decode, 64 sequences/GPU, "
                        f"ctx U[1k,{args.ctx_max // 1024}k] (seed 0+rank), in-proj Q4_K, out-proj Q6_K, "
                        f"index BF16, F32 state/KV",
            "batch_per_gpu": B,
            "parallelism": f"sequence-sharded x{world} (no collective)",
            "l2": "working set per step >> 126 MB L2 (no flush needed)",
            "step_algorithmic_bytes": step_bytes,
            "step_bytes_breakdown": parts,
            "step_hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / hbm,
        },
        "roofline": {
            "kernel": "gdn_decode_fused (conv/gates + recurrence + gated norm; B=64, one GDN layer)",
            "bound": "hbm",
            "achieved": achieved,
            "peak": hbm,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / hbm,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": rec_bytes,
            "avg_launch_ms": rec_avg_ms,
            "launches_timed": rec_n.value,
        },
        "e2e": {"value": job_tokens_per_s(world, B, e2e_ms), "unit": "tok/s",
                "h2d_bytes_per_step": B * gd.hidden * 4, "d2h_bytes_per_step": B * gd.hidden * 4},
        "gpu_launches": int(launches),
        **({"kernel_breakdown": breakdown} if breakdown else {}),
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        threads = min(cpu_threads(), 16)
        v, impl, secs = cpu_block_sample(threads, threads, rank)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": threads,
                                "kind": "reference" if impl == "reference" else "port",
                                "sample": f"{threads} sequences x 1 token of the 4-layer block "
                                          f"({secs:.1f} s wall)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    # release
    for row in gdn_states:
        for s in row:
            s.close()
    for s in qsa_states:
        s.close()
    for L in gdn_layers:
        L.close()
    qsa_layer.close()
    prov.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def run_b200_prefill(args, rank, world, local_rank):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import kqb200
    from kqb200 import tp

    torch.cuda.set_device(local_rank)
    d = kqb200.abi.Diagnostic()
    kqb200.abi.check(kqb200.lib().kq_b200_set_device(local_rank, C.byref(d)), d)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
    gd, qd = dims()
    T = args.tokens
    gdn_w, qsa_w = prefill_weights()
    prov = kqb200.Provider(local_rank)
    lib = kqb200.lib()
    stream = torch.cuda.ExternalStream(lib.kq_b200_get_stream())
    exchange = tp.torch_exchange(stream) if world > 1 and not args.replicated_indexer else None
    block = tp.TensorParallelBlock(kqb200, prov, gdn_w, [qsa_w], rank, world, capacity=T, exchange=exchange)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4321)   # the same input on every rank (replicated activations)
    x = torch.randn(T, gd.hidden, device="cuda", generator=gen)
    bufs = [torch.empty(T, gd.hidden, device="cuda") for _ in range(block.layer_count)]
    torch.cuda.synchronize()

    def all_reduce(t):
        return dist.all_reduce(t, async_op=True)

    reduce = all_reduce if world > 1 else None

    def step(inp):
        block.reset()
        block.prefill(inp, bufs, T, reduce, slice_tokens=args.slice_tokens)

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step(x)
    kqb200.synchronize()
    torch.cuda.synchronize()

    lib.kq_b200_profile_kernel(b"proj")
    launches0 = lib.kq_b200_kernel_launch_count()
    with ClockSampler(local_rank) as clocks:
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                step(x)
            e1.record(stream)
        kqb200.synchronize()
        torch.cuda.synchronize()
        barrier()
    launches = lib.kq_b200_kernel_launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    proj_n, proj_ms = C.c_uint64(), C.c_double()
    lib.kq_b200_profile_read(C.byref(proj_n), C.byref(proj_ms))
    lib.kq_b200_profile_kernel(None)

    breakdown = {}
    if args.breakdown:
        for fam in ("proj", "proj_exact", "gdn_conv", "gdn_recurrence", "gdn_chunk_prep", "gdn_chunk_state",
                    "gdn_gate_norm", "qsa_prepare", "qsa_block_keys", "qsa_score", "qsa_select", "qsa_attend",
                    "qsa_combine"):
            lib.kq_b200_profile_kernel(fam.encode())
            with torch.cuda.stream(stream):
                step(x)
            kqb200.synchronize()
            torch.cuda.synchronize()
            n_, t_ = C.c_uint64(), C.c_double()
            lib.kq_b200_profile_read(C.byref(n_), C.byref(t_))
            breakdown[fam] = {"ms_per_step": t_.value, "launches_per_step": n_.value}
        lib.kq_b200_profile_kernel(None)

    # ---- end-to-end: pinned host input -> block -> host output, every step
    xh = torch.randn(T, gd.hidden, generator=torch.Generator().manual_seed(6)).pin_memory()
    yh = torch.empty(T, gd.hidden).pin_memory()
    xin = torch.empty_like(x)
    barrier()
    torch.cuda.synchronize()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(args.steps):
            xin.copy_(xh, non_blocking=True)
            step(xin)
            yh.copy_(bufs[-1], non_blocking=True)
        f1.record(stream)
    kqb200.synchronize()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = f0.elapsed_time(f1) / args.steps
    assert torch.isfinite(yh).all(), "non-finite block output"

    ms, e2e_ms = max_over_ranks([ms, e2e_ms], world, torch.device("cuda", local_rank))
    total_flops, parts = prefill_flops(T)
    tc_flops = rank_tensor_core_flops(block, T)
    proj_step_ms = proj_ms.value / max(1, args.steps)
    achieved = tc_flops / (proj_step_ms * 1e-3) / 1e12
    peak, peak_kind = tensor_peak()
    line = {
        "metric": METRIC,
        "value": T * 1000.0 / ms,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": {
            "workload": f"config4: 4-layer block (3 GDN + 1 QSA) prefill of {T} tokens, batch 1, "
                        f"projections Q4_K, index BF16, F32 activations/state/KV",
            "parallelism": f"tensor-parallel x{world}: GDN by value-head group, QSA by query-head group "
                           f"(indexer {'replicated' if exchange is None else 'scores/top-k split by 64-token chunk, one all-reduce of the selections'}), "
                           f"NCCL all-reduce (f32) after each out-projection",
            "slice_tokens": args.slice_tokens,
            "l2": "working set per step (GBs of activations, KV, projections) >> 126 MB L2",
            "step_algorithmic_flops": total_flops,
            "step_flops_breakdown": parts,
            "step_tflops": total_flops / (ms * 1e-3) / 1e12,
        },
        "roofline": {
            "kernel": "proj (xconv + proj_umma: tcgen05 projection GEMMs of this rank's shards)",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "traffic": None,
            "algorithmic_flops_per_step": tc_flops,
            "ms_per_step": proj_step_ms,
            "launches_timed": proj_n.value,
            "note": "F32 operands as bf16 hi/lo pairs: three MMAs per algorithmic product",
        },
        "e2e": {"value": T * 1000.0 / e2e_ms, "unit": "tok/s",
                "h2d_bytes_per_step": T * gd.hidden * 4, "d2h_bytes_per_step": T * gd.hidden * 4},
        "gpu_launches": int(launches),
        **({"kernel_breakdown": breakdown} if breakdown else {}),
        "clocks": clocks.summary(),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, impl, secs = cpu_prefill_sample(args.cpu_tokens)
        line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": 1,
                                "kind": "reference" if impl == "reference" else "port",
                                "sample": f"first {args.cpu_tokens} tokens of the block prefill from empty "
                                          f"states, 1 thread ({secs:.1f} s wall)"}
    if rank == 0:
        print(json.dumps(line), flush=True)
    block.close()
    prov.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--breakdown", action="store_true", help="time every kernel family (extra steps)")
    ap.add_argument("--ctx-max", type=int, default=CTX_RANGE[1],
                    help="upper end of the context distribution (profiling runs use a small one)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                    help="decode: config 3 (default); prefill: config 4, tensor-parallel")
    ap.add_argument("--tokens", type=int, default=PREFILL_TOKENS, help="prefill length (config 4)")
    ap.add_argument("--slice-tokens", type=int, default=PREFILL_SLICE,
                    help="prefill tokens per layer call (all-reduce granularity)")
    ap.add_argument("--cpu-tokens", type=int, default=16, help="prefill tokens of the CPU baseline sample")
    ap.add_argument("--replicated-indexer", action="store_true",
                    help="prefill at N > 1: every rank selects for every token (no selection exchange)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "prefill":
        return run_b200_prefill(args, rank, world, local_rank)
    return run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
