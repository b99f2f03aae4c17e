"""GDN+QSA layer-block benchmark on B200: decode B=64 as
the headline, with the prefill configurations (2 and 4) as sub-records.

Headline workload per GPU: a 4-layer hybrid block (3 GDN layers + 1 QSA
layer, hidden 2048, GDN 16x128 key / 32x128 value heads, QSA 16 query / 2 KV
heads of 256, block 4, budget 2048) decoding one token for each of 64
independent sequences whose contexts are drawn uniformly from [1k, 32k]
(seed 0 + rank).  In-projections Q4_K, out-projections Q6_K, index
projections BF16; F32 state and KV caches.  A step = one token through the
whole block for all 64 sequences.  Multi-GPU: one process per GPU, each rank
serves its own 64 sequences (sequence sharding, no data-path collective;
weak scaling).

Sub-records of the same JSON line (default run; `--no-prefill` skips the
prefill ones):
  e2e_per_sequence      the decode step through the reference-shaped entry
                        points, one sequence per call with host buffers
  decode_b1             configs 0 and 1: batch-1 decode latency (one GPU)
  prefill_8k.gdn_layer  config 2: one GDN layer, Q6_K projections, 8192
                        tokens from a zero state (chunked WY-form recurrence)
  prefill_8k.block      the 4-layer block of config 4 on 8192 tokens
  prefill_131k          config 4: the 4-layer block (all projections Q4_K,
                        index BF16) on 131072 tokens
  moe_decode            the routed-expert MoE layer (512 experts, top-10,
                        shared expert) on a batch of 64 decode tokens
  layer_decode          one target GDN decoder layer (gated residuals, GDN,
                        MoE) decoding one token of each of 64 sequences
Every prefill runs tensor-parallel over the run's ranks (GDN by value-head
group, QSA by query-head group or by token within a KV-head group, the
indexer's selections exchanged once per layer call) with one NCCL
all-reduce of the partial outputs after every layer's out-projection
(strong scaling); at one GPU it is the plain layer.

Inputs are synthetic and seeded (no dataset): weights and states are drawn
with the distributions BASELINE.json names.  Every timed step's working set
(GBs of state, KV, weights and activations) is larger than the 126 MB L2, so
no L2 flush is needed between steps.

Timing: W warm-up steps, then exactly K steps between barrier +
synchronize on both sides, CUDA events on the library stream, max over
ranks.  The per-kernel timing behind `roofline` is a separate pass of the
same steps with events around that kernel family's launches (events between
kernels break the programmatic-dependent-launch overlap, so they stay out of
the headline region).  `e2e` repeats the step through the public API with
the step's inputs copied from pinned host memory and its outputs read back
inside the timed region.

Arms:
  default          the B200 library through its C-ABI (kestrel-q_b200)
  --impl reference the reference's own CPU operators (oracle/_ref, compiled
                   from Kestrel-Q's C sources) on the host cores, same
                   metric, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import functools
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
PREFILL_TOKENS = 131072
PREFILL_SLICE = 16384
CPU_PREFILL_TOKENS = 16


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
    """Config 3: the block's weights (one model, replicated on every rank)."""
    from kqb200 import synth
    gd, qd = dims()
    gdn = [synth.gdn_layer(l, gd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
           for l in range(GDN_LAYERS)]
    qsa = synth.qsa_layer(7, qd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_BF16)
    return gdn, qsa


def prefill_weights():
    """Config 4: the block with every projection Q4_K (index projections BF16)."""
    from kqb200 import synth
    gd, qd = dims()
    gdn = [synth.gdn_layer(20 + l, gd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_Q4_K)
           for l in range(GDN_LAYERS)]
    qsa = synth.qsa_layer(27, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
    return gdn, [qsa]


def gdn_prefill_weights():
    """Config 2: one GDN layer with every projection Q6_K."""
    from kqb200 import synth
    gd, _ = dims()
    return [synth.gdn_layer(202, gd, synth.TYPE_Q6_K, synth.TYPE_Q6_K, synth.TYPE_Q6_K)], []


PREFILL_KINDS = {
    "gdn_layer": ("config2: one GDN layer prefill from a zero state, batch 1, Q6_K projections, F32 state",
                  gdn_prefill_weights),
    "block": ("config4: 4-layer block (3 GDN + 1 QSA) prefill, batch 1, projections Q4_K, index BF16, "
              "F32 activations/state/KV", prefill_weights),
}


def wy_flops_per_chunk_head(C: int = 64, d: int = 128) -> int:
    """FLOPs of the chunked WY form for one head and one chunk of C tokens
    (dk = dv = d): K K^T and Q K^T (2 C^2 d each), the two triangular solves
    for W and U (C^2 d each), the causal P delta (C^2 d), and W S, Q S,
    K^T delta against the d x d state (2 C d^2 each)."""
    return 7 * C * C * d + 6 * C * d * d


def prefill_flops(T: int, gdn_layers: int = GDN_LAYERS, qsa_layers: int = 1):
    """Algorithmic FLOPs of one T-token prefill (all ranks together), by part."""
    gd, qd = dims()
    H, C, Vd, Hv = gd.hidden, gd.conv_channels, gd.value_width, gd.value_heads
    gdn_proj = gdn_layers * (2 * T * H * (C + Vd + 2 * Hv) + 2 * T * Vd * H)
    chunks = (T + 63) // 64
    wy = gdn_layers * Hv * chunks * wy_flops_per_chunk_head(64, gd.key_dim)
    parts = {"gdn_proj": gdn_proj, "gdn_wy": wy}
    if qsa_layers:
        qw, kvw = qd.q_width, qd.kv_width
        iw = qd.index_heads * qd.index_dim + qd.index_dim
        pos = np.arange(T, dtype=np.int64)
        nb = (pos + 1) // qd.block
        ntok = np.minimum(nb, qd.budget // qd.block) * qd.block + (pos + 1) % qd.block
        parts["qsa_proj"] = qsa_layers * (2 * T * H * (2 * qw + 2 * kvw) + 2 * T * qw * H + 2 * T * H * iw)
        parts["qsa_indexer"] = qsa_layers * int(2 * qd.index_heads * qd.index_dim * nb.sum())
        parts["qsa_attention"] = qsa_layers * int(4 * qd.query_heads * qd.head_dim * ntok.sum())
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
    """HBM bytes one decode step must move at minimum (per GPU): every
    weight once, GDN state and conv state read + written once, QSA K/V read
    only for the selected tokens, cached block keys once, new K/V/raw rows
    written, and the block's activations."""
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
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)   # let the sampler start before the timed work
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

def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_block_sample(n_seqs: int, threads: int, rank: int = 0):
    """The reference's own F32 operators (oracle/_ref when built, else the
    restatement) decoding one token of the 4-layer block for `n_seqs`
    sequences of the workload, `threads` sequences in parallel.
    Returns (tokens_per_second, kind, seconds)."""
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


def cpu_prefill_sample(kind: str, tokens: int):
    """The reference's own F32 operators (oracle/_ref when built, else the
    restatement) prefilling the first `tokens` tokens of a prefill workload
    (PREFILL_KINDS) from empty states, one thread (the reference's prefill
    of one sequence is sequential).  Returns (tokens_per_second, kind, seconds)."""
    from oracle import oracle as O
    impl = "reference" if O.ref_available() else "port"
    gd, qd = dims()
    gdn, qsa = PREFILL_KINDS[kind][1]()
    gw = [O.gdn_weights_f32(L) for L in gdn]
    qw = [O.qsa_weights_f32(L) for L in qsa]
    x = np.random.default_rng(99).normal(size=(tokens, gd.hidden)).astype(np.float32)
    conv = np.zeros(gd.conv_channels * gd.conv_kernel, np.float32)
    rec = np.zeros(gd.value_heads * gd.key_dim * gd.value_dim, np.float32)
    z = np.zeros((tokens, qd.kv_width), np.float32)
    zr = np.zeros((tokens, qd.index_dim), np.float32)
    t0 = time.perf_counter()
    h = x
    for w in gw:
        st, h, _, _ = O.gdn_run(gd, w, h, conv, rec, impl=impl)
        assert st == 0
    for w in qw:
        st, h, *_ = O.qsa_run(qd, w, h, z, z, zr, 0, tokens, impl=impl)
        assert st == 0
    elapsed = time.perf_counter() - t0
    return tokens / elapsed, impl, elapsed


def cpu_prefill_record(kind: str, tokens: int = CPU_PREFILL_TOKENS):
    v, impl, secs = cpu_prefill_sample(kind, tokens)
    return {"value": v, "unit": "tok/s", "cores": 1, "kind": "reference" if impl == "reference" else "port",
            "sample": f"first {tokens} tokens of the {kind} prefill from empty states, 1 thread "
                      f"({secs:.1f} s wall)"}


# ---------------------------------------------------------------- MoE

MOE_BATCH = 64
MOE_POOL = 16   # distinct input batches cycled through the timed steps
MOE_CPU_TOKENS = 8


@functools.lru_cache(maxsize=1)
def moe_weights():
    """The target MoE layer (512 experts, top-10, hidden 2560, routed and
    shared intermediate 640): gate/up Q4_K, down and shared Q8_0, router and
    shared gate F32 (src/kq_moe.c:27-54 type masks)."""
    from kqb200 import synth
    return synth.moe_layer(11, synth.MoeDims())


def moe_routes(w, x: np.ndarray) -> np.ndarray:
    """Selected experts [T][K] of tokens x from the F32 router (host float64
    product: byte accounting only, near ties do not matter there)."""
    d = w.dims
    R = w.router.data.view(np.float32).reshape(d.experts, d.hidden).astype(np.float64)
    logits = x.astype(np.float64) @ R.T
    return np.argpartition(-logits, d.top_k - 1, axis=1)[:, :d.top_k]


def moe_step_bytes(w, x: np.ndarray):
    """Algorithmic HBM bytes of one MoE call over the tokens x: each selected
    expert's gate/up/down rows once, the shared expert, the router, the
    activations in and out.  Returns (total, experts part, distinct experts)."""
    d = w.dims
    per_expert = (w.gate.nbytes + w.up.nbytes + w.down.nbytes) // d.experts
    distinct = len(np.unique(moe_routes(w, x)))
    shared = w.shared_gate.nbytes + w.shared_up.nbytes + w.shared_down.nbytes + d.hidden * 4
    io = 2 * x.shape[0] * d.hidden * 4
    return distinct * per_expert + shared + w.router.nbytes + io, distinct * per_expert, distinct


def cpu_moe_sample(w, tokens: int, threads: int):
    """The reference's own MoE operators on the host cores: per token
    kq_moe_route_f32, then kq_moe_execute_routed_expert_f32 for each selected
    expert and for the shared expert (F32 weights; the selected experts are
    dequantised outside the timed spans).  Returns (tokens/s, kind, threads)."""
    from oracle import oracle as O
    if not O.ref_available():
        return None, "unavailable", 0
    d = w.dims
    H, I, S = d.hidden, d.routed, d.shared
    router = np.ascontiguousarray(w.router.data.view(np.float32).reshape(d.experts, H))
    xs = np.random.default_rng(77).normal(size=(tokens, H)).astype(np.float32)

    def rows(t, e, n):
        rb = t.row_bytes
        return O.dequantize(t.type_id, t.data[e * n * rb:(e + 1) * n * rb]).reshape(n, -1)

    shared = (O.dequantize(w.shared_gate.type_id, w.shared_gate.data).reshape(S, H),
              O.dequantize(w.shared_up.type_id, w.shared_up.data).reshape(S, H),
              O.dequantize(w.shared_down.type_id, w.shared_down.data).reshape(H, S))

    def one(i):
        ref = O.RefMoe(d)
        try:
            x = xs[i]
            spent = 0.0
            t0 = time.perf_counter()
            ids, wt = ref.route(router, x)
            spent += time.perf_counter() - t0
            y = np.zeros(H, np.float32)
            for p in sorted(range(d.top_k), key=lambda q: ids[q]):
                e = int(ids[p])
                g, u, dn = rows(w.gate, e, I), rows(w.up, e, I), rows(w.down, e, H)
                t0 = time.perf_counter()
                out = ref.expert(g, u, dn, x)
                spent += time.perf_counter() - t0
                y = y + out * wt[p]
            t0 = time.perf_counter()
            ref.expert(*shared, x)
            spent += time.perf_counter() - t0
            return spent
        finally:
            ref.close()

    spans = [0.0] * threads
    with cf.ThreadPoolExecutor(max_workers=threads) as pool:
        for i, t in enumerate(pool.map(one, range(tokens))):
            spans[i % threads] += t
    return tokens / max(spans), "reference", threads


def cpu_moe_record(w=None, tokens: int = MOE_CPU_TOKENS):
    w = w if w is not None else moe_weights()
    threads = min(cpu_threads(), tokens)
    v, kind, threads = cpu_moe_sample(w, tokens, threads)
    if v is None:
        return {"unavailable": "reference library not built"}
    return {"value": v, "unit": "tok/s", "cores": threads, "kind": kind,
            "sample": f"{tokens} tokens, one per thread: kq_moe_route_f32 + kq_moe_execute_routed_expert_f32 for "
                      f"the 10 selected experts and the shared expert (F32 weights, dequantised outside the timing)"}


def moe_record(args, cx: Ctx, cpu: bool):
    """The routed-expert MoE layer decoding a batch of 64 tokens (one per
    sequence), target geometry.  A step = one kq_b200_moe_execute_async call
    over 64 tokens; the inputs cycle through 16 seeded batches so the set of
    selected experts changes every step.  Bound: HBM (each selected expert's
    weights once per step)."""
    torch, kqb200 = cx.torch, cx.kq
    w = moe_weights()
    d = w.dims
    B, H = MOE_BATCH, d.hidden
    prov = kqb200.Provider(cx.local_rank)
    layer = kqb200.MoeLayer(d, w, prov, layer=0)
    try:
        rng = np.random.default_rng(500 + cx.rank)
        xs = [rng.normal(size=(B, H)).astype(np.float32) for _ in range(MOE_POOL)]
        xd = [torch.from_numpy(x).cuda() for x in xs]
        y = torch.empty(B, H, device="cuda")
        torch.cuda.synchronize()
        it = [0]

        def step():
            kqb200.moe_execute_async(layer, xd[it[0] % MOE_POOL].data_ptr(), B, y.data_ptr())
            it[0] += 1

        with torch.cuda.stream(cx.stream):
            for _ in range(args.warmup):
                step()
        cx.sync()
        steps = args.moe_steps
        it[0] = 0
        launches0 = cx.lib.kq_b200_kernel_launch_count()
        with ClockSampler(cx.local_rank) as clocks:
            ms = cx.timed(steps, step)
        launches = cx.lib.kq_b200_kernel_launch_count() - launches0
        assert torch.isfinite(y).all(), "non-finite MoE output"
        it[0] = 0
        gu_ms, gu_n = cx.family_ms("moe_gate_up", steps, step)
        it[0] = 0
        dn_ms, dn_n = cx.family_ms("moe_down", steps, step)
        # end to end: the reference-shaped synchronous entry point with host
        # activations (kq_moe_execute_quantized, 64 tokens per call)
        it[0] = 0

        def e2e_step():
            st, out, *_ = layer.execute_quantized(xs[it[0] % MOE_POOL])
            it[0] += 1
            assert st == 0

        e2e_step()
        it[0] = 0
        e2e_ms = cx.timed(max(3, steps // 4), e2e_step)
        ms, e2e_ms, gu_ms, dn_ms = max_over_ranks([ms, e2e_ms, gu_ms, dn_ms], cx.world, cx.device)
        acc = [moe_step_bytes(w, xs[i % MOE_POOL]) for i in range(MOE_POOL)]
        step_bytes = float(np.mean([a[0] for a in acc]))
        distinct = float(np.mean([a[2] for a in acc]))
        per_expert_gu = (w.gate.nbytes + w.up.nbytes) // d.experts
        gu_bytes = distinct * per_expert_gu
        hbm, peak_kind = peaks()
        gu_avg = gu_ms / max(1.0, gu_n)
        achieved = gu_bytes / (gu_avg * 1e-3) / 1e9
        rec = {
            "workload": "MoE layer decode, 64 tokens/GPU (one per sequence), 512 experts top-10 + shared expert, "
                        "hidden 2560, intermediate 640, gate/up Q4_K, down/shared Q8_0, router F32",
            "value": job_tokens_per_s(cx.world, B, ms), "unit": "tok/s", "ms_per_step": ms, "steps": steps,
            "step_algorithmic_bytes": step_bytes, "distinct_experts_per_step": distinct,
            "step_hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / hbm,
            "roofline": {
                "kernel": "moe_gate_up (grouped Q4_K gate+up GEMV of the selected experts, SwiGLU epilogue)",
                "bound": "hbm", "achieved": achieved, "peak": hbm, "peak_kind": peak_kind, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": None,
                "algorithmic_bytes_per_launch": gu_bytes, "avg_launch_ms": gu_avg,
                "down_ms_per_step": dn_ms, "down_frac": distinct * (w.down.nbytes // d.experts) /
                (dn_ms / max(1.0, dn_n) * 1e-3) / 1e9 / hbm,
                "timing": "CUDA events around each launch of the kernel, in a pass of its own"},
            "e2e": {"value": job_tokens_per_s(cx.world, B, e2e_ms), "unit": "tok/s", "ms_per_step": e2e_ms,
                    "api": "kq_moe_execute_quantized, 64 tokens per call, host activations",
                    "h2d_bytes_per_step": B * H * 4, "d2h_bytes_per_step": B * H * 4},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if cpu and cx.rank == 0:
            rec["cpu_baseline"] = cpu_moe_record(w)
        return rec
    finally:
        layer.close()
        prov.close()


# ---------------------------------------------------------------- layer

LAYER_BRANCHES, LAYER_RANK = 4, 320
LAYER_CPU_TOKENS = 4


def decoder_layer_weights():
    """One target GDN decoder layer: GDN at the target model's geometry
    (hidden 2560, 16 x 128 key / 48 x 128 value heads; projections typed as
    in config 3: in Q4_K, out Q6_K, alpha/beta Q4_K), the target MoE
    (moe_weights) and gated residuals over 4 branches of rank 320 (BF16)."""
    from kqb200 import synth
    gd = synth.GdnDims(hidden=2560, key_heads=16, value_heads=48, key_dim=128, value_dim=128)
    gw = synth.gdn_layer(31, gd, synth.TYPE_Q4_K, synth.TYPE_Q6_K, synth.TYPE_Q4_K)
    gr = {"attn": synth.gr_weights(32, gd.hidden, LAYER_BRANCHES, LAYER_RANK),
          "moe": synth.gr_weights(33, gd.hidden, LAYER_BRANCHES, LAYER_RANK)}
    return gd, gw, gr


def cpu_layer_record(tokens: int = LAYER_CPU_TOKENS):
    """The reference's own operators for one decode token of the layer, per
    token: kq_layer_gr_read_f32, the GDN decode (kq_gdn_prefill_f32 on one
    token), kq_layer_gr_write_f32, the MoE gated residual, kq_moe_route_f32
    with kq_moe_execute_routed_expert_f32 for the selected and the shared
    expert, and the final write (F32 weights, dequantised outside the timed
    spans).  One token per thread."""
    from oracle import oracle as O
    if not O.ref_available():
        return {"unavailable": "reference library not built"}
    gd, gw, gr = decoder_layer_weights()
    mw = moe_weights()
    md = mw.dims
    H, I, S = md.hidden, md.routed, md.shared
    gwf = O.gdn_weights_f32(gw)

    def deq(t):
        return O.dequantize(t.type_id, t.data).reshape(-1)

    grf = {k: {"norm": g.norm, "down": deq(g.down), "up": deq(g.up), "inject": deq(g.inject)} for k, g in gr.items()}
    router = np.ascontiguousarray(mw.router.data.view(np.float32).reshape(md.experts, H))
    shared = (deq(mw.shared_gate).reshape(S, H), deq(mw.shared_up).reshape(S, H), deq(mw.shared_down).reshape(H, S))

    def rows(t, e, n):
        rb = t.row_bytes
        return O.dequantize(t.type_id, t.data[e * n * rb:(e + 1) * n * rb]).reshape(n, -1)

    def one(i):
        rng = np.random.default_rng(900 + i)
        x = rng.normal(0, 1, LAYER_BRANCHES * H).astype(np.float32)
        conv = rng.normal(0, 1, gd.conv_channels * 4).astype(np.float32)
        rec = (rng.normal(0, 0.02, gd.value_heads * gd.key_dim * gd.value_dim)).astype(np.float32)
        gr_ref, moe_ref = O.RefLayerGr(H, LAYER_BRANCHES, LAYER_RANK), O.RefMoe(md)
        try:
            spent = 0.0
            t0 = time.perf_counter()
            mixed, awg = gr_ref.read(grf["attn"], x)
            st, block, _, _ = O.gdn_run(gd, gwf, mixed, conv, rec, impl="reference")
            assert st == 0
            after = gr_ref.write(x, block, awg)
            moe_in, mwg = gr_ref.read(grf["moe"], after)
            ids, wt = moe_ref.route(router, moe_in)
            spent += time.perf_counter() - t0
            y = np.zeros(H, np.float32)
            for p in sorted(range(md.top_k), key=lambda q: ids[q]):
                e = int(ids[p])
                g, u, dn = rows(mw.gate, e, I), rows(mw.up, e, I), rows(mw.down, e, H)
                t0 = time.perf_counter()
                y = y + moe_ref.expert(g, u, dn, moe_in) * wt[p]
                spent += time.perf_counter() - t0
            t0 = time.perf_counter()
            moe_ref.expert(*shared, moe_in)
            gr_ref.write(after, y, mwg)
            spent += time.perf_counter() - t0
            return spent
        finally:
            gr_ref.close()
            moe_ref.close()

    threads = min(cpu_threads(), tokens)
    spans = [0.0] * threads
    with cf.ThreadPoolExecutor(max_workers=threads) as pool:
        for i, t in enumerate(pool.map(one, range(tokens))):
            spans[i % threads] += t
    return {"value": tokens / max(spans), "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{tokens} decode tokens of the target GDN layer, one per thread: the reference's gated "
                      f"residual, GDN and MoE operators (F32 weights, dequantised outside the timed spans)"}


def layer_record(args, cx: Ctx, cpu: bool):
    """One target GDN decoder layer (gated residual, GDN, gated residual,
    MoE) decoding one token for each of 64 sequences per step through
    kq_b200_layer_decode_batch; the inputs cycle through 16 seeded batches.
    Bound: HBM (the step's weights, the selected experts' weights, the GDN
    states)."""
    torch, kqb200 = cx.torch, cx.kq
    gd, gw, gr = decoder_layer_weights()
    mw = moe_weights()
    B, W = MOE_BATCH, LAYER_BRANCHES * gd.hidden
    prov = kqb200.Provider(cx.local_rank)
    mixer = kqb200.GdnLayer(gd, gw, prov, layer=0)
    moe = kqb200.MoeLayer(mw.dims, mw, prov, layer=0)
    layer = kqb200.DecoderLayer(1, gd.hidden, LAYER_BRANCHES, LAYER_RANK, 1e-6, mixer, moe, gr, prov)
    states = [layer.state() for _ in range(B)]
    try:
        # the states start from zero: a decode step's work does not depend on them
        gen = torch.Generator(device="cuda")
        gen.manual_seed(4321 + cx.rank)
        xs = [torch.randn(B, W, device="cuda", generator=gen) for _ in range(MOE_POOL)]
        y = torch.empty(B, W, device="cuda")
        torch.cuda.synchronize()
        it = [0]

        def step():
            kqb200.layer_decode_batch(layer, states, xs[it[0] % MOE_POOL].data_ptr(), y.data_ptr())
            it[0] += 1

        with torch.cuda.stream(cx.stream):
            for _ in range(args.warmup):
                step()
        cx.sync()
        steps = args.moe_steps
        launches0 = cx.lib.kq_b200_kernel_launch_count()
        with ClockSampler(cx.local_rank) as clocks:
            ms = cx.timed(steps, step)
        launches = cx.lib.kq_b200_kernel_launch_count() - launches0
        assert torch.isfinite(y).all(), "non-finite layer output"
        xh = torch.randn(B, W, generator=torch.Generator().manual_seed(6)).pin_memory()
        yh = torch.empty(B, W).pin_memory()

        def e2e_step():
            xs[0].copy_(xh, non_blocking=True)
            kqb200.layer_decode_batch(layer, states, xs[0].data_ptr(), y.data_ptr())
            yh.copy_(y, non_blocking=True)

        e2e_ms = cx.timed(max(3, steps // 4), e2e_step)
        ms, e2e_ms = max_over_ranks([ms, e2e_ms], cx.world, cx.device)
        hbm, peak_kind = peaks()
        xhost = [x.cpu().numpy() for x in xs[:4]]
        moe_bytes = float(np.mean([moe_step_bytes(mw, x[:, :gd.hidden])[0] for x in xhost]))
        gdn_w = sum(t.nbytes for t in (gw.qkv, gw.gate, gw.beta, gw.alpha, gw.output))
        gdn_state = B * 2 * 4 * (gd.value_heads * gd.key_dim * gd.value_dim + gd.conv_channels * 4)
        gr_bytes = 2 * sum(t.nbytes for t in (gr["attn"].down, gr["attn"].up, gr["attn"].inject))
        step_bytes = moe_bytes + gdn_w + gdn_state + gr_bytes + 2 * B * W * 4
        rec = {
            "workload": "target GDN decoder layer decode, 64 sequences/GPU: gated residual (4 branches, rank 320, "
                        "BF16), GDN (hidden 2560, 16x128 key / 48x128 value heads, Q4_K in / Q6_K out), gated "
                        "residual, MoE (512 experts top-10 + shared, Q4_K / Q8_0)",
            "value": job_tokens_per_s(cx.world, B, ms), "unit": "tok/s", "ms_per_step": ms, "steps": steps,
            "step_algorithmic_bytes": step_bytes,
            "step_hbm_frac": step_bytes / (ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind,
            "e2e": {"value": job_tokens_per_s(cx.world, B, e2e_ms), "unit": "tok/s", "ms_per_step": e2e_ms,
                    "h2d_bytes_per_step": B * W * 4, "d2h_bytes_per_step": B * W * 4},
            "gpu_launches": int(launches),
            "clocks": clocks.summary(),
        }
        if cpu and cx.rank == 0:
            rec["cpu_baseline"] = cpu_layer_record()
        return rec
    finally:
        for s in states:
            s.close()
        layer.close()
        moe.close()
        mixer.close()
        prov.close()


def run_reference(args, rank, world):
    """The reference arm: rank 0 alone times the reference's CPU operators on
    every host core it may use; other ranks exit at once."""
    if rank != 0:
        return 0
    from oracle import oracle as O
    if not O.PORT_LIB.exists():
        O.build()
    threads = cpu_threads()
    if args.workload == "prefill":
        return run_reference_prefill(args, world)
    n = threads
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
                         "sample": f"{n} sequences x 1 token of the 4-layer block, {threads} threads "
                                   f"(one sequence per thread)"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_prefill:
        line["prefill_8k"] = {k: {"impl": "reference", "cpu_baseline": cpu_prefill_record(k)}
                              for k in ("gdn_layer", "block")}
        line["prefill_131k"] = {"impl": "reference", "cpu_baseline": cpu_prefill_record("block")}
    if not args.no_moe:
        line["moe_decode"] = {"impl": "reference", "cpu_baseline": cpu_moe_record()}
        line["layer_decode"] = {"impl": "reference", "cpu_baseline": cpu_layer_record()}
    print(json.dumps(line), flush=True)
    return 0


def run_reference_prefill(args, world):
    vals, kind = [], "reference"
    cpu_prefill_sample("block", 2)
    t_all = time.perf_counter()
    for _ in range(args.steps):
        v, impl, _ = cpu_prefill_sample("block", args.cpu_tokens)
        kind = "reference" if impl == "reference" else "port"
        vals.append(v)
    elapsed = time.perf_counter() - t_all
    value = statistics.median(vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * elapsed / max(1, args.steps),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": PREFILL_KINDS["block"][0],
                   "sample": f"first {args.cpu_tokens} tokens of the prefill per step"},
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": 1, "kind": kind,
                         "sample": f"first {args.cpu_tokens} tokens of the 4-layer block prefill from empty "
                                   f"states, 1 thread"},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- B200 arm

class Ctx:
    """Per-rank plumbing: device, library stream, process group."""

    def __init__(self, rank, world, local_rank):
        import ctypes as C

        import torch
        import torch.distributed as dist

        import kqb200
        self.rank, self.world, self.local_rank = rank, world, local_rank
        self.torch, self.dist, self.kq = torch, dist, kqb200
        torch.cuda.set_device(local_rank)
        d = kqb200.abi.Diagnostic()
        kqb200.abi.check(kqb200.lib().kq_b200_set_device(local_rank, C.byref(d)), d)
        if world > 1:
            import datetime
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        self.lib = kqb200.lib()
        self.stream = torch.cuda.ExternalStream(self.lib.kq_b200_get_stream())
        self.device = torch.device("cuda", local_rank)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def sync(self):
        self.kq.synchronize()
        self.torch.cuda.synchronize()

    def timed(self, steps, fn):
        """Device time of `steps` calls of fn() on the library stream (ms per
        step), bracketed by barrier + synchronize on both sides."""
        torch = self.torch
        self.barrier()
        self.sync()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(self.stream):
            e0.record(self.stream)
            for _ in range(steps):
                fn()
            e1.record(self.stream)
        self.sync()
        self.barrier()
        return e0.elapsed_time(e1) / steps

    def family_ms(self, family, steps, fn):
        """Per-step device time of one kernel family (events around its
        launches), over `steps` extra calls of fn(); returns (ms, launches)."""
        import ctypes as C
        self.lib.kq_b200_profile_kernel(family.encode())
        with self.torch.cuda.stream(self.stream):
            for _ in range(steps):
                fn()
        self.sync()
        n_, t_ = C.c_uint64(), C.c_double()
        self.lib.kq_b200_profile_read(C.byref(n_), C.byref(t_))
        self.lib.kq_b200_profile_kernel(None)
        return t_.value / steps, n_.value / steps

    def close(self):
        if self.world > 1:
            self.dist.barrier()
            self.dist.destroy_process_group()


class RefShaped:
    """The reference-shaped synchronous entry points (kq_gdn_execute_quantized,
    kq_qsa_execute_quantized: src/kq_gdn_internal.h:81-96,
    src/kq_qsa_internal.h:94-102) called the way the reference's layer code
    calls them (src/kq_layer.c:746-765): one sequence per call, host buffers,
    caller-owned scratch, which this keeps allocated across calls."""

    def __init__(self, cx: Ctx):
        self.cx = cx
        self.lib = cx.lib
        self.abi = cx.kq.abi
        self.buffers = {}

    def _buf(self, key, floats):
        b = self.buffers.get(key)
        if b is None or b.size < floats:
            b = np.empty(max(1, floats), np.float32)
            self.buffers[key] = b
        return b

    def gdn(self, layer, state, x: np.ndarray, y: np.ndarray):
        import ctypes as C
        dm = layer.dims
        scratch = self._buf(("gs", id(layer)), self.lib.kq_gdn_config_scratch_bytes(layer.handle) // 4 + 1)
        conv = dm.conv_channels * dm.conv_kernel
        wscratch = self._buf(("gw", id(layer)), 2 * dm.value_heads + 2 * conv + dm.value_dim + 65536 // 4 + 64)
        d = self.abi.Diagnostic()
        self.abi.check(self.lib.kq_gdn_execute_quantized(
            layer.handle, layer.provider.handle, x.ctypes.data, x.shape[0], None, y.ctypes.data, y.size,
            state.handle, scratch.ctypes.data, scratch.nbytes, wscratch.ctypes.data, wscratch.nbytes, None, None,
            C.byref(d)), d)

    def qsa(self, layer, state, x: np.ndarray, y: np.ndarray):
        import ctypes as C
        dm = layer.dims
        need = C.c_uint64()
        d = self.abi.Diagnostic()
        self.abi.check(self.lib.kq_qsa_required_scratch_bytes(layer.handle, state.handle, x.shape[0],
                                                               C.byref(need), C.byref(d)), d)
        scratch = self._buf(("qs", id(layer)), need.value // 4 + 1)
        wscratch = self._buf(("qw", id(layer)), (65536 + 8 * (dm.head_dim + dm.index_dim) * 4) // 4 + 64)
        self.abi.check(self.lib.kq_qsa_execute_quantized(
            layer.handle, layer.provider.handle, x.ctypes.data, x.shape[0], y.ctypes.data, y.size, state.handle,
            scratch.ctypes.data, scratch.nbytes, wscratch.ctypes.data, wscratch.nbytes,
            self.abi.SELECTION_OBSERVER(), None, None, C.byref(d)), d)


def decode_record(args, cx: Ctx):
    """Config 3 decode: the headline record."""
    import ctypes as C
    torch, kqb200 = cx.torch, cx.kq
    rank, world = cx.rank, cx.world
    gd, qd = dims()
    gdn_w, qsa_w = layer_weights()
    ctx = contexts(rank, ctx_max=args.ctx_max)
    B = BATCH
    steps_total = args.warmup + 3 * args.steps + 80
    prov = kqb200.Provider(cx.local_rank)
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
            kqb200.abi.check(cx.lib.kq_gdn_state_import_f32(s.handle, conv.data_ptr(), conv.numel(),
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
        kqb200.abi.check(cx.lib.kq_qsa_state_import_f32(s.handle, k.data_ptr(), k.numel(), v.data_ptr(),
                                                        v.numel(), r.data_ptr(), r.numel(), L, C.byref(dd)), dd)
        del k, v, r
        qsa_states.append(s)
    torch.cuda.synchronize()
    bufs = [torch.randn(B, gd.hidden, device="cuda", generator=gen) for _ in range(GDN_LAYERS + 2)]
    torch.cuda.synchronize()

    def step(x_ptr, y_ptr):
        h_in = x_ptr
        for l in range(GDN_LAYERS):
            kqb200.gdn_decode_batch(gdn_layers[l], gdn_states[l], h_in, bufs[l + 1].data_ptr())
            h_in = bufs[l + 1].data_ptr()
        kqb200.qsa_decode_batch(qsa_layer, qsa_states, h_in, y_ptr)

    x0, y0 = bufs[0].data_ptr(), bufs[GDN_LAYERS + 1].data_ptr()
    with torch.cuda.stream(cx.stream):
        for _ in range(args.warmup):
            step(x0, y0)
    cx.sync()

    # ---- device-resident timed region (no per-launch events)
    launches0 = cx.lib.kq_b200_kernel_launch_count()
    with ClockSampler(cx.local_rank) as clocks:
        ms = cx.timed(args.steps, lambda: step(x0, y0))
    launches = cx.lib.kq_b200_kernel_launch_count() - launches0

    # ---- the roofline kernel, timed in a pass of its own
    rec_ms, rec_n = cx.family_ms("gdn_recurrence", args.steps, lambda: step(x0, y0))
    breakdown = {}
    if args.breakdown:
        for fam in ("proj", "proj_exact", "gdn_recurrence", "qsa_prepare", "qsa_score", "qsa_select",
                    "qsa_attend", "qsa_combine"):
            t, n = cx.family_ms(fam, 5, lambda: step(x0, y0))
            breakdown[fam] = {"ms_per_step": t, "launches_per_step": n}

    # ---- end-to-end: pinned host input -> block -> host result, every step
    xh = torch.randn(B, gd.hidden, generator=torch.Generator().manual_seed(5)).pin_memory()
    yh = torch.empty(B, gd.hidden).pin_memory()

    def e2e_step():
        bufs[0].copy_(xh, non_blocking=True)
        step(x0, y0)
        yh.copy_(bufs[GDN_LAYERS + 1], non_blocking=True)

    e2e_ms = cx.timed(args.steps, e2e_step)
    assert torch.isfinite(yh).all(), "non-finite block output"

    # ---- end-to-end through the reference-shaped entry points, one
    # sequence per call (the drop-in path a reference host takes)
    rs = RefShaped(cx)
    xs = np.random.default_rng(7).normal(size=(B, 1, gd.hidden)).astype(np.float32)
    hs = [np.empty((1, gd.hidden), np.float32) for _ in range(GDN_LAYERS + 1)]

    def per_sequence_step():
        for b in range(B):
            h = xs[b]
            for l in range(GDN_LAYERS):
                rs.gdn(gdn_layers[l], gdn_states[l][b], h, hs[l])
                h = hs[l]
            rs.qsa(qsa_layer, qsa_states[b], h, hs[GDN_LAYERS])

    per_seq_step_ms = 0.0
    if args.per_sequence_steps > 0:
        per_sequence_step()
        per_seq_step_ms = cx.timed(args.per_sequence_steps, per_sequence_step)
        assert np.isfinite(hs[GDN_LAYERS]).all(), "non-finite per-sequence output"

    ms, e2e_ms, rec_ms, per_seq_step_ms = max_over_ranks([ms, e2e_ms, rec_ms, per_seq_step_ms], world, cx.device)
    step_bytes, parts = algorithmic_bytes(gdn_w, qsa_w, ctx, B)
    hbm, peak_kind = peaks()
    rec_avg_ms = rec_ms / max(1.0, rec_n)
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
            "kernel": "gdn_decode_persist (conv/gates + recurrence + gated norm, persistent with next-item prefetch; B=64, one GDN layer)",
            "bound": "hbm",
            "achieved": achieved,
            "peak": hbm,
            "peak_kind": peak_kind,
            "unit": "GB/s",
            "frac": achieved / hbm,
            "traffic": traffic,
            "algorithmic_bytes_per_launch": rec_bytes,
            "avg_launch_ms": rec_avg_ms,
            "launches_timed": int(rec_n * args.steps),
            "timing": "CUDA events around each launch of the kernel, in a pass of its own after the timed region",
        },
        "e2e": {"value": job_tokens_per_s(world, B, e2e_ms), "unit": "tok/s",
                "h2d_bytes_per_step": B * gd.hidden * 4, "d2h_bytes_per_step": B * gd.hidden * 4},
        **({"e2e_per_sequence": {
            "value": job_tokens_per_s(world, B, per_seq_step_ms), "unit": "tok/s",
            "ms_per_step": per_seq_step_ms, "steps": args.per_sequence_steps,
            "calls_per_step": B * (GDN_LAYERS + 1),
            "api": "kq_gdn_execute_quantized / kq_qsa_execute_quantized, one sequence per call, host "
                   "activations, synchronous (the reference layer's calling pattern)",
            "h2d_bytes_per_step": B * (GDN_LAYERS + 1) * gd.hidden * 4,
            "d2h_bytes_per_step": B * (GDN_LAYERS + 1) * gd.hidden * 4}} if args.per_sequence_steps > 0 else {}),
        "gpu_launches": int(launches),
        **({"kernel_breakdown": breakdown} if breakdown else {}),
        "clocks": clocks.summary(),
    }
    for row in gdn_states:
        for s in row:
            s.close()
    for s in qsa_states:
        s.close()
    for L in gdn_layers:
        L.close()
    qsa_layer.close()
    prov.close()
    return line


def decode_b1_record(args, cx: Ctx, cpu: bool):
    """BASELINE configs 0 and 1: one decode token at batch 1, as latency.
    `device_ms`: the batched device entry point with one sequence (inputs in
    HBM); `api_ms`: the reference-shaped synchronous entry point with host
    buffers; `cpu_ms`: the reference's own operator on one host core."""
    import ctypes as C
    torch, kqb200 = cx.torch, cx.kq
    from kqb200 import synth
    gd, qd = dims()
    hbm, peak_kind = peaks()
    steps = args.b1_steps
    out = {}
    prov = kqb200.Provider(cx.local_rank)
    rs = RefShaped(cx)
    try:
        # config 0: GDN, Q8_0 qkv / gate / out, F32 alpha / beta
        gw = synth.gdn_layer(0, gd, synth.TYPE_Q8_0, synth.TYPE_Q8_0, synth.TYPE_F32)
        layer = kqb200.GdnLayer(gd, gw, prov, layer=0)
        st = kqb200.GdnState(layer)
        conv0, rec0 = synth.gdn_state(1, gd)
        st.load(conv0, rec0)
        x = torch.from_numpy(synth.hidden(2, 1, gd.hidden)).cuda()
        y = torch.empty_like(x)
        torch.cuda.synchronize()
        run = lambda: kqb200.gdn_decode_batch(layer, [st], x.data_ptr(), y.data_ptr())
        for _ in range(args.warmup):
            run()
        dev_ms = cx.timed(steps, run)
        xh, yh = synth.hidden(3, 1, gd.hidden), np.empty((1, gd.hidden), np.float32)
        rs.gdn(layer, st, xh, yh)
        api_ms = cx.timed(steps, lambda: rs.gdn(layer, st, xh, yh))
        w_bytes = sum(t.nbytes for t in (gw.qkv, gw.gate, gw.beta, gw.alpha, gw.output))
        tok_bytes = w_bytes + 2 * 4 * (gd.value_heads * gd.key_dim * gd.value_dim + gd.conv_channels * 4)
        rec = {"workload": "config0: GDN layer decode, batch 1, Q8_0 qkv/gate/out, F32 alpha/beta, F32 state",
               "device_ms": dev_ms, "device_tok_s": 1000.0 / dev_ms, "api_ms": api_ms,
               "api_tok_s": 1000.0 / api_ms, "steps": steps,
               "algorithmic_bytes_per_token": tok_bytes,
               "hbm_frac": tok_bytes / (dev_ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind}
        if cpu:
            from oracle import oracle as O
            impl = "reference" if O.ref_available() else "port"
            wf = O.gdn_weights_f32(gw)
            xs = synth.hidden(4, 3, gd.hidden)
            t0 = time.perf_counter()
            for i in range(3):
                assert O.gdn_run(gd, wf, xs[i:i + 1], conv0, rec0, impl=impl)[0] == 0
            rec["cpu_ms"] = (time.perf_counter() - t0) * 1000.0 / 3
            rec["cpu_kind"] = impl
        out["config0_gdn"] = rec
        st.close()
        layer.close()

        # config 1: QSA, context 4096 (4095 prior positions), Q4_K q/k/v/o, BF16 index
        qw = synth.qsa_layer(2, qd, synth.TYPE_Q4_K, synth.TYPE_Q4_K, synth.TYPE_BF16)
        qlayer = kqb200.QsaLayer(qd, qw, prov, layer=3)
        L = 4095
        qs = kqb200.QsaState(qlayer, L + 2 * steps + args.warmup + 8)
        k0, v0, r0 = synth.qsa_cache(5, qd, L)
        qs.load(k0, v0, r0)
        xq = torch.from_numpy(synth.hidden(6, 1, qd.hidden)).cuda()
        yq = torch.empty_like(xq)
        torch.cuda.synchronize()
        run = lambda: kqb200.qsa_decode_batch(qlayer, [qs], xq.data_ptr(), yq.data_ptr())
        for _ in range(args.warmup):
            run()
        dev_ms = cx.timed(steps, run)
        xh, yh = synth.hidden(7, 1, qd.hidden), np.empty((1, qd.hidden), np.float32)
        api_ms = cx.timed(steps, lambda: rs.qsa(qlayer, qs, xh, yh))
        w_bytes = sum(t.nbytes for t in (qw.query, qw.key, qw.value, qw.output, qw.index_query, qw.index_key))
        tok_bytes = w_bytes + qd.budget * 2 * qd.kv_width * 4 + (L + 1) // qd.block * qd.index_dim * 4
        rec = {"workload": "config1: QSA layer decode, batch 1, context 4096, Q4_K q/k/v/o, BF16 index, F32 KV",
               "device_ms": dev_ms, "device_tok_s": 1000.0 / dev_ms, "api_ms": api_ms,
               "api_tok_s": 1000.0 / api_ms, "steps": steps,
               "algorithmic_bytes_per_token": tok_bytes,
               "hbm_frac": tok_bytes / (dev_ms * 1e-3) / 1e9 / hbm, "peak_kind": peak_kind}
        if cpu:
            from oracle import oracle as O
            impl = "reference" if O.ref_available() else "port"
            wf = O.qsa_weights_f32(qw)
            xs = synth.hidden(8, 3, qd.hidden)
            t0 = time.perf_counter()
            for i in range(3):
                assert O.qsa_run(qd, wf, xs[i:i + 1], k0, v0, r0, L, L + 1, impl=impl)[0] == 0
            rec["cpu_ms"] = (time.perf_counter() - t0) * 1000.0 / 3
            rec["cpu_kind"] = impl
        out["config1_qsa"] = rec
        qs.close()
        qlayer.close()
    finally:
        prov.close()
    return out


def prefill_record(args, cx: Ctx, kind: str, T: int, steps: int, warmup: int, cpu: bool):
    """One prefill workload (PREFILL_KINDS) of T tokens, tensor-parallel over
    the ranks; returns its record (every rank takes the same collective
    steps)."""
    torch, kqb200 = cx.torch, cx.kq
    from kqb200 import tp
    rank, world = cx.rank, cx.world
    gd, _ = dims()
    gdn_w, qsa_w = PREFILL_KINDS[kind][1]()
    prov = kqb200.Provider(cx.local_rank)
    exchange = tp.torch_exchange(cx.stream) if world > 1 and not args.replicated_indexer else None
    block = tp.TensorParallelBlock(kqb200, prov, gdn_w, qsa_w, rank, world, capacity=T, exchange=exchange)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4321)   # the same input on every rank (replicated activations)
    x = torch.randn(T, gd.hidden, device="cuda", generator=gen)
    bufs = [torch.empty(T, gd.hidden, device="cuda") for _ in range(block.layer_count)]
    torch.cuda.synchronize()
    reduce = (lambda t: cx.dist.all_reduce(t, async_op=True)) if world > 1 else None
    slice_tokens = min(args.slice_tokens, T)

    def step(inp):
        block.reset()
        block.prefill(inp, bufs, T, reduce, slice_tokens=slice_tokens)

    with torch.cuda.stream(cx.stream):
        for _ in range(warmup):
            step(x)
    cx.sync()
    launches0 = cx.lib.kq_b200_kernel_launch_count()
    with ClockSampler(cx.local_rank) as clocks:
        ms = cx.timed(steps, lambda: step(x))
    launches = cx.lib.kq_b200_kernel_launch_count() - launches0
    proj_ms, proj_n = cx.family_ms("proj", steps, lambda: step(x))
    breakdown = {}
    if args.breakdown:
        for fam in ("proj", "proj_exact", "gdn_conv", "gdn_chunk_prep", "gdn_chunk_state", "gdn_gate_norm",
                    "qsa_prepare", "qsa_block_keys", "qsa_score", "qsa_select", "qsa_attend", "qsa_combine"):
            t, n = cx.family_ms(fam, 1, lambda: step(x))
            breakdown[fam] = {"ms_per_step": t, "launches_per_step": n}

    xh = torch.randn(T, gd.hidden, generator=torch.Generator().manual_seed(6)).pin_memory()
    yh = torch.empty(T, gd.hidden).pin_memory()
    xin = torch.empty_like(x)

    def e2e_step():
        xin.copy_(xh, non_blocking=True)
        step(xin)
        yh.copy_(bufs[-1], non_blocking=True)

    e2e_ms = cx.timed(steps, e2e_step)
    assert torch.isfinite(yh).all(), "non-finite prefill output"
    ms, e2e_ms, proj_ms = max_over_ranks([ms, e2e_ms, proj_ms], world, cx.device)
    n_gdn, n_qsa = len(gdn_w), len(qsa_w)
    total_flops, parts = prefill_flops(T, n_gdn, n_qsa)
    tc_flops = rank_tensor_core_flops(block, T)
    achieved = tc_flops / (proj_ms * 1e-3) / 1e12
    peak, peak_kind = tensor_peak()
    qsa_split = ("" if not n_qsa else
                 f", QSA by query-head group (indexer "
                 f"{'replicated' if exchange is None else 'scores/top-k split by 64-token chunk, selections all-reduced'})")
    rec = {
        "value": T * 1000.0 / ms,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": ms,
        "scaling": "strong",
        "workload": f"{PREFILL_KINDS[kind][0]}, {T} tokens",
        "parallelism": (f"tensor-parallel x{world}: GDN by value-head group{qsa_split}, "
                        f"NCCL all-reduce (f32) after each out-projection" if world > 1 else "one GPU"),
        "slice_tokens": slice_tokens,
        "step_algorithmic_flops": total_flops,
        "step_flops_breakdown": parts,
        "step_tflops": total_flops / (ms * 1e-3) / 1e12,
        "roofline": {
            "kernel": "proj (activation tiles + proj_umma: tcgen05 projection GEMMs of this rank's shards)",
            "bound": "tensor",
            "achieved": achieved,
            "peak": peak,
            "peak_kind": peak_kind,
            "unit": "TFLOP/s",
            "frac": achieved / peak,
            "bf16_pipe_frac": 3.0 * achieved / peak,
            "traffic": None,
            "algorithmic_flops_per_step": tc_flops,
            "ms_per_step": proj_ms,
            "launches_per_step": proj_n,
            "note": "F32 operands as bf16 hi/lo pairs: three bf16 MMAs per algorithmic product "
                    "(bf16_pipe_frac = 3 x frac)",
        },
        "e2e": {"value": T * 1000.0 / e2e_ms, "unit": "tok/s",
                "h2d_bytes_per_step": T * gd.hidden * 4, "d2h_bytes_per_step": T * gd.hidden * 4},
        "gpu_launches": int(launches),
        **({"kernel_breakdown": breakdown} if breakdown else {}),
        "clocks": clocks.summary(),
    }
    if cpu and rank == 0 and world == 1:
        rec["cpu_baseline"] = cpu_prefill_record(kind, args.cpu_tokens)
    block.close()
    prov.close()
    del x, bufs, xin
    torch.cuda.empty_cache()
    return rec


def run_b200(args, rank, world, local_rank):
    cx = Ctx(rank, world, local_rank)
    cpu = not args.no_cpu_baseline
    if args.workload == "prefill":
        rec = prefill_record(args, cx, "block", args.tokens, args.steps, args.warmup, cpu)
        line = {"metric": METRIC, "value": rec["value"], "unit": "tok/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": rec["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": rec["workload"], "parallelism": rec["parallelism"],
                           "slice_tokens": rec["slice_tokens"],
                           "l2": "working set per step (GBs of activations, KV, projections) >> 126 MB L2",
                           "step_algorithmic_flops": rec["step_algorithmic_flops"],
                           "step_flops_breakdown": rec["step_flops_breakdown"], "step_tflops": rec["step_tflops"]},
                **{k: rec[k] for k in ("roofline", "e2e", "gpu_launches", "clocks", "kernel_breakdown",
                                       "cpu_baseline") if k in rec}}
    else:
        line = decode_record(args, cx)
        if rank == 0 and world == 1 and cpu:
            threads = cpu_threads()
            v, impl, secs = cpu_block_sample(threads, threads, rank)
            line["cpu_baseline"] = {"value": v, "unit": "tok/s", "cores": threads,
                                    "kind": "reference" if impl == "reference" else "port",
                                    "sample": f"{threads} sequences x 1 token of the 4-layer block, one sequence "
                                              f"per thread ({secs:.1f} s wall)"}
        if world == 1 and args.b1_steps > 0:
            line["decode_b1"] = decode_b1_record(args, cx, cpu)
        if not args.no_moe:
            line["moe_decode"] = moe_record(args, cx, cpu)
            line["layer_decode"] = layer_record(args, cx, cpu)
        if not args.no_prefill:
            ps, pw = args.prefill_steps, args.prefill_warmup
            line["prefill_8k"] = {k: prefill_record(args, cx, k, 8192, ps, pw, cpu) for k in ("gdn_layer", "block")}
            line["prefill_131k"] = prefill_record(args, cx, "block", PREFILL_TOKENS, ps, pw, cpu)
    if rank == 0:
        print(json.dumps(line), flush=True)
    cx.close()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="headline decode record only")
    ap.add_argument("--no-moe", action="store_true", help="skip the MoE decode sub-record")
    ap.add_argument("--moe-steps", type=int, default=50, help="timed steps of the MoE decode sub-record")
    ap.add_argument("--breakdown", action="store_true", help="time every kernel family (extra passes)")
    ap.add_argument("--ctx-max", type=int, default=CTX_RANGE[1],
                    help="upper end of the context distribution (profiling runs use a small one)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill"],
                    help="decode: config 3 headline with the prefill sub-records (default); "
                         "prefill: config 4 alone (--tokens) as the line's own record")
    ap.add_argument("--tokens", type=int, default=PREFILL_TOKENS, help="prefill length (--workload prefill)")
    ap.add_argument("--prefill-steps", type=int, default=3, help="timed steps of each prefill sub-record")
    ap.add_argument("--prefill-warmup", type=int, default=3, help="warm-up steps of each prefill sub-record")
    ap.add_argument("--slice-tokens", type=int, default=PREFILL_SLICE,
                    help="prefill tokens per layer call (all-reduce granularity)")
    ap.add_argument("--per-sequence-steps", type=int, default=3,
                    help="decode steps timed through the reference-shaped entry points, one sequence per call")
    ap.add_argument("--b1-steps", type=int, default=50, help="steps of the batch-1 latency records (configs 0, 1)")
    ap.add_argument("--cpu-tokens", type=int, default=CPU_PREFILL_TOKENS,
                    help="prefill tokens of the CPU baseline sample")
    ap.add_argument("--replicated-indexer", action="store_true",
                    help="prefill at N > 1: every rank selects for every token (no selection exchange)")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    return run_b200(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
