"""Tensor-parallel prefill of a GDN/QSA block: head groups per rank, one
all-reduce after each output projection.

A GDN layer is split by value-head group: rank r of N keeps value heads
[r*Hv/N, (r+1)*Hv/N) and the key heads they read, [r*Hk/N, (r+1)*Hk/N)
(value head h reads key head h // (Hv/Hk), src/kq_gdn_qwen38.c:631-648, so
the groups stay aligned).  Its share of the in-projection is the q, k, v
rows of those heads (src/kq_gdn_qwen38.c:558-579), the gate rows and the
alpha/beta rows of its value heads, and the matching conv channels; the
recurrence and gated norm are local.  Its share of the out-projection is the
columns of its value heads, so the rank's output is a partial sum of
y = W_out . gated (src/kq_gdn_qwen38.c:826-831).

A QSA layer is split by query-head group: rank r keeps query heads
[r*Hq/N, (r+1)*Hq/N) with their interleaved [q | gate] rows
(src/kq_qsa_qwen38.c:569-571) and the key/value heads they read (head h
reads h // (Hq/Hkv)); ranks that share a key/value head both compute it.
Every rank holds the whole indexer (index projections and block keys), so
any rank can select for any token; with a selection exchange the block
scores and top-k are split by 64-token chunk (chunk c on rank c % N) and one
all-reduce of the selection rows gives every rank every token's blocks,
otherwise each rank selects for every token itself.  The out-projection
columns of the group again give a partial sum (src/kq_qsa_qwen38.c:783-787).
With more ranks than key/value heads (and a selection exchange), the ranks
that share a key/value head split the tokens instead of the query heads:
each holds every query head of its key/value head and runs the attention,
gate and out-projection for its contiguous share of the tokens, writing
zero rows elsewhere, so every rank reads only its share of the KV cache and
the same all-reduce completes the output.

Each shard is an ordinary layer of the smaller geometry, bound to the
library through the same config API; only the partial outputs need the
all-reduce.  The sum over ranks is taken in a different order than the
reference's single sequential dot, so results agree within tolerance, not
bit for bit.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import replace
from typing import Callable, Sequence

import numpy as np

from . import synth
from .synth import GEOMETRY, QTensor


# ----------------------------------------------------------------- slicing

def rows(t: QTensor, r0: int, r1: int) -> QTensor:
    """Rows [r0, r1) of a GGUF matrix (whole rows of blocks)."""
    rb = t.row_bytes
    return QTensor(t.type_id, r1 - r0, t.cols, t.data[r0 * rb:r1 * rb].copy())


def cols(t: QTensor, c0: int, c1: int) -> QTensor:
    """Columns [c0, c1) of a GGUF matrix; both ends on block boundaries."""
    be, bb = GEOMETRY[t.type_id]
    if c0 % be or c1 % be:
        raise ValueError(f"column range [{c0}, {c1}) is not aligned to {be}-value blocks")
    m = t.data.reshape(t.rows, t.row_bytes)
    part = np.ascontiguousarray(m[:, c0 // be * bb:c1 // be * bb])
    return QTensor(t.type_id, t.rows, c1 - c0, part.reshape(-1))


def cat_rows(*ts: QTensor) -> QTensor:
    t0 = ts[0]
    assert all(t.type_id == t0.type_id and t.cols == t0.cols for t in ts)
    return QTensor(t0.type_id, sum(t.rows for t in ts), t0.cols, np.concatenate([t.data for t in ts]))


def _check(world: int, rank: int, *counts: int) -> None:
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    for n in counts:
        if n % world:
            raise ValueError(f"{n} heads do not split over {world} ranks")


# ----------------------------------------------------------------- GDN

def gdn_head_range(dims: synth.GdnDims, rank: int, world: int):
    """(k0, nk, v0, nv): the key and value heads of `rank`."""
    _check(world, rank, dims.key_heads, dims.value_heads)
    nk, nv = dims.key_heads // world, dims.value_heads // world
    return rank * nk, nk, rank * nv, nv


def gdn_channels(dims: synth.GdnDims, rank: int, world: int) -> np.ndarray:
    """Conv channels (= qkv rows) of `rank`, in the shard's own order q | k | v."""
    k0, nk, v0, nv = gdn_head_range(dims, rank, world)
    dk, dv, kw = dims.key_dim, dims.value_dim, dims.key_heads * dims.key_dim
    return np.concatenate([np.arange(k0 * dk, (k0 + nk) * dk),
                           kw + np.arange(k0 * dk, (k0 + nk) * dk),
                           2 * kw + np.arange(v0 * dv, (v0 + nv) * dv)])


def shard_gdn(w: synth.GdnLayerWeights, rank: int, world: int) -> synth.GdnLayerWeights:
    d = w.dims
    k0, nk, v0, nv = gdn_head_range(d, rank, world)
    dk, dv, kw, K = d.key_dim, d.value_dim, d.key_heads * d.key_dim, d.conv_kernel
    qkv = cat_rows(rows(w.qkv, k0 * dk, (k0 + nk) * dk),
                   rows(w.qkv, kw + k0 * dk, kw + (k0 + nk) * dk),
                   rows(w.qkv, 2 * kw + v0 * dv, 2 * kw + (v0 + nv) * dv))
    ch = gdn_channels(d, rank, world)
    conv = w.conv.reshape(d.conv_channels, K)[ch].reshape(-1).copy()
    return synth.GdnLayerWeights(
        dims=replace(d, key_heads=nk, value_heads=nv),
        qkv=qkv,
        gate=rows(w.gate, v0 * dv, (v0 + nv) * dv),
        beta=rows(w.beta, v0, v0 + nv),
        alpha=rows(w.alpha, v0, v0 + nv),
        output=cols(w.output, v0 * dv, (v0 + nv) * dv),
        a_log=w.a_log[v0:v0 + nv].copy(),
        conv=conv,
        dt_bias=w.dt_bias[v0:v0 + nv].copy(),
        norm=w.norm.copy(),
    )


def shard_gdn_state(dims: synth.GdnDims, conv: np.ndarray, rec: np.ndarray, rank: int, world: int):
    """The conv history [C][K] and recurrent state [Hv][dk][dv] of a shard."""
    _, _, v0, nv = gdn_head_range(dims, rank, world)
    ch = gdn_channels(dims, rank, world)
    c = conv.reshape(dims.conv_channels, dims.conv_kernel)[ch].reshape(-1).copy()
    r = rec.reshape(dims.value_heads, -1)[v0:v0 + nv].reshape(-1).copy()
    return c, r


# ----------------------------------------------------------------- QSA

def qsa_head_range(dims: synth.QsaDims, rank: int, world: int):
    """(q0, nq, kv0, nkv): the query heads of `rank` and the key/value heads they read."""
    _check(world, rank, dims.query_heads)
    rep = dims.query_heads // dims.kv_heads
    nq = dims.query_heads // world
    if nq % rep and rep % nq:
        raise ValueError(f"{nq} query heads per rank do not align with groups of {rep}")
    q0 = rank * nq
    kv0, kv1 = q0 // rep, (q0 + nq - 1) // rep + 1
    return q0, nq, kv0, kv1 - kv0


def shard_qsa(w: synth.QsaLayerWeights, rank: int, world: int) -> synth.QsaLayerWeights:
    d = w.dims
    q0, nq, kv0, nkv = qsa_head_range(d, rank, world)
    hd = d.head_dim
    return synth.QsaLayerWeights(
        dims=replace(d, query_heads=nq, kv_heads=nkv),
        query=rows(w.query, q0 * 2 * hd, (q0 + nq) * 2 * hd),
        key=rows(w.key, kv0 * hd, (kv0 + nkv) * hd),
        value=rows(w.value, kv0 * hd, (kv0 + nkv) * hd),
        output=cols(w.output, q0 * hd, (q0 + nq) * hd),
        index_query=w.index_query,
        index_key=w.index_key,
        query_norm=w.query_norm.copy(),
        key_norm=w.key_norm.copy(),
        index_query_norm=w.index_query_norm.copy(),
        index_key_norm=w.index_key_norm.copy(),
    )


def qsa_token_part(dims: synth.QsaDims, rank: int, world: int):
    """(key/value head group, member, members) when `world` ranks split a QSA
    layer's tokens within key/value-head groups (world a multiple of the
    key/value head count and larger than it), else None."""
    if world <= dims.kv_heads or world % dims.kv_heads:
        return None
    members = world // dims.kv_heads
    return rank // members, rank % members, members


def shard_qsa_cache(dims: synth.QsaDims, key: np.ndarray, value: np.ndarray, raw: np.ndarray,
                    rank: int, world: int):
    """Cache rows of a shard: its key/value heads, and the whole raw index keys."""
    _, _, kv0, nkv = qsa_head_range(dims, rank, world)
    hd = dims.head_dim
    sl = slice(kv0 * hd, (kv0 + nkv) * hd)
    return np.ascontiguousarray(key[:, sl]), np.ascontiguousarray(value[:, sl]), raw.copy()


# ----------------------------------------------------------------- block

class TensorParallelBlock:
    """The layers of one hybrid block (GDN layers, then QSA layers), each
    sharded over `world` ranks, with the states of one sequence.

    `prefill(x, y, T)` runs T tokens: every layer reads the full
    activations [T][H] (replicated on every rank), writes its partial output,
    and `all_reduce` (in place, sum over ranks) completes it before the next
    layer reads it.  The tokens go through in slices of `slice_tokens`, so
    that the all-reduce of one slice overlaps the next slice's kernels when
    `all_reduce` returns a handle with `wait()` (asynchronous collectives).
    """

    def __init__(self, kq, provider, gdn_weights: Sequence[synth.GdnLayerWeights],
                 qsa_weights: Sequence[synth.QsaLayerWeights], rank: int, world: int, capacity: int,
                 layer_base: int = 0, exchange: Callable | None = None):
        """`exchange(words_ptr, count, stream_ptr) -> int`, when given,
        enqueues on the library stream a sum over the ranks of `count` int32
        words at `words_ptr` (device memory) and returns 0; the QSA layers
        then split the indexer's selections by token chunk."""
        self.kq = kq
        self.rank, self.world = rank, world
        self._exchange = None
        if exchange is not None and world > 1:
            self._exchange = kq.abi.EXCHANGE_FN(lambda p, n, st, _u: int(exchange(p, n, st)))
        self.gdn_layers, self.gdn_states = [], []
        self.qsa_layers, self.qsa_states = [], []
        for i, w in enumerate(gdn_weights):
            sw = shard_gdn(w, rank, world)
            layer = kq.GdnLayer(sw.dims, sw, provider, layer=layer_base + i)
            self.gdn_layers.append(layer)
            self.gdn_states.append(kq.GdnState(layer))
        self.token_parts = []
        for i, w in enumerate(qsa_weights):
            part = qsa_token_part(w.dims, rank, world) if self._exchange is not None else None
            if part is None:
                sw = shard_qsa(w, rank, world)
                self.token_parts.append((0, 1))
            else:
                group, member, members = part
                sw = shard_qsa(w, group, w.dims.kv_heads)
                self.token_parts.append((member, members))
            layer = kq.QsaLayer(sw.dims, sw, provider, layer=layer_base + len(gdn_weights) + i)
            self.qsa_layers.append(layer)
            self.qsa_states.append(kq.QsaState(layer, capacity))

    @property
    def layer_count(self) -> int:
        return len(self.gdn_layers) + len(self.qsa_layers)

    def reset(self) -> None:
        lib, abi = self.kq.lib(), self.kq.abi
        for s in self.gdn_states:
            d = abi.Diagnostic()
            abi.check(lib.kq_gdn_state_reset(s.handle, C.byref(d)), d)
        for s in self.qsa_states:
            d = abi.Diagnostic()
            abi.check(lib.kq_qsa_state_reset(s.handle, C.byref(d)), d)

    def run_layer(self, index: int, x_ptr: int, tokens: int, y_ptr: int) -> None:
        """Partial output of layer `index` for `tokens` tokens (asynchronous)."""
        if index < len(self.gdn_states):
            self.kq.gdn_prefill_async(self.gdn_states[index], x_ptr, tokens, y_ptr)
        elif self._exchange is not None:
            q = index - len(self.gdn_states)
            part, parts = self.token_parts[q]
            self.kq.qsa_prefill_sharded_async(self.qsa_states[q], x_ptr, tokens, y_ptr, self.rank, self.world,
                                              self._exchange, part, parts)
        else:
            self.kq.qsa_prefill_async(self.qsa_states[index - len(self.gdn_states)], x_ptr, tokens, y_ptr)

    def prefill(self, x, buffers: Sequence, tokens: int, all_reduce: Callable | None,
                slice_tokens: int | None = None) -> None:
        """x: device [T][H] f32 (torch); buffers: one device [T][H] f32 output
        per layer; the block's output is buffers[-1].  `all_reduce(t)` sums a
        tensor over the ranks in place (None for one rank) and may return a
        handle with `wait()`."""
        S = tokens if slice_tokens is None else max(1, min(slice_tokens, tokens))
        pending = {}
        src = x
        for layer in range(self.layer_count):
            dst = buffers[layer]
            t0 = 0
            while t0 < tokens:
                n = min(S, tokens - t0)
                h = pending.pop((layer - 1, t0), None)
                if h is not None:
                    h.wait()
                self.run_layer(layer, src[t0:t0 + n].data_ptr(), n, dst[t0:t0 + n].data_ptr())
                if all_reduce is not None:
                    h = all_reduce(dst[t0:t0 + n])
                    if h is not None:
                        pending[(layer, t0)] = h
                t0 += n
            src = dst
        for h in pending.values():
            h.wait()

    def close(self) -> None:
        for s in self.gdn_states + self.qsa_states:
            s.close()
        for layer in self.gdn_layers + self.qsa_layers:
            layer.close()
        self.gdn_states, self.qsa_states, self.gdn_layers, self.qsa_layers = [], [], [], []


class DeviceWords:
    """A device array the library owns, seen by torch (CUDA array interface)."""

    def __init__(self, ptr: int, count: int, typestr: str = "<i4"):
        self.__cuda_array_interface__ = {"shape": (int(count),), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None, "stream": None}


def torch_exchange(lib_stream):
    """A selection exchange over torch.distributed (NCCL): an in-place
    all-reduce (sum) of the words on the library stream."""
    import torch
    import torch.distributed as dist

    def exchange(ptr: int, count: int, _stream: int) -> int:
        t = torch.as_tensor(DeviceWords(ptr, count), device="cuda")
        with torch.cuda.stream(lib_stream):
            dist.all_reduce(t)
        return 0

    return exchange
