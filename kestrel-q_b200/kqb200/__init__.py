"""Python host mirror of the Kestrel-Q operator ABI on the B200.

The product is the C-ABI library ``kestrel-q_b200/lib/libkqb200.so``
(include/*.h); this package binds it with ctypes for tests, the benchmark and
Python callers, keeping the reference's names, argument meaning and error
behaviour (every non-OK ``kq_status`` raises :class:`KQError`).
Device memory for batched calls comes from torch (plumbing only).
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np

from . import abi, synth
from .abi import KQError, lib

__all__ = ["abi", "synth", "lib", "KQError", "Provider", "GdnLayer", "GdnState", "QsaLayer",
           "QsaState", "build"]


def build(force: bool = False):
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location(
        "kqb200_build", Path(__file__).resolve().parent.parent / "build.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.build(force)


def _ptr(a) -> int | None:
    if a is None:
        return None
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return int(a)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


class Provider:
    """Device-resident weight provider (kq_b200_provider_create)."""

    def __init__(self, device: int = 0):
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_b200_provider_create(device, C.byref(self.handle), C.byref(d)), d)
        self.device = device

    def add_matrix(self, name: str, role: int, t: synth.QTensor) -> int:
        out = C.c_void_p()
        d = abi.Diagnostic()
        data = np.ascontiguousarray(t.data)
        abi.check(lib().kq_b200_provider_add_matrix(self.handle, name.encode(), role, t.type_id, t.rows,
                                                    t.cols, data.ctypes.data, data.size, C.byref(out),
                                                    C.byref(d)), d)
        return out.value

    def add_vector(self, name: str, role: int, values: np.ndarray) -> int:
        v = _f32(values)
        out = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_b200_provider_add_vector_f32(self.handle, name.encode(), role, v.ctypes.data,
                                                        v.size, C.byref(out), C.byref(d)), d)
        return out.value

    def linear(self, tensor: int, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        xv = _f32(x)
        y = np.empty(rows, np.float32)
        d = abi.Diagnostic()
        abi.check(lib().kq_weight_provider_linear_f32(self.handle, tensor, 0, 0xFFFFFFFF, rows, cols,
                                                      xv.ctypes.data, y.ctypes.data, rows, None, 0,
                                                      C.byref(d)), d)
        return y

    def close(self):
        if self.handle:
            lib().kq_weight_provider_close(self.handle)
            self.handle = C.c_void_p()


# roles (include/kq_model.h)
ROLE = {"a_log": 6, "conv": 7, "dt_bias": 8, "alpha": 9, "beta": 10, "qkv": 11, "gate": 12, "norm": 13,
        "out": 14, "k_norm": 15, "k": 16, "o": 17, "q_norm": 18, "q": 19, "v": 20, "index_qk": 21,
        "index_k_norm": 22, "index_q_norm": 23, "moe_router": 24, "routed_down": 25, "routed_gate_up": 26,
        "shared_down": 27, "shared_gate": 28, "shared_up": 29, "shared_gate_weight": 30, "hc_norm": 2, "hc_down": 3, "hc_up": 4, "hc_inject": 5}


class GdnLayer:
    """A GDN test config (kq_gdn_test_config_create), optionally bound to
    provider weights (kq_b200_gdn_config_bind)."""

    def __init__(self, dims: synth.GdnDims, weights: synth.GdnLayerWeights | None = None,
                 provider: Provider | None = None, layer: int = 0, activation_dtype: int = 0):
        gd = abi.GdnDimensions(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim,
                               dims.value_dim, dims.conv_kernel, dims.eps, activation_dtype)
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_gdn_test_config_create(C.byref(gd), C.byref(self.handle), C.byref(d)), d)
        self.dims = dims
        self.provider = provider
        if weights is not None:
            assert provider is not None
            p = provider
            t = abi.GdnTensors(
                a_log=p.add_vector(f"l{layer}.gdn.a_log", ROLE["a_log"], weights.a_log),
                conv=p.add_vector(f"l{layer}.gdn.conv", ROLE["conv"], weights.conv),
                dt_bias=p.add_vector(f"l{layer}.gdn.dt_bias", ROLE["dt_bias"], weights.dt_bias),
                alpha=p.add_matrix(f"l{layer}.gdn.alpha", ROLE["alpha"], weights.alpha),
                beta=p.add_matrix(f"l{layer}.gdn.beta", ROLE["beta"], weights.beta),
                qkv=p.add_matrix(f"l{layer}.gdn.qkv", ROLE["qkv"], weights.qkv),
                gate=p.add_matrix(f"l{layer}.gdn.gate", ROLE["gate"], weights.gate),
                norm=p.add_vector(f"l{layer}.gdn.norm", ROLE["norm"], weights.norm),
                output=p.add_matrix(f"l{layer}.gdn.out", ROLE["out"], weights.output))
            abi.check(lib().kq_b200_gdn_config_bind(self.handle, p.handle, C.byref(t), C.byref(d)), d)

    @property
    def scratch_bytes(self) -> int:
        return lib().kq_gdn_config_scratch_bytes(self.handle)

    def close(self):
        if self.handle:
            lib().kq_gdn_config_close(self.handle)
            self.handle = C.c_void_p()


class GdnState:
    def __init__(self, layer: GdnLayer):
        self.layer = layer
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_gdn_state_create(layer.handle, C.byref(self.handle), C.byref(d)), d)

    def load(self, conv: np.ndarray, rec: np.ndarray, initialized: int = 1):
        c, r = _f32(conv), _f32(rec)
        d = abi.Diagnostic()
        abi.check(lib().kq_gdn_state_import_f32(self.handle, c.ctypes.data, c.size, r.ctypes.data, r.size,
                                                initialized, C.byref(d)), d)

    def save(self):
        L = lib()
        nc = L.kq_gdn_config_conv_state_element_count(self.layer.handle)
        nr = L.kq_gdn_config_recurrent_element_count(self.layer.handle)
        c = np.empty(nc, np.float32)
        r = np.empty(nr, np.float32)
        init = C.c_int()
        d = abi.Diagnostic()
        abi.check(L.kq_gdn_state_export_f32(self.handle, c.ctypes.data, nc, r.ctypes.data, nr, C.byref(init),
                                            C.byref(d)), d)
        return c, r, init.value

    def execute_quantized(self, x: np.ndarray, mask: np.ndarray | None = None) -> np.ndarray:
        xv = _f32(x)
        T = xv.shape[0]
        H = self.layer.dims.hidden
        y = np.empty((T, H), np.float32)
        scratch = np.empty(max(1, self.layer.scratch_bytes // 4), np.float32)
        wscratch = np.empty(self._weight_scratch_floats(), np.float32)
        m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        d = abi.Diagnostic()
        abi.check(lib().kq_gdn_execute_quantized(self.layer.handle, self.layer.provider.handle, xv.ctypes.data, T,
                                                 _ptr(m), y.ctypes.data, y.size, self.handle,
                                                 scratch.ctypes.data, scratch.nbytes, wscratch.ctypes.data,
                                                 wscratch.nbytes, None, None, C.byref(d)), d)
        return y

    def _weight_scratch_floats(self) -> int:
        dm = self.layer.dims
        conv = dm.conv_channels * dm.conv_kernel
        return 2 * dm.value_heads + 2 * conv + dm.value_dim + 65536 // 4 + 64

    def close(self):
        if self.handle:
            lib().kq_gdn_state_close(self.handle)
            self.handle = C.c_void_p()


def gdn_decode_batch(layer: GdnLayer, states: Sequence[GdnState], x_ptr: int, y_ptr: int) -> None:
    arr = (C.c_void_p * len(states))(*[s.handle.value for s in states])
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_gdn_decode_batch(layer.handle, arr, len(states), x_ptr, y_ptr, C.byref(d)), d)


class QsaLayer:
    def __init__(self, dims: synth.QsaDims, weights: synth.QsaLayerWeights | None = None,
                 provider: Provider | None = None, layer: int = 3, activation_dtype: int = 0):
        qd = abi.QsaDimensions(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads,
                               dims.index_dim, dims.block, dims.budget, dims.max_context, dims.rotary,
                               dims.eps, dims.theta, activation_dtype)
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_qsa_test_config_create(C.byref(qd), C.byref(self.handle), C.byref(d)), d)
        self.dims = dims
        self.provider = provider
        if weights is not None:
            assert provider is not None
            p = provider
            t = abi.QsaTensors(
                query=p.add_matrix(f"l{layer}.qsa.q", ROLE["q"], weights.query),
                key=p.add_matrix(f"l{layer}.qsa.k", ROLE["k"], weights.key),
                value=p.add_matrix(f"l{layer}.qsa.v", ROLE["v"], weights.value),
                output=p.add_matrix(f"l{layer}.qsa.o", ROLE["o"], weights.output),
                query_norm=p.add_vector(f"l{layer}.qsa.q_norm", ROLE["q_norm"], weights.query_norm),
                key_norm=p.add_vector(f"l{layer}.qsa.k_norm", ROLE["k_norm"], weights.key_norm),
                index_query=p.add_matrix(f"l{layer}.qsa.iq", ROLE["index_qk"], weights.index_query),
                index_key=p.add_matrix(f"l{layer}.qsa.ik", ROLE["index_qk"], weights.index_key),
                index_query_norm=p.add_vector(f"l{layer}.qsa.iq_norm", ROLE["index_q_norm"],
                                              weights.index_query_norm),
                index_key_norm=p.add_vector(f"l{layer}.qsa.ik_norm", ROLE["index_k_norm"],
                                            weights.index_key_norm))
            abi.check(lib().kq_b200_qsa_config_bind(self.handle, p.handle, C.byref(t), C.byref(d)), d)

    def close(self):
        if self.handle:
            lib().kq_qsa_config_close(self.handle)
            self.handle = C.c_void_p()


class QsaState:
    def __init__(self, layer: QsaLayer, capacity: int):
        self.layer = layer
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_qsa_state_create(layer.handle, capacity, C.byref(self.handle), C.byref(d)), d)

    @property
    def length(self) -> int:
        return lib().kq_qsa_state_length(self.handle)

    def load(self, key: np.ndarray, value: np.ndarray, raw: np.ndarray):
        k, v, r = _f32(key), _f32(value), _f32(raw)
        d = abi.Diagnostic()
        abi.check(lib().kq_qsa_state_import_f32(self.handle, k.ctypes.data, k.size, v.ctypes.data, v.size,
                                                r.ctypes.data, r.size, k.shape[0] if k.ndim == 2 else
                                                k.size // self.layer.dims.kv_width, C.byref(d)), d)

    def save(self):
        dm = self.layer.dims
        n = self.length
        k = np.empty((n, dm.kv_width), np.float32)
        v = np.empty((n, dm.kv_width), np.float32)
        r = np.empty((n, dm.index_dim), np.float32)
        ln = C.c_uint64()
        d = abi.Diagnostic()
        abi.check(lib().kq_qsa_state_export_f32(self.handle, k.ctypes.data, k.size, v.ctypes.data, v.size,
                                                r.ctypes.data, r.size, C.byref(ln), C.byref(d)), d)
        return k, v, r

    def execute_quantized(self, x: np.ndarray, want_selection: bool = False):
        xv = _f32(x)
        T = xv.shape[0]
        dm = self.layer.dims
        y = np.empty((T, dm.hidden), np.float32)
        need = C.c_uint64()
        d = abi.Diagnostic()
        # an impossible request (e.g. beyond capacity) is left to the
        # operator's own validation, which reports the reference's status
        if lib().kq_qsa_required_scratch_bytes(self.layer.handle, self.handle, T, C.byref(need), C.byref(d)) != 0:
            need.value = 4
        scratch = np.empty(max(1, need.value // 4), np.float32)
        wscratch = np.empty((65536 + 8 * (dm.head_dim + dm.index_dim) * 4) // 4 + 64, np.float32)
        sels = []

        def on_sel(sel_p, _user):
            s = sel_p.contents
            sels.append({
                "position": s.absolute_position,
                "scores": np.ctypeslib.as_array(s.candidate_scores, (s.candidate_count,)).copy()
                if s.candidate_count else np.empty(0, np.float32),
                "selected": np.ctypeslib.as_array(s.selected_block_ids, (s.selected_block_count,)).copy()
                if s.selected_block_count else np.empty(0, np.uint32),
                "tokens": np.ctypeslib.as_array(s.selected_token_positions, (s.selected_token_count,)).copy(),
                "tail": s.tail_count,
            })

        cb = abi.SELECTION_OBSERVER(on_sel) if want_selection else abi.SELECTION_OBSERVER()
        abi.check(lib().kq_qsa_execute_quantized(self.layer.handle, self.layer.provider.handle, xv.ctypes.data,
                                                 T, y.ctypes.data, y.size, self.handle, scratch.ctypes.data,
                                                 scratch.nbytes, wscratch.ctypes.data, wscratch.nbytes, cb,
                                                 None, None, C.byref(d)), d)
        return (y, sels) if want_selection else y

    def close(self):
        if self.handle:
            lib().kq_qsa_state_close(self.handle)
            self.handle = C.c_void_p()


def qsa_decode_batch(layer: QsaLayer, states: Sequence[QsaState], x_ptr: int, y_ptr: int) -> None:
    arr = (C.c_void_p * len(states))(*[s.handle.value for s in states])
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_qsa_decode_batch(layer.handle, arr, len(states), x_ptr, y_ptr, C.byref(d)), d)


class MoeLayer:
    """An MoE test config (kq_moe_test_config_create), optionally bound to
    provider weights (kq_b200_moe_config_bind): router F32 matrix, gate/up as
    one split semantic of two expert stacks, down as an expert stack, the
    shared expert's three matrices and its [1 x H] gate weight."""

    def __init__(self, dims: synth.MoeDims, weights: synth.MoeLayerWeights | None = None,
                 provider: Provider | None = None, layer: int = 0, activation_dtype: int = 0):
        md = abi.MoeDimensions(dims.hidden, dims.experts, dims.top_k, dims.routed, dims.shared, activation_dtype)
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_moe_test_config_create(C.byref(md), C.byref(self.handle), C.byref(d)), d)
        self.dims = dims
        self.provider = provider
        self.tensors = None
        if weights is not None:
            assert provider is not None
            p, L = provider, lib()
            E, H, I = dims.experts, dims.hidden, dims.routed

            def stack(name, role, t, rows, cols):
                out = C.c_void_p()
                data = np.ascontiguousarray(t.data)
                abi.check(L.kq_b200_provider_add_expert_stack(p.handle, name.encode(), role, t.type_id, E, rows, cols,
                                                              data.ctypes.data, data.size, C.byref(out),
                                                              C.byref(d)), d)
                return out.value

            gu = C.c_void_p()
            g, u = np.ascontiguousarray(weights.gate.data), np.ascontiguousarray(weights.up.data)
            abi.check(L.kq_b200_provider_add_expert_gate_up(p.handle, f"l{layer}.moe.gate_up".encode(),
                                                            weights.gate.type_id, E, I, H, g.ctypes.data, g.size,
                                                            u.ctypes.data, u.size, C.byref(gu), C.byref(d)), d)
            gw = synth.f32_tensor(weights.shared_gate_weight.reshape(1, -1))
            t = abi.MoeTensors(
                router=p.add_matrix(f"l{layer}.moe.router", ROLE["moe_router"], weights.router),
                routed_down=stack(f"l{layer}.moe.down", ROLE["routed_down"], weights.down, H, I),
                routed_gate_up=gu.value,
                shared_down=p.add_matrix(f"l{layer}.moe.shared_down", ROLE["shared_down"], weights.shared_down),
                shared_gate=p.add_matrix(f"l{layer}.moe.shared_gate", ROLE["shared_gate"], weights.shared_gate),
                shared_up=p.add_matrix(f"l{layer}.moe.shared_up", ROLE["shared_up"], weights.shared_up),
                shared_gate_weight=p.add_matrix(f"l{layer}.moe.shared_gate_weight", ROLE["shared_gate_weight"], gw))
            self.tensors = t
            abi.check(L.kq_b200_moe_config_bind(self.handle, p.handle, C.byref(t), C.byref(d)), d)

    @property
    def scratch_bytes(self) -> int:
        return lib().kq_moe_config_scratch_bytes(self.handle)

    def _run(self, fn, first, x, route: bool, checkpoints: bool):
        xv = _f32(x)
        T = xv.shape[0]
        y = np.zeros((T, self.dims.hidden), np.float32)
        scratch = np.zeros(self.scratch_bytes // 4 + 1, np.float32)
        routes, cps = [], []

        def on_route(p, _u):
            r = p.contents
            routes.append({"token": int(r.token_index),
                           "logits": np.ctypeslib.as_array(r.router_logits, (r.expert_count,)).copy(),
                           "probabilities": np.ctypeslib.as_array(r.router_probabilities, (r.expert_count,)).copy(),
                           "ids": np.ctypeslib.as_array(r.selected_expert_ids, (r.selected_count,)).copy(),
                           "weights": np.ctypeslib.as_array(r.selected_weights, (r.selected_count,)).copy()})

        def on_cp(p, _u):
            c = p.contents
            cps.append((int(c.kind), int(c.token_index), int(c.expert_id), int(c.top_k_position),
                        np.ctypeslib.as_array(c.values, (c.value_count,)).copy()))

        rcb = abi.MOE_ROUTE_OBSERVER(on_route) if route else abi.MOE_ROUTE_OBSERVER()
        ccb = abi.MOE_CHECKPOINT_OBSERVER(on_cp) if checkpoints else abi.MOE_CHECKPOINT_OBSERVER()
        d = abi.Diagnostic()
        st = fn(*first, xv.ctypes.data, T, y.ctypes.data, y.size, scratch.ctypes.data, scratch.nbytes, rcb, ccb,
                None, C.byref(d))
        return st, y, routes, cps, d

    def execute_quantized(self, x: np.ndarray, route: bool = False, checkpoints: bool = False):
        """(status, y, routes, checkpoints, diagnostic) of kq_moe_execute_quantized."""
        ws = np.zeros(16384 + 1, np.float32)
        L = lib()

        def call(cfg, prov, xp, T, yp, cap, sp, sb, rcb, ccb, user, dp):
            return L.kq_moe_execute_quantized(cfg, prov, xp, T, yp, cap, sp, sb, ws.ctypes.data, ws.nbytes, rcb, ccb,
                                              user, dp)
        return self._run(call, (self.handle, self.provider.handle), x, route, checkpoints)

    def execute_f32(self, w: dict, x: np.ndarray, route: bool = False, checkpoints: bool = False):
        """(status, y, routes, checkpoints, diagnostic) of kq_moe_execute_f32
        with canonical F32 weights `w` (abi.MOE_WEIGHT_FIELDS)."""
        arrs = {k: _f32(np.asarray(w[k]).reshape(-1)) for k in abi.MOE_WEIGHT_FIELDS}
        mw = abi.MoeWeightsF32()
        for k in abi.MOE_WEIGHT_FIELDS:
            setattr(mw, k, arrs[k].ctypes.data)
            setattr(mw, k + "_count", arrs[k].size)
        return self._run(lib().kq_moe_execute_f32, (self.handle, C.byref(mw)), x, route, checkpoints)

    def close(self):
        if self.handle:
            lib().kq_moe_config_close(self.handle)
            self.handle = C.c_void_p()


class DecoderLayer:
    """A decoder layer (kq_layer_test_config_create) over a GdnLayer or
    QsaLayer mixer and a MoeLayer, optionally with provider gated-residual
    tensors (kq_b200_layer_config_bind).  family: 1 GDN, 2 QSA."""

    def __init__(self, family: int, hidden: int, branches: int, rank: int, eps: float, mixer, moe: MoeLayer,
                 gr: dict | None = None, provider: Provider | None = None, layer: int = 0):
        self.family, self.hidden, self.branches, self.rank = family, hidden, branches, rank
        self.mixer, self.moe, self.provider = mixer, moe, provider
        ld = abi.LayerDimensions(layer, hidden, branches, rank, eps, family)
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_layer_test_config_create(C.byref(ld), mixer.handle if family == 1 else None,
                                                    mixer.handle if family == 2 else None, moe.handle, None, None,
                                                    C.byref(self.handle), C.byref(d)), d)
        if gr is not None:
            p = provider
            t = abi.LayerTensors()
            for side, prefix in (("attn", "attention"), ("moe", "moe")):
                g = gr[side]
                setattr(t, f"{prefix}_norm", p.add_vector(f"l{layer}.{side}_gr.norm", ROLE["hc_norm"], g.norm))
                setattr(t, f"{prefix}_down", p.add_matrix(f"l{layer}.{side}_gr.down", ROLE["hc_down"], g.down))
                setattr(t, f"{prefix}_up", p.add_matrix(f"l{layer}.{side}_gr.up", ROLE["hc_up"], g.up))
                setattr(t, f"{prefix}_inject", p.add_matrix(f"l{layer}.{side}_gr.inject", ROLE["hc_inject"], g.inject))
            abi.check(lib().kq_b200_layer_config_bind(self.handle, p.handle, C.byref(t), C.byref(d)), d)

    @property
    def width(self) -> int:
        return self.hidden * self.branches

    def state(self, capacity: int = 0) -> "DecoderLayerState":
        return DecoderLayerState(self, capacity)

    def close(self):
        if self.handle:
            lib().kq_layer_config_close(self.handle)
            self.handle = C.c_void_p()


class DecoderLayerState:
    def __init__(self, layer: DecoderLayer, capacity: int = 0):
        self.layer = layer
        self.handle = C.c_void_p()
        d = abi.Diagnostic()
        abi.check(lib().kq_layer_state_create(layer.handle, capacity, C.byref(self.handle), C.byref(d)), d)

    @property
    def position(self) -> int:
        return lib().kq_layer_state_position(self.handle)

    def rollback_last(self, tokens: int) -> int:
        d = abi.Diagnostic()
        return lib().kq_layer_state_rollback_last(self.handle, tokens, C.byref(d))

    def _scratch(self, T: int, quantized: bool):
        need = C.c_uint64()
        d = abi.Diagnostic()
        fn = lib().kq_layer_required_quantized_scratch_bytes if quantized else lib().kq_layer_required_scratch_bytes
        abi.check(fn(self.layer.handle, self.handle, T, C.byref(need), C.byref(d)), d)
        return np.zeros(need.value // 4 + 1, np.float32)

    def _observer(self, checkpoints: bool):
        cps = []

        def on_cp(p, _u):
            c = p.contents
            cps.append((int(c.kind), int(c.token_index), int(c.rank),
                        tuple(int(c.dimensions[i]) for i in range(c.rank)),
                        np.ctypeslib.as_array(c.values, (c.value_count,)).copy()))

        return cps, (abi.LAYER_CHECKPOINT_OBSERVER(on_cp) if checkpoints else abi.LAYER_CHECKPOINT_OBSERVER())

    def run_f32(self, weights: dict, x: np.ndarray, mask: np.ndarray | None = None, checkpoints: bool = False):
        """kq_layer_prefill_f32 with F32 arrays: weights = {"attn": {norm, down,
        up, inject}, "moe_gr": {...}, "mixer": {fields}, "moe": {fields}}.
        Returns (status, y, checkpoints, metrics, diagnostic)."""
        L = self.layer
        keep = []

        def arr(a):
            v = _f32(np.asarray(a).reshape(-1))
            keep.append(v)
            return v

        lw = abi.LayerWeightsF32()
        for side, dst in (("attn", lw.attention_gr), ("moe_gr", lw.moe_gr)):
            for k in abi.GR_FIELDS:
                v = arr(weights[side][k])
                setattr(dst, k, v.ctypes.data)
                setattr(dst, k + "_count", v.size)
        fields = abi.GDN_WEIGHT_FIELDS if L.family == 1 else abi.QSA_WEIGHT_FIELDS
        mw = abi.GdnWeightsF32() if L.family == 1 else abi.QsaWeightsF32()
        for k in fields:
            v = arr(weights["mixer"][k])
            setattr(mw, k, v.ctypes.data)
            setattr(mw, k + "_count", v.size)
        ew = abi.MoeWeightsF32()
        for k in abi.MOE_WEIGHT_FIELDS:
            v = arr(weights["moe"][k])
            setattr(ew, k, v.ctypes.data)
            setattr(ew, k + "_count", v.size)
        if L.family == 1:
            lw.gdn = C.cast(C.pointer(mw), C.c_void_p)
        else:
            lw.qsa = C.cast(C.pointer(mw), C.c_void_p)
        lw.moe = C.cast(C.pointer(ew), C.c_void_p)
        xv = _f32(x).reshape(-1, L.width)
        T = xv.shape[0]
        y = np.zeros_like(xv)
        scratch = self._scratch(T, False)
        cps, cb = self._observer(checkpoints)
        m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        met = abi.LayerMetrics()
        d = abi.Diagnostic()
        st = lib().kq_layer_prefill_f32(L.handle, C.byref(lw), xv.ctypes.data, None, T,
                                        None if m is None else m.ctypes.data, y.ctypes.data, y.size, self.handle,
                                        scratch.ctypes.data, scratch.nbytes, cb, None, C.byref(met), C.byref(d))
        return st, y, cps, met, d

    def run_quantized(self, x: np.ndarray, mask: np.ndarray | None = None, checkpoints: bool = False):
        """kq_layer_prefill_quantized_f32 (provider-bound config)."""
        L = self.layer
        xv = _f32(x).reshape(-1, L.width)
        T = xv.shape[0]
        y = np.zeros_like(xv)
        scratch = self._scratch(T, True)
        cps, cb = self._observer(checkpoints)
        m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
        met = abi.LayerMetrics()
        d = abi.Diagnostic()
        st = lib().kq_layer_prefill_quantized_f32(L.handle, L.provider.handle, xv.ctypes.data, None, T,
                                                  None if m is None else m.ctypes.data, y.ctypes.data, y.size,
                                                  self.handle, scratch.ctypes.data, scratch.nbytes, cb, None,
                                                  C.byref(met), C.byref(d))
        return st, y, cps, met, d

    def close(self):
        if self.handle:
            lib().kq_layer_state_close(self.handle)
            self.handle = C.c_void_p()


def layer_decode_batch(layer: DecoderLayer, states: Sequence[DecoderLayerState], x_ptr: int, y_ptr: int) -> None:
    arr = (C.c_void_p * len(states))(*[s.handle.value for s in states])
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_layer_decode_batch(layer.handle, arr, len(states), x_ptr, y_ptr, C.byref(d)), d)


def moe_execute_async(layer: MoeLayer, x_ptr: int, tokens: int, y_ptr: int) -> None:
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_moe_execute_async(layer.handle, x_ptr, tokens, y_ptr, C.byref(d)), d)


def gdn_prefill_async(state: GdnState, x_ptr: int, tokens: int, y_ptr: int) -> None:
    """T tokens of one sequence on device buffers, asynchronous on the library stream."""
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_gdn_prefill_async(state.layer.handle, state.handle, x_ptr, tokens, y_ptr,
                                              C.byref(d)), d)


def qsa_prefill_async(state: QsaState, x_ptr: int, tokens: int, y_ptr: int) -> None:
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_qsa_prefill_async(state.layer.handle, state.handle, x_ptr, tokens, y_ptr,
                                              C.byref(d)), d)


def qsa_prefill_sharded_async(state: QsaState, x_ptr: int, tokens: int, y_ptr: int, rank: int, world: int,
                              exchange, token_part: int = 0, token_parts: int = 1) -> None:
    """Tensor-parallel QSA prefill of one rank: the indexer's scores and top-k
    of this rank's 64-token chunk groups, `exchange` (an abi.EXCHANGE_FN,
    kept alive by the caller) sums the selection buffer over the ranks, then
    attention for every chunk, or with token_parts > 1 for token part
    `token_part` only (zero output rows elsewhere)."""
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_qsa_prefill_split_async(state.layer.handle, state.handle, x_ptr, tokens, y_ptr, rank,
                                                    world, token_part, token_parts, exchange, None, C.byref(d)), d)


def synchronize() -> None:
    d = abi.Diagnostic()
    abi.check(lib().kq_b200_synchronize(C.byref(d)), d)
