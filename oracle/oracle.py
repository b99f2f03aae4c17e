"""ctypes wrapper of the CPU oracle (TEST INFRASTRUCTURE ONLY).

Two implementations of the reference algorithm, selected by ``impl``:

  "port"       oracle/_build/libkqoracle.so — this repository's C restatement
               (kq_oracle.c), including Q6_K which the reference lacks;
  "reference"  oracle/_ref/libkqref.so — Kestrel-Q's own hot-path C sources
               compiled from the reference tree by ``make -C oracle ref``.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
PORT_LIB = HERE / "_build" / "libkqoracle.so"
REF_LIB = HERE / "_ref" / "libkqref.so"

u32, u64, f32, vp = C.c_uint32, C.c_uint64, C.c_float, C.c_void_p

GEOMETRY = {0: (1, 4), 30: (1, 2), 8: (32, 34), 12: (256, 144), 14: (256, 210)}


class _GdnDims(C.Structure):   # kqo_gdn_dims
    _fields_ = [("hidden_size", u32), ("key_heads", u32), ("value_heads", u32), ("key_dim", u32),
                ("value_dim", u32), ("conv_kernel", u32), ("rms_norm_epsilon", f32)]


class _GdnWeights(C.Structure):   # kqo_gdn_weights
    _fields_ = [(n, vp) for n in ["a_log", "conv", "dt_bias", "alpha", "beta", "qkv", "gate", "norm", "output"]]


class _QsaDims(C.Structure):   # kqo_qsa_dims
    _fields_ = [("hidden_size", u32), ("query_heads", u32), ("kv_heads", u32), ("head_dim", u32),
                ("index_heads", u32), ("index_dim", u32), ("block_size", u32), ("token_budget", u32),
                ("rotary_dim", u32), ("rms_norm_epsilon", f32), ("rope_theta", f32)]


QSA_FIELDS = ["query", "key", "value", "output", "query_norm", "key_norm", "index_query", "index_key",
              "index_query_norm", "index_key_norm"]
GDN_FIELDS = ["a_log", "conv", "dt_bias", "alpha", "beta", "qkv", "gate", "norm", "output"]


class _QsaWeights(C.Structure):   # kqo_qsa_weights
    _fields_ = [(n, vp) for n in QSA_FIELDS]


# reference ABI structures (Kestrel-Q src/kq_gdn_internal.h:11-20,
# src/kq_qsa_internal.h:11-25, include/kq_gdn.h:64-83, include/kq_qsa.h:82-103)
class _RefGdnDims(C.Structure):
    _fields_ = [("hidden_size", u32), ("key_head_count", u32), ("value_head_count", u32),
                ("key_head_dimension", u32), ("value_head_dimension", u32), ("conv_kernel_size", u32),
                ("rms_norm_epsilon", f32), ("activation_dtype", C.c_int)]


class _RefQsaDims(C.Structure):
    _fields_ = [("hidden_size", u32), ("query_head_count", u32), ("key_value_head_count", u32),
                ("head_dimension", u32), ("index_query_head_count", u32), ("index_head_dimension", u32),
                ("block_size", u32), ("token_budget", u32), ("max_context", u32), ("rotary_dimension", u32),
                ("rms_norm_epsilon", f32), ("rope_theta", f32), ("activation_dtype", C.c_int)]


def _pairs(names):
    out = []
    for n in names:
        out += [(n, vp), (n + "_count", u64)]
    return out


class _RefGdnWeights(C.Structure):
    _fields_ = _pairs(GDN_FIELDS)


class _RefQsaWeights(C.Structure):
    _fields_ = _pairs(QSA_FIELDS)


class _Diag(C.Structure):
    _fields_ = [("status", C.c_int), ("message", C.c_char * 256)]


class _RefSelection(C.Structure):
    _fields_ = [("token_index", u64), ("absolute_position", u64), ("candidate_block_ids", C.POINTER(u32)),
                ("candidate_scores", C.POINTER(f32)), ("candidate_count", u64),
                ("selected_block_ids", C.POINTER(u32)), ("selected_block_count", u64),
                ("selected_token_positions", C.POINTER(u32)), ("selected_token_count", u64),
                ("tail_count", u64)]


_SEL_CB = C.CFUNCTYPE(None, C.POINTER(_RefSelection), vp)
_port = None
_ref = None


def build() -> None:
    """Builds the restatement, and the reference when its sources are present."""
    subprocess.run(["make", "-s", "-C", str(HERE), "port"], check=True)
    if Path("/root/reference/src/kq_gdn.c").exists():
        subprocess.run(["make", "-s", "-C", str(HERE), "ref"], check=True)


def port():
    global _port
    if _port is None:
        if not PORT_LIB.exists():
            build()
        _port = C.CDLL(str(PORT_LIB))
    return _port


def ref_available() -> bool:
    return REF_LIB.exists()


def ref():
    global _ref
    if _ref is None:
        if not REF_LIB.exists():
            raise RuntimeError("reference oracle not built (make -C oracle ref)")
        _ref = C.CDLL(str(REF_LIB))
    return _ref


def _a(x) -> np.ndarray:
    return np.ascontiguousarray(x, dtype=np.float32)


# ------------------------------------------------------------------ numerics

def dequantize(type_id: int, packed: np.ndarray, impl: str = "port") -> np.ndarray:
    be, bb = GEOMETRY[type_id]
    data = np.ascontiguousarray(packed, np.uint8)
    n = data.size // bb * be
    out = np.empty(n, np.float32)
    if impl == "port":
        st = port().kqo_dequantize(u32(type_id), data.ctypes.data_as(vp), u64(data.size),
                                   out.ctypes.data_as(vp), u64(n))
    else:
        cnt = u64()
        d = _Diag()
        st = ref().kq_dequantize_blocks_f32(u32(type_id), data.ctypes.data_as(vp), u64(data.size),
                                            out.ctypes.data_as(vp), u64(n), C.byref(cnt), C.byref(d))
    if st != 0:
        raise RuntimeError(f"oracle dequantize failed: {st}")
    return out


def matvec(type_id: int, packed: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
    """y[b, r] in the reference's sequential row-dot order."""
    xv = _a(x).reshape(-1, cols)
    y = np.empty((xv.shape[0], rows), np.float32)
    data = np.ascontiguousarray(packed, np.uint8)
    st = port().kqo_matvec(u32(type_id), data.ctypes.data_as(vp), u64(rows), u64(cols),
                           xv.ctypes.data_as(vp), u64(xv.shape[0]), y.ctypes.data_as(vp))
    if st != 0:
        raise RuntimeError(f"oracle matvec failed: {st}")
    return y


def row_dot_ref(type_id: int, packed: np.ndarray, x: np.ndarray) -> float:
    data = np.ascontiguousarray(packed, np.uint8)
    xv = _a(x)
    out = f32()
    d = _Diag()
    st = ref().kq_quantized_row_dot_f32(u32(type_id), data.ctypes.data_as(vp), u64(data.size),
                                        xv.ctypes.data_as(vp), u64(xv.size), C.byref(out), C.byref(d))
    if st != 0:
        raise RuntimeError(f"reference row dot failed: {st} {d.message}")
    return out.value


# ------------------------------------------------------------------ GDN

def gdn_run(dims, w: dict, x: np.ndarray, conv: np.ndarray, rec: np.ndarray, mask=None, impl: str = "port"):
    """Runs T tokens; returns (status, y[T,H], conv', rec')."""
    xv = _a(x).reshape(-1, dims.hidden)
    T = xv.shape[0]
    y = np.zeros((T, dims.hidden), np.float32)
    conv2, rec2 = _a(conv).copy(), _a(rec).copy()
    ws = {k: _a(w[k]) for k in GDN_FIELDS}
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    if impl == "port":
        gd = _GdnDims(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim,
                      dims.conv_kernel, dims.eps)
        gw = _GdnWeights(*[ws[k].ctypes.data for k in GDN_FIELDS])
        st = port().kqo_gdn_run(C.byref(gd), C.byref(gw), xv.ctypes.data_as(vp), u64(T),
                                None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp),
                                conv2.ctypes.data_as(vp), rec2.ctypes.data_as(vp))
        return st, y, conv2, rec2
    L = ref()
    gd = _RefGdnDims(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim,
                     dims.conv_kernel, dims.eps, 0)
    cfg, state = vp(), vp()
    d = _Diag()
    if L.kq_gdn_test_config_create(C.byref(gd), C.byref(cfg), C.byref(d)) != 0:
        raise RuntimeError(d.message)
    try:
        if L.kq_gdn_state_create(cfg, C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        init = 0 if (not conv2.any() and not rec2.any()) else 1
        st = L.kq_gdn_state_import_f32(state, conv2.ctypes.data_as(vp), u64(conv2.size), rec2.ctypes.data_as(vp),
                                       u64(rec2.size), C.c_int(init), C.byref(d))
        if st != 0:
            raise RuntimeError(d.message)
        L.kq_gdn_config_scratch_bytes.restype = u64
        sb = L.kq_gdn_config_scratch_bytes(cfg)
        scratch = np.empty(sb // 4 + 1, np.float32)
        gw = _RefGdnWeights()
        for k in GDN_FIELDS:
            setattr(gw, k, ws[k].ctypes.data)
            setattr(gw, k + "_count", ws[k].size)
        st = L.kq_gdn_prefill_f32(cfg, C.byref(gw), xv.ctypes.data_as(vp), u64(T),
                                  None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp), u64(y.size),
                                  state, scratch.ctypes.data_as(vp), u64(sb), None, None, C.byref(d))
        init_out = C.c_int()
        L.kq_gdn_state_export_f32(state, conv2.ctypes.data_as(vp), u64(conv2.size), rec2.ctypes.data_as(vp),
                                  u64(rec2.size), C.byref(init_out), C.byref(d))
        return st, y, conv2, rec2
    finally:
        if state:
            L.kq_gdn_state_close(state)
        L.kq_gdn_config_close(cfg)


# ------------------------------------------------------------------ QSA

def qsa_run(dims, w: dict, x: np.ndarray, key: np.ndarray, value: np.ndarray, raw: np.ndarray, length: int,
            capacity: int, impl: str = "port"):
    """Runs T tokens on caches holding `length` prior rows.

    Returns (status, y[T,H], key', value', raw', new_length, selections) with
    one selection dict per token (scores, selected block ids)."""
    xv = _a(x).reshape(-1, dims.hidden)
    T = xv.shape[0]
    y = np.zeros((T, dims.hidden), np.float32)
    kc = np.zeros((capacity, dims.kv_width), np.float32)
    vc = np.zeros((capacity, dims.kv_width), np.float32)
    rc = np.zeros((capacity, dims.index_dim), np.float32)
    kc[:length], vc[:length], rc[:length] = key[:length], value[:length], raw[:length]
    ws = {k: _a(w[k]) for k in QSA_FIELDS}
    topk = dims.budget // dims.block
    max_blocks = capacity // dims.block
    sels = []
    if impl == "port":
        qd = _QsaDims(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads, dims.index_dim,
                      dims.block, dims.budget, dims.rotary, dims.eps, dims.theta)
        qw = _QsaWeights(*[ws[k].ctypes.data for k in QSA_FIELDS])
        ln = u64(length)
        sel = np.zeros((T, topk), np.uint32)
        cnt = np.zeros(T, np.uint32)
        scores = np.zeros((T, max(1, max_blocks)), np.float32)
        st = port().kqo_qsa_run(C.byref(qd), C.byref(qw), xv.ctypes.data_as(vp), u64(T), y.ctypes.data_as(vp),
                                kc.ctypes.data_as(vp), vc.ctypes.data_as(vp), rc.ctypes.data_as(vp), u64(capacity),
                                C.byref(ln), sel.ctypes.data_as(vp), cnt.ctypes.data_as(vp),
                                scores.ctypes.data_as(vp))
        for t in range(T):
            nb = (length + t + 1) // dims.block
            sels.append({"scores": scores[t, :nb].copy(), "selected": sel[t, :cnt[t]].copy()})
        n = ln.value
        return st, y, kc[:n], vc[:n], rc[:n], n, sels
    L = ref()
    qd = _RefQsaDims(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads, dims.index_dim,
                     dims.block, dims.budget, max(capacity, dims.max_context if dims.max_context else capacity),
                     dims.rotary, dims.eps, dims.theta, 0)
    cfg, state = vp(), vp()
    d = _Diag()
    if L.kq_qsa_test_config_create(C.byref(qd), C.byref(cfg), C.byref(d)) != 0:
        raise RuntimeError(d.message)
    try:
        if L.kq_qsa_state_create(cfg, u64(capacity), C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        st = L.kq_qsa_state_import_f32(state, kc.ctypes.data_as(vp), u64(length * dims.kv_width),
                                       vc.ctypes.data_as(vp), u64(length * dims.kv_width), rc.ctypes.data_as(vp),
                                       u64(length * dims.index_dim), u64(length), C.byref(d))
        if st != 0:
            raise RuntimeError(d.message)
        need = u64()
        L.kq_qsa_required_scratch_bytes(cfg, state, u64(T), C.byref(need), C.byref(d))
        scratch = np.empty(need.value // 4 + 1, np.float32)
        qw = _RefQsaWeights()
        for k in QSA_FIELDS:
            setattr(qw, k, ws[k].ctypes.data)
            setattr(qw, k + "_count", ws[k].size)

        def on_sel(p, _u):
            s = p.contents
            nb = s.candidate_count
            sels.append({"scores": np.ctypeslib.as_array(s.candidate_scores, (nb,)).copy() if nb else
                         np.zeros(0, np.float32),
                         "selected": np.ctypeslib.as_array(s.selected_block_ids, (s.selected_block_count,)).copy()
                         if s.selected_block_count else np.zeros(0, np.uint32)})

        cb = _SEL_CB(on_sel)
        st = L.kq_qsa_prefill_f32(cfg, C.byref(qw), xv.ctypes.data_as(vp), u64(T), y.ctypes.data_as(vp),
                                  u64(y.size), state, scratch.ctypes.data_as(vp), need, cb, None, None, C.byref(d))
        ln = u64()
        L.kq_qsa_state_length.restype = u64
        n = L.kq_qsa_state_length(state)
        k2 = np.zeros((max(n, 1), dims.kv_width), np.float32)
        v2 = np.zeros_like(k2)
        r2 = np.zeros((max(n, 1), dims.index_dim), np.float32)
        L.kq_qsa_state_export_f32(state, k2.ctypes.data_as(vp), u64(k2.size), v2.ctypes.data_as(vp), u64(v2.size),
                                  r2.ctypes.data_as(vp), u64(r2.size), C.byref(ln), C.byref(d))
        return st, y, k2[:n], v2[:n], r2[:n], n, sels
    finally:
        if state:
            L.kq_qsa_state_close(state)
        L.kq_qsa_config_close(cfg)


def select_blocks(scores: np.ndarray, limit: int) -> np.ndarray:
    s = _a(scores)
    out = np.zeros(max(1, limit), np.uint32)
    port().kqo_select_blocks.restype = u64
    n = port().kqo_select_blocks(s.ctypes.data_as(vp), u64(s.size), u64(limit), out.ctypes.data_as(vp))
    return out[:n]


# ------------------------------------------------------------------ helpers

def gdn_weights_f32(layer) -> dict:
    """Canonical F32 weights of a synth.GdnLayerWeights (dequantised here)."""
    def dq(t):
        return dequantize(t.type_id, t.data).reshape(t.rows, t.cols)
    return {"a_log": layer.a_log, "conv": layer.conv, "dt_bias": layer.dt_bias, "alpha": dq(layer.alpha),
            "beta": dq(layer.beta), "qkv": dq(layer.qkv), "gate": dq(layer.gate), "norm": layer.norm,
            "output": dq(layer.output)}


def qsa_weights_f32(layer) -> dict:
    def dq(t):
        return dequantize(t.type_id, t.data).reshape(t.rows, t.cols)
    return {"query": dq(layer.query), "key": dq(layer.key), "value": dq(layer.value), "output": dq(layer.output),
            "query_norm": layer.query_norm, "key_norm": layer.key_norm, "index_query": dq(layer.index_query),
            "index_key": dq(layer.index_key), "index_query_norm": layer.index_query_norm,
            "index_key_norm": layer.index_key_norm}


# ------------------------------------------------------------------ checkpoints

_PORT_CB = C.CFUNCTYPE(None, u32, u64, u32, C.POINTER(u64), C.POINTER(f32), u64, vp)


class _RefGdnCheckpoint(C.Structure):   # include/kq_gdn.h:46-53
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 4),
                ("values", C.POINTER(f32)), ("value_count", u64)]


class _RefQsaCheckpoint(C.Structure):   # include/kq_qsa.h:38-45
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 3),
                ("values", C.POINTER(f32)), ("value_count", u64)]


_REF_GDN_CB = C.CFUNCTYPE(None, C.POINTER(_RefGdnCheckpoint), vp)
_REF_QSA_CB = C.CFUNCTYPE(None, C.POINTER(_RefQsaCheckpoint), vp)


def _record(out, kind, token, rank, dims, values, count):
    vals = np.ctypeslib.as_array(values, (count,)).copy() if count else np.zeros(0, np.float32)
    out.append({"kind": int(kind), "token": int(token), "rank": int(rank),
                "dims": tuple(int(dims[i]) for i in range(rank)), "values": vals})


def gdn_checkpoints(dims, w: dict, x: np.ndarray, conv: np.ndarray, rec: np.ndarray, mask=None,
                    impl: str = "port"):
    """Every checkpoint of a GDN run, in emission order: a list of dicts
    (kind, token, rank, dims, values).  impl "port": the restatement's
    kqo_gdn_run_observed; "reference": the reference's kq_gdn_prefill_f32 with
    a checkpoint observer.  Returns (status, checkpoints)."""
    xv = _a(x).reshape(-1, dims.hidden)
    T = xv.shape[0]
    y = np.zeros((T, dims.hidden), np.float32)
    conv2, rec2 = _a(conv).copy(), _a(rec).copy()
    ws = {k: _a(w[k]) for k in GDN_FIELDS}
    m = None if mask is None else np.ascontiguousarray(mask, np.uint8)
    out = []
    if impl == "port":
        cb = _PORT_CB(lambda kind, tok, rank, dp, vals, n, _u: _record(out, kind, tok, rank, dp, vals, n))
        gd = _GdnDims(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim,
                      dims.conv_kernel, dims.eps)
        gw = _GdnWeights(*[ws[k].ctypes.data for k in GDN_FIELDS])
        st = port().kqo_gdn_run_observed(C.byref(gd), C.byref(gw), xv.ctypes.data_as(vp), u64(T),
                                         None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp),
                                         conv2.ctypes.data_as(vp), rec2.ctypes.data_as(vp), cb, None)
        return st, out
    L = ref()
    cb = _REF_GDN_CB(lambda p, _u: _record(out, p.contents.kind, p.contents.token_index, p.contents.rank,
                                           p.contents.dimensions, p.contents.values, p.contents.value_count))
    gd = _RefGdnDims(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim,
                     dims.conv_kernel, dims.eps, 0)
    cfg, state = vp(), vp()
    d = _Diag()
    if L.kq_gdn_test_config_create(C.byref(gd), C.byref(cfg), C.byref(d)) != 0:
        raise RuntimeError(d.message)
    try:
        if L.kq_gdn_state_create(cfg, C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        init = 0 if (not conv2.any() and not rec2.any()) else 1
        if L.kq_gdn_state_import_f32(state, conv2.ctypes.data_as(vp), u64(conv2.size), rec2.ctypes.data_as(vp),
                                     u64(rec2.size), C.c_int(init), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        L.kq_gdn_config_scratch_bytes.restype = u64
        sb = L.kq_gdn_config_scratch_bytes(cfg)
        scratch = np.empty(sb // 4 + 1, np.float32)
        gw = _RefGdnWeights()
        for k in GDN_FIELDS:
            setattr(gw, k, ws[k].ctypes.data)
            setattr(gw, k + "_count", ws[k].size)
        st = L.kq_gdn_prefill_f32(cfg, C.byref(gw), xv.ctypes.data_as(vp), u64(T),
                                  None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp), u64(y.size),
                                  state, scratch.ctypes.data_as(vp), u64(sb), cb, None, C.byref(d))
        return st, out
    finally:
        if state:
            L.kq_gdn_state_close(state)
        L.kq_gdn_config_close(cfg)


def qsa_checkpoints(dims, w: dict, x: np.ndarray, key: np.ndarray, value: np.ndarray, raw: np.ndarray,
                    length: int, capacity: int, impl: str = "port"):
    """Every checkpoint of a QSA run over caches holding `length` prior rows,
    in emission order (see gdn_checkpoints).  Returns (status, checkpoints)."""
    xv = _a(x).reshape(-1, dims.hidden)
    T = xv.shape[0]
    y = np.zeros((T, dims.hidden), np.float32)
    kc = np.zeros((capacity, dims.kv_width), np.float32)
    vc = np.zeros((capacity, dims.kv_width), np.float32)
    rc = np.zeros((capacity, dims.index_dim), np.float32)
    kc[:length], vc[:length], rc[:length] = key[:length], value[:length], raw[:length]
    ws = {k: _a(w[k]) for k in QSA_FIELDS}
    out = []
    if impl == "port":
        cb = _PORT_CB(lambda kind, tok, rank, dp, vals, n, _u: _record(out, kind, tok, rank, dp, vals, n))
        qd = _QsaDims(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads, dims.index_dim,
                      dims.block, dims.budget, dims.rotary, dims.eps, dims.theta)
        qw = _QsaWeights(*[ws[k].ctypes.data for k in QSA_FIELDS])
        ln = u64(length)
        st = port().kqo_qsa_run_observed(C.byref(qd), C.byref(qw), xv.ctypes.data_as(vp), u64(T),
                                         y.ctypes.data_as(vp), kc.ctypes.data_as(vp), vc.ctypes.data_as(vp),
                                         rc.ctypes.data_as(vp), u64(capacity), C.byref(ln), None, None, None, cb,
                                         None)
        return st, out
    L = ref()
    cb = _REF_QSA_CB(lambda p, _u: _record(out, p.contents.kind, p.contents.token_index, p.contents.rank,
                                           p.contents.dimensions, p.contents.values, p.contents.value_count))
    qd = _RefQsaDims(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads, dims.index_dim,
                     dims.block, dims.budget, max(capacity, dims.max_context if dims.max_context else capacity),
                     dims.rotary, dims.eps, dims.theta, 0)
    cfg, state = vp(), vp()
    d = _Diag()
    if L.kq_qsa_test_config_create(C.byref(qd), C.byref(cfg), C.byref(d)) != 0:
        raise RuntimeError(d.message)
    try:
        if L.kq_qsa_state_create(cfg, u64(capacity), C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        if L.kq_qsa_state_import_f32(state, kc.ctypes.data_as(vp), u64(length * dims.kv_width),
                                     vc.ctypes.data_as(vp), u64(length * dims.kv_width), rc.ctypes.data_as(vp),
                                     u64(length * dims.index_dim), u64(length), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        need = u64()
        L.kq_qsa_required_scratch_bytes(cfg, state, u64(T), C.byref(need), C.byref(d))
        scratch = np.empty(need.value // 4 + 1, np.float32)
        qw = _RefQsaWeights()
        for k in QSA_FIELDS:
            setattr(qw, k, ws[k].ctypes.data)
            setattr(qw, k + "_count", ws[k].size)
        st = L.kq_qsa_prefill_f32(cfg, C.byref(qw), xv.ctypes.data_as(vp), u64(T), y.ctypes.data_as(vp),
                                  u64(y.size), state, scratch.ctypes.data_as(vp), need, _SEL_CB(), cb, None,
                                  C.byref(d))
        return st, out
    finally:
        if state:
            L.kq_qsa_state_close(state)
        L.kq_qsa_config_close(cfg)


# ------------------------------------------------------------------ state descriptors

def gdn_state_roundtrip_ref(dims, dtype: int, conv: np.ndarray, rec: np.ndarray, x: np.ndarray, w: dict):
    """The reference (compiled kq_gdn.c) with activation dtype `dtype` (0 F32,
    1 BF16; src/kq_gdn.c:109-122,599-701): imports the state, exports it
    again, and tries one F32 execution (src/kq_gdn_qwen38.c:393-397).
    Returns (create status, exported conv, exported rec, execute status)."""
    L = ref()
    gd = _RefGdnDims(dims.hidden, dims.key_heads, dims.value_heads, dims.key_dim, dims.value_dim,
                     dims.conv_kernel, dims.eps, dtype)
    cfg, state = vp(), vp()
    d = _Diag()
    st = L.kq_gdn_test_config_create(C.byref(gd), C.byref(cfg), C.byref(d))
    if st != 0:
        return st, None, None, None
    try:
        if L.kq_gdn_state_create(cfg, C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        c, r = _a(conv).copy(), _a(rec).copy()
        if L.kq_gdn_state_import_f32(state, c.ctypes.data_as(vp), u64(c.size), r.ctypes.data_as(vp), u64(r.size),
                                     C.c_int(1), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        c2, r2 = np.zeros_like(c), np.zeros_like(r)
        init = C.c_int()
        L.kq_gdn_state_export_f32(state, c2.ctypes.data_as(vp), u64(c2.size), r2.ctypes.data_as(vp), u64(r2.size),
                                  C.byref(init), C.byref(d))
        L.kq_gdn_config_scratch_bytes.restype = u64
        sb = L.kq_gdn_config_scratch_bytes(cfg)
        scratch = np.empty(sb // 4 + 1, np.float32)
        gw = _RefGdnWeights()
        ws = {k: _a(w[k]) for k in GDN_FIELDS}
        for k in GDN_FIELDS:
            setattr(gw, k, ws[k].ctypes.data)
            setattr(gw, k + "_count", ws[k].size)
        xv = _a(x).reshape(-1, dims.hidden)
        y = np.zeros_like(xv)
        est = L.kq_gdn_prefill_f32(cfg, C.byref(gw), xv.ctypes.data_as(vp), u64(xv.shape[0]), None,
                                   y.ctypes.data_as(vp), u64(y.size), state, scratch.ctypes.data_as(vp), u64(sb),
                                   None, None, C.byref(d))
        return 0, c2, r2, est
    finally:
        if state:
            L.kq_gdn_state_close(state)
        L.kq_gdn_config_close(cfg)


def qsa_state_roundtrip_ref(dims, dtype: int, key: np.ndarray, value: np.ndarray, raw: np.ndarray, length: int,
                            capacity: int, x: np.ndarray | None = None, w: dict | None = None):
    """The reference (compiled kq_qsa.c) with activation dtype `dtype`
    (src/kq_qsa.c:80-93,513-620): imports `length` cache rows, exports them
    again and, given `x` and `w`, tries one F32 prefill of `x`.  Returns
    (create status, key, value, raw, exported length, execute status or
    None)."""
    L = ref()
    qd = _RefQsaDims(dims.hidden, dims.query_heads, dims.kv_heads, dims.head_dim, dims.index_heads, dims.index_dim,
                     dims.block, dims.budget, max(capacity, dims.max_context if dims.max_context else capacity),
                     dims.rotary, dims.eps, dims.theta, dtype)
    cfg, state = vp(), vp()
    d = _Diag()
    st = L.kq_qsa_test_config_create(C.byref(qd), C.byref(cfg), C.byref(d))
    if st != 0:
        return st, None, None, None, 0, None
    try:
        if L.kq_qsa_state_create(cfg, u64(capacity), C.byref(state), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        k, v, r = _a(key)[:length].copy(), _a(value)[:length].copy(), _a(raw)[:length].copy()
        if L.kq_qsa_state_import_f32(state, k.ctypes.data_as(vp), u64(k.size), v.ctypes.data_as(vp), u64(v.size),
                                     r.ctypes.data_as(vp), u64(r.size), u64(length), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        k2, v2, r2 = np.zeros_like(k), np.zeros_like(v), np.zeros_like(r)
        ln = u64()
        L.kq_qsa_state_export_f32(state, k2.ctypes.data_as(vp), u64(k2.size), v2.ctypes.data_as(vp), u64(v2.size),
                                  r2.ctypes.data_as(vp), u64(r2.size), C.byref(ln), C.byref(d))
        est = None
        if x is not None:
            xv = _a(x).reshape(-1, dims.hidden)
            T = xv.shape[0]
            need = u64()
            L.kq_qsa_required_scratch_bytes(cfg, state, u64(T), C.byref(need), C.byref(d))
            scratch = np.empty(need.value // 4 + 1, np.float32)
            ws = {k: _a(w[k]) for k in QSA_FIELDS}
            qw = _RefQsaWeights()
            for k in QSA_FIELDS:
                setattr(qw, k, ws[k].ctypes.data)
                setattr(qw, k + "_count", ws[k].size)
            y = np.zeros_like(xv)
            est = L.kq_qsa_prefill_f32(cfg, C.byref(qw), xv.ctypes.data_as(vp), u64(T), y.ctypes.data_as(vp),
                                       u64(y.size), state, scratch.ctypes.data_as(vp), need, None, None, None,
                                       C.byref(d))
        return 0, k2, v2, r2, ln.value, est
    finally:
        if state:
            L.kq_qsa_state_close(state)
        L.kq_qsa_config_close(cfg)


# ------------------------------------------------------------------ MoE

MOE_FIELDS = ["router", "routed_gate", "routed_up", "routed_down", "shared_gate", "shared_up", "shared_down",
              "shared_gate_weight"]


class _MoeDims(C.Structure):   # kqo_moe_dims
    _fields_ = [("hidden_size", u32), ("expert_count", u32), ("top_k", u32), ("routed_intermediate_size", u32),
                ("shared_intermediate_size", u32)]


class _MoeWeights(C.Structure):   # kqo_moe_weights
    _fields_ = [(n, vp) for n in MOE_FIELDS]


class _RefMoeDims(C.Structure):   # src/kq_moe_internal.h:10-17
    _fields_ = [("hidden_size", u32), ("expert_count", u32), ("top_k", u32), ("routed_intermediate_size", u32),
                ("shared_intermediate_size", u32), ("activation_dtype", C.c_int)]


class _RefMoeWeights(C.Structure):   # include/kq_moe.h:72-89
    _fields_ = _pairs(MOE_FIELDS)


class _RefMoeRoute(C.Structure):   # include/kq_moe.h:58-66
    _fields_ = [("token_index", u64), ("router_logits", C.POINTER(f32)), ("router_probabilities", C.POINTER(f32)),
                ("expert_count", u64), ("selected_expert_ids", C.POINTER(u32)),
                ("selected_weights", C.POINTER(f32)), ("selected_count", u32)]


class _RefMoeCheckpoint(C.Structure):   # include/kq_moe.h:43-52
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("expert_id", u32), ("top_k_position", u32),
                ("rank", u32), ("dimensions", u64 * 2), ("values", C.POINTER(f32)), ("value_count", u64)]


_REF_ROUTE_CB = C.CFUNCTYPE(None, C.POINTER(_RefMoeRoute), vp)
_REF_MOE_CB = C.CFUNCTYPE(None, C.POINTER(_RefMoeCheckpoint), vp)
_PORT_MOE_CB = C.CFUNCTYPE(None, u32, u64, u32, u32, u32, C.POINTER(u64), C.POINTER(f32), u64, vp)


def moe_weights_f32(layer) -> dict:
    """Canonical F32 arrays of a synth.MoeLayerWeights (quantized stacks
    dequantized with the oracle's bit-exact decoders)."""
    def deq(t):
        return dequantize(t.type_id, t.data).reshape(-1)
    return {"router": deq(layer.router), "routed_gate": deq(layer.gate), "routed_up": deq(layer.up),
            "routed_down": deq(layer.down), "shared_gate": deq(layer.shared_gate), "shared_up": deq(layer.shared_up),
            "shared_down": deq(layer.shared_down), "shared_gate_weight": _a(layer.shared_gate_weight).reshape(-1)}


def moe_run(dims, w: dict, x: np.ndarray, impl: str = "port", checkpoints: bool = False):
    """T tokens through the MoE operator.  Returns (status, y[T,H], route,
    checkpoints) with route = dict(logits [T,E], probabilities [T,E], ids
    [T,K] in top-k order, weights [T,K]) and checkpoints a list of (kind,
    token, expert, position, values) in emission order (empty unless asked)."""
    xv = _a(x).reshape(-1, dims.hidden)
    T, E, K = xv.shape[0], dims.experts, dims.top_k
    y = np.zeros((T, dims.hidden), np.float32)
    ws = {k: _a(w[k]).reshape(-1) for k in MOE_FIELDS}
    route = {"logits": np.zeros((T, E), np.float32), "probabilities": np.zeros((T, E), np.float32),
             "ids": np.zeros((T, K), np.uint32), "weights": np.zeros((T, K), np.float32)}
    cps = []
    if impl == "port":
        md = _MoeDims(dims.hidden, E, K, dims.routed, dims.shared)
        mw = _MoeWeights(*[ws[k].ctypes.data for k in MOE_FIELDS])

        def on_cp(kind, token, expert, position, rank, dp, values, count, _u):
            cps.append((int(kind), int(token), int(expert), int(position),
                        np.ctypeslib.as_array(values, (count,)).copy()))

        cb = _PORT_MOE_CB(on_cp) if checkpoints else _PORT_MOE_CB()
        st = port().kqo_moe_run_observed(C.byref(md), C.byref(mw), xv.ctypes.data_as(vp), u64(T),
                                         y.ctypes.data_as(vp), route["logits"].ctypes.data_as(vp),
                                         route["probabilities"].ctypes.data_as(vp), route["ids"].ctypes.data_as(vp),
                                         route["weights"].ctypes.data_as(vp), cb, None)
        return st, y, route, cps
    L = ref()
    qd = _RefMoeDims(dims.hidden, E, K, dims.routed, dims.shared, 0)
    cfg = vp()
    d = _Diag()
    if L.kq_moe_test_config_create(C.byref(qd), C.byref(cfg), C.byref(d)) != 0:
        raise RuntimeError(d.message)
    try:
        L.kq_moe_config_scratch_bytes.restype = u64
        sb = L.kq_moe_config_scratch_bytes(cfg)
        scratch = np.empty(sb // 4 + 1, np.float32)
        mw = _RefMoeWeights()
        for k in MOE_FIELDS:
            setattr(mw, k, ws[k].ctypes.data)
            setattr(mw, k + "_count", ws[k].size)

        def on_route(p, _u):
            r = p.contents
            t = r.token_index
            route["logits"][t] = np.ctypeslib.as_array(r.router_logits, (r.expert_count,))
            route["probabilities"][t] = np.ctypeslib.as_array(r.router_probabilities, (r.expert_count,))
            route["ids"][t] = np.ctypeslib.as_array(r.selected_expert_ids, (r.selected_count,))
            route["weights"][t] = np.ctypeslib.as_array(r.selected_weights, (r.selected_count,))

        def on_cp(p, _u):
            c = p.contents
            cps.append((int(c.kind), int(c.token_index), int(c.expert_id), int(c.top_k_position),
                        np.ctypeslib.as_array(c.values, (c.value_count,)).copy()))

        rcb = _REF_ROUTE_CB(on_route)
        ccb = _REF_MOE_CB(on_cp) if checkpoints else _REF_MOE_CB()
        st = L.kq_moe_execute_f32(cfg, C.byref(mw), xv.ctypes.data_as(vp), u64(T), y.ctypes.data_as(vp),
                                  u64(y.size), scratch.ctypes.data_as(vp), u64(sb), rcb, ccb, None, C.byref(d))
        return st, y, route, cps
    finally:
        L.kq_moe_config_close(cfg)


class RefMoe:
    """The reference's own MoE operators (oracle/_ref) on one test config:
    kq_moe_route_f32 and kq_moe_execute_routed_expert_f32 with F32 weights
    (src/kq_moe_qwen38.c:276-376,461-568).  Used as the CPU baseline of the
    MoE decode record: every selected expert and the shared expert run
    through the reference's expert operator."""

    def __init__(self, dims):
        L = ref()
        self.L, self.dims = L, dims
        self.cfg = vp()
        d = _Diag()
        qd = _RefMoeDims(dims.hidden, dims.experts, dims.top_k, dims.routed, dims.shared, 0)
        if L.kq_moe_test_config_create(C.byref(qd), C.byref(self.cfg), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        L.kq_moe_config_one_expert_workspace_bytes.restype = u64
        self.scratch = np.empty(L.kq_moe_config_one_expert_workspace_bytes(self.cfg) // 4 + 1, np.float32)
        self.out = np.empty(dims.hidden, np.float32)

    def route(self, router: np.ndarray, x: np.ndarray):
        E, K = self.dims.experts, self.dims.top_k
        lg, pr = np.empty(E, np.float32), np.empty(E, np.float32)
        ids, w = np.empty(K, np.uint32), np.empty(K, np.float32)
        d = _Diag()
        st = self.L.kq_moe_route_f32(self.cfg, router.ctypes.data_as(vp), u64(router.size), x.ctypes.data_as(vp),
                                     lg.ctypes.data_as(vp), u64(E), pr.ctypes.data_as(vp), u64(E),
                                     ids.ctypes.data_as(vp), u64(K), w.ctypes.data_as(vp), u64(K), C.byref(d))
        if st != 0:
            raise RuntimeError(d.message)
        return ids, w

    def expert(self, gate: np.ndarray, up: np.ndarray, down: np.ndarray, x: np.ndarray) -> np.ndarray:
        ew = (_RefExpertWeights)(gate.ctypes.data, gate.size, up.ctypes.data, up.size, down.ctypes.data, down.size)
        d = _Diag()
        st = self.L.kq_moe_execute_routed_expert_f32(self.cfg, C.byref(ew), u32(0), x.ctypes.data_as(vp),
                                                     self.out.ctypes.data_as(vp), u64(self.out.size),
                                                     self.scratch.ctypes.data_as(vp), u64(self.scratch.nbytes),
                                                     C.byref(d))
        if st != 0:
            raise RuntimeError(d.message)
        return self.out.copy()

    def close(self):
        self.L.kq_moe_config_close(self.cfg)


class _RefExpertWeights(C.Structure):   # include/kq_moe.h:91-98
    _fields_ = _pairs(["gate", "up", "down"])


# ------------------------------------------------------------------ layer

GR_FIELDS = ["norm", "down", "up", "inject"]


class _LayerDims(C.Structure):   # kqo_layer_dims
    _fields_ = [("hidden_size", u32), ("branch_count", u32), ("gr_rank", u32), ("rms_epsilon", f32),
                ("family", u32)]


class _GrWeights(C.Structure):   # kqo_gr_weights
    _fields_ = [(n, vp) for n in GR_FIELDS]


class _RefLayerDims(C.Structure):   # src/kq_layer_internal.h:10-17
    _fields_ = [("layer_id", u32), ("hidden_size", u32), ("branch_count", u32), ("gr_rank", u32),
                ("rms_epsilon", f32), ("family", C.c_int)]


class _RefGrWeights(C.Structure):   # include/kq_layer.h kq_layer_gr_weights_f32
    _fields_ = _pairs(GR_FIELDS)


class _RefLayerWeights(C.Structure):   # include/kq_layer.h kq_layer_weights_f32
    _fields_ = [("attention_gr", _RefGrWeights), ("moe_gr", _RefGrWeights), ("gdn", vp), ("qsa", vp), ("moe", vp),
                ("ple_value", vp), ("ple_provider", vp)]


class _RefLayerCheckpoint(C.Structure):   # include/kq_layer.h kq_layer_checkpoint
    _fields_ = [("kind", C.c_int), ("token_index", u64), ("rank", u32), ("dimensions", u64 * 3),
                ("values", C.POINTER(f32)), ("value_count", u64)]


_REF_LAYER_CB = C.CFUNCTYPE(None, C.POINTER(_RefLayerCheckpoint), vp)


def layer_sequence(impl: str, ld, gr: dict, mixer_dims, mixer_w: dict, moe_dims, moe_w: dict, blocks, masks=None,
                   capacity: int = 64, checkpoints: bool = False):
    """Runs the token blocks `blocks` ([T_i][B*H] each) one after another
    through one decoder layer from a zero state.  ld: (hidden, branches,
    rank, eps, family 1 GDN / 2 QSA); gr: {"attn": {norm, down, up, inject},
    "moe": {...}}.  Returns a list of (status, output, checkpoints)."""
    hidden, branches, rank, eps, family = ld
    gw = {side: {k: _a(gr[side][k]).reshape(-1) for k in GR_FIELDS} for side in ("attn", "moe")}
    mw = {k: _a(moe_w[k]).reshape(-1) for k in MOE_FIELDS}
    fields = GDN_FIELDS if family == 1 else QSA_FIELDS
    xw = {k: _a(mixer_w[k]).reshape(-1) for k in fields}
    out = []
    if impl == "port":
        ldm = _LayerDims(hidden, branches, rank, eps, family)
        grs = [_GrWeights(*[gw[s][k].ctypes.data for k in GR_FIELDS]) for s in ("attn", "moe")]
        md = _MoeDims(moe_dims.hidden, moe_dims.experts, moe_dims.top_k, moe_dims.routed, moe_dims.shared)
        mws = _MoeWeights(*[mw[k].ctypes.data for k in MOE_FIELDS])
        if family == 1:
            d = mixer_dims
            gd = _GdnDims(d.hidden, d.key_heads, d.value_heads, d.key_dim, d.value_dim, d.conv_kernel, d.eps)
            gws = _GdnWeights(*[xw[k].ctypes.data for k in GDN_FIELDS])
            conv = np.zeros(d.conv_channels * d.conv_kernel, np.float32)
            rec = np.zeros(d.value_heads * d.key_dim * d.value_dim, np.float32)
        else:
            d = mixer_dims
            qd = _QsaDims(d.hidden, d.query_heads, d.kv_heads, d.head_dim, d.index_heads, d.index_dim, d.block,
                          d.budget, d.rotary, d.eps, d.theta)
            qws = _QsaWeights(*[xw[k].ctypes.data for k in QSA_FIELDS])
            kc = np.zeros((capacity, d.kv_width), np.float32)
            vc = np.zeros((capacity, d.kv_width), np.float32)
            rc = np.zeros((capacity, d.index_dim), np.float32)
            length = u64(0)
        for bi, x in enumerate(blocks):
            xv = _a(x).reshape(-1, hidden * branches)
            y = np.zeros_like(xv)
            cps = []

            def on_cp(kind, token, rank_, dp, values, count, _u):
                cps.append((int(kind), int(token), int(rank_), tuple(int(dp[i]) for i in range(rank_)),
                            np.ctypeslib.as_array(values, (count,)).copy()))

            cb = _PORT_CB(on_cp) if checkpoints else _PORT_CB()
            m = None if masks is None or masks[bi] is None else np.ascontiguousarray(masks[bi], np.uint8)
            if family == 1:
                st = port().kqo_layer_run_observed(
                    C.byref(ldm), C.byref(grs[0]), C.byref(grs[1]), C.byref(gd), C.byref(gws),
                    conv.ctypes.data_as(vp), rec.ctypes.data_as(vp), None, None, None, None, None, u64(0), None,
                    C.byref(md), C.byref(mws), xv.ctypes.data_as(vp), u64(xv.shape[0]),
                    None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp), cb, None)
            else:
                st = port().kqo_layer_run_observed(
                    C.byref(ldm), C.byref(grs[0]), C.byref(grs[1]), None, None, None, None, C.byref(qd),
                    C.byref(qws), kc.ctypes.data_as(vp), vc.ctypes.data_as(vp), rc.ctypes.data_as(vp), u64(capacity),
                    C.byref(length), C.byref(md), C.byref(mws), xv.ctypes.data_as(vp), u64(xv.shape[0]), None,
                    y.ctypes.data_as(vp), cb, None)
            out.append((st, y, cps))
        return out
    L = ref()
    d0 = _Diag()
    sub = vp()
    if family == 1:
        d = mixer_dims
        g = _RefGdnDims(d.hidden, d.key_heads, d.value_heads, d.key_dim, d.value_dim, d.conv_kernel, d.eps, 0)
        if L.kq_gdn_test_config_create(C.byref(g), C.byref(sub), C.byref(d0)) != 0:
            raise RuntimeError(d0.message)
        sw = _RefGdnWeights()
    else:
        d = mixer_dims
        q = _RefQsaDims(d.hidden, d.query_heads, d.kv_heads, d.head_dim, d.index_heads, d.index_dim, d.block,
                        d.budget, capacity, d.rotary, d.eps, d.theta, 0)
        if L.kq_qsa_test_config_create(C.byref(q), C.byref(sub), C.byref(d0)) != 0:
            raise RuntimeError(d0.message)
        sw = _RefQsaWeights()
    for k in fields:
        setattr(sw, k, xw[k].ctypes.data)
        setattr(sw, k + "_count", xw[k].size)
    moe_cfg = vp()
    if L.kq_moe_test_config_create(C.byref(_RefMoeDims(moe_dims.hidden, moe_dims.experts, moe_dims.top_k,
                                                       moe_dims.routed, moe_dims.shared, 0)),
                                   C.byref(moe_cfg), C.byref(d0)) != 0:
        raise RuntimeError(d0.message)
    rmw = _RefMoeWeights()
    for k in MOE_FIELDS:
        setattr(rmw, k, mw[k].ctypes.data)
        setattr(rmw, k + "_count", mw[k].size)
    lcfg, state = vp(), vp()
    rd = _RefLayerDims(0 if family == 1 else 3, hidden, branches, rank, eps, family)
    st = L.kq_layer_test_config_create(C.byref(rd), sub if family == 1 else None, sub if family == 2 else None,
                                       moe_cfg, None, None, C.byref(lcfg), C.byref(d0))
    if st != 0:
        raise RuntimeError(f"layer config: {st} {d0.message}")
    lw = _RefLayerWeights()
    for side, dst in (("attn", lw.attention_gr), ("moe", lw.moe_gr)):
        for k in GR_FIELDS:
            setattr(dst, k, gw[side][k].ctypes.data)
            setattr(dst, k + "_count", gw[side][k].size)
    lw.gdn = C.cast(C.pointer(sw), vp) if family == 1 else None
    lw.qsa = C.cast(C.pointer(sw), vp) if family == 2 else None
    lw.moe = C.cast(C.pointer(rmw), vp)
    try:
        if L.kq_layer_state_create(lcfg, u64(capacity if family == 2 else 0), C.byref(state), C.byref(d0)) != 0:
            raise RuntimeError(d0.message)
        for bi, x in enumerate(blocks):
            xv = _a(x).reshape(-1, hidden * branches)
            T = xv.shape[0]
            y = np.zeros_like(xv)
            need = u64()
            L.kq_layer_required_scratch_bytes(lcfg, state, u64(T), C.byref(need), C.byref(d0))
            scratch = np.zeros(need.value // 4 + 1, np.float32)
            cps = []

            def on_cp(p, _u):
                c = p.contents
                cps.append((int(c.kind), int(c.token_index), int(c.rank),
                            tuple(int(c.dimensions[i]) for i in range(c.rank)),
                            np.ctypeslib.as_array(c.values, (c.value_count,)).copy()))

            cb = _REF_LAYER_CB(on_cp) if checkpoints else _REF_LAYER_CB()
            m = None if masks is None or masks[bi] is None else np.ascontiguousarray(masks[bi], np.uint8)
            st = L.kq_layer_prefill_f32(lcfg, C.byref(lw), xv.ctypes.data_as(vp), None, u64(T),
                                        None if m is None else m.ctypes.data_as(vp), y.ctypes.data_as(vp),
                                        u64(y.size), state, scratch.ctypes.data_as(vp), need, cb, None, None,
                                        C.byref(d0))
            out.append((st, y, cps))
        return out
    finally:
        if state:
            L.kq_layer_state_close(state)
        L.kq_layer_config_close(lcfg)
        L.kq_moe_config_close(moe_cfg)
        if family == 1:
            L.kq_gdn_config_close(sub)
        else:
            L.kq_qsa_config_close(sub)


class RefLayerGr:
    """The reference's gated-residual read and write
    (kq_layer_gr_read_f32 / kq_layer_gr_write_f32, src/kq_layer_qwen38.c:
    166-209) on a reference test layer config of the given geometry (GDN
    family; the sub-configs only carry the hidden size).  Used as part of the
    CPU baseline of the layer decode record."""

    def __init__(self, hidden: int, branches: int, rank: int, eps: float = 1e-6):
        L = ref()
        self.L, self.H, self.B, self.R = L, hidden, branches, rank
        d = _Diag()
        self.g, self.m, self.cfg = vp(), vp(), vp()
        if L.kq_gdn_test_config_create(C.byref(_RefGdnDims(hidden, 1, 1, 4, 4, 4, 1e-6, 0)), C.byref(self.g),
                                       C.byref(d)) != 0:
            raise RuntimeError(d.message)
        if L.kq_moe_test_config_create(C.byref(_RefMoeDims(hidden, 1, 1, 1, 1, 0)), C.byref(self.m), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        if L.kq_layer_test_config_create(C.byref(_RefLayerDims(0, hidden, branches, rank, eps, 1)), self.g, None,
                                         self.m, None, None, C.byref(self.cfg), C.byref(d)) != 0:
            raise RuntimeError(d.message)
        W = hidden * branches
        self.nm, self.rg = np.empty(W, np.float32), np.empty(W, np.float32)
        self.rank = np.empty(rank, np.float32)
        L.kq_layer_gr_write_f32.restype = None

    def read(self, w: dict, branches: np.ndarray):
        """(mixed [H], write gate [B]) of one token's branches [B*H]."""
        gw = _RefGrWeights()
        ws = {k: _a(w[k]).reshape(-1) for k in GR_FIELDS}
        for k in GR_FIELDS:
            setattr(gw, k, ws[k].ctypes.data)
            setattr(gw, k + "_count", ws[k].size)
        x = _a(branches).reshape(-1)
        mixed, wg = np.empty(self.H, np.float32), np.empty(self.B, np.float32)
        d = _Diag()
        st = self.L.kq_layer_gr_read_f32(self.cfg, C.byref(gw), x.ctypes.data_as(vp), self.nm.ctypes.data_as(vp),
                                         self.rg.ctypes.data_as(vp), mixed.ctypes.data_as(vp),
                                         self.rank.ctypes.data_as(vp), wg.ctypes.data_as(vp), C.byref(d))
        if st != 0:
            raise RuntimeError(d.message)
        return mixed, wg

    def write(self, branches: np.ndarray, block: np.ndarray, wg: np.ndarray) -> np.ndarray:
        x, b, g = _a(branches).reshape(-1), _a(block).reshape(-1), _a(wg).reshape(-1)
        out = np.empty_like(x)
        self.L.kq_layer_gr_write_f32(self.cfg, x.ctypes.data_as(vp), b.ctypes.data_as(vp), g.ctypes.data_as(vp),
                                     out.ctypes.data_as(vp))
        return out

    def close(self):
        self.L.kq_layer_config_close(self.cfg)
        self.L.kq_moe_config_close(self.m)
        self.L.kq_gdn_config_close(self.g)
