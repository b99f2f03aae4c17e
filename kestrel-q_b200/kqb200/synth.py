"""Seeded synthetic GGUF weights and states for the BASELINE configurations.

No dataset or checkpoint is involved: every tensor is drawn from a numpy
generator with the shapes and distributions the benchmark configurations
name (GGUF Q8_0 / Q4_K / Q6_K blocks, N(0,1) activations, N(0,0.02)
recurrent state, ...).  Block layouts follow the public GGUF formats:

  Q8_0  34 B / 32 values : fp16 d, 32 x int8 code          value = code * d
  Q4_K 144 B / 256 values: fp16 d, fp16 dmin, 12 B packed 6-bit (scale, min)
                           pairs, 128 B of 4-bit codes      value = d*sc*q - dmin*m
  Q6_K 210 B / 256 values: 128 B low nibbles, 64 B high bit pairs,
                           16 x int8 scales, fp16 d         value = d*sc*(q - 32)
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

TYPE_F32, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_BF16 = 0, 8, 12, 14, 30
GEOMETRY = {TYPE_F32: (1, 4), TYPE_BF16: (1, 2), TYPE_Q8_0: (32, 34),
            TYPE_Q4_K: (256, 144), TYPE_Q6_K: (256, 210)}
TYPE_NAMES = {TYPE_F32: "F32", TYPE_BF16: "BF16", TYPE_Q8_0: "Q8_0", TYPE_Q4_K: "Q4_K", TYPE_Q6_K: "Q6_K"}


@dataclass
class QTensor:
    """rows x cols matrix stored as consecutive GGUF rows of `type_id` blocks."""
    type_id: int
    rows: int
    cols: int
    data: np.ndarray  # uint8, rows * row_bytes

    @property
    def row_bytes(self) -> int:
        be, bb = GEOMETRY[self.type_id]
        return self.cols // be * bb

    @property
    def nbytes(self) -> int:
        return int(self.data.size)


def _f16_bytes(values: np.ndarray) -> np.ndarray:
    return values.astype(np.float16).view(np.uint8).reshape(values.shape + (2,))


def pack_q8_0(rng: np.random.Generator, rows: int, cols: int,
              d_range=(0.001, 0.01)) -> QTensor:
    nb = cols // 32
    out = np.empty((rows, nb, 34), np.uint8)
    out[..., 0:2] = _f16_bytes(rng.uniform(*d_range, size=(rows, nb)))
    out[..., 2:] = rng.integers(-127, 128, size=(rows, nb, 32), dtype=np.int16).astype(np.int8).view(np.uint8)
    return QTensor(TYPE_Q8_0, rows, cols, out.reshape(-1))


def pack_q4_k(rng: np.random.Generator, rows: int, cols: int,
              d_range=(0.5e-4, 2.5e-4), dmin_range=(0.5e-3, 1.5e-3)) -> QTensor:
    nb = cols // 256
    out = np.empty((rows, nb, 144), np.uint8)
    out[..., 0:2] = _f16_bytes(rng.uniform(*d_range, size=(rows, nb)))
    out[..., 2:4] = _f16_bytes(rng.uniform(*dmin_range, size=(rows, nb)))
    out[..., 4:] = rng.integers(0, 256, size=(rows, nb, 140), dtype=np.uint8)
    return QTensor(TYPE_Q4_K, rows, cols, out.reshape(-1))


def pack_q6_k(rng: np.random.Generator, rows: int, cols: int,
              d_range=(1.0e-5, 2.5e-5)) -> QTensor:
    nb = cols // 256
    out = np.empty((rows, nb, 210), np.uint8)
    out[..., 0:192] = rng.integers(0, 256, size=(rows, nb, 192), dtype=np.uint8)
    out[..., 192:208] = rng.integers(-127, 128, size=(rows, nb, 16), dtype=np.int16).astype(np.int8).view(np.uint8)
    out[..., 208:210] = _f16_bytes(rng.uniform(*d_range, size=(rows, nb)))
    return QTensor(TYPE_Q6_K, rows, cols, out.reshape(-1))


def to_bf16_bits(values: np.ndarray) -> np.ndarray:
    bits = np.ascontiguousarray(values, np.float32).view(np.uint32).astype(np.uint64)
    rounded = (bits + 0x7FFF + ((bits >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def pack_bf16(rng: np.random.Generator, rows: int, cols: int, std=0.02) -> QTensor:
    vals = rng.normal(0.0, std, size=(rows, cols)).astype(np.float32)
    return QTensor(TYPE_BF16, rows, cols, to_bf16_bits(vals).view(np.uint8).reshape(-1))


def pack_f32(rng: np.random.Generator, rows: int, cols: int, std=0.02) -> QTensor:
    vals = rng.normal(0.0, std, size=(rows, cols)).astype(np.float32)
    return QTensor(TYPE_F32, rows, cols, vals.view(np.uint8).reshape(-1))


def f32_tensor(values: np.ndarray) -> QTensor:
    v = np.ascontiguousarray(values, np.float32)
    return QTensor(TYPE_F32, v.shape[0], v.shape[1], v.view(np.uint8).reshape(-1))


PACKERS = {TYPE_Q8_0: pack_q8_0, TYPE_Q4_K: pack_q4_k, TYPE_Q6_K: pack_q6_k,
           TYPE_BF16: pack_bf16, TYPE_F32: pack_f32}


def pack(type_id: int, rng: np.random.Generator, rows: int, cols: int) -> QTensor:
    return PACKERS[type_id](rng, rows, cols)


# ----------------------------------------------------------------- GDN

@dataclass
class GdnDims:
    hidden: int = 2048
    key_heads: int = 16
    value_heads: int = 32
    key_dim: int = 128
    value_dim: int = 128
    conv_kernel: int = 4
    eps: float = 1e-6

    @property
    def conv_channels(self) -> int:
        return 2 * self.key_heads * self.key_dim + self.value_heads * self.value_dim

    @property
    def value_width(self) -> int:
        return self.value_heads * self.value_dim


@dataclass
class GdnLayerWeights:
    dims: GdnDims
    qkv: QTensor
    gate: QTensor
    beta: QTensor
    alpha: QTensor
    output: QTensor
    a_log: np.ndarray
    conv: np.ndarray
    dt_bias: np.ndarray
    norm: np.ndarray


def gdn_layer(seed: int, dims: GdnDims, in_type: int = TYPE_Q8_0, out_type: int = TYPE_Q8_0,
              gate_type: int | None = None) -> GdnLayerWeights:
    """One GDN layer: qkv/z projections and out-proj in the given GGUF types,
    alpha/beta projections in `gate_type` (F32 = the reference target type),
    A_log ~ U(-1,1), dt_bias ~ N(0,0.1), conv taps ~ U(-0.5,0.5), norm ~ 1."""
    rng = np.random.default_rng(seed)
    H, C, Vd, Hv = dims.hidden, dims.conv_channels, dims.value_width, dims.value_heads
    gt = in_type if gate_type is None else gate_type
    return GdnLayerWeights(
        dims=dims,
        qkv=pack(in_type, rng, C, H),
        gate=pack(in_type, rng, Vd, H),
        beta=pack(gt, rng, Hv, H),
        alpha=pack(gt, rng, Hv, H),
        output=pack(out_type, rng, H, Vd),
        a_log=rng.uniform(-1.0, 1.0, Hv).astype(np.float32),
        conv=rng.uniform(-0.5, 0.5, C * dims.conv_kernel).astype(np.float32),
        dt_bias=rng.normal(0.0, 0.1, Hv).astype(np.float32),
        norm=(1.0 + rng.normal(0.0, 0.05, dims.value_dim)).astype(np.float32),
    )


def gdn_state(seed: int, dims: GdnDims, zero: bool = False):
    rng = np.random.default_rng(seed)
    C, K = dims.conv_channels, dims.conv_kernel
    n = dims.value_heads * dims.key_dim * dims.value_dim
    if zero:
        return np.zeros(C * K, np.float32), np.zeros(n, np.float32)
    return (rng.normal(0.0, 1.0, C * K).astype(np.float32),
            rng.normal(0.0, 0.02, n).astype(np.float32))


# ----------------------------------------------------------------- QSA

@dataclass
class QsaDims:
    hidden: int = 2048
    query_heads: int = 16
    kv_heads: int = 2
    head_dim: int = 256
    index_heads: int = 4
    index_dim: int = 128
    block: int = 4
    budget: int = 2048
    max_context: int = 262144
    rotary: int = 64
    eps: float = 1e-6
    theta: float = 1.0e7

    @property
    def q_width(self) -> int:
        return self.query_heads * self.head_dim

    @property
    def kv_width(self) -> int:
        return self.kv_heads * self.head_dim


@dataclass
class QsaLayerWeights:
    dims: QsaDims
    query: QTensor
    key: QTensor
    value: QTensor
    output: QTensor
    index_query: QTensor
    index_key: QTensor
    query_norm: np.ndarray
    key_norm: np.ndarray
    index_query_norm: np.ndarray
    index_key_norm: np.ndarray


def qsa_layer(seed: int, dims: QsaDims, proj_type: int = TYPE_Q4_K, out_type: int | None = None,
              index_type: int = TYPE_BF16) -> QsaLayerWeights:
    """One QSA layer: q(+gate)/k/v/o in `proj_type` (o in `out_type`), the
    index projections in `index_type` (BF16 = the reference target type),
    (1+w)-form norm deltas ~ N(0, 0.1)."""
    rng = np.random.default_rng(seed)
    H = dims.hidden
    ot = proj_type if out_type is None else out_type
    return QsaLayerWeights(
        dims=dims,
        query=pack(proj_type, rng, 2 * dims.q_width, H),
        key=pack(proj_type, rng, dims.kv_width, H),
        value=pack(proj_type, rng, dims.kv_width, H),
        output=pack(ot, rng, H, dims.q_width),
        index_query=pack(index_type, rng, dims.index_heads * dims.index_dim, H),
        index_key=pack(index_type, rng, dims.index_dim, H),
        query_norm=rng.normal(0.0, 0.1, dims.head_dim).astype(np.float32),
        key_norm=rng.normal(0.0, 0.1, dims.head_dim).astype(np.float32),
        index_query_norm=rng.normal(0.0, 0.1, dims.index_dim).astype(np.float32),
        index_key_norm=rng.normal(0.0, 0.1, dims.index_dim).astype(np.float32),
    )


def qsa_cache(seed: int, dims: QsaDims, length: int):
    """K / V / raw-index-key cache rows ~ N(0,1) for `length` prior tokens."""
    rng = np.random.default_rng(seed)
    k = rng.normal(0.0, 1.0, (length, dims.kv_width)).astype(np.float32)
    v = rng.normal(0.0, 1.0, (length, dims.kv_width)).astype(np.float32)
    r = rng.normal(0.0, 1.0, (length, dims.index_dim)).astype(np.float32)
    return k, v, r


# ----------------------------------------------------------------- MoE

@dataclass
class MoeDims:
    """Routed experts + gated shared expert (target: 512 experts, top-10,
    hidden 2560, routed / shared intermediate 640)."""
    hidden: int = 2560
    experts: int = 512
    top_k: int = 10
    routed: int = 640
    shared: int = 640


@dataclass
class MoeLayerWeights:
    dims: MoeDims
    router: QTensor              # [E][H] F32
    gate: QTensor                # [E*I][H] expert stack (expert-major rows)
    up: QTensor                  # [E*I][H]
    down: QTensor                # [E*H][I]
    shared_gate: QTensor         # [S][H]
    shared_up: QTensor           # [S][H]
    shared_down: QTensor         # [H][S]
    shared_gate_weight: np.ndarray  # [H] F32


def moe_layer(seed: int, dims: MoeDims, gate_up_type: int = TYPE_Q4_K, down_type: int = TYPE_Q8_0,
              shared_type: int = TYPE_Q8_0) -> MoeLayerWeights:
    """One MoE layer in the target's GGUF types (gate/up Q4_K, down Q8_0,
    shared Q8_0, router and shared gate F32 ~ N(0, 0.02)).  Q8_0 scales are
    drawn so that decoded values stay within +-0.05 (std ~0.015), the scale of
    trained FFN weights; with N(0,1) inputs the SwiGLU activations stay O(10)."""
    rng = np.random.default_rng(seed)
    E, H, I, S = dims.experts, dims.hidden, dims.routed, dims.shared

    def small(t, rows, cols):
        return pack_q8_0(rng, rows, cols, d_range=(1e-4, 4e-4)) if t == TYPE_Q8_0 else pack(t, rng, rows, cols)
    return MoeLayerWeights(
        dims=dims,
        router=pack_f32(rng, E, H),
        gate=pack(gate_up_type, rng, E * I, H),
        up=pack(gate_up_type, rng, E * I, H),
        down=small(down_type, E * H, I),
        shared_gate=small(shared_type, S, H),
        shared_up=small(shared_type, S, H),
        shared_down=small(shared_type, H, S),
        shared_gate_weight=rng.normal(0.0, 0.02, H).astype(np.float32),
    )


# ----------------------------------------------------------------- layer

@dataclass
class GrWeights:
    """One gated residual over B branches of width H (W = B*H)."""
    norm: np.ndarray    # [W] F32, (1 + w) form
    down: QTensor       # [rank][W]
    up: QTensor         # [W][rank]
    inject: QTensor     # [B][W]


def gr_weights(seed: int, hidden: int, branches: int, rank: int, type_id: int = TYPE_BF16) -> GrWeights:
    """Gated-residual tensors: norm deltas ~ N(0, 0.05), projections
    ~ N(0, 0.02) in `type_id`."""
    rng = np.random.default_rng(seed)
    W = hidden * branches
    return GrWeights(norm=rng.normal(0.0, 0.05, W).astype(np.float32), down=pack(type_id, rng, rank, W),
                     up=pack(type_id, rng, W, rank), inject=pack(type_id, rng, branches, W))


def hidden(seed: int, rows: int, width: int) -> np.ndarray:
    return np.random.default_rng(seed).normal(0.0, 1.0, (rows, width)).astype(np.float32)
