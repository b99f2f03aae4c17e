"""Precision budget of the tensor-core QSA attention, on CPU.

For head_dim 256 the GPU attention (qsa_attend_tc_kernel in
kestrel-q_b200/csrc/kernels_qsa.cu) reads bf16 hi / lo copies of the K and
V cache rows, scales Q by log2(e) / sqrt(d) before splitting it, takes
every product as a_hi b_hi + a_hi b_lo + a_lo b_hi with F32 accumulation,
keeps a softmax reference point that is raised only when a logit exceeds it
by more than 12 (base-2 units), and splits the weights exp2(logit - m)
into bf16 pairs for the P V product.  The reference computes
softmax(q . k / sqrt(d)) v in F32 (src/kq_qsa_qwen38.c:716-773).  This
test restates the GPU arithmetic in numpy (rounding emulated bit by bit)
and checks it against the same attention in F64, within the tolerance of
the GPU parity tests (|a - b| <= 2e-3 + 1e-3 |b|), for diffuse and for
peaked attention over 2048 selected tokens.  It pins the design, not the
CUDA code; the GPU tests check the kernel against the oracle.
"""
import numpy as np
import pytest

HD, HEADS, TILE = 256, 8, 16
LOG2E = np.float32(1.4426950408889634)


def bf16(x):
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def split(x):
    x = np.asarray(x, np.float32)
    hi = bf16(x)
    return hi, bf16(x - hi)


def mm3(ah, al, bh, bl):
    f = np.float32
    return (ah @ bh).astype(f) + (ah @ bl).astype(f) + (al @ bh).astype(f)


def attention_split(q, k, v):
    """One (token, KV head): q [HEADS][HD], k, v [n][HD]."""
    f = np.float32
    qh, ql = split(q * (LOG2E / np.float32(np.sqrt(HD))))
    kh, kl = split(k)
    vh, vl = split(v)
    m = np.full(HEADS, -np.inf, f)
    l = np.zeros(HEADS, f)
    o = np.zeros((HEADS, HD), f)
    for t0 in range(0, len(k), TILE):
        sl = slice(t0, t0 + TILE)
        lg = mm3(kh[sl], kl[sl], qh.T, ql.T).T          # [HEADS][tile], base-2 units
        if (lg > (m + 12.0)[:, None]).any():
            m_new = np.maximum(m, lg.max(axis=1))
            corr = np.where(np.isinf(m), 0.0, np.exp2(m - m_new)).astype(f)
            l *= corr
            o *= corr[:, None]
            m = m_new
        p = np.exp2(lg - m[:, None]).astype(f)
        l += p.sum(axis=1)
        ph, pl = split(p)
        o += mm3(ph, pl, vh[sl], vl[sl])
    return o / l[:, None]


def attention_f64(q, k, v):
    s = (q.astype(np.float64) @ k.T.astype(np.float64)) / np.sqrt(HD)
    w = np.exp(s - s.max(axis=1, keepdims=True))
    return (w / w.sum(axis=1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("sharp", [1.0, 6.0])
def test_split_attention_within_tolerance(sharp):
    """sharp 1: RMS-normed q and k (logits of a few units, diffuse
    weights); sharp 6: logits of tens, a few tokens dominate, and the
    reference point is raised along the way."""
    rng = np.random.default_rng(11)
    n = 2048 + 3
    k = rng.normal(size=(n, HD)).astype(np.float32)
    v = rng.normal(size=(n, HD)).astype(np.float32)
    q = (sharp * rng.normal(size=(HEADS, HD))).astype(np.float32)
    q[:, :] += sharp * 0.5 * k[n // 3]          # one strongly matching key
    got = attention_split(q, k, v)
    want = attention_f64(q, k, v)
    excess = np.abs(got - want) - (2e-3 + 1e-3 * np.abs(want))
    assert excess.max() <= 0, excess.max()
