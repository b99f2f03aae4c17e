"""Precision budget of the chunked GDN prefill, on CPU.

The GPU prefill (kestrel-q_b200/csrc/kernels_gdn_chunk.cu) rewrites the
token-by-token delta rule of the reference (src/kq_gdn_qwen38.c:705-761:
S <- e^g S; delta = beta (v - S^T k); S <- S + k delta^T; o = S^T q) per
64-token chunk in the WY form and runs its products on the tensor cores
with F32 operands split into hi / lo parts: L = K K^T and P = Q K^T as TF32
pairs, delta = U - W S, O = e^G (Q S) + P delta and the state update as
bf16 pairs, each product taken as a_hi b_hi + a_hi b_lo + a_lo b_hi with
F32 accumulation.  This test restates that arithmetic in numpy (rounding
emulated bit by bit) and checks, over 16 chunks with weak and strong
decays, that it stays within the tolerance the GPU parity tests use
(|a - b| <= 2e-3 + 1e-3 |b|) of the token recurrence evaluated in F64.
It pins the design, not the CUDA code; the GPU tests check the kernels
against the oracle.
"""
import numpy as np
import pytest

C, D = 64, 128


def bf16(x):
    """Round-to-nearest-even to bf16, returned as float32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16) << 16
    return b.astype(np.uint32).view(np.float32)


def tf32(x):
    """Round to nearest (ties away) to TF32, returned as float32."""
    b = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    b = (b + 0x1000) & ~np.uint64(0x1FFF)
    return b.astype(np.uint32).view(np.float32)


def split(x, rnd):
    x = np.asarray(x, np.float32)
    hi = rnd(x)
    return hi, rnd(x - hi)


def mm3(a, b, rnd):
    """a @ b as the three-term split product, F32 accumulation."""
    ah, al = split(a, rnd)
    bh, bl = split(b, rnd)
    f = np.float32
    return (ah @ bh).astype(f) + (ah @ bl).astype(f) + (al @ bh).astype(f)


def pair(x):
    """Value stored as a bf16 hi / lo pair."""
    h, l = split(x, bf16)
    return h + l


def token_recurrence(q, k, v, beta, g, s0):
    s = s0.astype(np.float64).copy()
    out = np.zeros((len(q), D))
    for t in range(len(q)):
        s *= np.exp(g[t])
        delta = beta[t] * (v[t] - s.T @ k[t])
        s += np.outer(k[t], delta)
        out[t] = s.T @ q[t]
    return out, s


def chunked_split(q, k, v, beta, g, s0):
    f = np.float32
    s = s0.astype(f).copy()
    out = np.zeros((len(q), D), f)
    for c0 in range(0, len(q), C):
        qc, kc, vc = q[c0:c0 + C], k[c0:c0 + C], v[c0:c0 + C]
        bc, gc = beta[c0:c0 + C], g[c0:c0 + C]
        n = len(qc)
        G = np.cumsum(gc.astype(f)).astype(f)
        lower = np.tril(np.ones((n, n), bool), -1)
        # e^(G_i - G_j) only where j <= i (exponent <= 0), as the kernel does
        decay = np.exp(np.where(np.tril(np.ones((n, n), bool)), G[:, None] - G[None, :], 0)).astype(f)
        L = np.where(lower, mm3(kc, kc.T, tf32) * decay, 0).astype(f)
        P = pair(np.where(lower | np.eye(n, dtype=bool), mm3(qc, kc.T, tf32) * decay, 0))
        # forward substitution in F32, in place
        W = (np.exp(G)[:, None] * kc).astype(f)
        U = vc.astype(f).copy()
        for i in range(n):
            W[i] = bc[i] * (W[i] - L[i, :i] @ W[:i])
            U[i] = bc[i] * (U[i] - L[i, :i] @ U[:i])
        W = pair(W)
        delta = U - mm3(W, s, bf16)
        o = np.exp(G)[:, None] * mm3(pair(qc), s, bf16) + mm3(P, delta, bf16)
        dprime = np.exp(G[-1] - G)[:, None] * delta
        s = np.exp(G[-1]) * s + mm3(pair(kc).T, dprime, bf16)
        out[c0:c0 + n] = o
    return out, s


def within(a, b, atol=2e-3, rtol=1e-3):
    return np.abs(np.asarray(a, np.float64) - b) - (atol + rtol * np.abs(b))


@pytest.mark.parametrize("g_lo,g_hi", [(-0.05, -0.001), (-3.0, -0.5)])
def test_chunked_split_products_stay_within_tolerance(g_lo, g_hi):
    rng = np.random.default_rng(7)
    T = 16 * C + 37   # ragged last chunk
    unit = lambda x: x / np.linalg.norm(x, axis=1, keepdims=True)
    q = unit(rng.normal(size=(T, D))).astype(np.float32)
    k = unit(rng.normal(size=(T, D))).astype(np.float32)
    v = rng.normal(size=(T, D)).astype(np.float32)
    beta = rng.uniform(0.05, 0.95, T).astype(np.float32)
    g = rng.uniform(g_lo, g_hi, T).astype(np.float32)
    s0 = (0.1 * rng.normal(size=(D, D))).astype(np.float32)
    want_o, want_s = token_recurrence(q, k, v, beta, g, s0)
    got_o, got_s = chunked_split(q, k, v, beta, g, s0)
    assert within(got_o, want_o).max() <= 0, within(got_o, want_o).max()
    assert within(got_s, want_s).max() <= 0, within(got_s, want_s).max()
    # and far inside it: the worst output error is ~1e-5 on outputs of O(1)
    assert np.abs(got_o - want_o).max() < 1e-4


def test_split_product_error_bounds():
    """One three-term product of 128-term dots: the error against the
    exact dot, relative to sum |a_i b_i|, is ~2^-21 with TF32 pairs and
    ~2^-16 with bf16 pairs (bounds below with a factor 4 of slack)."""
    rng = np.random.default_rng(3)
    a = rng.normal(size=(64, D)).astype(np.float32)
    b = rng.normal(size=(D, 64)).astype(np.float32)
    exact = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)
    assert (np.abs(mm3(a, b, tf32) - exact) / scale).max() < 2.0 ** -19
    assert (np.abs(mm3(a, b, bf16) - exact) / scale).max() < 2.0 ** -14
