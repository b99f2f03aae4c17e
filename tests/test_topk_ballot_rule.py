"""The MoE route kernel's top-k scan (moe_route_kernel, kernels_moe.cu) against
the reference's sequential rule (src/kq_moe_qwen38.c:211-245), on the CPU.

The reference keeps the first K experts, then lets expert i replace the
worst member (lowest probability, lowest id among equal probabilities) when
its probability is strictly greater.  The kernel tests 32 experts per warp
ballot against the current worst and inserts the hits one at a time in
index order, testing the rest of the chunk again against the new worst.
Both are restated here step for step; the selected sets (and the member
positions) must agree on inputs with many ties, where the order of
replacements decides which of the tied experts survive.
"""
import numpy as np


def sequential_rule(p, k):
    ids = list(range(k))

    def worst():
        w = 0
        for pos in range(1, k):
            c, cw = ids[pos], ids[w]
            if p[c] < p[cw] or (p[c] == p[cw] and c < cw):
                w = pos
        return w

    w = worst()
    for i in range(k, len(p)):
        if p[i] > p[ids[w]]:
            ids[w] = i
            w = worst()
    return ids


def ballot_rule(p, k):
    """Lane l < k holds member l; the worst is the lane minimising (value, id)."""
    e = len(p)
    my_id = [lane if lane < k else 0xFFFFFFFF for lane in range(32)]
    my_v = [float(p[lane]) if lane < k else np.inf for lane in range(32)]

    def find_worst():
        key, lane = min(((my_v[l], my_id[l]), l) for l in range(32))
        return lane, key[0]

    wpos, wv = find_worst()
    for base in range(k, e, 32):
        v = [float(p[base + l]) if base + l < e else -np.inf for l in range(32)]
        m = sum(1 << l for l in range(32) if v[l] > wv)
        while m:
            l = (m & -m).bit_length() - 1
            my_id[wpos], my_v[wpos] = base + l, v[l]
            wpos, wv = find_worst()
            m &= ~((2 << l) - 1) & 0xFFFFFFFF
            m &= sum(1 << j for j in range(32) if v[j] > wv)
    return my_id[:k]


def test_ballot_scan_equals_sequential_rule():
    rng = np.random.default_rng(0)
    for trial in range(1500):
        e = int(rng.integers(12, 600))
        k = int(rng.integers(1, min(32, e) + 1))
        if trial % 2:   # few distinct values: long runs of ties across chunks
            p = rng.integers(0, int(rng.integers(1, 20)), e).astype(np.float32)
        else:
            p = rng.random(e).astype(np.float32)
        assert ballot_rule(p, k) == sequential_rule(p, k), (trial, e, k)
