"""Allocation-free batched linear (kq_b200_provider_linear_batch_f32_static).

Collected last on purpose: it must give the allocating entry point's results
(and the CPU oracle's) both in a fresh process and after every other test has
run.  Each shape is called twice in a row, because the entry point's scratch
array keeps the previous call's contents.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3   # the parity tolerance of the other GPU tests
LIMIT_EXCEEDED = 14


def _close(a, b, what):
    a = np.asarray(a, np.float64).reshape(-1)
    b = np.asarray(b, np.float64).reshape(-1)
    bad = np.nonzero(np.abs(a - b) > ATOL + RTOL * np.abs(b))[0]
    assert bad.size == 0, f"{what}: {bad.size} values out of tolerance"


@pytest.mark.parametrize("type_id,rows,cols,batch", [(12, 520, 2048, 64), (14, 2048, 4096, 100), (8, 96, 512, 5)])
def test_static_linear_matches_allocating_entry(kq, oracle, type_id, rows, cols, batch):
    """Two calls in a row: each must equal the allocating entry point and the
    CPU oracle's row dots, batches above 8 must have run the tensor-core GEMM
    (check + activation tiles + GEMM = three launches; the CUDA-core
    fallback would be two), and a warmed-up call must leave the device's free
    memory unchanged."""
    import torch
    from kqb200 import synth
    rng = np.random.default_rng(rows * 7 + batch)
    q = synth.pack(type_id, rng, rows, cols)
    p = kq.Provider(0)
    lib = kq.lib()
    try:
        h = p.add_matrix("m", 11, q)
        for call in range(2):
            xn = rng.normal(size=(batch, cols)).astype(np.float32)
            x = torch.from_numpy(xn).cuda()
            y_ref = torch.full((batch, rows), float("nan"), device="cuda")
            y_static = torch.full((batch, rows), float("nan"), device="cuda")
            torch.cuda.synchronize()
            d = kq.abi.Diagnostic()
            st = lib.kq_b200_provider_linear_batch_f32(p.handle, h, rows, cols, x.data_ptr(), batch,
                                                       y_ref.data_ptr(), C.byref(d))
            assert st == 0, d.text()
            kq.synchronize()
            free0 = torch.cuda.mem_get_info()[0]
            n0 = lib.kq_b200_kernel_launch_count()
            st = lib.kq_b200_provider_linear_batch_f32_static(p.handle, h, rows, cols, x.data_ptr(), batch,
                                                              y_static.data_ptr(), None, C.byref(d))
            assert st == 0, d.text()
            launched = lib.kq_b200_kernel_launch_count() - n0
            free1 = torch.cuda.mem_get_info()[0]
            if batch > 8:
                assert launched == 3, f"tensor-core path did not run ({launched} launches)"
            if call == 1:
                assert free1 == free0, f"free device memory changed by {free0 - free1} bytes"
            ys = y_static.cpu().numpy()
            _close(ys, y_ref.cpu().numpy(), f"type {type_id} call {call} vs allocating entry")
            _close(ys, oracle.matvec(type_id, q.data, rows, cols, xn), f"type {type_id} call {call} vs oracle")
    finally:
        p.close()


def test_static_linear_rejects_oversize_batch(kq):
    import torch
    from kqb200 import synth
    rows, cols, batch = 64, 2048, 1024   # 16 x 32 tiles of 16 KiB = 8 MiB > 4 MiB
    q = synth.pack(12, np.random.default_rng(3), rows, cols)
    p = kq.Provider(0)
    try:
        h = p.add_matrix("m", 11, q)
        x = torch.zeros((batch, cols), device="cuda")
        y = torch.zeros((batch, rows), device="cuda")
        d = kq.abi.Diagnostic()
        st = kq.lib().kq_b200_provider_linear_batch_f32_static(p.handle, h, rows, cols, x.data_ptr(), batch,
                                                               y.data_ptr(), None, C.byref(d))
        assert st == LIMIT_EXCEEDED, d.text()
        assert "static scratch" in d.text()
    finally:
        p.close()
