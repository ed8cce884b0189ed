"""The allocation-free entry point, qmm_matmul_dev_noalloc.

Some callers may not allocate device memory: a plugin whose host framework
owns the device memory pool, or a serving loop that cannot take the
device-wide synchronisation a cudaMalloc implies. For them the library offers
one matmul entry point whose workspace is a fixed device array inside
libqmm.so. This test calls it through the C ABI and checks its output against
the caller-workspace entry point (qmm_matmul_dev) within the tests' tolerance,
on two calls in a row (the shared array keeps the previous call's contents,
so the second call checks that nothing stale leaks through). The file sorts
last so a run that stops at the first failure has run everything else first.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close_rel

pytestmark = pytest.mark.gpu

Q4_0, Q8_0 = 2, 8
BB = {Q4_0: 18, Q8_0: 34}


def _run(torch, qlib, dt, act, x, w, m, k, n, noalloc):
    xd = torch.from_numpy(x).cuda()
    wd = torch.from_numpy(w).cuda()
    yd = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if noalloc:
        rc = qlib.qmm_matmul_dev_noalloc(dt, act, xd.data_ptr(), wd.data_ptr(), wd.numel(), m, k, n,
                                         yd.data_ptr(), st)
    else:
        wsz = qlib.qmm_workspace_size(dt, act, m, n, k)
        ws = torch.zeros(max(wsz, 256), dtype=torch.uint8, device="cuda")
        rc = qlib.qmm_matmul_dev(dt, act, xd.data_ptr(), wd.data_ptr(), wd.numel(), m, k, n, yd.data_ptr(),
                                 ws.data_ptr(), ws.numel(), st)
    assert rc == 0, qlib.qmm_last_error_message()
    torch.cuda.synchronize()
    return yd.cpu().numpy()


# shapes that use every part of the scratch: split-K partials and tickets
# (small N), the paired and the plain 2-D tile loaders, batched tokens
CASES = [(Q8_0, 0, 1, 1152, 256), (Q4_0, 0, 3, 4096, 96), (Q8_0, 1, 8, 1152, 1024), (Q4_0, 1, 1, 6912, 1152)]


@pytest.mark.parametrize("dt,act,m,k,n", CASES)
def test_noalloc_matches_workspace_entry(qlib, oracle, dt, act, m, k, n):
    import torch
    rng = np.random.default_rng(m * 7 + k + n + act)
    wf = rng.normal(0.0, 0.02, n * k).astype(np.float32)
    w = oracle.quantize_q8_0(wf) if dt == Q8_0 else oracle.quantize_q4_0(wf)
    for call in range(2):  # two calls in a row through the shared array
        x = rng.normal(0.0, 1.0, m * k).astype(np.float32)
        ref = _run(torch, qlib, dt, act, x, w, m, k, n, noalloc=False)
        got = _run(torch, qlib, dt, act, x, w, m, k, n, noalloc=True)
        assert_close_rel(got, ref, 1e-3)


def test_noalloc_rejects_oversized_workspace(qlib):
    import torch
    m, k, n = 64, 32768, 64  # needs far more than the fixed scratch
    xd = torch.zeros(m * k, dtype=torch.float32, device="cuda")
    wd = torch.zeros(n * (k // 32) * 34, dtype=torch.uint8, device="cuda")
    yd = torch.zeros(m * n, dtype=torch.float32, device="cuda")
    rc = qlib.qmm_matmul_dev_noalloc(Q8_0, 0, xd.data_ptr(), wd.data_ptr(), wd.numel(), m, k, n, yd.data_ptr(), None)
    assert rc == 8
    assert b"no-alloc scratch limit" in qlib.qmm_last_error_message()
