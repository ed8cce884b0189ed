"""The allocation-free entry point, qmm_matmul_dev_noalloc.

Some callers cannot allocate device memory: a plugin whose host framework owns
the device memory pool (every byte it may touch is handed to it), or a serving
loop that cannot take the device-wide synchronisation a cudaMalloc implies.
For them the library offers one matmul entry point whose workspace is a fixed
device array inside libqmm.so. This test calls it through the C ABI and checks
its output against the oracle (the reference's CPU path restated): bit for bit
for the Q8_0-activation modes, within the 1e-3 contract for f32 activations.
Each case runs two calls in a row: the shared array keeps the previous call's
contents, so the second call checks that nothing stale (split-K partials,
tickets) leaks through. Every f32 case is chosen so that it plans onto a
kernel that really uses the scratch array (qmm_workspace_size > 0: the
streaming GEMV with K split, or the band GEMV with K split), not the resident
kernel, which needs none. The file sorts last so a run that stops at the first
failure has run everything else first.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import assert_close_rel

pytestmark = pytest.mark.gpu

Q4_0, Q8_0 = 2, 8
BB = {Q4_0: 18, Q8_0: 34}


def _noalloc(torch, qlib, dt, act, xd, wd, m, k, n):
    yd = torch.full((m * n,), float("nan"), dtype=torch.float32, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = qlib.qmm_matmul_dev_noalloc(dt, act, xd.data_ptr(), wd.data_ptr(), wd.numel(), m, k, n, yd.data_ptr(), st)
    assert rc == 0, qlib.qmm_last_error_message()
    torch.cuda.synchronize()
    return yd.cpu().numpy()


def _oracle(oracle, dt, act, x, w, m, k, n):
    if dt == Q8_0:
        fn = oracle.matmul_f32_q8_v2 if act else oracle.matmul_f32_q8
    else:
        fn = oracle.matmul_f32_q4_native if act else oracle.matmul_f32_q4
    return fn(x, w, m, k, n)


# (dtype, act, m, k, n, needs scratch):
#  * Q8_0 f32, M = 20, K = 1152 (1224-byte rows, not a 16-byte pitch): the
#    streaming GEMV (paired-row loader) with K split over warps -> x records,
#    side records, split-K partials and tickets in the scratch array;
#  * Q8_0 f32, M = 1, 8192 -> 16384 (142 MB, too large for the resident
#    kernel): the band GEMV with K split in two slices -> partials and tickets;
#  * Q4_0 f32, M = 24, 4096 -> 96: the streaming GEMV (more tokens than the
#    resident kernel takes), K split over warps;
#  * Q8_0 / Q4_0 with Q8_0 activations: the streaming GEMV's quantised
#    activation records (these must match the reference bit for bit).
CASES = [(Q8_0, 0, 20, 1152, 256, True), (Q8_0, 0, 1, 8192, 16384, True), (Q4_0, 0, 24, 4096, 96, True),
         (Q8_0, 1, 8, 1152, 1024, True), (Q4_0, 1, 1, 6912, 1152, True)]


@pytest.mark.parametrize("dt,act,m,k,n,scratch", CASES)
def test_noalloc_matches_oracle(qlib, oracle, dt, act, m, k, n, scratch):
    import torch
    if scratch:
        assert qlib.qmm_workspace_size(dt, act, m, n, k) > 0, "case no longer plans onto a kernel with scratch"
    rng = np.random.default_rng(m * 7 + k + n + act)
    wf = rng.normal(0.0, 0.02, n * k).astype(np.float32)
    w = oracle.quantize_q8_0(wf) if dt == Q8_0 else oracle.quantize_q4_0(wf)
    wd = torch.from_numpy(w).cuda()
    for call in range(2):  # two calls in a row through the shared array
        x = rng.normal(0.0, 1.0, m * k).astype(np.float32)
        got = _noalloc(torch, qlib, dt, act, torch.from_numpy(x).cuda(), wd, m, k, n)
        ref = _oracle(oracle, dt, act, x, w, m, k, n)
        if act:
            np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))
        else:
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
