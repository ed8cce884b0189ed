"""The bounded-wait failure path on the GPU, in the allowed form: a wait on a
shared-memory barrier that nothing completes, with a short probe limit, gives
up, records a timeout in the device error word and returns; the host reads
QMM_ERR_TIMEOUT through qmm_device_status and the context stays usable. No
kernel here faults, traps or hangs (every wait of the library is bounded the
same way; the self-test only shortens the bound)."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ERR_TIMEOUT = 7


def test_bounded_wait_timeout_is_reported_and_cleared(qlib, oracle):
    import torch
    from conftest import assert_close_rel
    torch.cuda.init()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert qlib.qmm_device_status(0) == 0, qlib.qmm_last_error_message()
    assert qlib.qmm_selftest_bounded_wait(4096, st) == 0, qlib.qmm_last_error_message()
    rc = qlib.qmm_device_status(0)
    assert rc == ERR_TIMEOUT
    assert b"timed out" in qlib.qmm_last_error_message()
    # the word was cleared by the read, and the context still runs the hot path
    assert qlib.qmm_device_status(0) == 0
    m, k, n = 2, 1152, 1024
    rng = np.random.default_rng(3)
    w = oracle.quantize_q8_0(rng.normal(0, 0.02, n * k).astype(np.float32))
    x = rng.normal(0, 1, m * k).astype(np.float32)
    xd, wd = torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()
    yd = torch.empty(m * n, dtype=torch.float32, device="cuda")
    ws = torch.zeros(max(qlib.qmm_workspace_size(8, 0, m, n, k), 256), dtype=torch.uint8, device="cuda")
    assert qlib.qmm_matmul_dev(8, 0, xd.data_ptr(), wd.data_ptr(), wd.numel(), m, k, n, yd.data_ptr(),
                               ws.data_ptr(), ws.numel(), st) == 0
    torch.cuda.synchronize()
    assert_close_rel(yd.cpu().numpy(), oracle.matmul_f32_q8(x, w, m, k, n))
    assert qlib.qmm_device_status(0) == 0


def test_two_timeouts_in_a_row(qlib):
    import torch
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for _ in range(2):
        assert qlib.qmm_selftest_bounded_wait(1, st) == 0
        assert qlib.qmm_device_status(0) == ERR_TIMEOUT
    assert qlib.qmm_device_status(0) == 0
