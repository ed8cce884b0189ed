"""Tensor parallelism over NCCL on 2 GPUs (skipped with fewer): the
column-parallel and row-parallel linears of machinelearning_b200/tp.py against
the oracle's single-process result. Column-parallel Q8_0-activation outputs
are bit-exact (each output keeps the reference's block order); f32-activation
outputs and row-parallel sums meet the 1e-3 contract."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

Q4_0, Q8_0 = 2, 8


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int):
    import datetime
    import sys

    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import oracle
    from conftest import assert_close_rel
    from machinelearning_b200.tp import ColumnParallelLinear, RowParallelLinear

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        oracle.build()
        for dt, m, k, n in [(Q4_0, 1, 1152, 6912), (Q8_0, 8, 6912, 1152), (Q4_0, 32, 8192, 512)]:
            rng = np.random.default_rng(k + n + m)
            wf = rng.normal(0, 0.02, n * k).astype(np.float32)
            w = oracle.quantize_q8_0(wf) if dt == Q8_0 else oracle.quantize_q4_0(wf)
            x = rng.normal(0, 1, (m, k)).astype(np.float32)
            xd = torch.from_numpy(x).cuda()
            f32 = oracle.matmul_f32_q8 if dt == Q8_0 else oracle.matmul_f32_q4
            native = oracle.matmul_f32_q8_v2 if dt == Q8_0 else oracle.matmul_f32_q4_native
            ref = f32(x.ravel(), w, m, k, n)
            ref_native = native(x.ravel(), w, m, k, n)

            col = ColumnParallelLinear(dt, n, k, w, rank)
            assert_close_rel(col(xd).cpu().numpy().ravel(), ref, 1e-3, 4e-3 if m >= 17 else None)
            col.local.set_native_q4_matmul(True)
            col.local.set_native_q8_matmul(True)
            yn = col(xd).cpu().numpy().ravel()
            assert np.array_equal(yn.view(np.uint32), ref_native.view(np.uint32)), "column-parallel native"

            row = RowParallelLinear(dt, n, k, w, rank)
            assert_close_rel(row(xd).cpu().numpy().ravel(), ref, 1e-3, 4e-3 if m >= 17 else None)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_nccl_world2():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
