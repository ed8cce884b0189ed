"""Tensor-parallel sharding and joins (machinelearning_b200/tp.py) on CPU:
world_size-2 gloo process groups, each rank computing its shard with the
oracle (the reference's CPU path restated), joined with the same collectives
the GPU path uses. Column-parallel results must be bit-identical to the
single-process result; row-parallel sums within f32 rounding."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from machinelearning_b200.tp import column_shard, join_columns, row_shard, x_row_slice

Q4_0, Q4_1, Q8_0 = 2, 3, 8
MATMUL = {(Q8_0, 0): "matmul_f32_q8", (Q8_0, 1): "matmul_f32_q8_v2", (Q4_0, 0): "matmul_f32_q4",
          (Q4_0, 1): "matmul_f32_q4_native", (Q4_1, 0): "matmul_f32_q4_1", (Q4_1, 1): "matmul_f32_q4_1_native"}
CASES = [(Q8_0, 0, 3, 256, 64), (Q8_0, 1, 3, 256, 64), (Q4_0, 0, 5, 512, 96), (Q4_0, 1, 2, 128, 32),
         (Q4_1, 0, 4, 256, 40), (Q4_1, 1, 1, 64, 8)]


def make_case(oracle, dt, m, k, n, seed):
    rng = np.random.default_rng(seed)
    wf = rng.normal(0, 0.02, n * k).astype(np.float32)
    w = {Q8_0: oracle.quantize_q8_0, Q4_0: oracle.quantize_q4_0, Q4_1: oracle.quantize_q4_1}[dt](wf)
    x = rng.normal(0, 1, (m, k)).astype(np.float32)
    return w, x


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import datetime

    import oracle

    oracle.build()
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        for ci, (dt, act, m, k, n) in enumerate(CASES):
            w, x = make_case(oracle, dt, m, k, n, seed=10 + ci)
            fn = getattr(oracle, MATMUL[(dt, act)])
            full = fn(x.ravel(), w, m, k, n).reshape(m, n)

            # column-parallel: this rank's output rows, all_gather, reorder
            nl = n // world
            y = torch.from_numpy(fn(x.ravel(), column_shard(w, n, k, dt, rank, world), m, k, nl).copy())
            parts = [torch.empty(m * nl) for _ in range(world)]
            dist.all_gather(parts, y.reshape(-1))
            yc = join_columns(torch.cat(parts), m, nl, world).numpy()
            np.testing.assert_array_equal(yc.view(np.uint32), full.view(np.uint32),
                                          err_msg=f"column-parallel case {ci} not bit-identical")

            # row-parallel: this rank's K blocks of every row and of x, all_reduce
            kl = k // world
            xs = np.ascontiguousarray(x_row_slice(x, k, rank, world))
            yr = torch.from_numpy(fn(xs.ravel(), row_shard(w, n, k, dt, rank, world), m, kl, n).copy())
            dist.all_reduce(yr)
            err = np.linalg.norm(yr.numpy().reshape(m, n) - full) / max(np.linalg.norm(full), 1e-30)
            assert err < 1e-5, f"row-parallel case {ci}: relative error {err}"
    finally:
        dist.destroy_process_group()


def test_tp_gloo_world2():
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)


def test_shard_helpers(oracle):
    dt, n, k = Q4_0, 8, 128
    w, x = make_case(oracle, dt, 2, k, n, seed=1)
    rb = (k // 32) * 18
    assert np.array_equal(column_shard(w, n, k, dt, 1, 2), w[4 * rb:8 * rb])
    r0, r1 = row_shard(w, n, k, dt, 0, 2), row_shard(w, n, k, dt, 1, 2)
    assert r0.size == r1.size == n * 2 * 18
    # re-interleaving the two block halves gives back every row
    both = np.concatenate([r0.reshape(n, 36), r1.reshape(n, 36)], axis=1).reshape(-1)
    assert np.array_equal(both, w)
    assert x_row_slice(x, k, 1, 2).shape == (2, 64)
    g = np.arange(2 * 3 * 4, dtype=np.float32)  # [world=2][m=3][nl=4]
    assert np.array_equal(join_columns(g, 3, 4, 2)[1], np.r_[g[4:8], g[16:20]])
    with pytest.raises(ValueError):
        column_shard(w, n, k, dt, 0, 3)
