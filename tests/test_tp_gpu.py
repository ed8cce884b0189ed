"""Tensor parallelism through the library's NCCL C ABI (include/qmm_tp.h).

One GPU: a one-rank communicator (real NCCL) runs the column- and row-parallel
forwards, which must equal the single-GPU Linear bit for bit; a stream wait
that runs past its limit returns QMM_ERR_TIMEOUT and aborts the communicator;
an init whose peer never joins returns QMM_ERR_TIMEOUT (host bootstrap only:
no kernel runs).

Two GPUs (skipped with fewer): the column-parallel, row-parallel and
Megatron-paired feed-forward and the sharded Gemma-3 decode step against the
oracle's single-process result
(column-parallel Q8_0-activation outputs bit-exact; f32 outputs and sums within
the 1e-3 contract), first with NCCL joins, then again with joins over peer
memory (qmm_tp_enable_peer: band GEMV and f16 GEMM epilogues writing every
rank's buffer, the copy kernel for the rest, a sharded decode step replayed
from a captured graph); a peer join whose peer never signals returns
QMM_ERR_TIMEOUT after its 2 s limit; then a rank that leaves between steps:
the other learns it on the host (StepGuard) before launching its next
collective and returns QMM_ERR_TIMEOUT. NVLS is off in these tests.
"""
from __future__ import annotations

import ctypes
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

Q4_0, Q8_0 = 2, 8
OK, ERR_NCCL, ERR_TIMEOUT = 0, 6, 7
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _weights(oracle, dt, n, k, seed):
    wf = np.random.default_rng(seed).normal(0, 0.02, n * k).astype(np.float32)
    return oracle.quantize_q8_0(wf) if dt == Q8_0 else oracle.quantize_q4_0(wf)


def test_world1_comm_matches_linear(oracle, qlib):
    from machinelearning_b200.linear import Linear, QuantWeight
    from machinelearning_b200.tp import ColumnParallelLinear, RowParallelLinear, TpComm

    torch.cuda.set_device(0)
    comm = TpComm.init(TpComm.unique_id(), 1, 0, 0, timeout_s=60.0)
    try:
        for dt, m, k, n in [(Q4_0, 1, 1152, 6912), (Q8_0, 8, 1024, 1152), (Q4_0, 32, 4096, 512)]:
            w = _weights(oracle, dt, n, k, seed=k + n)
            x = torch.from_numpy(np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float32)).cuda()
            ref = Linear(QuantWeight.from_host(dt, n, k, w, 0))(x)
            col, row = ColumnParallelLinear(dt, n, k, w, 0, comm), RowParallelLinear(dt, n, k, w, 0, comm)
            yc, yr = col(x), row(x)
            assert comm.wait(30.0) == OK
            assert torch.equal(yc, ref) and torch.equal(yr, ref)
            ya = comm.all_reduce(yc.clone())
            assert comm.wait(30.0) == OK and torch.equal(ya, ref)
        assert comm.status() == OK
    finally:
        assert comm.close() == OK


def test_world1_wait_limit_aborts(qlib):
    from machinelearning_b200.tp import TpComm

    torch.cuda.set_device(0)
    comm = TpComm.init(TpComm.unique_id(), 1, 0, 0, timeout_s=60.0)
    torch.cuda._sleep(int(1.5e9))  # a bounded spin (~1 s) the wait's limit cuts short
    rc = comm.wait(0.05)
    assert rc == ERR_TIMEOUT, rc
    assert b"aborted" in qlib.qmm_last_error_message()
    assert comm.status() == ERR_NCCL  # an aborted communicator refuses further work
    torch.cuda.synchronize()
    assert comm.close() == OK


_MISSING_PEER = r"""
import sys, time
sys.path.insert(0, ROOT)
import torch
from machinelearning_b200 import _lib
from machinelearning_b200.tp import TpComm
torch.cuda.set_device(0)
t0 = time.monotonic()
try:
    TpComm.init(TpComm.unique_id(), 2, 0, 0, timeout_s=2.0)
    print("RESULT ok")
except _lib.QmmError as e:
    print(f"RESULT {e.status} {time.monotonic() - t0:.2f}")
"""


def test_init_with_missing_peer_times_out():
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    p = subprocess.run([sys.executable, "-c", f"ROOT = {ROOT!r}\n" + _MISSING_PEER], env=env, capture_output=True,
                       text=True, timeout=180)
    assert p.returncode == 0, p.stderr[-3000:]
    line = [ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1].split()
    assert int(line[1]) == ERR_TIMEOUT and 2.0 <= float(line[2]) < 60.0, line


def _worker(rank: int, world: int, port: int):
    import datetime

    import torch.distributed as dist

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import oracle
    from conftest import assert_close_rel
    from machinelearning_b200._lib import GELU
    from machinelearning_b200.tp import (ColumnParallelLinear, ParallelFeedForward, RowParallelLinear, StepGuard,
                                         TpComm, default_store)

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    comm = TpComm.from_group(rank, timeout_s=60.0)
    oracle.build()
    _parity_pass(comm, rank, oracle, assert_close_rel, GELU)
    # the same joins over peer memory: band GEMV (M = 1, 16384 x 8192) and
    # f16 GEMM (M = 32) epilogues store into every rank's buffer over NVLink,
    # the other kernels' results are pushed by a copy kernel; one flag-barrier
    # kernel per call. Column results stay bit-identical to one GPU.
    comm.enable_peer(64 << 20)
    _parity_pass(comm, rank, oracle, assert_close_rel, GELU,
                 extra=[(Q4_0, 1, 8192, 16384), (Q8_0, 1, 4096, 8192), (Q4_0, 32, 8192, 2048), (Q8_0, 32, 4096, 4096)])
    # a join whose peer never signals: rank 0 runs a row-parallel forward that
    # rank 1 skips (a dropped message); rank 0's bounded wait runs out and the
    # next wait returns QMM_ERR_TIMEOUT. Rank 1 stays alive until rank 0's
    # kernels are done (the gloo barrier), so no write reaches freed memory.
    short = TpComm.from_group(rank, timeout_s=60.0)
    short.enable_peer(1 << 20, join_timeout_s=2.0)
    w = _weights(oracle, Q8_0, 256, 1024, seed=5)
    row = RowParallelLinear(Q8_0, 256, 1024, w, rank, short)
    xs = torch.ones(1, 512, device="cuda")
    if rank == 0:
        row.forward_local(xs)
        rc = short.wait(30.0)
        assert rc == ERR_TIMEOUT, rc
    torch.cuda.synchronize()
    dist.barrier()
    short.abort()
    short.close()
    _leave_test(comm, rank, world, StepGuard, default_store)


def _parity_pass(comm, rank, oracle, assert_close_rel, GELU, extra=()):
    from machinelearning_b200.tp import ColumnParallelLinear, ParallelFeedForward, RowParallelLinear

    for dt, m, k, n in [(Q4_0, 1, 1152, 6912), (Q8_0, 8, 6912, 1152), (Q4_0, 32, 8192, 512), *extra]:
        w = _weights(oracle, dt, n, k, seed=k + n + m)
        x = np.random.default_rng(m).normal(0, 1, (m, k)).astype(np.float32)
        xd = torch.from_numpy(x).cuda()
        f32 = oracle.matmul_f32_q8 if dt == Q8_0 else oracle.matmul_f32_q4
        native = oracle.matmul_f32_q8_v2 if dt == Q8_0 else oracle.matmul_f32_q4_native
        ref, ref_native = f32(x.ravel(), w, m, k, n), native(x.ravel(), w, m, k, n)
        col = ColumnParallelLinear(dt, n, k, w, rank, comm)
        yc = col(xd)
        assert comm.wait(60.0) == OK
        assert_close_rel(yc.cpu().numpy().ravel(), ref, 1e-3, 4e-3 if 17 <= m <= 32 else None)
        col.local.set_native_q4_matmul(True)
        col.local.set_native_q8_matmul(True)
        yn = col(xd)
        assert comm.wait(60.0) == OK
        assert np.array_equal(yn.cpu().numpy().ravel().view(np.uint32), ref_native.view(np.uint32))
        row = RowParallelLinear(dt, n, k, w, rank, comm)
        yr = row(xd)
        assert comm.wait(60.0) == OK
        assert_close_rel(yr.cpu().numpy().ravel(), ref, 1e-3, 4e-3 if 17 <= m <= 32 else None)
    # Megatron pairing: gelu(x gate^T) * (x up^T) -> down, one all-reduce
    dim, hidden, m = 1024, 2048, 4
    gw, uw = _weights(oracle, Q4_0, hidden, dim, 11), _weights(oracle, Q4_0, hidden, dim, 12)
    dw = _weights(oracle, Q4_0, dim, hidden, 13)
    x = np.random.default_rng(14).normal(0, 1, (m, dim)).astype(np.float32)
    ffn = ParallelFeedForward(Q4_0, dim, hidden, gw, uw, dw, rank, comm, GELU)
    y = ffn(torch.from_numpy(x).cuda())
    assert comm.wait(60.0) == OK
    g = oracle.matmul_f32_q4(x.ravel(), gw, m, dim, hidden).reshape(m, hidden)
    u = oracle.matmul_f32_q4(x.ravel(), uw, m, dim, hidden).reshape(m, hidden)
    h = (oracle.gelu(g.ravel()).reshape(m, hidden) * u).astype(np.float32)
    assert_close_rel(y.cpu().numpy().ravel(), oracle.matmul_f32_q4(h.ravel(), dw, m, hidden, dim), 1e-3)
    # the sharded Gemma-3 decode step (FFN Megatron-paired, lm_head by
    # vocabulary rows) against the oracle's pass, batch 1 and 3, 3 positions
    from oracle.decode import decode_step
    from test_decode_gpu import host_weights, small_config

    from machinelearning_b200.decode import Gemma3Decoder
    cfg = small_config(256)
    hw = host_weights(oracle, cfg, seed=21)
    for B in (1, 3):
        dec = Gemma3Decoder(cfg, hw, batch=B, device=rank, comm=comm)
        kc = [np.zeros((B, cfg.n_kv_heads, cfg.ctx, cfg.head_dim), np.float32) for _ in range(cfg.n_layers)]
        vc = [np.zeros_like(kc[0]) for _ in range(cfg.n_layers)]
        rng = np.random.default_rng(31 + B)  # the same token ids on both ranks
        dec.set_position(0)
        for pos in range(3):
            if pos == 1 and comm.peer_bytes:
                dec.capture()  # joins over peer memory: later steps replay one graph
                assert dec.graph is not None
            tokens = rng.integers(0, cfg.vocab, B)
            got = dec.step(tokens)
            dec.wait(60.0)
            ref = decode_step(cfg, hw, tokens, pos, kc, vc)
            assert_close_rel(got.cpu().numpy().ravel(), ref.ravel(), 1e-3)
        dec.close()


def _leave_test(comm, rank, world, StepGuard, default_store):
    # rank 1 leaves between steps; rank 0 learns it on the host, launches nothing
    guard = StepGuard(default_store(), rank, world, timeout_s=3.0, prefix="tp_gpu_leave")
    buf = torch.ones(1024, device="cuda")
    codes = []
    for step in range(3):
        if rank == 1 and step == 2:
            break
        codes.append(guard.run(step, lambda: buf, lambda t: (comm.all_reduce(t), comm.wait(30.0))))
        if codes[-1]:
            break
    # no finalize handshake with a departed peer: both sides abort
    comm.abort()
    torch.cuda.synchronize()
    comm.close()
    if rank == 0:
        assert codes == [OK, OK, ERR_TIMEOUT], (codes, guard.last_error)
    else:
        assert codes == [OK, OK]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp_nccl_world2():
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    mp.spawn(_worker, args=(2, _free_port()), nprocs=2, join=True)
