"""Failure handling of the tensor-parallel path, on the host (no GPU).

1. The C ABI's communicator control (include/qmm_tp.h) against a stand-in
   NCCL (tests/fake_nccl/fake_nccl.c, built here with gcc and loaded through
   QMM_NCCL_LIBRARY in a fresh process): an init that never completes or fails
   returns QMM_ERR_TIMEOUT / QMM_ERR_NCCL within its limit and aborts the
   communicator; a peer error reported by NCCL aborts it and turns every
   later call into QMM_ERR_NCCL; a collective that never completes times out.
2. StepGuard (machinelearning_b200/tp.py) on world-2 gloo ranks: a rank that
   raises, a rank that leaves between steps, and a rank that drops its part of
   a collective. The surviving rank returns a status code instead of hanging.
"""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
FAKE_SRC = os.path.join(ROOT, "tests", "fake_nccl", "fake_nccl.c")
OK, ERR_NCCL, ERR_TIMEOUT, ERR_INVALID_INPUT, ERR_CUDA = 0, 6, 7, 8, 5


@pytest.fixture(scope="module")
def fake_nccl(tmp_path_factory):
    out = str(tmp_path_factory.mktemp("fake_nccl") / "libfake_nccl.so")
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", "-o", out, FAKE_SRC], check=True)
    return out


_SCENARIOS = r"""
import ctypes, json, sys, time
sys.path.insert(0, ROOT)
fake = ctypes.CDLL(FAKE)            # the same object the library will dlopen
from machinelearning_b200 import _lib
L = _lib.lib()
res = {"available": L.qmm_tp_available()}
uid = (ctypes.c_uint8 * 128)()
res["uid"] = L.qmm_tp_unique_id(uid)
cnt = lambda name: ctypes.c_int.in_dll(fake, name).value
def init(mode, timeout):
    fake.fake_nccl_set_mode(mode)
    h = ctypes.c_void_p()
    t0 = time.monotonic()
    rc = L.qmm_tp_init(uid, 2, 0, -1, timeout, ctypes.byref(h))
    return rc, time.monotonic() - t0, h
rc, dt, h = init(1, 0.3)
res["hang"] = [rc, dt, cnt("fake_nccl_aborts"), h.value, L.qmm_last_error_message().decode()]
rc, dt, h = init(2, 5.0)
res["init_error"] = [rc, dt, cnt("fake_nccl_aborts"), h.value]
res["bad_rank"] = L.qmm_tp_init(uid, 2, 2, -1, 1.0, ctypes.byref(ctypes.c_void_p()))
res["bad_timeout"] = L.qmm_tp_init(uid, 2, 0, -1, 0.0, ctypes.byref(ctypes.c_void_p()))
# a healthy communicator, then a peer error after its first collective
rc, dt, h = init(3, 5.0)
buf = ctypes.create_string_buffer(64)
res["remote"] = [rc, L.qmm_tp_status(h), L.qmm_tp_all_reduce_f32(h, buf, 4, None), L.qmm_tp_status(h),
                 cnt("fake_nccl_aborts"), L.qmm_tp_all_reduce_f32(h, buf, 4, None), L.qmm_tp_destroy(h),
                 cnt("fake_nccl_destroys")]
# a collective that never completes: the communicator's own limit
fake.fake_nccl_set_mode(4)
h = ctypes.c_void_p()
rc = L.qmm_tp_init(uid, 2, 0, -1, 0.3, ctypes.byref(h))
t0 = time.monotonic()
rc2 = L.qmm_tp_all_gather_f32(h, buf, buf, 4, None)
res["collective_hang"] = [rc, rc2, time.monotonic() - t0, cnt("fake_nccl_aborts"),
                          L.qmm_last_error_message().decode(), L.qmm_tp_status(h), L.qmm_tp_destroy(h)]
# healthy: finalize + destroy, explicit abort
rc, dt, h = init(0, 5.0)
r = ctypes.c_int(); w = ctypes.c_int()
res["healthy"] = [rc, L.qmm_tp_rank(h, ctypes.byref(r), ctypes.byref(w)), r.value, w.value,
                  L.qmm_tp_all_reduce_f32(h, buf, 0, None), L.qmm_tp_destroy(h), cnt("fake_nccl_finalizes"),
                  cnt("fake_nccl_destroys"), cnt("fake_nccl_aborts")]
rc, dt, h = init(0, 5.0)
res["abort"] = [rc, L.qmm_tp_abort(h), L.qmm_tp_status(h), L.qmm_tp_destroy(h), cnt("fake_nccl_aborts"),
                cnt("fake_nccl_destroys")]
# peer joins: argument checks, and a setup that cannot allocate (no GPU here)
# fails with a status and leaves the communicator usable for NCCL joins
rc, dt, h = init(0, 5.0)
res["peer"] = [L.qmm_tp_enable_peer(None, 1024, 0.0), L.qmm_tp_enable_peer(h, 0, 0.0),
               L.qmm_tp_enable_peer(h, 1 << 20, 0.0), L.qmm_tp_status(h),
               L.qmm_tp_all_reduce_f32(h, buf, 4, None), L.qmm_tp_destroy(h)]
res["null"] = [L.qmm_tp_status(None), L.qmm_tp_destroy(None), L.qmm_tp_abort(None)]
print("RESULT " + json.dumps(res))
"""


def test_communicator_control_with_stand_in_nccl(fake_nccl):
    env = dict(os.environ, QMM_NCCL_LIBRARY=fake_nccl)
    code = f"ROOT = {ROOT!r}\nFAKE = {fake_nccl!r}\n" + _SCENARIOS
    p = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stderr[-3000:]
    res = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith("RESULT ")][-1][7:])
    assert res["available"] == 1 and res["uid"] == OK
    rc, dt, aborts, handle, msg = res["hang"]
    assert rc == ERR_TIMEOUT and 0.3 <= dt < 5.0 and aborts == 1 and handle is None, res["hang"]
    assert "aborted" in msg
    rc, dt, aborts, handle = res["init_error"]
    assert rc == ERR_NCCL and aborts == 1 and handle is None and dt < 5.0, res["init_error"]
    assert res["bad_rank"] == ERR_INVALID_INPUT and res["bad_timeout"] == ERR_INVALID_INPUT
    # init ok, status ok, collective ok; then the peer error aborts; later calls refuse
    assert res["remote"] == [OK, OK, OK, ERR_NCCL, 1, ERR_NCCL, OK, 0], res["remote"]
    rc, rc2, dt, aborts, msg, st, d = res["collective_hang"]
    assert rc == OK and rc2 == ERR_TIMEOUT and 0.3 <= dt < 5.0 and aborts == 1, res["collective_hang"]
    assert st == ERR_NCCL and d == OK
    assert res["healthy"] == [OK, OK, 0, 2, OK, OK, 1, 1, 0], res["healthy"]
    assert res["abort"] == [OK, OK, ERR_NCCL, OK, 1, 0], res["abort"]
    assert res["null"] == [ERR_INVALID_INPUT, OK, ERR_INVALID_INPUT]
    assert res["peer"] == [ERR_INVALID_INPUT, ERR_INVALID_INPUT, ERR_CUDA, OK, OK, OK], res["peer"]


# ---- StepGuard on gloo ranks ---------------------------------------------------------------------

def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _guard_worker(rank: int, world: int, port: int, scenario: str, q):
    import datetime

    import torch
    import torch.distributed as dist

    from machinelearning_b200.tp import StepGuard

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    store = dist.distributed_c10d._get_default_store()
    # the guard's limit is above the collectives' (3 s): a rank waiting at a
    # step meets a peer's posted collective failure before its own limit
    guard = StepGuard(store, rank, world, timeout_s=6.0, prefix=f"t_{scenario}")
    codes = []
    t0 = time.monotonic()
    try:
        for step in range(4):
            def compute():
                if scenario == "raise" and rank == 1 and step == 2:
                    raise RuntimeError("injected failure in rank 1's compute")
                return torch.full((8,), float(rank + step))

            def join(t):
                if scenario == "drop" and rank == 1 and step == 2:
                    return  # this rank's message never goes out
                dist.all_reduce(t)
                assert float(t[0]) == sum(r + step for r in range(world))

            if scenario == "leave" and rank == 1 and step == 2:
                break  # leaves between steps: nothing in flight
            try:
                rc = guard.run(step, compute, join)
            except RuntimeError as e:
                codes.append(("raised", str(e)))
                break
            codes.append(rc)
            if rc:
                break
    finally:
        q.put((rank, codes, guard.last_error, time.monotonic() - t0))
        if scenario == "ok":
            dist.destroy_process_group()


def _run_guard(scenario: str):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_guard_worker, args=(r, 2, port, scenario, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, codes, err, dt = q.get(timeout=120)
        out[rank] = (codes, err, dt)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def test_step_guard_healthy():
    out = _run_guard("ok")
    assert out[0][0] == [OK] * 4 and out[1][0] == [OK] * 4


def test_step_guard_rank_raises():
    out = _run_guard("raise")
    assert out[1][0] == [OK, OK, ("raised", "injected failure in rank 1's compute")]
    # rank 0 learns of it on the host before launching step 2's collective
    assert out[0][0] == [OK, OK, ERR_NCCL], out[0]
    assert "rank 1" in out[0][1] and "injected failure" in out[0][1]
    assert out[0][2] < 30


def test_step_guard_rank_leaves_between_steps():
    out = _run_guard("leave")
    assert out[1][0] == [OK, OK]
    assert out[0][0] == [OK, OK, ERR_TIMEOUT], out[0]
    assert "[1]" in out[0][1]
    assert out[0][2] < 30


def test_step_guard_dropped_message():
    out = _run_guard("drop")
    # rank 0's collective times out (3 s process-group limit) and is returned as a code;
    # rank 1 then meets rank 0's posted failure at the next step
    assert out[0][0] == [OK, OK, ERR_TIMEOUT], out[0]
    assert out[1][0][:2] == [OK, OK] and out[1][0][-1] == ERR_NCCL, out[1]
    assert out[0][2] < 30 and out[1][2] < 30
