"""Tensor parallelism for the quantised linear layers: one process per GPU,
joins over NCCL (NVLink / NVSwitch on a B200 box).

Every output of a quantised matmul is an independent dot product over whole
32-weight blocks (reference llmserve/llmmodel/kernel/main/src/core/quantize.rs:
458-484), so a projection shards without any repacking of its GGUF bytes:

* column-parallel (q / k / v / gate / up / lm_head): rank r holds output rows
  [r*N/W, (r+1)*N/W) -- one contiguous byte range of the weight -- and every
  rank sees all of x. The y shards are joined with all_gather (rank-major
  [W][M][N/W]) and reordered to [M][N]. Each output keeps its block order, so
  results are bit-identical to one GPU.
* row-parallel (o / down): rank r holds blocks [r*nb/W, (r+1)*nb/W) of every
  row -- a strided byte sub-range, copied once at load -- and the matching K
  slice of x. The partial [M][N] outputs are summed with all_reduce (the sum
  order changes, so results agree within the usual tolerance, not bitwise).
  Q8_0 activation blocks never straddle a shard (shards are whole blocks), so
  the Q8_0-activation modes quantise exactly the blocks one GPU would.

The shard/join helpers are plain numpy / torch (tested on CPU with gloo).
ColumnParallelLinear / RowParallelLinear call the library's tensor-parallel
C ABI (include/qmm_tp.h): the local GEMV/GEMM and the NCCL join are enqueued by
libqmm.so on the caller's current stream, over a non-blocking communicator
whose every wait has a host-side time limit (TpComm). StepGuard is the host
side of failure handling between steps: ranks agree through the
process-group store that every rank reached a step, a rank that fails tells
the others before they launch the step's collectives, and failures come back
as the library's status codes instead of hangs.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._lib import BLOCK_BYTES, ERR_NCCL, ERR_TIMEOUT, OK, QmmError
from .linear import Linear, QuantWeight, _stream_ptr

QK = 32


def _split(total: int, world: int, rank: int) -> tuple[int, int]:
    if total % world:
        raise ValueError(f"{total} does not split evenly over {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def column_shard(weight: np.ndarray, n: int, k: int, dtype: int, rank: int, world: int) -> np.ndarray:
    """Bytes of output rows [rank*n/world, (rank+1)*n/world): a contiguous range."""
    row_bytes = (k // QK) * BLOCK_BYTES[dtype]
    w = np.asarray(weight, dtype=np.uint8).reshape(-1)
    if w.size < n * row_bytes:
        raise ValueError("weight buffer shorter than n*k/32 blocks")
    r0, r1 = _split(n, world, rank)
    return w[r0 * row_bytes:r1 * row_bytes]


def row_shard(weight: np.ndarray, n: int, k: int, dtype: int, rank: int, world: int) -> np.ndarray:
    """Blocks [rank*nb/world, (rank+1)*nb/world) of every row, as a new [n][nb/world]
    block matrix (byte-for-byte blocks, rows re-strided)."""
    bb = BLOCK_BYTES[dtype]
    nb = k // QK
    w = np.asarray(weight, dtype=np.uint8).reshape(-1)[: n * nb * bb].reshape(n, nb * bb)
    b0, b1 = _split(nb, world, rank)
    return np.ascontiguousarray(w[:, b0 * bb:b1 * bb]).reshape(-1)


def x_row_slice(x, k: int, rank: int, world: int):
    """The K slice of x ([..., k]) that a row-parallel shard multiplies."""
    b0, b1 = _split(k // QK, world, rank)
    return x[..., b0 * QK:b1 * QK]


def join_columns(gathered, m: int, n_local: int, world: int):
    """Rank-major [world][m][n_local] (all_gather's layout) -> [m][world * n_local]."""
    g = gathered.reshape(world, m, n_local)
    if isinstance(g, torch.Tensor):
        return g.permute(1, 0, 2).reshape(m, world * n_local)
    return np.transpose(g, (1, 0, 2)).reshape(m, world * n_local)




# ---- native communicator (include/qmm_tp.h) -------------------------------------------------

class TpComm:
    """An NCCL communicator owned by libqmm.so (qmm_tp_init): non-blocking,
    every wait bounded by `timeout_s`; a failure aborts it and surfaces as
    QMM_ERR_NCCL / QMM_ERR_TIMEOUT."""

    def __init__(self, handle: int, rank: int, world: int, device: int, timeout_s: float):
        self._h = ctypes.c_void_p(handle)
        self.rank, self.world, self.device, self.timeout_s = rank, world, device, timeout_s
        self.peer_bytes = 0  # join buffer size once enable_peer ran

    @staticmethod
    def available() -> bool:
        return bool(_lib.lib().qmm_tp_available())

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * _lib.TP_UNIQUE_ID_BYTES)()
        _lib.check(_lib.lib().qmm_tp_unique_id(buf))
        return bytes(buf)

    @classmethod
    def init(cls, uid: bytes, world: int, rank: int, device: int, timeout_s: float = 60.0) -> "TpComm":
        if len(uid) != _lib.TP_UNIQUE_ID_BYTES:
            raise ValueError("unique id must be 128 bytes")
        buf = (ctypes.c_uint8 * _lib.TP_UNIQUE_ID_BYTES).from_buffer_copy(uid)
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().qmm_tp_init(buf, int(world), int(rank), int(device), float(timeout_s), ctypes.byref(h)))
        return cls(h.value, rank, world, device, timeout_s)

    @classmethod
    def from_group(cls, device: int, group=None, timeout_s: float = 60.0) -> "TpComm":
        """Rank 0 of `group` makes the unique id; the group's own backend carries it."""
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        obj = [cls.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        return cls.init(obj[0], world, rank, device, timeout_s)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    def enable_peer(self, nbytes: int, join_timeout_s: float = 0.0) -> None:
        """Joins over peer memory (qmm_tp_enable_peer): column / row forwards
        whose joined result fits in `nbytes` are written straight into every
        rank's buffer over NVLink and joined by one flag-barrier kernel instead
        of an NCCL collective; a join waits at most `join_timeout_s` for the
        peers (<= 0: the communicator's limit). Collective: every rank calls it."""
        _lib.check(_lib.lib().qmm_tp_enable_peer(self._h, int(nbytes), float(join_timeout_s)))
        self.peer_bytes = int(nbytes)

    def status(self) -> int:
        """One poll of the communicator's error state (a status code, never raises)."""
        return _lib.lib().qmm_tp_status(self._h)

    def wait(self, timeout_s: float | None = None, stream: torch.cuda.Stream | None = None) -> int:
        """Waits for `stream`'s work (default: the current stream) with the
        communicator watched; a status code (QMM_ERR_TIMEOUT / QMM_ERR_NCCL
        abort the communicator)."""
        sp = stream.cuda_stream if stream is not None else _stream_ptr(self.device)
        return _lib.lib().qmm_tp_wait(self._h, ctypes.c_void_p(sp),
                                      float(timeout_s if timeout_s is not None else self.timeout_s))

    def all_gather(self, send: torch.Tensor) -> torch.Tensor:
        out = torch.empty(self.world * send.numel(), dtype=torch.float32, device=send.device)
        _lib.check(_lib.lib().qmm_tp_all_gather_f32(self._h, send.data_ptr(), out.data_ptr(), send.numel(),
                                                    ctypes.c_void_p(_stream_ptr(self.device))))
        return out

    def all_reduce(self, buf: torch.Tensor) -> torch.Tensor:
        _lib.check(_lib.lib().qmm_tp_all_reduce_f32(self._h, buf.data_ptr(), buf.numel(),
                                                    ctypes.c_void_p(_stream_ptr(self.device))))
        return buf

    def abort(self) -> None:
        if self._h is not None and self._h.value:
            _lib.lib().qmm_tp_abort(self._h)

    def close(self) -> int:
        rc = OK
        if self._h is not None and self._h.value:
            rc = _lib.lib().qmm_tp_destroy(self._h)
            self._h = None
        return rc

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _act_of(linear: Linear) -> int:
    return linear.act_mode()


class ColumnParallelLinear:
    """Output rows split over the communicator's ranks; forward returns the
    full y on every rank (qmm_tp_column_forward: local product + all-gather)."""

    def __init__(self, dtype: int, n: int, k: int, weight_host, device: int, comm: TpComm):
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.n, self.k, self.n_local = n, k, n // self.world
        shard = column_shard(np.frombuffer(weight_host, dtype=np.uint8) if isinstance(weight_host, (bytes, bytearray))
                             else weight_host, n, k, dtype, self.rank, self.world)
        self.local = Linear(QuantWeight.from_host(dtype, self.n_local, k, shard, device))

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x = x.float().contiguous()
        m = x.numel() // self.k
        if out is None:
            out = torch.empty((*x.shape[:-1], self.n), dtype=torch.float32, device=x.device)
        _lib.check(_lib.lib().qmm_tp_column_forward(self.comm.handle, self.local.weight.handle, x.data_ptr(), m,
                                                    out.data_ptr(), _act_of(self.local),
                                                    ctypes.c_void_p(_stream_ptr(self.local.weight.device))))
        return out

    __call__ = forward


class RowParallelLinear:
    """K blocks split over the communicator's ranks; forward takes the full x
    (or, with forward_local, this rank's K slice) and returns the summed y on
    every rank (qmm_tp_row_forward: local product + all-reduce)."""

    def __init__(self, dtype: int, n: int, k: int, weight_host, device: int, comm: TpComm):
        self.comm = comm
        self.world, self.rank = comm.world, comm.rank
        self.n, self.k, self.k_local = n, k, k // self.world
        buf = np.ascontiguousarray(np.frombuffer(weight_host, dtype=np.uint8) if isinstance(
            weight_host, (bytes, bytearray)) else np.asarray(weight_host, dtype=np.uint8).ravel())
        h = ctypes.c_void_p()
        _lib.check(_lib.lib().qmm_weight_create_row_shard(int(dtype), int(n), int(k), buf.ctypes.data, buf.size,
                                                          self.rank, self.world, int(device), ctypes.byref(h)))
        self.local = Linear(QuantWeight(h.value, dtype, n, self.k_local, device))

    def forward_local(self, x_local: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        x_local = x_local.float().contiguous()
        m = x_local.numel() // self.k_local
        if out is None:
            out = torch.empty((*x_local.shape[:-1], self.n), dtype=torch.float32, device=x_local.device)
        _lib.check(_lib.lib().qmm_tp_row_forward(self.comm.handle, self.local.weight.handle, x_local.data_ptr(), m,
                                                 out.data_ptr(), _act_of(self.local),
                                                 ctypes.c_void_p(_stream_ptr(self.local.weight.device))))
        return out

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        m = x.numel() // self.k
        xs = x_row_slice(x.reshape(m, self.k), self.k, self.rank, self.world)
        return self.forward_local(xs, out).reshape(*x.shape[:-1], self.n)

    __call__ = forward


class ParallelFeedForward:
    """Megatron pairing of a gated feed-forward block (feed_forward.rs:198-251):
    gate/up column shards fused on each rank (qmm_weight_fuse_gate_up), the
    gated product of this rank's hidden slice computed locally, and down as a
    row-parallel linear over exactly that slice: one all-reduce per block and
    no all-gather in between. hidden/world must be a multiple of 32."""

    def __init__(self, dtype: int, dim: int, hidden: int, gate_host, up_host, down_host, device: int,
                 comm: TpComm, act_fn: int):
        from .fused import fuse_gate_up
        self.comm, self.act_fn = comm, act_fn
        world, rank = comm.world, comm.rank
        if hidden % (32 * world):
            raise ValueError(f"hidden {hidden} does not split into whole blocks over {world} ranks")
        self.dim, self.hidden, self.h_local = dim, hidden, hidden // world

        def col(host):
            return QuantWeight.from_host(dtype, self.h_local, dim,
                                         column_shard(np.asarray(host, dtype=np.uint8).ravel(), hidden, dim, dtype,
                                                      rank, world), device)
        g, u = col(gate_host), col(up_host)
        self.gate_up = fuse_gate_up(g, u)
        g.close()
        u.close()
        self.down = RowParallelLinear(dtype, dim, hidden, down_host, device, comm)

    def forward(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        from .fused import gated_forward
        h = gated_forward(self.gate_up, x, self.act_fn)
        return self.down.forward_local(h, out)

    __call__ = forward


# ---- failure handling between steps -----------------------------------------------------------

def _is_timeout(e: BaseException) -> bool:
    return "timeout" in str(e).lower() or "timed out" in str(e).lower()


class StepGuard:
    """Host-side agreement on each step through a torch.distributed Store.

    ``run(step, compute, join)`` returns a status code and never hangs:

    * every rank posts that it reached the step, and waits (polling, at most
      ``timeout_s``) until all ranks have, or until one posted a failure:
      QMM_ERR_TIMEOUT names the ranks that never arrived (one that left between
      steps), QMM_ERR_NCCL carries a peer's posted failure;
    * ``compute()`` (the rank-local work) raising posts the failure before any
      collective is launched, then re-raises on that rank;
    * before ``join(out)`` (the collectives) the ranks agree again, so a
      peer's failure in its compute stops the others on the host;
    * an error inside ``join`` (a collective that timed out, a communicator
      abort: QmmError carries the library's code) is posted and returned.
    """

    def __init__(self, store, rank: int, world: int, timeout_s: float = 10.0, prefix: str = "qmm_tp",
                 poll_s: float = 0.001):
        self.store, self.rank, self.world = store, rank, world
        self.timeout_s, self.prefix, self.poll_s = timeout_s, prefix, poll_s
        self.last_error = ""

    def _key(self, *parts) -> str:
        return "/".join((self.prefix,) + tuple(str(p) for p in parts))

    def post_failure(self, reason: str) -> None:
        self.store.set(self._key("failed"), f"rank {self.rank}: {reason}")

    def peer_failure(self) -> str | None:
        k = self._key("failed")
        if self.store.check([k]):
            return self.store.get(k).decode(errors="replace")
        return None

    def agree(self, tag: str) -> int:
        import time
        self.store.set(self._key(tag, self.rank), "1")
        keys = [self._key(tag, r) for r in range(self.world)]
        t0 = time.monotonic()
        while True:
            failed = self.peer_failure()
            if failed is not None:
                self.last_error = failed
                return ERR_NCCL
            if self.store.check(keys):
                return OK
            if time.monotonic() - t0 > self.timeout_s:
                missing = [r for r, k in enumerate(keys) if not self.store.check([k])]
                self.last_error = f"ranks {missing} did not reach {tag} within {self.timeout_s} s"
                return ERR_TIMEOUT
            time.sleep(self.poll_s)

    def run(self, step: int, compute, join=None) -> int:
        rc = self.agree(f"s{step}/begin")
        if rc:
            return rc
        try:
            out = compute()
        except BaseException as e:
            self.post_failure(f"step {step} compute: {e!r}")
            raise
        if join is None:
            return OK
        rc = self.agree(f"s{step}/join")
        if rc:
            return rc
        try:
            join(out)
        except QmmError as e:
            self.last_error = str(e)
            self.post_failure(f"step {step} join: {e}")
            return e.status
        except Exception as e:  # a collective of torch.distributed
            self.last_error = str(e)
            self.post_failure(f"step {step} join: {e!r}")
            return ERR_TIMEOUT if _is_timeout(e) else ERR_NCCL
        return OK


def default_store():
    """The default process group's store (for StepGuard)."""
    return dist.distributed_c10d._get_default_store()


__all__ = ["column_shard", "row_shard", "x_row_slice", "join_columns", "TpComm", "ColumnParallelLinear",
           "RowParallelLinear", "ParallelFeedForward", "StepGuard", "default_store"]
