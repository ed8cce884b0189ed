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

The shard/join helpers are plain numpy / torch (tested on CPU with gloo);
ColumnParallelLinear / RowParallelLinear run the library's GEMV/GEMM on the
local shard and join with torch.distributed collectives on the current stream.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist

from ._lib import BLOCK_BYTES
from .linear import Linear, QuantWeight

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


class ColumnParallelLinear:
    """Output rows split over the ranks of `group`; forward returns the full y on every rank."""

    def __init__(self, dtype: int, n: int, k: int, weight_host, device: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n, self.k, self.n_local = n, k, n // self.world
        shard = column_shard(np.frombuffer(weight_host, dtype=np.uint8) if isinstance(weight_host, (bytes, bytearray))
                             else weight_host, n, k, dtype, self.rank, self.world)
        self.local = Linear(QuantWeight.from_host(dtype, self.n_local, k, shard, device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = x.numel() // self.k
        y = self.local.forward(x.reshape(m, self.k))
        gathered = torch.empty(self.world * m * self.n_local, dtype=torch.float32, device=x.device)
        dist.all_gather_into_tensor(gathered, y.reshape(-1), group=self.group)
        return join_columns(gathered, m, self.n_local, self.world).reshape(*x.shape[:-1], self.n)

    __call__ = forward


class RowParallelLinear:
    """K blocks split over the ranks of `group`; forward takes the full x and
    returns the summed y on every rank."""

    def __init__(self, dtype: int, n: int, k: int, weight_host, device: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.n, self.k, self.k_local = n, k, k // self.world
        shard = row_shard(np.frombuffer(weight_host, dtype=np.uint8) if isinstance(weight_host, (bytes, bytearray))
                          else weight_host, n, k, dtype, self.rank, self.world)
        self.local = Linear(QuantWeight.from_host(dtype, n, self.k_local, shard, device))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        m = x.numel() // self.k
        xs = x_row_slice(x.reshape(m, self.k), self.k, self.rank, self.world).contiguous()
        y = self.local.forward(xs)
        dist.all_reduce(y, group=self.group)
        return y.reshape(*x.shape[:-1], self.n)

    __call__ = forward
