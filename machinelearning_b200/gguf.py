"""GGUF -> HBM: upload quantised weight tensors byte for byte, no repacking.

The parser restates the reference's header reader
(llmserve/llmmodel/gguf/main/src/core/parser.rs:162-232): magic "GGUF",
version 2 or 3, u64 tensor and metadata counts, metadata key/value pairs
(value types 0-12, arrays recursive), then per tensor: name, u32 dimension
count, u64 dimensions (innermost first), u32 GGML type, u64 offset. Tensor
data starts at the header end rounded up to 32 bytes (the reference's fixed
alignment; it does not read general.alignment). A tensor's byte size is
n_blocks * block_bytes (parser.rs:511-518) and must lie inside the file.

upload() maps the file (zero-copy, as the reference's load_tensors_mmap,
parser.rs:501-576) and copies each Q4_0 / Q8_0 / Q4_1 matrix's exact file
range to the GPU with one host-to-device copy into a library-owned
qmm_weight. With verify=True the device copy's checksum (computed on the GPU
by the library) must equal the checksum of the file range computed here.
"""
from __future__ import annotations

import ctypes
import mmap
import os
import struct
from dataclasses import dataclass, field

import numpy as np

from . import _lib
from .linear import QuantWeight

GGUF_MAGIC = b"GGUF"
ALIGNMENT = 32

# GGML type id -> (block elements, block bytes) (reference gguf api/types.rs)
GGML_TYPES = {
    0: ("F32", 1, 4), 1: ("F16", 1, 2), 2: ("Q4_0", 32, 18), 3: ("Q4_1", 32, 20), 6: ("Q5_0", 32, 22),
    7: ("Q5_1", 32, 24), 8: ("Q8_0", 32, 34), 9: ("Q8_1", 32, 40), 10: ("Q2_K", 256, 84), 11: ("Q3_K", 256, 110),
    12: ("Q4_K", 256, 144), 13: ("Q5_K", 256, 176), 14: ("Q6_K", 256, 210), 15: ("Q8_K", 256, 292),
}
UPLOADABLE = (2, 3, 8)  # the block types the matmul kernels read


class GgufError(ValueError):
    """Malformed or unsupported GGUF input (the reference's GgufError)."""


@dataclass
class TensorInfo:
    name: str
    dims: list[int]  # GGUF order: innermost first
    ggml_type: int
    offset: int      # relative to the data section

    @property
    def shape(self) -> list[int]:
        return list(reversed(self.dims))

    @property
    def n_elements(self) -> int:
        n = 1
        for d in self.dims:
            n *= d
        return n

    @property
    def nbytes(self) -> int:
        _, per, bb = GGML_TYPES[self.ggml_type]
        return (self.n_elements // per) * bb if per > 1 else self.n_elements * bb


@dataclass
class GGUFFile:
    version: int
    metadata: dict = field(default_factory=dict)
    tensors: list[TensorInfo] = field(default_factory=list)
    data_offset: int = 0

    @classmethod
    def parse(cls, data) -> "GGUFFile":
        """Parse the header, metadata and tensor infos of a GGUF image (bytes,
        mmap or any buffer)."""
        cur = _Cursor(memoryview(data))
        if bytes(cur.read(4)) != GGUF_MAGIC:
            raise GgufError("invalid GGUF magic")
        version = cur.u32()
        if version < 2 or version > 3:
            raise GgufError(f"unsupported GGUF version: {version}")
        n_tensors, n_meta = cur.u64(), cur.u64()
        meta = {}
        for _ in range(n_meta):
            key = cur.string()
            meta[key] = cur.value(cur.u32())
        infos = []
        for _ in range(n_tensors):
            name = cur.string()
            dims = [cur.u64() for _ in range(cur.u32())]
            t = cur.u32()
            if t not in GGML_TYPES:
                raise GgufError(f"unsupported GGML type: {t}")
            infos.append(TensorInfo(name, dims, t, cur.u64()))
        return cls(version, meta, infos, (cur.pos + ALIGNMENT - 1) & ~(ALIGNMENT - 1))

    @classmethod
    def parse_file(cls, path: str) -> "GGUFFile":
        with open(path, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
            return cls.parse(mm)

    def tensor_range(self, info: TensorInfo, file_size: int) -> tuple[int, int]:
        start = self.data_offset + info.offset
        end = start + info.nbytes
        if end > file_size:
            raise GgufError(f"tensor '{info.name}' data exceeds file bounds")
        return start, end


class _Cursor:
    def __init__(self, buf: memoryview):
        self.buf, self.pos = buf, 0

    def read(self, n: int) -> memoryview:
        if self.pos + n > len(self.buf):
            raise GgufError("unexpected end of GGUF file")
        v = self.buf[self.pos:self.pos + n]
        self.pos += n
        return v

    def _unpack(self, fmt: str, n: int):
        return struct.unpack("<" + fmt, self.read(n))[0]

    def u32(self) -> int:
        return self._unpack("I", 4)

    def u64(self) -> int:
        return self._unpack("Q", 8)

    def string(self) -> str:
        return bytes(self.read(self.u64())).decode("utf-8", errors="replace")

    def value(self, t: int):
        scalars = {0: ("B", 1), 1: ("b", 1), 2: ("H", 2), 3: ("h", 2), 4: ("I", 4), 5: ("i", 4), 6: ("f", 4),
                   10: ("Q", 8), 11: ("q", 8), 12: ("d", 8)}
        if t in scalars:
            return self._unpack(*scalars[t])
        if t == 7:
            return self._unpack("B", 1) != 0
        if t == 8:
            return self.string()
        if t == 9:
            et, count = self.u32(), self.u64()
            return [self.value(et) for _ in range(count)]
        raise GgufError(f"unknown GGUF value type: {t}")


def checksum(data) -> int:
    """Position-weighted checksum of a byte range: sum over its little-endian
    32-bit words w_i (the tail zero-padded) of w_i * (2i + 1), modulo 2^64.
    The library computes the same value on the GPU (qmm_checksum_dev)."""
    b = np.frombuffer(data, dtype=np.uint8)
    total = 0
    chunk = 1 << 24  # words per step (bounded temporary memory)
    nwords = (b.size + 3) // 4
    tail = b.size - (b.size // 4) * 4
    words = b[: (b.size // 4) * 4].view("<u4")
    for w0 in range(0, nwords, chunk):
        w1 = min(nwords, w0 + chunk)
        if w1 <= words.size:
            w = words[w0:w1].astype(np.uint64)
        else:
            last = np.zeros(4, np.uint8)
            last[:tail] = b[words.size * 4:]
            w = np.concatenate([words[w0:].astype(np.uint64), last.view("<u4").astype(np.uint64)])
        idx = np.arange(w0, w0 + w.size, dtype=np.uint64) * np.uint64(2) + np.uint64(1)
        with np.errstate(over="ignore"):
            total = (total + int(np.sum(w * idx, dtype=np.uint64))) & 0xFFFFFFFFFFFFFFFF
    return total


def device_checksum(weight: QuantWeight) -> int:
    out = ctypes.c_ulonglong(0)
    _lib.check(_lib.lib().qmm_weight_checksum(weight.handle, ctypes.byref(out)))
    return out.value


def upload(path: str, device: int = 0, names=None, verify: bool = True) -> dict:
    """Upload every Q4_0 / Q8_0 / Q4_1 matrix of a GGUF file (or those in
    `names`) to `device`: {name: QuantWeight}, weights [shape[0] rows,
    shape[1] inputs]. Other tensor types are not uploaded (the reference
    keeps F32/F16 as raw tensors and dequantises K-quants on the host)."""
    gf = GGUFFile.parse_file(path)
    out = {}
    with open(path, "rb") as f, mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ) as mm:
        size = len(mm)
        view = memoryview(mm)
        try:
            for info in gf.tensors:
                if names is not None and info.name not in names:
                    continue
                if info.ggml_type not in UPLOADABLE or len(info.dims) != 2:
                    continue
                k, n = info.dims  # innermost first: in_features, then rows
                start, end = gf.tensor_range(info, size)
                raw = np.frombuffer(view[start:end], dtype=np.uint8)  # zero-copy file range
                w = QuantWeight.from_host(info.ggml_type, n, k, raw, device)
                if verify:
                    got, want = device_checksum(w), checksum(view[start:end])
                    if got != want:
                        w.close()
                        raise GgufError(f"tensor '{info.name}': device checksum {got:#x} != file {want:#x}")
                out[info.name] = w
                del raw
        finally:
            view.release()
    return out


def write_gguf(path: str, tensors, metadata=None, version: int = 3) -> None:
    """Write a GGUF image: tensors = [(name, ggml_type, shape [rows, inputs], raw bytes)].
    (For tests and fixtures: the layout the parser above reads.)"""
    def s(x: str) -> bytes:
        e = x.encode()
        return struct.pack("<Q", len(e)) + e

    def val(v):
        if isinstance(v, bool):
            return struct.pack("<I", 7) + struct.pack("<B", int(v))
        if isinstance(v, int):
            return struct.pack("<I", 4) + struct.pack("<I", v)
        if isinstance(v, float):
            return struct.pack("<I", 6) + struct.pack("<f", v)
        if isinstance(v, str):
            return struct.pack("<I", 8) + s(v)
        if isinstance(v, list):
            assert all(isinstance(x, int) for x in v)
            return struct.pack("<I", 9) + struct.pack("<IQ", 4, len(v)) + b"".join(struct.pack("<I", x) for x in v)
        raise TypeError(type(v))

    metadata = metadata or {}
    head = GGUF_MAGIC + struct.pack("<IQQ", version, len(tensors), len(metadata))
    for kk, v in metadata.items():
        head += s(kk) + val(v)
    offs, off = [], 0
    for name, t, shape, raw in tensors:
        offs.append(off)
        off += len(raw)
        off = (off + ALIGNMENT - 1) & ~(ALIGNMENT - 1)
    for (name, t, shape, raw), o in zip(tensors, offs):
        dims = list(reversed(shape))
        head += s(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", t, o)
    pad = (-len(head)) % ALIGNMENT
    with open(path, "wb") as f:
        f.write(head + b"\0" * pad)
        for (name, t, shape, raw), o in zip(tensors, offs):
            cur = f.tell() - len(head) - pad
            f.write(b"\0" * (o - cur))
            f.write(bytes(raw))
