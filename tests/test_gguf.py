"""GGUF -> HBM upload (machinelearning_b200/gguf.py): the header parser against
the reference's own parser tests (gguf/main/src/core/parser.rs:1153-1170) and
its rules, the host checksum, and on the GPU a byte-for-byte upload verified
by the device checksum and used by the matmul."""
from __future__ import annotations

import ctypes
import struct

import numpy as np
import pytest

from machinelearning_b200.gguf import ALIGNMENT, GGUFFile, GgufError, checksum, write_gguf

Q4_0, Q4_1, Q8_0 = 2, 3, 8


# ---- the reference's parser tests ----------------------------------------------------------

def test_magic_check():  # parser.rs:1153-1156
    with pytest.raises(GgufError):
        GGUFFile.parse(bytes(20))


def test_valid_minimal():  # parser.rs:1159-1170
    data = b"GGUF" + struct.pack("<I", 3) + struct.pack("<Q", 0) + struct.pack("<Q", 0)
    g = GGUFFile.parse(data)
    assert g.version == 3 and g.metadata == {} and g.tensors == []


# ---- parser rules -----------------------------------------------------------------------------

@pytest.mark.parametrize("version", [1, 4])
def test_unsupported_version(version):
    with pytest.raises(GgufError):
        GGUFFile.parse(b"GGUF" + struct.pack("<IQQ", version, 0, 0))


def test_truncated():
    with pytest.raises(GgufError):
        GGUFFile.parse(b"GGUF" + struct.pack("<I", 3) + b"\x01")


def _tensors(oracle):
    rng = np.random.default_rng(5)
    q4 = oracle.quantize_q4_0(rng.normal(0, 0.02, 64 * 256).astype(np.float32))
    q8 = oracle.quantize_q8_0(rng.normal(0, 0.02, 48 * 128).astype(np.float32))
    q41 = oracle.quantize_q4_1(rng.normal(0, 0.02, 32 * 384).astype(np.float32))
    f32 = rng.normal(0, 1, 16).astype(np.float32).tobytes()
    return [("blk.0.ffn_up.weight", Q4_0, [64, 256], q4.tobytes()),
            ("output_norm.weight", 0, [16], f32),
            ("blk.0.attn_q.weight", Q8_0, [48, 128], q8.tobytes()),
            ("blk.0.ffn_down.weight", Q4_1, [32, 384], q41.tobytes())]


def test_parse_written_file(oracle, tmp_path):
    path = str(tmp_path / "m.gguf")
    tensors = _tensors(oracle)
    meta = {"general.architecture": "gemma3", "gemma3.block_count": 26, "gemma3.rope.freq_base": 10000.0,
            "general.flag": True, "tokenizer.ids": [1, 2, 3]}
    write_gguf(path, tensors, meta)
    g = GGUFFile.parse_file(path)
    assert g.version == 3
    assert g.metadata["general.architecture"] == "gemma3" and g.metadata["gemma3.block_count"] == 26
    assert g.metadata["tokenizer.ids"] == [1, 2, 3] and g.metadata["general.flag"] is True
    assert g.data_offset % ALIGNMENT == 0
    data = open(path, "rb").read()
    for info, (name, t, shape, raw) in zip(g.tensors, tensors):
        assert info.name == name and info.ggml_type == t and info.shape == shape
        start, end = g.tensor_range(info, len(data))
        assert data[start:end] == raw  # the exact bytes, nothing repacked
        assert info.nbytes == len(raw)


def test_tensor_out_of_bounds(oracle, tmp_path):
    path = str(tmp_path / "m.gguf")
    write_gguf(path, _tensors(oracle))
    data = open(path, "rb").read()
    g = GGUFFile.parse(data)
    with pytest.raises(GgufError):
        g.tensor_range(g.tensors[-1], len(data) - 1)


def test_checksum_known_values():
    assert checksum(bytes([1, 0, 0, 0, 2, 0, 0, 0])) == 1 * 1 + 2 * 3
    assert checksum(bytes([1, 0, 0, 0, 5])) == 1 + 5 * 3  # tail word zero-padded
    assert checksum(b"") == 0
    big = np.full(1 << 20, 0xFFFFFFFF, dtype="<u4").tobytes()
    n = 1 << 20
    assert checksum(big) == (0xFFFFFFFF * n * n) % (1 << 64)  # sum of (2i+1) = n^2, mod 2^64


# ---- GPU: upload, device checksum, matmul on the uploaded bytes -------------------------------

@pytest.mark.gpu
def test_upload_verified_and_usable(oracle, qlib, tmp_path):
    import torch

    from machinelearning_b200.gguf import device_checksum, upload
    from machinelearning_b200.linear import Linear

    path = str(tmp_path / "m.gguf")
    tensors = _tensors(oracle)
    write_gguf(path, tensors, {"general.architecture": "gemma3"})
    ws = upload(path, device=0, verify=True)
    assert set(ws) == {"blk.0.ffn_up.weight", "blk.0.attn_q.weight", "blk.0.ffn_down.weight"}  # not the F32 norm
    fns = {Q4_0: (oracle.matmul_f32_q4, oracle.matmul_f32_q4_native),
           Q8_0: (oracle.matmul_f32_q8, oracle.matmul_f32_q8_v2),
           Q4_1: (oracle.matmul_f32_q4_1, oracle.matmul_f32_q4_1_native)}
    for name, t, shape, raw in tensors:
        if name not in ws:
            continue
        n, k = shape
        w = ws[name]
        assert (w.dtype, w.n, w.k) == (t, n, k)
        assert device_checksum(w) == checksum(raw)
        x = np.random.default_rng(n + k).normal(0, 1, (3, k)).astype(np.float32)
        lin = Linear(w)
        y = lin(torch.from_numpy(x).cuda()).cpu().numpy().ravel()
        ref = fns[t][0](x.ravel(), np.frombuffer(raw, np.uint8), 3, k, n)
        assert np.linalg.norm(y - ref) <= 1e-3 * np.linalg.norm(ref)
        lin.set_native_q4_matmul(True)
        lin.set_native_q8_matmul(True)
        yn = lin(torch.from_numpy(x).cuda()).cpu().numpy().ravel()
        assert np.array_equal(yn.view(np.uint32), fns[t][1](x.ravel(), np.frombuffer(raw, np.uint8), 3, k, n).view(np.uint32))
    # a changed byte changes the device checksum of the same range
    buf = torch.from_numpy(np.frombuffer(tensors[0][3], np.uint8).copy()).cuda()
    out = ctypes.c_ulonglong()
    assert qlib.qmm_checksum_dev(buf.data_ptr(), buf.numel(), None, ctypes.byref(out)) == 0
    assert out.value == checksum(tensors[0][3])
    buf[100] ^= 1
    assert qlib.qmm_checksum_dev(buf.data_ptr(), buf.numel(), None, ctypes.byref(out)) == 0
    assert out.value != checksum(tensors[0][3])
