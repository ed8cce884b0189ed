"""A Gemma-3 decode step on one GPU: the quantised projections of this
library around the decode kernels of ``csrc/qmm_decode.cu``.

Mirrors the reference's single-token forward pass with a KV cache
(``LlmModel::forward_with_cache_pass``, llmserve/llmmodel/model/main/src/core/
forward.rs:107-239, on the Gemma-3 assembly of model.rs:726-907):

    x = embed(tokens) * emb_scale
    per layer:  h = rmsnorm(x, attn_norm)
                q|k|v = h . Wqkv^T (one fused Q4_0 matmul)
                q, k = rope(rmsnorm_per_head(q|k)); k, v -> cache[pos]
                a = softmax(q . K^T / sqrt(query_pre_attn_scalar)) V
                x += rmsnorm(a . Wo^T, post_attn_norm)
                f = down(gelu(gate(h2)) * up(h2)),  h2 = rmsnorm(x, ffn_norm)
                x += rmsnorm(f, post_ffn_norm)
    logits = rmsnorm(x, norm) . Emb^T      (Q8_0, tied with the embedding)

Per layer: one fused QKV matmul, one gate/up matmul with the GeGLU epilogue,
o and down, plus five small kernels (the post-norm + residual add is fused
with the next pre-norm). The decode position lives in device memory, so
``capture()`` records a whole step once as a CUDA graph that ``step()``
replays while the graph itself advances the position.
"""
from __future__ import annotations

import ctypes
import dataclasses
import math

import numpy as np
import torch

from . import _lib
from ._lib import GELU
from .fused import fuse_gate_up
from .linear import QuantWeight, _stream_ptr

Q4_0, Q8_0 = 2, 8


@dataclasses.dataclass
class Gemma3Config:
    hidden: int = 1152
    n_layers: int = 26
    n_heads: int = 4
    n_kv_heads: int = 1
    head_dim: int = 256
    ffn: int = 6912
    vocab: int = 262144
    ctx: int = 512
    eps: float = 1e-6
    offset: float = 1.0
    rope_local: float = 10000.0
    rope_global: float = 1000000.0
    pattern: int = 6
    query_pre_attn_scalar: float = 256.0
    emb_scale: float = float(np.float32(math.sqrt(1152.0)))

    @classmethod
    def gemma3_1b(cls, ctx: int = 512) -> "Gemma3Config":
        """Gemma-3-1B: 26 layers, hidden 1152, 4 query heads / 1 KV head of
        256, GeGLU FFN 6912, vocabulary 262144."""
        return cls(ctx=ctx)


def rope_tables(head_dim: int, ctx: int, theta: float):
    """cos/sin [ctx][head_dim/2] in f32 as the reference builds them
    (layers/main/src/core/rope.rs:113-128)."""
    half = head_dim // 2
    i = np.arange(half, dtype=np.float32)
    freq = (np.float32(1.0) / np.power(np.float32(theta), np.float32(2.0) * i / np.float32(head_dim),
                                       dtype=np.float32)).astype(np.float32)
    ang = (np.arange(ctx, dtype=np.float32)[:, None] * freq[None, :]).astype(np.float32)
    return np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)


def _quant_weight(dt: int, n: int, k: int, data, device: int, kpad: int = 0) -> QuantWeight:
    """A library weight from block bytes; kpad > k: each row padded with
    zero blocks (scale 0: every product 0) to kpad columns."""
    bb = 34 if dt == Q8_0 else 18
    if kpad > k:
        t = data if isinstance(data, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(data, dtype=np.uint8))
        t = t.to(torch.device("cuda", device))
        padded = torch.zeros(n, (kpad // 32) * bb, dtype=torch.uint8, device=t.device)
        padded[:, :(k // 32) * bb] = t.view(n, (k // 32) * bb)
        return QuantWeight.from_device(dt, n, kpad, padded.reshape(-1))
    if isinstance(data, torch.Tensor):
        return QuantWeight.from_device(dt, n, k, data)
    return QuantWeight.from_host(dt, n, k, np.ascontiguousarray(data, dtype=np.uint8), device)


def padded_k(k: int, batch: int) -> int:
    """Columns a batch-matmul weight of k columns is padded to. Batches of 17
    to 128 run on the tensor-core GEMMs; the decode-batch GEMM reads row
    pitches of 0 or 8 mod 16 bytes in place (Q4_0 / Q8_0 rows are 18 / 34
    bytes per 32 columns: k/32 a multiple of 4); larger batches run on the
    prefill GEMM, which needs a 16-byte pitch (k/32 a multiple of 8) and also
    takes 17..32 tokens where the pitch allows; smaller batches keep k (GEMV)."""
    nb = k // 32
    if batch < 17 or nb % 8 == 0 or (batch <= 128 and nb % 4 == 0):
        return k
    return (k // 256 + 1) * 256


def _rows(data, n: int, row_bytes: int, r0: int, r1: int):
    """Rows [r0, r1) of an [n][row_bytes] byte matrix (numpy or CUDA tensor)."""
    if isinstance(data, torch.Tensor):
        return data.view(n, row_bytes)[r0:r1].contiguous().view(-1)
    return np.ascontiguousarray(np.asarray(data, dtype=np.uint8).reshape(n, row_bytes)[r0:r1]).ravel()


def _cols(data, n: int, row_bytes: int, c0: int, c1: int):
    """Bytes [c0, c1) of every row of an [n][row_bytes] byte matrix."""
    if isinstance(data, torch.Tensor):
        return data.view(n, row_bytes)[:, c0:c1].contiguous().view(-1)
    return np.ascontiguousarray(np.asarray(data, dtype=np.uint8).reshape(n, row_bytes)[:, c0:c1]).ravel()


def band_k(k: int) -> int:
    """Columns the lm_head is padded to at batch 1: a 16-byte row pitch lets its
    one-token matmul stream through the band GEMV."""
    return k if (k // 32) % 8 == 0 else (k // 256 + 1) * 256


class Gemma3Decoder:
    """Weights: the dict layout of the parity oracle (``emb`` Q8_0 bytes,
    ``final_norm``, per layer ``qkv``/``o``/``gate``/``up``/``down`` Q4_0 bytes
    and the six norm vectors), as host numpy arrays or CUDA uint8 tensors.

    ``comm`` (a ``tp.TpComm`` of W > 1 ranks, one decoder per rank) shards the
    step tensor-parallel: the feed-forward block Megatron-style (gate/up rows
    [r F/W, (r+1) F/W) fused on each rank, down over the same K slice, one
    all-reduce) and the tied lm_head by vocabulary rows (one all-gather of the
    logits). Attention (4 query heads, 1 KV head) and the norms are replicated
    on every rank. The sharded step runs its launches directly (the library's
    non-blocking communicator is not captured in a CUDA graph)."""

    def __init__(self, cfg: Gemma3Config, weights: dict, batch: int, device: int = 0, fused_attention: bool = True,
                 comm=None):
        self.cfg, self.batch, self.device = cfg, batch, device
        self.comm = comm if comm is not None and comm.world > 1 else None
        W, R = (self.comm.world, self.comm.rank) if self.comm else (1, 0)
        if cfg.ffn % (32 * W) or cfg.vocab % W:
            raise ValueError(f"ffn {cfg.ffn} / vocab {cfg.vocab} do not shard over {W} ranks")
        self.ffn_local, self.vocab_local = cfg.ffn // W, cfg.vocab // W
        self.fused_attention = fused_attention  # QK-norm/RoPE/cache append inside the attention kernel
        dev = torch.device("cuda", device)
        self.dev = dev
        H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        self.lib = _lib.lib()

        def vec(a):
            return torch.as_tensor(np.asarray(a, np.float32) if not isinstance(a, torch.Tensor) else a,
                                   dtype=torch.float32).to(dev).contiguous()

        self.emb = _quant_weight(Q8_0, cfg.vocab, H, weights["emb"], device)
        self.kh = kh = padded_k(H, batch)  # K of the matmuls that read the hidden state
        # the lm_head also at batch 1: a 16-byte row pitch lets its one-token
        # matmul stream through the band kernel
        self.klm = klm = kh if batch != 1 else band_k(H)
        Fl, Vl = self.ffn_local, self.vocab_local
        if self.comm:  # this rank's vocabulary rows
            lm = _rows(weights["emb"], cfg.vocab, (H // 32) * 34, R * Vl, (R + 1) * Vl)
            self.lm_head = _quant_weight(Q8_0, Vl, H, lm, device, klm)
        else:
            self.lm_head = self.emb if klm == H else _quant_weight(Q8_0, cfg.vocab, H, weights["emb"], device, klm)
        self.final_norm = vec(weights["final_norm"])
        self.layers = []
        nqkv = (nq + 2 * nkv) * hd
        rb_h, rb_f = (H // 32) * 18, (cfg.ffn // 32) * 18
        for lw in weights["layers"]:
            gate = _quant_weight(Q4_0, Fl, H, _rows(lw["gate"], cfg.ffn, rb_h, R * Fl, (R + 1) * Fl), device, kh)
            up = _quant_weight(Q4_0, Fl, H, _rows(lw["up"], cfg.ffn, rb_h, R * Fl, (R + 1) * Fl), device, kh)
            down = lw["down"] if W == 1 else _cols(lw["down"], H, rb_f, R * (Fl // 32) * 18, (R + 1) * (Fl // 32) * 18)
            layer = {
                "qkv": _quant_weight(Q4_0, nqkv, H, lw["qkv"], device, kh),
                "o": _quant_weight(Q4_0, H, nq * hd, lw["o"], device),
                "gate_up": fuse_gate_up(gate, up),
                "down": _quant_weight(Q4_0, H, Fl, down, device),
            }
            gate.close()
            up.close()
            for key in ("attn_norm", "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm", "k_norm"):
                layer[key] = vec(lw[key])
            self.layers.append(layer)
        tabs = {t: rope_tables(hd, cfg.ctx, t) for t in (cfg.rope_local, cfg.rope_global)}
        self.rope = {t: (vec(c), vec(s)) for t, (c, s) in tabs.items()}
        B = batch
        z = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=dev)  # noqa: E731
        self.k_cache = z(cfg.n_layers, B, nkv, cfg.ctx, hd)
        self.v_cache = z(cfg.n_layers, B, nkv, cfg.ctx, hd)
        self.tokens = torch.zeros(B, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.x, self.h, self.o = z(B, H), z(B, H), z(B, H)
        self.hp = self.h if kh == H else z(B, kh)  # h with a zero tail to kh columns
        self.hl = self.hp if klm == kh else z(B, klm)  # the same for the lm_head
        self.qkv, self.q, self.attn = z(B, nqkv), z(B, nq * hd), z(B, nq * hd)
        self.ff = z(B, Fl)
        self.logits = z(B, cfg.vocab)
        self.part = z(int(self.lib.qmm_attention_partial_floats(B, nq, hd, cfg.ctx)))
        self.inv_scale = float(np.float32(1.0) / np.float32(math.sqrt(cfg.query_pre_attn_scalar)))
        self.stream = torch.cuda.Stream(dev)
        self.graph = None
        need = max(self.lib.qmm_workspace_size(dt, 0, B, n, k) for dt, n, k in
                   [(Q4_0, nqkv, kh), (Q4_0, H, nq * hd), (Q4_0, 2 * Fl, kh), (Q4_0, H, Fl),
                    (Q8_0, Vl, klm)])
        _lib.check(self.lib.qmm_reserve_workspace(device, ctypes.c_void_p(self.stream.cuda_stream), need + (1 << 20)))

    # ---- one step, issued on self.stream ---------------------------------------------
    def _launch(self, advance: bool):
        cfg, L, B = self.cfg, self.lib, self.batch
        H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
        sp = ctypes.c_void_p(self.stream.cuda_stream)
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        ck = _lib.check
        ck(L.qmm_embed_q8_dev(ctypes.c_void_p(self.emb.device_ptr()), cfg.vocab, H, P(self.tokens), B, cfg.emb_scale, P(self.x), sp))
        # normed hidden states go straight into hp (rows kh wide, zero tail)
        ck(L.qmm_rmsnorm_dev(P(self.x), P(self.layers[0]["attn_norm"]), cfg.offset, cfg.eps, B, H, P(self.hp), self.kh,
                             sp))
        for li, lw in enumerate(self.layers):
            theta = cfg.rope_global if (li + 1) % cfg.pattern == 0 else cfg.rope_local
            cos, sin = self.rope[theta]
            ck(L.qmm_linear_forward(lw["qkv"].handle, P(self.hp), B, P(self.qkv), 0, sp))
            if self.fused_attention:
                ck(L.qmm_attention_decode_fused_dev(P(self.qkv), B, nq, nkv, hd, P(lw["q_norm"]), P(lw["k_norm"]),
                                                    cfg.offset, cfg.eps, P(cos), P(sin), P(self.pos), cfg.ctx,
                                                    P(self.k_cache[li]), P(self.v_cache[li]), self.inv_scale,
                                                    P(self.part), P(self.attn), sp))
            else:
                ck(L.qmm_qk_rope_cache_dev(P(self.qkv), B, nq, nkv, hd, P(lw["q_norm"]), P(lw["k_norm"]), cfg.offset,
                                           cfg.eps, P(cos), P(sin), P(self.pos), cfg.ctx, P(self.q),
                                           P(self.k_cache[li]), P(self.v_cache[li]), sp))
                ck(L.qmm_attention_decode_dev(P(self.q), P(self.k_cache[li]), P(self.v_cache[li]), B, nq, nkv, hd,
                                              P(self.pos), cfg.ctx, self.inv_scale, P(self.part), P(self.attn), sp))
            ck(L.qmm_linear_forward(lw["o"].handle, P(self.attn), B, P(self.o), 0, sp))
            ck(L.qmm_residual_rmsnorm_dev(P(self.x), P(self.o), P(lw["post_attn_norm"]), P(lw["ffn_norm"]),
                                          cfg.offset, cfg.eps, B, H, P(self.hp), self.kh, sp))
            ck(L.qmm_gated_forward(lw["gate_up"].handle, P(self.hp), B, P(self.ff), GELU, sp))
            if self.comm:  # this rank's K slice of down, summed over the ranks
                ck(L.qmm_tp_row_forward(self.comm.handle, lw["down"].handle, P(self.ff), B, P(self.o), 0, sp))
            else:
                ck(L.qmm_linear_forward(lw["down"].handle, P(self.ff), B, P(self.o), 0, sp))
            nxt = self.layers[li + 1]["attn_norm"] if li + 1 < len(self.layers) else self.final_norm
            ck(L.qmm_residual_rmsnorm_dev(P(self.x), P(self.o), P(lw["post_ffn_norm"]), P(nxt), cfg.offset, cfg.eps,
                                          B, H, P(self.hp), self.kh, sp))
        if self.hl is not self.hp:  # batch 1: only the lm_head reads a padded copy
            with torch.cuda.stream(self.stream):
                self.hl[:, :H].copy_(self.hp)
        if self.comm:  # this rank's vocabulary rows, gathered into [B][vocab]
            ck(L.qmm_tp_column_forward(self.comm.handle, self.lm_head.handle, P(self.hl), B, P(self.logits), 0, sp))
        else:
            ck(L.qmm_linear_forward(self.lm_head.handle, P(self.hl), B, P(self.logits), 0, sp))
        if advance:
            ck(L.qmm_add_int_dev(P(self.pos), 1, sp))

    def set_position(self, pos: int) -> None:
        if not 0 <= pos < self.cfg.ctx:
            raise ValueError(f"position {pos} outside the cache (0..{self.cfg.ctx - 1})")
        self.stream.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(self.stream):
            self.pos.fill_(pos)

    def set_tokens(self, tokens) -> None:
        t = torch.as_tensor(np.asarray(tokens, dtype=np.int32))
        if t.numel() != self.batch:
            raise ValueError(f"{t.numel()} tokens for a batch of {self.batch}")
        with torch.cuda.stream(self.stream):
            self.tokens.copy_(t, non_blocking=False)

    def capture(self, advance: bool = True) -> None:
        """Record one step (and, with ``advance``, the position increment) as a
        CUDA graph; later ``step()`` calls replay it. A sharded decoder is
        captured only when every join of the step goes over peer memory
        (TpComm.enable_peer with room for the logits and the FFN partials);
        NCCL joins are not captured, so it keeps launching directly."""
        if self.comm and not self.comm.peer_bytes >= 4 * self.batch * max(
                self.cfg.vocab, self.comm.world * self.cfg.hidden):
            self.graph = None
            return
        # one direct launch first (it rewrites this position's cache rows with
        # the same values): kernel attributes are set outside the capture
        with torch.cuda.stream(self.stream):
            self._launch(False)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=self.stream):
            self._launch(advance)
        self.graph = g

    def step(self, tokens=None, advance: bool = True) -> torch.Tensor:
        """Logits [batch][vocab] of one step at the current position (tokens:
        host ids, or None to reuse the device token buffer). Without a graph
        the kernels are launched directly."""
        if tokens is not None:
            self.set_tokens(tokens)
        if self.graph is not None:
            with torch.cuda.stream(self.stream):
                self.graph.replay()
        else:
            with torch.cuda.stream(self.stream):
                self._launch(advance)
        # work queued on the caller's stream after this call sees the logits
        torch.cuda.current_stream(self.dev).wait_stream(self.stream)
        return self.logits

    def wait(self, timeout_s: float = 60.0) -> None:
        """Waits for the step's work; a sharded decoder through its
        communicator (a stuck or failed collective raises QmmError with
        QMM_ERR_TIMEOUT / QMM_ERR_NCCL instead of hanging)."""
        if self.comm:
            _lib.check(self.comm.wait(timeout_s, self.stream))
        else:
            self.stream.synchronize()

    def close(self) -> None:
        self.graph = None
        for lw in self.layers:
            for key in ("qkv", "o", "gate_up", "down"):
                lw[key].close()
        if self.lm_head is not self.emb:
            self.lm_head.close()
        self.emb.close()


def random_weights(cfg: Gemma3Config, seed: int, device: int = 0) -> dict:
    """Seeded random-init weights in the oracle's dict layout, quantised on the
    device by this library's bit-exact quantisers (weights ~N(0, 0.02), norm
    vectors ~N(0, 0.1)): CUDA uint8 tensors for the block bytes."""
    dev = torch.device("cuda", device)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    L = _lib.lib()
    H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim

    def quant(dt, n, k):
        wf = torch.randn(n * k, generator=gen, device=dev) * 0.02
        out = torch.empty(n * (k // 32) * (34 if dt == Q8_0 else 18), dtype=torch.uint8, device=dev)
        _lib.check(L.qmm_quantize_dev(dt, 0, ctypes.c_void_p(wf.data_ptr()), wf.numel(),
                                      ctypes.c_void_p(out.data_ptr()), None,
                                      ctypes.c_void_p(_stream_ptr(device))))
        torch.cuda.synchronize(dev)
        return out

    def norm(n):
        return torch.randn(n, generator=gen, device=dev) * 0.1

    w = {"emb": quant(Q8_0, cfg.vocab, H), "final_norm": norm(H), "layers": []}
    for _ in range(cfg.n_layers):
        w["layers"].append({
            "qkv": quant(Q4_0, (nq + 2 * nkv) * hd, H), "o": quant(Q4_0, H, nq * hd),
            "gate": quant(Q4_0, cfg.ffn, H), "up": quant(Q4_0, cfg.ffn, H), "down": quant(Q4_0, H, cfg.ffn),
            "attn_norm": norm(H), "post_attn_norm": norm(H), "ffn_norm": norm(H), "post_ffn_norm": norm(H),
            "q_norm": norm(hd), "k_norm": norm(hd)})
    return w
