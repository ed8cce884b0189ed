"""TEST INFRASTRUCTURE ONLY -- the parity oracle of a Gemma-3 decode step.

A numpy restatement of the reference's single-token forward pass with a KV
cache, on the same quantised block bytes the device model uses; its matmuls
are the C oracle's ``matmul_f32_q4`` / ``matmul_f32_q8`` (the reference's
f32-activation paths). Only ``tests/`` may import it, as the checker.

Reference, in order:
  embeddings and final projection  llmserve/llmmodel/model/main/src/core/forward.rs:107-239
  Gemma-3 assembly (norm offset 1, global RoPE every ``pattern``-th layer,
  attention scale sqrt(query_pre_attn_scalar))  model/main/src/core/model.rs:726-907
  sandwich block                   llmserve/llmmodel/layers/main/src/core/transformer_block.rs:424-449
  attention decode (q/k norm, RoPE, cache, softmax(q.k / scale) v; no mask
  for one token)                   llmserve/llmmodel/layers/main/src/core/attention.rs:454-610
  RMSNorm                          main/features/tensor/src/core/tensor/math.rs:21-80, 334-380
  RoPE tables and rotation         llmserve/llmmodel/layers/main/src/core/rope.rs:7-130
  GeGLU feed-forward               llmserve/llmmodel/layers/main/src/core/feed_forward.rs:198-251
"""
from __future__ import annotations

import numpy as np

from . import Q4_0, Q8_0, gelu, matmul_f32_q4, matmul_f32_q8, to_f32

F = np.float32


def rope_tables(head_dim: int, ctx: int, theta: float, scaling: float = 1.0):
    """cos/sin [ctx][head_dim/2]: freq_i = (1 / theta^(2i/hd)) / scaling,
    angle = pos * freq_i, all in f32 (rope.rs:113-128)."""
    half = head_dim // 2
    i = np.arange(half, dtype=F)
    freq = (F(1.0) / np.power(F(theta), F(2.0) * i / F(head_dim), dtype=F)).astype(F) / F(scaling)
    ang = (np.arange(ctx, dtype=F)[:, None] * freq[None, :]).astype(F)
    return np.cos(ang).astype(F), np.sin(ang).astype(F)


def rmsnorm(x, w, offset: float, eps: float):
    """x / sqrt(mean(x^2) + eps) * (w + offset) over the last axis."""
    x = np.asarray(x, F)
    ss = np.sum(x * x, axis=-1, keepdims=True, dtype=F)
    inv = F(1.0) / np.sqrt(ss / F(x.shape[-1]) + F(eps))
    return ((x * inv) * (np.asarray(w, F) + F(offset))).astype(F)


def rope(x, cos, sin):
    """First half x1*cos - x2*sin, second half x1*sin + x2*cos (rope.rs:7-48)."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return np.concatenate([x1 * cos - x2 * sin, x1 * sin + x2 * cos], axis=-1).astype(F)


def decode_step(cfg, w, tokens, pos: int, k_cache, v_cache):
    """Logits [B][vocab] of one decode step at position ``pos``; k_cache /
    v_cache [layers][B][n_kv][ctx][head_dim] are updated in place.

    ``cfg``: hidden, n_layers, n_heads, n_kv_heads, head_dim, ffn, vocab, ctx,
    eps, offset, rope_local, rope_global, pattern, query_pre_attn_scalar,
    emb_scale. ``w``: "emb" (Q8_0 [vocab][hidden] bytes, tied with the output
    projection), "final_norm", and per layer "qkv" (Q4_0 bytes of the q, k, v
    rows in that order), "o", "gate", "up", "down", "attn_norm",
    "post_attn_norm", "ffn_norm", "post_ffn_norm", "q_norm", "k_norm"."""
    B = len(tokens)
    H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    rb = (H // 32) * 34  # Q8_0 bytes per embedding row: only the gathered rows are dequantised
    emb = np.asarray(w["emb"], np.uint8)
    x = np.stack([to_f32(Q8_0, emb[t * rb:(t + 1) * rb], H) for t in np.asarray(tokens)])
    x = (x * F(cfg.emb_scale)).astype(F)
    tables = {t: rope_tables(hd, cfg.ctx, t) for t in (cfg.rope_local, cfg.rope_global)}
    inv_scale = F(1.0) / F(np.sqrt(F(cfg.query_pre_attn_scalar)))
    for li, lw in enumerate(w["layers"]):
        h = rmsnorm(x, lw["attn_norm"], cfg.offset, cfg.eps)
        qkv = matmul_f32_q4(h.ravel(), lw["qkv"], B, H, (nq + 2 * nkv) * hd).reshape(B, nq + 2 * nkv, hd)
        q = rmsnorm(qkv[:, :nq], lw["q_norm"], cfg.offset, cfg.eps)
        k = rmsnorm(qkv[:, nq:nq + nkv], lw["k_norm"], cfg.offset, cfg.eps)
        v = qkv[:, nq + nkv:]
        cos, sin = tables[cfg.rope_global if (li + 1) % cfg.pattern == 0 else cfg.rope_local]
        q = rope(q, cos[pos], sin[pos])
        k = rope(k, cos[pos], sin[pos])
        k_cache[li][:, :, pos] = k
        v_cache[li][:, :, pos] = v
        ctx = np.zeros((B, nq, hd), F)
        for b in range(B):
            for hh in range(nq):
                kv = hh // (nq // nkv)
                s = (k_cache[li][b, kv, :pos + 1] @ q[b, hh]).astype(F) * inv_scale
                p = np.exp(s - s.max()).astype(F)
                p = (p / p.sum(dtype=F)).astype(F)
                ctx[b, hh] = p @ v_cache[li][b, kv, :pos + 1]
        o = matmul_f32_q4(ctx.ravel(), lw["o"], B, nq * hd, H).reshape(B, H)
        x = (x + rmsnorm(o, lw["post_attn_norm"], cfg.offset, cfg.eps)).astype(F)
        h2 = rmsnorm(x, lw["ffn_norm"], cfg.offset, cfg.eps)
        g = matmul_f32_q4(h2.ravel(), lw["gate"], B, H, cfg.ffn).reshape(B, cfg.ffn)
        u = matmul_f32_q4(h2.ravel(), lw["up"], B, H, cfg.ffn).reshape(B, cfg.ffn)
        f = (gelu(g) * u).astype(F)
        d = matmul_f32_q4(f.ravel(), lw["down"], B, cfg.ffn, H).reshape(B, H)
        x = (x + rmsnorm(d, lw["post_ffn_norm"], cfg.offset, cfg.eps)).astype(F)
    x = rmsnorm(x, w["final_norm"], cfg.offset, cfg.eps)
    return matmul_f32_q8(x.ravel(), w["emb"], B, H, cfg.vocab).reshape(B, cfg.vocab)
