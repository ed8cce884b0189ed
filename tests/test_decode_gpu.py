"""Gemma-3 decode step on the GPU (machinelearning_b200/decode.py) against the
oracle's restatement of the reference's forward pass with a KV cache
(oracle/decode.py), on the same quantised block bytes: a small model of the
Gemma-3 shape (6 layers so that layer 5 takes the global RoPE base, 4 query
heads sharing 1 KV head, sandwich norms, GeGLU, tied Q8_0 embedding), several
consecutive positions, batch 3. Logits within the 1e-3 contract."""
from __future__ import annotations

import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

Q4_0, Q8_0 = 2, 8


def small_config(hidden=256):
    from machinelearning_b200.decode import Gemma3Config
    return Gemma3Config(hidden=hidden, n_layers=6, n_heads=4, n_kv_heads=1, head_dim=64, ffn=512, vocab=640, ctx=16,
                        emb_scale=float(np.float32(math.sqrt(float(hidden)))))


def host_weights(oracle, cfg, seed):
    rng = np.random.default_rng(seed)
    H, nq, nkv, hd = cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim
    q4 = lambda n, k: oracle.quantize_q4_0(rng.normal(0, 0.05, n * k).astype(np.float32))  # noqa: E731
    norm = lambda n: rng.normal(0, 0.1, n).astype(np.float32)  # noqa: E731
    w = {"emb": oracle.quantize_q8_0(rng.normal(0, 0.05, cfg.vocab * H).astype(np.float32)),
         "final_norm": norm(H), "layers": []}
    for _ in range(cfg.n_layers):
        w["layers"].append({
            "qkv": q4((nq + 2 * nkv) * hd, H), "o": q4(H, nq * hd), "gate": q4(cfg.ffn, H), "up": q4(cfg.ffn, H),
            "down": q4(H, cfg.ffn), "attn_norm": norm(H), "post_attn_norm": norm(H), "ffn_norm": norm(H),
            "post_ffn_norm": norm(H), "q_norm": norm(hd), "k_norm": norm(hd)})
    return w


@pytest.fixture(scope="module")
def torch_cuda():
    import torch
    assert torch.cuda.is_available()
    return torch


# (graph, batch, hidden): batch 20 with hidden 288 (9 blocks a row) runs the
# hidden-state matmuls on the tensor-core GEMM over zero-padded 16-byte rows
# fused: QK-norm / RoPE / cache append inside the attention kernel, or the
# separate kernels (both C-ABI forms)
@pytest.mark.parametrize("use_graph,B,hidden,fused", [(False, 3, 256, True), (True, 3, 256, True),
                                                      (True, 20, 288, True), (False, 3, 256, False),
                                                      (True, 20, 288, False), (True, 1, 288, True)])
def test_decode_steps_match_oracle(oracle, torch_cuda, use_graph, B, hidden, fused):
    from conftest import assert_close_rel
    from oracle.decode import decode_step

    from machinelearning_b200.decode import Gemma3Decoder
    cfg = small_config(hidden)
    w = host_weights(oracle, cfg, seed=11)
    model = Gemma3Decoder(cfg, w, batch=B, fused_attention=fused)
    assert model.kh == (512 if B == 20 else hidden)
    assert model.klm == (512 if hidden == 288 and B in (1, 20) else hidden)  # batch 1: padded lm_head only
    kc = [np.zeros((B, cfg.n_kv_heads, cfg.ctx, cfg.head_dim), np.float32) for _ in range(cfg.n_layers)]
    vc = [np.zeros_like(kc[0]) for _ in range(cfg.n_layers)]
    rng = np.random.default_rng(12)
    model.set_position(0)
    if use_graph:
        model.capture()
    for pos in range(5):
        tokens = rng.integers(0, cfg.vocab, B)
        got = model.step(tokens).cpu().numpy()
        ref = decode_step(cfg, w, tokens, pos, kc, vc)
        # norm-wise 1e-3 always; per element, the GEMM path (f16-rounded
        # operands, outliers ~4e-3 of the rms per matmul) compounds over the
        # layers, so its guard is 1e-2 of the rms
        assert_close_rel(got.ravel(), ref.ravel(), 1e-3, 1e-2 if model.kh != hidden else None)
    assert int(model.pos.item()) == 5
    model.close()


def test_decode_cache_and_attention_pieces(oracle, torch_cuda):
    """The cache after a step holds the reference's normed, rotated k and raw v
    at the step's position (and nothing elsewhere)."""
    from oracle.decode import decode_step

    from machinelearning_b200.decode import Gemma3Decoder
    cfg = small_config()
    w = host_weights(oracle, cfg, seed=21)
    B = 2
    model = Gemma3Decoder(cfg, w, batch=B)
    kc = [np.zeros((B, cfg.n_kv_heads, cfg.ctx, cfg.head_dim), np.float32) for _ in range(cfg.n_layers)]
    vc = [np.zeros_like(kc[0]) for _ in range(cfg.n_layers)]
    tokens = np.array([5, 600])
    model.set_position(3)
    model.step(tokens)
    decode_step(cfg, w, tokens, 3, kc, vc)
    k_dev = model.k_cache.cpu().numpy()
    v_dev = model.v_cache.cpu().numpy()
    for li in range(cfg.n_layers):
        np.testing.assert_allclose(k_dev[li], kc[li], rtol=2e-3, atol=2e-4)
        np.testing.assert_allclose(v_dev[li], vc[li], rtol=2e-3, atol=2e-4)
    assert not k_dev[:, :, :, :3].any() and not k_dev[:, :, :, 4:].any()
    model.close()


# ---- BASELINE configs[3] at its own shapes --------------------------------------------------
# Gemma-3-1B: 26 layers, hidden 1152, 4 query heads / 1 KV head of 256, GeGLU
# 6912, tied Q8_0 vocabulary 262144, KV context 512. The cache is pre-filled
# with the same random keys/values on both sides (positions before the step),
# so a step at position p attends over p + 1 entries: p = 0 (one entry), 31 /
# 32 (either side of a 32-position attention chunk), 511 (the full context,
# 16 chunks). Batch 1 runs the resident / band GEMVs and the 262144-row padded
# lm_head, batch 16 the two-token-tile GEMVs, batch 64 the f16 tensor-core GEMM
# on the unpadded K = 1152 rows (paired-row view; exact activations, d*q
# rounded to f16 once: ~2e-4 norm-wise per matmul). The logits and the cache
# rows the step writes meet the 1e-3 norm-wise contract at every batch; per
# element, batch 64's weight rounding compounds over 26 layers (measured up to
# ~5e-3 of the rms on B200), so its guard is 1e-2 of the rms, as for the other
# GEMM-path decode test.

@pytest.fixture(scope="module")
def gemma_1b(torch_cuda, oracle):
    from machinelearning_b200.decode import Gemma3Config, random_weights
    cfg = Gemma3Config.gemma3_1b(ctx=512)
    w = random_weights(cfg, seed=4242, device=0)
    host = {"emb": w["emb"].cpu().numpy(), "final_norm": w["final_norm"].cpu().numpy(),
            "layers": [{k: v.cpu().numpy() for k, v in lw.items()} for lw in w["layers"]]}
    return cfg, w, host


def _prefill_cache(cfg, B, pos, seed):
    """Random cache contents for positions < pos (zero elsewhere), shaped
    [layers][B][n_kv][ctx][head_dim] like the decoder's cache."""
    rng = np.random.default_rng(seed)
    shape = (cfg.n_layers, B, cfg.n_kv_heads, cfg.ctx, cfg.head_dim)
    k = np.zeros(shape, np.float32)
    v = np.zeros(shape, np.float32)
    if pos:
        k[:, :, :, :pos] = rng.standard_normal((cfg.n_layers, B, cfg.n_kv_heads, pos, cfg.head_dim), np.float32)
        v[:, :, :, :pos] = rng.standard_normal((cfg.n_layers, B, cfg.n_kv_heads, pos, cfg.head_dim),
                                               np.float32) * np.float32(0.7)
    return k, v


@pytest.mark.parametrize("B,positions", [(1, (0, 31, 32, 511)), (16, (0, 31, 511)), (64, (32, 511))])
def test_gemma3_1b_decode_at_config_shapes(gemma_1b, torch_cuda, oracle, B, positions):
    from conftest import assert_close_rel
    from oracle.decode import decode_step

    from machinelearning_b200.decode import Gemma3Decoder
    cfg, w, host = gemma_1b
    model = Gemma3Decoder(cfg, w, batch=B)
    rng = np.random.default_rng(77 + B)
    try:
        for pos in positions:
            kc, vc = _prefill_cache(cfg, B, pos, seed=1000 * B + pos)
            model.k_cache.copy_(torch_cuda.from_numpy(kc))
            model.v_cache.copy_(torch_cuda.from_numpy(vc))
            model.set_position(pos)
            tokens = rng.integers(0, cfg.vocab, B)
            got = model.step(tokens).cpu().numpy()
            ref = decode_step(cfg, host, tokens, pos, list(kc), list(vc))
            rel = assert_close_rel(got.ravel(), ref.ravel(), 1e-3, 1e-2 if B > 16 else None)
            print(f"batch {B} position {pos}: norm-wise relative error {rel:.2e}")
            # the step wrote the reference's k (normed, rotated) and v at the position
            for dcache, hcache in ((model.k_cache, kc), (model.v_cache, vc)):
                assert_close_rel(dcache[:, :, :, pos].cpu().numpy().ravel(), hcache[:, :, :, pos].ravel(), 1e-3,
                                 1e-2 if B > 16 else None)
    finally:
        model.close()
