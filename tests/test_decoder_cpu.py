"""Host-side pieces of the small decoder (RMSNorm, RoPE tables, weight
generation and quantization rule) and the oracle decoder's KV cache, on the
CPU."""
import numpy as np
import pytest
import torch

from riallm_b200 import decoder as D


def test_rms_norm_and_rope_match_numpy():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(5, 64, generator=g)
    w = torch.rand(64, generator=g) + 0.5
    y = D.rms_norm(x, w, 1e-5).double().numpy()
    xd = x.double().numpy()
    want = xd / np.sqrt((xd * xd).mean(-1, keepdims=True) + 1e-5) * w.double().numpy()
    assert np.abs(y - want).max() < 1e-5
    cos, sin = D.rope_tables(torch.arange(3, 7), 16, 1e6)
    assert cos.shape == (4, 8)
    q = torch.randn(2, 4, 16, generator=g)
    r = D.apply_rope(q, cos, sin)
    # rotation keeps the norm of each (i, i + d/2) pair
    a = q[..., :8] ** 2 + q[..., 8:] ** 2
    b = r[..., :8] ** 2 + r[..., 8:] ** 2
    assert torch.allclose(a, b, atol=1e-5)
    # position 0 is the identity
    c0, s0 = D.rope_tables(torch.zeros(1, dtype=torch.long), 16, 1e6)
    assert torch.equal(D.apply_rope(q[:, :1], c0, s0), q[:, :1])


def test_synthetic_weights_layout():
    cfg = D.DecoderConfig(layers=1, hidden=64, heads=4, kv_heads=2, head_dim=16, vocab=128, experts=4,
                          intermediate=32)
    w = D.synthetic_weights(cfg, seed=3, device="cpu")
    assert w["model.layers.0.mlp.experts.gate_up_proj"].shape == (4, 64, 64)
    assert w["model.layers.0.mlp.experts.down_proj"].shape == (4, 64, 32)
    assert w["model.layers.0.self_attn.k_proj.weight"].shape == (32, 64)
    assert torch.equal(w["model.norm.weight"], torch.ones(64))
    w2 = D.synthetic_weights(cfg, seed=3, device="cpu")
    assert all(torch.equal(w[k], w2[k]) for k in w)


def test_oracle_decoder_cache_matches_full_prefill():
    """Decoding token by token through the KV cache gives the logits of one
    prefill over the whole sequence (the oracle decoder, small config)."""
    from oracle import oracle as O
    from oracle.decoder_ref import DecoderRef
    O.build()
    cfg = D.DecoderConfig(layers=2, hidden=128, heads=4, kv_heads=2, head_dim=32, vocab=256, experts=4,
                          top_k=2, intermediate=64)
    w = D.synthetic_weights(cfg, seed=5, device="cpu")
    qw, shapes = {}, {}
    for k, v in w.items():
        if v.numel() >= 4096:
            qw[k] = O.quantize(v.numpy().reshape(-1), O.FOUR_BIT)
            shapes[k] = tuple(v.shape)
        else:
            qw[k] = v.numpy()
    ids = np.random.default_rng(2).integers(0, cfg.vocab, 9)
    full = DecoderRef(cfg, qw, shapes).forward(ids, 0)
    inc = DecoderRef(cfg, qw, shapes)
    part = inc.forward(ids[:6], 0)
    assert np.allclose(part, full[:6], rtol=0, atol=1e-9)
    for i in range(6, 9):
        row = inc.forward(ids[i:i + 1], i)[0]
        assert np.abs(row - full[i]).max() <= 2e-2 * np.abs(full[i]).max()
