"""AutoModel.from_pretrained on a Mixtral-layout checkpoint written to disk
(config.json + safetensors shards with riallm's tensor names), against a
Decoder built in memory from the same weights: identical greedy tokens,
resident (prefetch_layers=false) and streamed (prefetch_layers=true,
prefetch_buffer_size=2) alike, and the quantized-shard cache reused on a
second load."""
import json
import os

import pytest
import torch

pytestmark = pytest.mark.gpu


def _write_checkpoint(path, cfg, w):
    """Mixtral names (block_sparse_moe.experts.e.w1/w3/w2) from the fused
    synthetic layout, bf16 like a released checkpoint, two shards and an
    index."""
    from riallm_b200.loader import write_safetensors
    I = cfg.intermediate
    shards = [{}, {}]
    for name, t in w.items():
        if name.endswith("mlp.experts.gate_up_proj") or name.endswith("mlp.experts.down_proj"):
            continue
        dst = name.replace(".mlp.gate.weight", ".block_sparse_moe.gate.weight")
        shards[0 if "layers.0." in name or "embed" in name else 1][dst] = t.to(torch.bfloat16).cpu()
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        gu, dn = w[p + "mlp.experts.gate_up_proj"], w[p + "mlp.experts.down_proj"]
        for e in range(cfg.experts):
            base = p + f"block_sparse_moe.experts.{e}."
            shards[l % 2][base + "w1.weight"] = gu[e, :I].to(torch.bfloat16).cpu()
            shards[l % 2][base + "w3.weight"] = gu[e, I:].to(torch.bfloat16).cpu()
            shards[l % 2][base + "w2.weight"] = dn[e].to(torch.bfloat16).cpu()
    wmap = {}
    for i, sh in enumerate(shards):
        fn = f"model-{i + 1:05d}-of-00002.safetensors"
        write_safetensors(os.path.join(path, fn), sh)
        wmap.update({k: fn for k in sh})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wmap}, f)
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({"model_type": "mixtral", "vocab_size": cfg.vocab, "hidden_size": cfg.hidden,
                   "num_hidden_layers": cfg.layers, "num_attention_heads": cfg.heads,
                   "num_key_value_heads": cfg.kv_heads, "intermediate_size": cfg.intermediate,
                   "max_position_embeddings": 4096, "rms_norm_eps": cfg.eps, "rope_theta": cfg.theta,
                   "num_local_experts": cfg.experts, "num_experts_per_tok": cfg.top_k}, f)


def test_from_pretrained_matches_in_memory_model(rb, tmp_path):
    from riallm_b200 import decoder as D
    from riallm_b200.auto_model import AutoModel
    cfg = D.DecoderConfig(vocab=4096)
    w = D.synthetic_weights(cfg, seed=0)
    # What the checkpoint holds: bf16 values (read back as float32).
    w = {k: (v if "norm" in k else v.to(torch.bfloat16).float()) for k, v in w.items()}
    _write_checkpoint(str(tmp_path), cfg, w)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab, (32,), generator=g)

    ref = D.Decoder(cfg, D.quantize_weights(w))
    want = prompt.tolist() + ref.generate(prompt.cuda(), 8)
    ref.close()

    opts = rb.ModelOptions(compression=rb.CompressionType.FourBit, prefetch_layers=False)
    m = AutoModel.from_pretrained(str(tmp_path), opts, cache_dir=str(tmp_path / "q"))
    assert m.config.num_experts() == cfg.experts and m.streamer is None
    assert m.generate(prompt, 8, 0.7, 0.9) == want
    m.close()
    assert os.path.exists(tmp_path / "q" / "layer_1.fourbit.safetensors")

    opts = rb.ModelOptions(compression=rb.CompressionType.FourBit, prefetch_layers=True, prefetch_buffer_size=2)
    m = AutoModel.from_pretrained(str(tmp_path), opts, cache_dir=str(tmp_path / "q"))  # cache hit
    assert m.streamer is not None and m.streamer.depth == 2
    assert m.generate(prompt, 8) == want
    st = m.stream_stats()
    # every forward streams each layer's MoE tensors once: a prefill + 7 decode steps
    assert st["copies"] == 8 * cfg.layers and st["bytes"] > 0
    m.close()

    # Routed streaming: decode steps copy only the experts they route to.
    m = AutoModel.from_pretrained(str(tmp_path), opts, cache_dir=str(tmp_path / "q"), routed_streaming=True)
    assert m.streamer.routed
    assert m.generate(prompt, 8) == want
    st2 = m.stream_stats()
    assert st2["copies"] == 8 * cfg.layers and st2["bytes"] < st["bytes"]
    m.close()
