"""Mixtral checkpoint -> fused layout -> GPU quantization -> shard cache ->
MoE block: the cached layer gives the same block output, bit for bit, as
quantizing the fused tensors directly."""
import pytest
import torch

from riallm_b200 import loader as L

pytestmark = pytest.mark.gpu


def test_cached_mixtral_layer_runs_the_block(rb, tmp_path):
    E, H, I, k = 8, 512, 512, 2
    g = torch.Generator().manual_seed(3)
    base = "model.layers.0.block_sparse_moe"
    shard = {f"{base}.gate.weight": (0.02 * torch.randn(E, H, generator=g)).to(torch.bfloat16)}
    for e in range(E):
        shard[f"{base}.experts.{e}.w1.weight"] = (0.02 * torch.randn(I, H, generator=g)).to(torch.bfloat16)
        shard[f"{base}.experts.{e}.w3.weight"] = (0.02 * torch.randn(I, H, generator=g)).to(torch.bfloat16)
        shard[f"{base}.experts.{e}.w2.weight"] = (0.02 * torch.randn(H, I, generator=g)).to(torch.bfloat16)
    L.write_safetensors(str(tmp_path / "ckpt" / "model.safetensors"), shard)
    idx = L.CheckpointIndex(str(tmp_path / "ckpt"))
    fused = L.mixtral_moe_layer(idx, 0, E)
    cache = L.QuantizedShardCache(str(tmp_path / "cache"), rb.CompressionType.FourBit)
    cache.layer(0, lambda: fused)
    loaded = cache.load(0)

    def dev(t):
        if isinstance(t, rb.QuantizedTensor):
            return rb.QuantizedTensor(t.data.cuda(), t.shape, t.qtype, t.scales.cuda(), t.zero_points.cuda(),
                                      t.block_size)
        return t.cuda()
    direct = {n: (rb.quantize_tensor(t.cuda(), rb.CompressionType.FourBit) if t.numel() >= 4096 else t.cuda())
              for n, t in fused.items()}
    x = torch.randn(24, H, device="cuda").to(torch.bfloat16)
    a = rb.apply_moe({n: dev(t) for n, t in loaded.items()}, x, k, E)
    b = rb.apply_moe(direct, x, k, E)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
