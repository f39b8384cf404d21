"""Layer packing for the streamer (host side, no GPU): every part lands
256-byte aligned in one blob and reads back unchanged."""
import torch

from riallm_b200 import CompressionType, QuantizedTensor
from riallm_b200.streaming import ALIGN, PackedLayer


def _q(n, seed):
    g = torch.Generator().manual_seed(seed)
    data = torch.randint(0, 256, (n // 2,), dtype=torch.uint8, generator=g)
    scales = torch.rand(n // 64, generator=g)
    zeros = torch.rand(n // 64, generator=g)
    return QuantizedTensor(data, (n // 256, 256), CompressionType.FourBit, scales, zeros, 64)


def test_packed_layer_round_trip():
    t = {"mlp.gate.weight": torch.randn(8, 256), "mlp.experts.gate_up_proj": _q(8 * 512 * 256, 1),
         "mlp.experts.down_proj": _q(8 * 256 * 256 + 64, 2)}
    p = PackedLayer(t, pinned=False)
    assert p.nbytes % ALIGN == 0
    for e in p.index.values():
        for off, nb in e.parts:
            assert off % ALIGN == 0 and off + nb <= p.nbytes
    v = p.views(p.blob)
    assert torch.equal(v["mlp.gate.weight"], t["mlp.gate.weight"])
    for name in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
        a, b = v[name], t[name]
        assert a.shape == b.shape and a.qtype == b.qtype and a.block_size == b.block_size
        assert torch.equal(a.data, b.data) and torch.equal(a.scales, b.scales)
        assert torch.equal(a.zero_points, b.zero_points)
