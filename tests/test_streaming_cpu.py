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


def _qe(E, rows, cols, seed):
    """A NF4 expert tensor [E, rows, cols] with random codes and parameters."""
    n = E * rows * cols
    g = torch.Generator().manual_seed(seed)
    return QuantizedTensor(torch.randint(0, 256, (n // 2,), dtype=torch.uint8, generator=g), (E, rows, cols),
                           CompressionType.FourBit, torch.rand(n // 64, generator=g), torch.rand(n // 64, generator=g),
                           64)


def test_expert_ranges_cover_routed_experts_and_next_parameters():
    """Copying only the ranges of experts {1, 3} of a 4-expert layer into an
    empty buffer reproduces those experts' codes, scales and zero points,
    and the first scale / zero point of the expert after each (the NF4 decode
    reads it for the last element of the expert's last block), and nothing
    else."""
    E = 4
    t = {"mlp.gate.weight": torch.randn(E, 128), "mlp.experts.gate_up_proj": _qe(E, 64, 128, 3),
         "mlp.experts.down_proj": _qe(E, 128, 32, 4)}
    p = PackedLayer(t, pinned=False)
    offs, sizes = p.expert_ranges([3, 1, 1])
    buf = torch.zeros_like(p.blob)
    for o, n in zip(offs, sizes):
        buf[o:o + n] = p.blob[o:o + n]
    v = p.views(buf)
    for name in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
        a, b = v[name], t[name]
        per_d = b.data.numel() // E
        per_p = b.scales.numel() // E
        for e in range(E):
            d_a, d_b = a.data[e * per_d:(e + 1) * per_d], b.data[e * per_d:(e + 1) * per_d]
            s_a, s_b = a.scales[e * per_p:(e + 1) * per_p], b.scales[e * per_p:(e + 1) * per_p]
            z_a, z_b = a.zero_points[e * per_p:(e + 1) * per_p], b.zero_points[e * per_p:(e + 1) * per_p]
            if e in (1, 3):
                assert torch.equal(d_a, d_b) and torch.equal(s_a, s_b) and torch.equal(z_a, z_b)
            elif e == 2:  # only its first parameters ride along with expert 1
                assert not d_a.any()
                assert s_a[0] == s_b[0] and z_a[0] == z_b[0] and not s_a[1:].any() and not z_a[1:].any()
            else:
                assert not d_a.any() and not s_a.any() and not z_a.any()
    assert not v["mlp.gate.weight"].any()  # the router is not part of the ranges
