"""Layer streaming on the GPU: blocks computed from streamed weights equal
those computed from resident weights bit for bit, the copies are accounted
for, and misuse of the slot ring is refused."""
import pytest
import torch

pytestmark = pytest.mark.gpu

H, I, E, K = 512, 512, 8, 2


def _layer_host(rb, seed):
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(seed)
    out = {}
    for name, shape in [("mlp.gate.weight", (E, H)), ("mlp.experts.gate_up_proj", (E, 2 * I, H)),
                        ("mlp.experts.down_proj", (E, H, I))]:
        q = rb.quantize_tensor(torch.empty(shape, device=dev).normal_(0.0, 0.02, generator=gen),
                               rb.CompressionType.FourBit)
        out[name] = rb.QuantizedTensor(q.data.cpu(), q.shape, q.qtype, q.scales.cpu(), q.zero_points.cpu(),
                                       q.block_size)
    return out


def _to_dev(rb, t):
    return {n: rb.QuantizedTensor(q.data.cuda(), q.shape, q.qtype, q.scales.cuda(), q.zero_points.cuda(),
                                  q.block_size) for n, q in t.items()}


@pytest.mark.parametrize("depth,n_layers", [(2, 5), (1, 3), (3, 3)])
def test_streamed_layers_match_resident(rb, depth, n_layers):
    from riallm_b200.streaming import LayerStreamer, PackedLayer
    host = [_layer_host(rb, 100 + i) for i in range(n_layers)]
    x = torch.randn(16, H, device="cuda").to(torch.bfloat16)
    ref = [rb.apply_moe(_to_dev(rb, t), x, K, E) for t in host]
    packed = [PackedLayer(t) for t in host]
    s = LayerStreamer(packed, depth=depth)
    outs = {}

    def fn(i, t):
        outs[i] = rb.apply_moe(t, x, K, E)
    s.run(fn)
    s.run(fn)  # a second pass reuses the ring
    torch.cuda.synchronize()
    for i in range(n_layers):
        assert torch.equal(outs[i], ref[i]), i
    st = s.stats()
    assert st["copies"] == 2 * n_layers
    assert st["bytes"] == 2 * sum(p.nbytes for p in packed)
    assert st["h2d_gbs"] > 0
    s.close()
    for p in packed:
        p.close()


def test_streamer_refuses_misuse(rb):
    from riallm_b200.streaming import LayerStreamer, PackedLayer
    packed = [PackedLayer(_layer_host(rb, 7)) for _ in range(3)]
    s = LayerStreamer(packed, depth=2)
    with pytest.raises(rb.ConfigError):
        s.acquire(0)          # not prefetched
    s.prefetch(0)
    s.prefetch(1)
    with pytest.raises(rb.ConfigError):
        s.prefetch(2)         # slot 0 still holds layer 0
    s.acquire(0)
    s.release(0)
    s.prefetch(2)             # now allowed
    s.acquire(1)
    s.release(1)
    s.acquire(2)
    s.release(2)
    torch.cuda.synchronize()
    s.close()
    for p in packed:
        p.close()
