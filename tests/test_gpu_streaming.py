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


def test_routed_streaming_decode_matches_resident(rb):
    """A decoder whose streamer copies, per decode step, only the experts
    the step's batch routes to (routers resident) produces the resident
    decoder's tokens and logits, and copies fewer bytes per step than whole
    layers. Prefills still copy whole layers."""
    from riallm_b200 import decoder as D
    from riallm_b200.streaming import LayerStreamer, PackedLayer
    cfg = D.DecoderConfig(layers=3)
    qw = D.synthetic_model(cfg, seed=7, device="cuda")
    names = ("mlp.gate.weight", "mlp.experts.gate_up_proj", "mlp.experts.down_proj")
    packed = [PackedLayer({n: qw[f"model.layers.{l}.{n}"] for n in names}) for l in range(cfg.layers)]
    st = LayerStreamer(packed, depth=2, routed=True)
    g = torch.Generator().manual_seed(3)
    prompt = torch.randint(0, cfg.vocab, (2, 20), generator=g).cuda()
    plain = D.Decoder(cfg, qw, max_batch=2, max_seq=64)
    t0, l0 = plain.generate(prompt, 5, keep_logits=True)
    plain.close()
    dec = D.Decoder(cfg, {k: v for k, v in qw.items() if ".mlp." not in k}, max_batch=2, max_seq=64, streamer=st)
    b0 = st.stats()["bytes"]
    dec.forward(prompt)  # prefill: whole layers
    b1 = st.stats()["bytes"]
    dec.reset()
    t1, l1 = dec.generate(prompt, 5, keep_logits=True)
    b2 = st.stats()["bytes"]
    dec.close()
    st.close()
    full = sum(p.nbytes for p in packed)
    for p in packed:
        p.close()
    assert b1 - b0 == full
    # generate = one prefill (full layers) + 4 routed decode steps
    assert b2 - b1 - full < 4 * full
    assert torch.equal(t0, t1)
    assert float((l1 - l0).abs().max() / l0.abs().max()) < 1e-5
