"""GPU parity of quantize / dequantize (src/quantization.rs) against the
oracle: bit-exact codes, scales, zero points and dequantized values."""
import numpy as np
import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def f32bits(t):
    return t.detach().cpu().numpy().view(np.uint32)


@pytest.fixture(scope="module")
def golden():
    return load_golden("quant.npz")


@pytest.mark.parametrize("qname,qt", [("nf4", 1), ("int8", 2)])
def test_quantize_dequantize_golden_bit_exact(rb, golden, qname, qt):
    for key in [k for k in golden if k.startswith("v_")]:
        n = int(key[2:])
        v = torch.from_numpy(golden[key]).cuda()
        q = rb.quantize_tensor(v, rb.CompressionType(qt))
        torch.cuda.synchronize()
        assert np.array_equal(q.data.cpu().numpy(), golden[f"{qname}_data_{n}"]), n
        assert np.array_equal(f32bits(q.scales), golden[f"{qname}_scales_{n}"].view(np.uint32)), n
        assert np.array_equal(f32bits(q.zero_points), golden[f"{qname}_zeros_{n}"].view(np.uint32)), n
        d = q.dequantize(torch.float32)
        assert np.array_equal(f32bits(d), golden[f"{qname}_deq_{n}"].view(np.uint32)), n
        db = q.dequantize(torch.bfloat16)
        assert torch.equal(db, d.to(torch.bfloat16)), n


@pytest.mark.parametrize("n", [1 << 22, (1 << 22) + 37])
@pytest.mark.parametrize("qt", [1, 2])
def test_large_tensor_matches_oracle(rb, oracle_lib, n, qt):
    O = oracle_lib
    rng = np.random.default_rng(n + qt)
    v = rng.normal(0, 0.02, n).astype(np.float32)
    ref = O.quantize(v, qt)
    q = rb.quantize_tensor(torch.from_numpy(v).cuda(), rb.CompressionType(qt))
    assert np.array_equal(q.data.cpu().numpy(), ref.data)
    assert np.array_equal(f32bits(q.scales), ref.scales.view(np.uint32))
    assert np.array_equal(f32bits(q.zero_points), ref.zero_points.view(np.uint32))
    assert np.array_equal(f32bits(q.dequantize()), O.dequantize(ref).view(np.uint32))


def test_codebook_mode(rb, oracle_lib):
    O = oracle_lib
    rng = np.random.default_rng(3)
    v = rng.normal(0, 0.5, 5000).astype(np.float32)
    q4 = rb.quantize_tensor(torch.from_numpy(v).cuda(), rb.CompressionType.FourBit)
    d = q4.dequantize(codebook=True).cpu().numpy()
    data = q4.data.cpu().numpy()
    e = np.arange(v.size)
    codes = np.where(e & 1, data[e >> 1] >> 4, data[e >> 1] & 15)
    b = np.minimum((e + 1) // 64, q4.scales.numel() - 1)
    scales = q4.scales.cpu().numpy()
    s = np.where((e + 1) // 64 < scales.size, scales[b], np.float32(1.0))
    assert np.array_equal(d.view(np.uint32), (O.NF4_TABLE[codes] * s).astype(np.float32).view(np.uint32))
    q8 = rb.quantize_tensor(torch.from_numpy(v).cuda(), rb.CompressionType.EightBit)
    d8 = q8.dequantize(codebook=True).cpu().numpy()
    c8 = q8.data.cpu().numpy().astype(np.float32)
    s8 = q8.scales.cpu().numpy()[e // 128]
    z8 = q8.zero_points.cpu().numpy()[e // 128]
    assert np.array_equal(d8.view(np.uint32), ((c8 * s8).astype(np.float32) + z8).astype(np.float32).view(np.uint32))


def test_compress_layer_state_dict_threshold(rb):
    """src/quantization.rs:289-296: only tensors with >= 4096 elements."""
    sd = {"big": torch.randn(64, 64, device="cuda"), "small": torch.randn(4095, device="cuda")}
    comp, meta = rb.compress_layer_state_dict(sd, rb.CompressionType.FourBit)
    assert set(meta) == {"big"} and comp["small"] is sd["small"]
    assert comp["big"].dtype == torch.uint8 and comp["big"].numel() == 2048
    back = rb.dequantize_layer_state_dict(comp, meta)
    assert back["big"].shape == (64, 64)


def test_errors(rb):
    with pytest.raises(rb.QuantizationError):
        rb.quantize_tensor(torch.randn(8, device="cuda"), rb.CompressionType.None_)
