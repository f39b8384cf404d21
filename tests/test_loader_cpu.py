"""Mixtral-layout loading, the quantized-shard cache and the reference's
quant-state JSON, on the CPU (the oracle's quantizer stands in for the GPU
kernel, which the GPU tests cover)."""
import json
import os

import numpy as np
import pytest
import torch

from riallm_b200 import CompressionType, ModelLoadingError, QuantizedTensor
from riallm_b200 import loader as L


def _oracle_quantize(t, c):
    from oracle import oracle as O
    q = O.quantize(t.detach().float().numpy().reshape(-1), int(c))
    return QuantizedTensor(torch.from_numpy(q.data.copy()), tuple(t.shape), CompressionType(int(c)),
                           torch.from_numpy(q.scales.copy()), torch.from_numpy(q.zero_points.copy()), q.block_size)


def test_safetensors_round_trip(tmp_path):
    g = torch.Generator().manual_seed(0)
    t = {"a": torch.randn(3, 5, generator=g), "b": torch.randn(7, generator=g).to(torch.bfloat16),
         "c": torch.randint(0, 255, (11,), dtype=torch.uint8, generator=g), "d": torch.arange(4, dtype=torch.int64),
         "empty": torch.empty(0, 4)}
    p = str(tmp_path / "x.safetensors")
    L.write_safetensors(p, t, {"k": "v"})
    back = L.read_safetensors(p)
    assert set(back) == set(t)
    for k in t:
        assert back[k].dtype == t[k].dtype and back[k].shape == t[k].shape and torch.equal(back[k], t[k])
    assert L.read_safetensors_metadata(p) == {"k": "v"}
    assert set(L.read_safetensors(p, ["a"])) == {"a"}
    with open(p, "rb") as f:
        n = int.from_bytes(f.read(8), "little")
    assert n % 8 == 0


def _fake_mixtral(tmp_path, E=4, H=256, I=128, layers=2):
    g = torch.Generator().manual_seed(1)
    ref = {}
    files = {}
    for l in range(layers):
        base = f"model.layers.{l}.block_sparse_moe"
        shard = {f"{base}.gate.weight": torch.randn(E, H, generator=g).to(torch.bfloat16)}
        for e in range(E):
            for w, shape in (("w1", (I, H)), ("w3", (I, H)), ("w2", (H, I))):
                shard[f"{base}.experts.{e}.{w}.weight"] = (0.02 * torch.randn(*shape, generator=g)).to(torch.bfloat16)
        fn = f"model-{l:05d}.safetensors"
        L.write_safetensors(str(tmp_path / fn), shard)
        files.update({k: fn for k in shard})
        ref[l] = shard
    with open(tmp_path / "model.safetensors.index.json", "w") as f:
        json.dump({"metadata": {}, "weight_map": files}, f)
    return ref


def test_mixtral_mapping_to_fused_layout(tmp_path):
    E, H, I = 4, 256, 128
    ref = _fake_mixtral(tmp_path, E, H, I)
    idx = L.CheckpointIndex(str(tmp_path))
    t = L.mixtral_moe_layer(idx, 1, E)
    base = "model.layers.1.block_sparse_moe"
    assert t["mlp.gate.weight"].shape == (E, H)
    assert t["mlp.experts.gate_up_proj"].shape == (E, 2 * I, H)
    assert t["mlp.experts.down_proj"].shape == (E, H, I)
    for e in range(E):
        assert torch.equal(t["mlp.experts.gate_up_proj"][e, :I], ref[1][f"{base}.experts.{e}.w1.weight"].float())
        assert torch.equal(t["mlp.experts.gate_up_proj"][e, I:], ref[1][f"{base}.experts.{e}.w3.weight"].float())
        assert torch.equal(t["mlp.experts.down_proj"][e], ref[1][f"{base}.experts.{e}.w2.weight"].float())
    # Without an index file the shards are scanned.
    os.remove(tmp_path / "model.safetensors.index.json")
    t2 = L.mixtral_moe_layer(L.CheckpointIndex(str(tmp_path)), 1, E)
    assert torch.equal(t2["mlp.experts.down_proj"], t["mlp.experts.down_proj"])
    with pytest.raises(ModelLoadingError, match="Tensor not found"):
        L.mixtral_moe_layer(idx, 5, E)


@pytest.mark.parametrize("qt", [CompressionType.FourBit, CompressionType.EightBit])
def test_quantized_shard_cache(tmp_path, qt):
    E, H, I = 4, 256, 128
    _fake_mixtral(tmp_path / "ckpt", E, H, I)
    idx = L.CheckpointIndex(str(tmp_path / "ckpt"))
    cache = L.QuantizedShardCache(str(tmp_path / "cache"), qt, quantize=_oracle_quantize)
    calls = []

    def src():
        calls.append(1)
        return L.mixtral_moe_layer(idx, 0, E)
    a = cache.layer(0, src)
    assert calls == [1] and cache.has(0)
    b = cache.layer(0, src)  # hit: no second quantization
    assert calls == [1]
    for name in ("mlp.experts.gate_up_proj", "mlp.experts.down_proj"):
        qa, qb = a[name], b[name]
        assert qb.qtype == qt and qb.shape == qa.shape and qb.block_size == qa.block_size
        assert torch.equal(qa.data, qb.data) and torch.equal(qa.scales, qb.scales)
        assert torch.equal(qa.zero_points, qb.zero_points)
    # the router weight (E*H = 1024 < 4096 elements) is kept as it is
    assert not isinstance(b["mlp.gate.weight"], QuantizedTensor)


def test_quant_state_json_matches_reference_format(tmp_path):
    q = _oracle_quantize(torch.randn(64 * 70), CompressionType.FourBit)
    p = str(tmp_path / "state.json")
    L.save_quant_state({"w": q}, p)
    with open(p) as f:
        d = json.load(f)
    assert set(d["w"]) == {"shape", "qtype", "scales", "zero_points", "block_size"}
    assert d["w"]["qtype"] == "FourBit" and d["w"]["block_size"] == 64
    back = L.load_quant_state(p)
    assert back["w"].qtype == CompressionType.FourBit
    assert np.array_equal(back["w"].scales.numpy(), q.scales.numpy())
    # The reference's loader ignores the stored qtype (always EightBit).
    assert L.load_quant_state(p, honor_qtype=False)["w"].qtype == CompressionType.EightBit
    assert L.load_quant_state(str(tmp_path / "missing.json")) == {}


def test_truncated_files_are_loading_errors(tmp_path):
    """A shard or quant-state file cut short (an interrupted write or copy)
    raises ModelLoadingError naming the file, never a bare decode error."""
    E, H, I = 4, 256, 128
    _fake_mixtral(tmp_path / "ckpt", E, H, I, layers=1)
    shard = tmp_path / "ckpt" / "model-00000.safetensors"
    full = shard.read_bytes()
    for cut in (4, 12, len(full) // 2, len(full) - 1):
        shard.write_bytes(full[:cut])
        with pytest.raises(ModelLoadingError, match="safetensors"):
            L.read_safetensors(str(shard))
    shard.write_bytes(full[:len(full) - 1])
    idx = L.CheckpointIndex(str(tmp_path / "ckpt"))
    with pytest.raises(ModelLoadingError, match="truncated"):
        L.mixtral_moe_layer(idx, 0, E)
    # A cached quantized shard cut short is refused too.
    shard.write_bytes(full)
    cache = L.QuantizedShardCache(str(tmp_path / "cache"), CompressionType.FourBit, quantize=_oracle_quantize)
    cache.layer(0, lambda: L.mixtral_moe_layer(L.CheckpointIndex(str(tmp_path / "ckpt")), 0, E))
    cp = cache.path(0)
    data = open(cp, "rb").read()
    with open(cp, "wb") as f:
        f.write(data[:-100])
    with pytest.raises(ModelLoadingError, match="truncated"):
        cache.load(0)
    q = _oracle_quantize(torch.randn(64 * 70), CompressionType.FourBit)
    p = str(tmp_path / "state.json")
    L.save_quant_state({"w": q}, p)
    text = open(p).read()
    with open(p, "w") as f:
        f.write(text[:len(text) // 2])
    with pytest.raises(ModelLoadingError, match="quant-state"):
        L.load_quant_state(p)
