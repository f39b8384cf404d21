"""Mixtral-layout MoE weight loading and a quantized-shard cache.

riallm has no mapping from Hugging Face Mixtral checkpoints to its fused
expert layout, and its `compress_layer_state_dict` / `save_quant_state`
(src/quantization.rs:278-381) are never wired into loading. This module:

* reads safetensors files (the format `SafetensorModelPersister` uses,
  src/persistence.rs:23-116) with a small reader of its own (the
  `safetensors` package is not required);
* maps a Mixtral layer's `block_sparse_moe` tensors onto the fused layout
  the MoE block takes: `mlp.gate.weight` [E,H] from `gate.weight`,
  `mlp.experts.gate_up_proj` [E,2I,H] with rows 0..I-1 from `experts.e.w1`
  (gate) and rows I..2I-1 from `experts.e.w3` (up), and
  `mlp.experts.down_proj` [E,H,I] from `experts.e.w2`;
* quantizes a layer once and caches it on disk (one safetensors shard per
  layer: uint8 codes, float32 scales and zero points, shapes and qtypes in
  the header metadata), so later loads skip quantization;
* writes and reads the reference's `save_quant_state` JSON.
"""
from __future__ import annotations

import json
import os
import struct
from typing import Callable, Dict, Iterable, Mapping, Optional

import numpy as np
import torch

from . import CompressionType, ModelLoadingError, QuantizationError, QuantizedTensor, TensorLike

# safetensors dtype names <-> torch dtypes
_DT = {"F32": torch.float32, "F16": torch.float16, "BF16": torch.bfloat16, "I64": torch.int64,
       "I32": torch.int32, "U8": torch.uint8, "I8": torch.int8, "BOOL": torch.bool}
_DT_INV = {v: k for k, v in _DT.items()}


def _read_header(f, path: str):
    """The JSON header of an open safetensors file and the data offset.
    A file cut short (or not a safetensors file) is a ModelLoadingError."""
    size = os.fstat(f.fileno()).st_size
    raw = f.read(8)
    if len(raw) < 8:
        raise ModelLoadingError(f"truncated safetensors file (no header length): {path}")
    (n,) = struct.unpack("<Q", raw)
    if n > size - 8:
        raise ModelLoadingError(f"truncated safetensors file (header of {n} bytes, file of {size}): {path}")
    try:
        header = json.loads(f.read(n))
    except (ValueError, UnicodeDecodeError) as exc:
        raise ModelLoadingError(f"corrupt safetensors header in {path}: {exc}") from None
    return header, 8 + n, size


def read_safetensors(path: str, names: Optional[Iterable[str]] = None) -> Dict[str, torch.Tensor]:
    """Tensors of a safetensors file (all, or those named), on the CPU.
    Raises ModelLoadingError when the file is shorter than its header says
    (a shard cut off mid-write or mid-copy)."""
    with open(path, "rb") as f:
        header, base, size = _read_header(f, path)
        want = set(names) if names is not None else None
        out = {}
        for name, info in header.items():
            if name == "__metadata__" or (want is not None and name not in want):
                continue
            b, e = info["data_offsets"]
            if not (0 <= b <= e) or base + e > size:
                raise ModelLoadingError(f"truncated safetensors file: tensor {name} needs bytes "
                                        f"[{base + b}, {base + e}) of a {size}-byte file {path}")
            f.seek(base + b)
            buf = bytearray(f.read(e - b))
            dt = _DT[info["dtype"]]
            t = torch.frombuffer(buf, dtype=torch.uint8) if e > b else torch.empty(0, dtype=torch.uint8)
            out[name] = t.view(dt).reshape(info["shape"]) if e > b else torch.empty(info["shape"], dtype=dt)
        return out


def read_safetensors_metadata(path: str) -> Dict[str, str]:
    with open(path, "rb") as f:
        return _read_header(f, path)[0].get("__metadata__", {})


def write_safetensors(path: str, tensors: Mapping[str, torch.Tensor], metadata: Optional[Dict[str, str]] = None):
    """Writes tensors (moved to the CPU) in safetensors layout, names sorted,
    data 8-byte aligned."""
    header = {}
    blobs = []
    off = 0
    for name in sorted(tensors):
        t = tensors[name].detach().contiguous().cpu()
        raw = t.reshape(-1).view(torch.uint8).numpy().tobytes() if t.numel() else b""
        header[name] = {"dtype": _DT_INV[t.dtype], "shape": list(t.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    if metadata:
        header["__metadata__"] = {k: str(v) for k, v in metadata.items()}
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for raw in blobs:
            f.write(raw)


class CheckpointIndex:
    """Tensor name -> file over a Hugging Face checkpoint directory (one or
    more *.safetensors files, with or without model.safetensors.index.json)."""

    def __init__(self, directory: str):
        self.dir = directory
        self.where: Dict[str, str] = {}
        idx = os.path.join(directory, "model.safetensors.index.json")
        if os.path.exists(idx):
            with open(idx) as f:
                for name, fn in json.load(f)["weight_map"].items():
                    self.where[name] = os.path.join(directory, fn)
        else:
            for fn in sorted(os.listdir(directory)):
                if fn.endswith(".safetensors"):
                    p = os.path.join(directory, fn)
                    with open(p, "rb") as f:
                        for name in _read_header(f, p)[0]:
                            if name != "__metadata__":
                                self.where[name] = p

    def get(self, names: Iterable[str]) -> Dict[str, torch.Tensor]:
        names = list(names)
        missing = [n for n in names if n not in self.where]
        if missing:
            raise ModelLoadingError(f"Tensor not found: {missing[0]}")
        by_file: Dict[str, list] = {}
        for n in names:
            by_file.setdefault(self.where[n], []).append(n)
        out = {}
        for p, ns in by_file.items():
            out.update(read_safetensors(p, ns))
        return out


def mixtral_moe_layer(ckpt: CheckpointIndex, layer: int, num_experts: int,
                      prefix: str = "model.layers") -> Dict[str, torch.Tensor]:
    """A Mixtral layer's MoE tensors in the fused layout (float32, CPU)."""
    base = f"{prefix}.{layer}.block_sparse_moe"
    names = [f"{base}.gate.weight"]
    for e in range(num_experts):
        names += [f"{base}.experts.{e}.w1.weight", f"{base}.experts.{e}.w3.weight", f"{base}.experts.{e}.w2.weight"]
    t = ckpt.get(names)
    gate = t[f"{base}.gate.weight"].float()
    gu = torch.stack([torch.cat([t[f"{base}.experts.{e}.w1.weight"].float(), t[f"{base}.experts.{e}.w3.weight"].float()], 0)
                      for e in range(num_experts)])
    dn = torch.stack([t[f"{base}.experts.{e}.w2.weight"].float() for e in range(num_experts)])
    if gu.shape[1] != 2 * dn.shape[2] or gu.shape[2] != dn.shape[1] or gate.shape != (num_experts, gu.shape[2]):
        raise ModelLoadingError(f"layer {layer}: inconsistent expert shapes {tuple(gate.shape)}, "
                                f"{tuple(gu.shape)}, {tuple(dn.shape)}")
    return {"mlp.gate.weight": gate, "mlp.experts.gate_up_proj": gu, "mlp.experts.down_proj": dn}


QuantizeFn = Callable[[torch.Tensor, CompressionType], QuantizedTensor]


def _default_quantize(t: torch.Tensor, c: CompressionType) -> QuantizedTensor:
    from . import quantize_tensor
    q = quantize_tensor(t.cuda(), c)
    return QuantizedTensor(q.data.cpu(), q.shape, q.qtype, q.scales.cpu(), q.zero_points.cpu(), q.block_size)


class QuantizedShardCache:
    """One safetensors shard per layer under `directory`: for every tensor of
    at least 4096 elements (compress_layer_state_dict's rule,
    src/quantization.rs:291-295) its uint8 codes under the tensor's name and
    float32 `<name>.scales` / `<name>.zero_points`; smaller tensors stay as
    they are. Shapes, qtypes and block sizes are in the header metadata."""

    def __init__(self, directory: str, compression: CompressionType,
                 quantize: Optional[QuantizeFn] = None):
        self.dir = directory
        self.compression = CompressionType(compression)
        if self.compression == CompressionType.None_:
            raise QuantizationError("No compression specified")
        self.quantize = quantize or _default_quantize

    def path(self, layer: int) -> str:
        return os.path.join(self.dir, f"layer_{layer}.{self.compression.name.lower()}.safetensors")

    def has(self, layer: int) -> bool:
        return os.path.exists(self.path(layer))

    def store(self, layer: int, tensors: Mapping[str, torch.Tensor]) -> Dict[str, TensorLike]:
        out: Dict[str, TensorLike] = {}
        blobs: Dict[str, torch.Tensor] = {}
        meta = {}
        for name, t in tensors.items():
            if t.numel() < 4096:
                out[name] = t
                blobs[name] = t
                continue
            q = self.quantize(t, self.compression)
            out[name] = q
            blobs[name] = q.data.cpu()
            blobs[name + ".scales"] = q.scales.cpu()
            blobs[name + ".zero_points"] = q.zero_points.cpu()
            meta[name] = json.dumps({"shape": list(q.shape), "qtype": q.qtype.name, "block_size": q.block_size})
        write_safetensors(self.path(layer), blobs, meta)
        return out

    def load(self, layer: int) -> Dict[str, TensorLike]:
        p = self.path(layer)
        if not os.path.exists(p):
            raise ModelLoadingError(f"Layer file not found: {p}")
        meta = read_safetensors_metadata(p)
        t = read_safetensors(p)
        out: Dict[str, TensorLike] = {}
        for name, v in t.items():
            if name.endswith(".scales") or name.endswith(".zero_points"):
                continue
            if name in meta:
                m = json.loads(meta[name])
                out[name] = QuantizedTensor(v, tuple(m["shape"]), CompressionType[m["qtype"]],
                                            t[name + ".scales"], t[name + ".zero_points"], int(m["block_size"]))
            else:
                out[name] = v
        return out

    def layer(self, layer: int, source: Callable[[], Mapping[str, torch.Tensor]]) -> Dict[str, TensorLike]:
        """The cached layer, quantizing source() and storing it on a miss."""
        return self.load(layer) if self.has(layer) else self.store(layer, source())


def save_quant_state(metadata: Mapping[str, QuantizedTensor], path: str):
    """src/quantization.rs:315-339: JSON of shape, qtype (Debug name),
    scales, zero_points and block_size per tensor (codes are stored
    separately)."""
    ser = {}
    for name, q in metadata.items():
        ser[name] = {"shape": [int(d) for d in q.shape], "qtype": q.qtype.name if q.qtype.name != "None_" else "None",
                     "scales": [float(v) for v in np.asarray(q.scales.cpu(), dtype=np.float32)],
                     "zero_points": [float(v) for v in np.asarray(q.zero_points.cpu(), dtype=np.float32)],
                     "block_size": int(q.block_size)}
    with open(path, "w") as f:
        json.dump(ser, f, indent=2)


def load_quant_state(path: str, honor_qtype: bool = True) -> Dict[str, QuantizedTensor]:
    """src/quantization.rs:342-381. The reference sets every qtype to
    EightBit regardless of the file; honor_qtype=False reproduces that, the
    default reads the stored name. Codes are empty (loaded separately);
    block_size defaults to 128 as there."""
    if not os.path.exists(path):
        return {}
    try:
        with open(path) as f:
            ser = json.load(f)
    except ValueError as exc:
        raise ModelLoadingError(f"corrupt quant-state file {path}: {exc}") from None
    out = {}
    for name, d in ser.items():
        qt = CompressionType.EightBit
        if honor_qtype:
            qt = {"FourBit": CompressionType.FourBit, "EightBit": CompressionType.EightBit,
                  "None": CompressionType.None_}.get(d.get("qtype", "EightBit"), CompressionType.EightBit)
        out[name] = QuantizedTensor(torch.empty(0, dtype=torch.uint8), tuple(int(v) for v in d["shape"]), qt,
                                    torch.tensor(d["scales"], dtype=torch.float32),
                                    torch.tensor(d["zero_points"], dtype=torch.float32),
                                    int(d.get("block_size", 128)))
    return out
