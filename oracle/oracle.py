"""CPU oracle for riallm's block quantization and MoE block forward.

TEST INFRASTRUCTURE ONLY. Only tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline / reference arm import this module, as the parity reference or
the timed CPU port. The product (riallm_b200) never imports it.

PARITY UNPINNED: the reference (Rust, candle 0.8) cannot be built or run
here and its tests pin no values (tests/integration_test.rs:124-148). The C
restatement (riallm_oracle.c) is pinned by hand-derived known answers on the
reference's own test inputs and cross-checked by the numpy mirror below,
which is written independently of the C code.

Two layers:
  * ctypes bindings to oracle/_build/libriallm_oracle.so (built by the
    Makefile beside this file);
  * a numpy mirror of src/quantization.rs (vectorised, independent of the C).
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libriallm_oracle.so")

NONE, FOUR_BIT, EIGHT_BIT = 0, 1, 2
BLOCK = {FOUR_BIT: 64, EIGHT_BIT: 128}

# src/quantization.rs:127-130
NF4_TABLE = np.array(
    [-1.0, -0.6962, -0.5250, -0.3900, -0.2750, -0.1750, -0.0850, -0.0150, 0.0,
     0.0150, 0.0850, 0.1750, 0.2750, 0.3900, 0.5250, 0.6962], dtype=np.float32)


def build() -> str:
    """Compile the C oracle with its Makefile; returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        u64, i32, vp, fp = ctypes.c_uint64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_float
        L.ro_num_blocks.restype = u64
        L.ro_num_blocks.argtypes = [i32, u64]
        L.ro_data_bytes.restype = u64
        L.ro_data_bytes.argtypes = [i32, u64]
        L.ro_quantize_nf4.argtypes = [vp, u64, vp, vp, vp]
        L.ro_quantize_int8.argtypes = [vp, u64, vp, vp, vp]
        L.ro_dequantize_nf4.restype = u64
        L.ro_dequantize_nf4.argtypes = [vp, u64, vp, u64, vp, u64, u64, u64, vp]
        L.ro_dequantize_int8.restype = u64
        L.ro_dequantize_int8.argtypes = [vp, u64, vp, u64, vp, u64, u64, vp]
        L.ro_tensor_span_f32.argtypes = [vp, u64, u64, i32, vp]
        L.ro_expf.restype = fp
        L.ro_expf.argtypes = [fp]
        L.ro_router.argtypes = [vp, i32, i32, i32, vp, i32, i32, vp, vp, vp, vp]
        L.ro_bucket.argtypes = [vp, i32, i32, i32, vp, vp, vp]
        L.ro_moe_forward.argtypes = [vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, vp, vp, i32]
        L.ro_f32_to_bf16.restype = ctypes.c_uint16
        L.ro_f32_to_bf16.argtypes = [fp]
        _lib = L
    return _lib


def _p(a: np.ndarray | None):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# --------------------------------------------------------------- QuantizedTensor

@dataclass
class QTensor:
    """Host copy of the reference's QuantizedTensor (src/quantization.rs:12-30)."""
    qtype: int
    data: np.ndarray          # uint8 (packed) or float32 (qtype NONE)
    scales: np.ndarray        # float32
    zero_points: np.ndarray   # float32
    numel: int
    block_size: int


class _CQT(ctypes.Structure):
    _fields_ = [("qtype", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("data", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("zero_points", ctypes.c_void_p), ("numel", ctypes.c_uint64),
                ("n_scales", ctypes.c_uint64), ("n_zero_points", ctypes.c_uint64)]


class _CMoeW(ctypes.Structure):
    _fields_ = [("gate", _CQT), ("gate_up_proj", _CQT), ("down_proj", _CQT),
                ("shared_gate_proj", _CQT), ("shared_up_proj", _CQT),
                ("shared_down_proj", _CQT), ("shared_expert_gate", _CQT),
                ("shared_intermediate", ctypes.c_int32)]


def _cqt(t: QTensor | None) -> _CQT:
    if t is None:
        return _CQT()
    return _CQT(t.qtype, t.block_size, _p(t.data), _p(t.scales), _p(t.zero_points),
                t.numel, t.scales.size, t.zero_points.size)


def quantize(v: np.ndarray, qtype: int) -> QTensor:
    """C oracle quantize (src/quantization.rs:111-245)."""
    v = np.ascontiguousarray(v, dtype=np.float32).reshape(-1)
    n = v.size
    if qtype == NONE:
        return QTensor(NONE, v.copy(), np.zeros(0, np.float32), np.zeros(0, np.float32), n, 0)
    L = lib()
    nb = L.ro_num_blocks(qtype, n)
    data = np.zeros(L.ro_data_bytes(qtype, n), np.uint8)
    scales = np.zeros(nb, np.float32)
    zeros = np.zeros(nb, np.float32)
    fn = L.ro_quantize_nf4 if qtype == FOUR_BIT else L.ro_quantize_int8
    fn(_p(v), n, _p(data), _p(scales), _p(zeros))
    return QTensor(qtype, data, scales, zeros, n, BLOCK[qtype])


def dequantize(t: QTensor) -> np.ndarray:
    """C oracle dequantize, literal loops of src/quantization.rs:45-95."""
    L = lib()
    if t.qtype == FOUR_BIT:
        out = np.zeros(2 * t.data.size, np.float32)
        w = L.ro_dequantize_nf4(_p(t.data), t.data.size, _p(t.scales), t.scales.size,
                                _p(t.zero_points), t.zero_points.size, t.numel,
                                t.block_size, _p(out))
        return out[:w]
    if t.qtype == EIGHT_BIT:
        out = np.zeros(t.data.size, np.float32)
        L.ro_dequantize_int8(_p(t.data), t.data.size, _p(t.scales), t.scales.size,
                             _p(t.zero_points), t.zero_points.size, t.block_size, _p(out))
        return out
    return t.data.astype(np.float32).copy()


def tensor_span(t: QTensor, start: int, length: int, bf16_round: bool = False) -> np.ndarray:
    out = np.zeros(length, np.float32)
    c = _cqt(t)
    lib().ro_tensor_span_f32(ctypes.byref(c), start, length, int(bf16_round), _p(out))
    return out


def expf(x: float) -> float:
    return lib().ro_expf(x)


def router(x: np.ndarray, wg: np.ndarray, k: int):
    """Returns (logits, probs, topk_idx, topk_w). x is bf16 bits (uint16) or float32."""
    T, H = x.shape
    E = wg.shape[0]
    x = np.ascontiguousarray(x)
    wg = np.ascontiguousarray(wg, dtype=np.float32)
    logits = np.zeros((T, E), np.float32)
    probs = np.zeros((T, E), np.float32)
    idx = np.zeros((T, k), np.int32)
    w = np.zeros((T, k), np.float32)
    lib().ro_router(_p(x), int(x.dtype == np.uint16), T, H, _p(wg), E, k,
                    _p(logits), _p(probs), _p(idx), _p(w))
    return logits, probs, idx, w


def bucket(topk_idx: np.ndarray, E: int):
    T, k = topk_idx.shape
    idx = np.ascontiguousarray(topk_idx, dtype=np.int32)
    counts = np.zeros(E, np.int32)
    offsets = np.zeros(E + 1, np.int32)
    perm = np.zeros(T * k, np.int32)
    lib().ro_bucket(_p(idx), T, k, E, _p(counts), _p(offsets), _p(perm))
    return counts, offsets, perm


@dataclass
class MoeWeights:
    """One layer's MoE tensors in the reference layout (src/model.rs:762,791-792)."""
    gate: QTensor            # [E, H]
    gate_up_proj: QTensor    # [E, 2I, H]
    down_proj: QTensor       # [E, H, I]
    shared_gate_proj: QTensor | None = None
    shared_up_proj: QTensor | None = None
    shared_down_proj: QTensor | None = None
    shared_expert_gate: QTensor | None = None
    shared_intermediate: int = 0


def moe_forward(w: MoeWeights, x: np.ndarray, T: int, H: int, I: int, E: int, k: int,
                n_threads: int = 0):
    """Whole block (src/model.rs:751-818). Returns (out f32 [T,H], idx, w, counts)."""
    cw = _CMoeW(_cqt(w.gate), _cqt(w.gate_up_proj), _cqt(w.down_proj),
                _cqt(w.shared_gate_proj), _cqt(w.shared_up_proj), _cqt(w.shared_down_proj),
                _cqt(w.shared_expert_gate), w.shared_intermediate)
    x = np.ascontiguousarray(x)
    out = np.zeros((T, H), np.float32)
    idx = np.zeros((T, k), np.int32)
    tw = np.zeros((T, k), np.float32)
    counts = np.zeros(E, np.int32)
    lib().ro_moe_forward(ctypes.byref(cw), _p(x), int(x.dtype == np.uint16), T, H, I, E, k,
                         _p(out), _p(idx), _p(tw), _p(counts), n_threads)
    return out, idx, tw, counts


# ------------------------------------------------------------------ bf16 helpers

def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round to nearest even, as torch and the CUDA cvt do."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------ numpy mirror
# Written from src/quantization.rs independently of riallm_oracle.c; tests
# require the two to agree bit for bit.

def np_quantize_nf4(v: np.ndarray):
    v = np.asarray(v, dtype=np.float32).reshape(-1)
    n = v.size
    nb = -(-n // 64)
    pad = np.zeros(nb * 64, np.float32)
    pad[:n] = v
    blocks = pad.reshape(nb, 64)
    lens = np.full(nb, 64)
    lens[-1] = n - (nb - 1) * 64
    valid = np.arange(64)[None, :] < lens[:, None]
    absmax = np.where(valid, np.abs(blocks), np.float32(0)).max(axis=1).astype(np.float32)
    sums = np.full(nb, -0.0, np.float32)
    for i in range(64):  # sequential f32 sum, element by element
        sums = np.where(valid[:, i], (sums + blocks[:, i]).astype(np.float32), sums)
    mean = (sums / lens.astype(np.float32)).astype(np.float32)
    norm = np.clip(blocks, np.float32(-1), np.float32(1))
    dist = np.abs(norm[:, :, None] - NF4_TABLE[None, None, :]).astype(np.float32)
    codes = np.argmin(dist, axis=2).astype(np.uint8)  # first minimum wins
    codes[~valid] = np.argmin(np.abs(np.float32(0) - NF4_TABLE))  # odd tail pads with q(0.0)
    pairs = codes.reshape(nb, 32, 2)
    packed = (pairs[:, :, 1] << 4) | pairs[:, :, 0]
    nbytes = (lens + 1) // 2
    data = np.concatenate([packed[b, :nbytes[b]] for b in range(nb)]) if nb > 1 else packed[0, :nbytes[0]]
    return data.astype(np.uint8), absmax, mean


def np_quantize_int8(v: np.ndarray):
    v = np.asarray(v, dtype=np.float32).reshape(-1)
    n = v.size
    nb = -(-n // 128)
    data = np.zeros(n, np.uint8)
    scales = np.zeros(nb, np.float32)
    zeros = np.zeros(nb, np.float32)
    with np.errstate(invalid="ignore", divide="ignore"):
        for b in range(nb):
            blk = v[b * 128:(b + 1) * 128]
            mn, mx = np.float32(blk.min()), np.float32(blk.max())
            scale = np.float32((mx - mn) / np.float32(255.0))
            scales[b], zeros[b] = scale, mn
            t = ((blk - mn) / scale).astype(np.float32)
            t = np.sign(t) * np.floor(np.abs(t) + np.float32(0.5))  # half away from zero
            t = np.where(np.isnan(t), 0, np.clip(t, 0, 255))
            data[b * 128:(b + 1) * 128] = t.astype(np.uint8)
    return data, scales, zeros


def np_dequantize_nf4(data, scales, zeros, numel, block_size=64):
    """Vectorised closed form: element e uses parameter block (e+1)//block_size."""
    e = np.arange(numel, dtype=np.int64)
    byte = np.asarray(data)[e >> 1]
    q = np.where(e & 1, (byte >> 4) & 15, byte & 15).astype(np.float32)
    b = (e + 1) // block_size
    s = np.where(b < scales.size, scales[np.minimum(b, scales.size - 1)], np.float32(1.0))
    z = np.where(b < zeros.size, zeros[np.minimum(b, zeros.size - 1)], np.float32(0.0))
    return ((q - z.astype(np.float32)).astype(np.float32) * s.astype(np.float32)).astype(np.float32)


def np_dequantize_int8(data, scales, zeros, block_size=128):
    e = np.arange(np.asarray(data).size, dtype=np.int64)
    b = e // block_size
    s = np.where(b < scales.size, scales[np.minimum(b, scales.size - 1)], np.float32(1.0))
    z = np.where(b < zeros.size, zeros[np.minimum(b, zeros.size - 1)], np.float32(0.0))
    return ((np.asarray(data).astype(np.float32) - z).astype(np.float32) * s).astype(np.float32)


# ------------------------------------------------------------- synthetic layers

def synthetic_layer(H: int, I: int, E: int, qtype: int, seed: int, std: float = 0.02,
                    shared_intermediate: int = 0):
    """Seeded N(0, std) MoE layer quantized like compress_layer_state_dict
    (src/quantization.rs:278-312: tensors with >= 4096 elements are quantized).
    Returns (MoeWeights, dict of float32 originals)."""
    rng = np.random.default_rng(seed)
    raw = {
        "gate": rng.normal(0.0, std, size=(E, H)).astype(np.float32),
        "gate_up_proj": rng.normal(0.0, std, size=(E, 2 * I, H)).astype(np.float32),
        "down_proj": rng.normal(0.0, std, size=(E, H, I)).astype(np.float32),
    }
    if shared_intermediate:
        Is = shared_intermediate
        raw["shared_gate_proj"] = rng.normal(0.0, std, size=(Is, H)).astype(np.float32)
        raw["shared_up_proj"] = rng.normal(0.0, std, size=(Is, H)).astype(np.float32)
        raw["shared_down_proj"] = rng.normal(0.0, std, size=(H, Is)).astype(np.float32)
        raw["shared_expert_gate"] = rng.normal(0.0, std, size=(1, H)).astype(np.float32)

    def q(name):
        a = raw[name]
        return quantize(a, qtype if a.size >= 4096 else NONE)

    w = MoeWeights(q("gate"), q("gate_up_proj"), q("down_proj"))
    if shared_intermediate:
        w.shared_gate_proj = q("shared_gate_proj")
        w.shared_up_proj = q("shared_up_proj")
        w.shared_down_proj = q("shared_down_proj")
        w.shared_expert_gate = q("shared_expert_gate")
        w.shared_intermediate = shared_intermediate
    return w, raw


def synthetic_x(T: int, H: int, seed: int, bf16: bool = True) -> np.ndarray:
    """Activations N(0,1); bf16 bits (uint16) when bf16, else float32."""
    x = np.random.default_rng(seed).normal(0.0, 1.0, size=(T, H)).astype(np.float32)
    return f32_to_bf16_bits(x).reshape(T, H) if bf16 else x
