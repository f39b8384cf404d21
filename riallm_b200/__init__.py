"""riallm_b200 -- B200-native (sm_100a) MoE block forward with block-quantized
weights, a drop-in for riallm's MoE / quantization path.

This module mirrors the reference's Rust interface for the path, over the C
ABI of libriallm_cuda.so (include/riallm_cuda.h):

  CompressionType, DeviceSpec, ModelOptions      src/config.rs:323-411
  QuantizedTensor, quantize_tensor,
  compress_layer_state_dict                      src/quantization.rs:12-312
  apply_moe (== apply_qwen3_5_moe)               src/model.rs:751-834
  RiallmError and its variants                   src/error.rs:8-47

torch is used only to hold device memory and to name CUDA streams. There is
no CPU fallback: without the compiled library every call raises.
"""
from __future__ import annotations

import ctypes
import enum
import os
from dataclasses import dataclass, field
from typing import Dict, Mapping, Optional, Union

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libriallm_cuda.so")

__all__ = [
    "CompressionType", "DeviceSpec", "ModelOptions", "QuantizedTensor", "quantize_tensor",
    "compress_layer_state_dict", "dequantize_layer_state_dict", "apply_moe", "route", "Context",
    "RiallmError", "ModelLoadingError", "MemoryError_", "ConfigError", "QuantizationError",
    "CudaError", "TimeoutError_", "lib", "AutoModel", "ModelConfig",
]


# ----------------------------------------------------------------- errors

class RiallmError(RuntimeError):
    """Base class, src/error.rs:8 (RiallmError)."""


class MemoryError_(RiallmError):
    """RiallmError::Memory."""


class QuantizationError(RiallmError):
    """RiallmError::Quantization."""


class ConfigError(RiallmError):
    """RiallmError::Config."""


class ModelLoadingError(RiallmError):
    """RiallmError::ModelLoading (e.g. "Tensor not found: ...")."""


class CudaError(RiallmError):
    """A CUDA runtime failure (RiallmError::Candle's role in the reference)."""


class TimeoutError_(RiallmError):
    """A bounded device-side wait expired; the kernel aborted cleanly."""


_STATUS = {1: MemoryError_, 2: QuantizationError, 3: ConfigError, 4: ModelLoadingError,
           5: CudaError, 6: TimeoutError_, 7: RiallmError}


# ------------------------------------------------------------- C library

class CQTensor(ctypes.Structure):
    _fields_ = [("qtype", ctypes.c_int32), ("block_size", ctypes.c_int32),
                ("data", ctypes.c_void_p), ("scales", ctypes.c_void_p),
                ("zero_points", ctypes.c_void_p), ("numel", ctypes.c_uint64),
                ("n_scales", ctypes.c_uint64), ("n_zero_points", ctypes.c_uint64)]


class CMoeWeights(ctypes.Structure):
    _fields_ = [("gate", CQTensor), ("gate_up_proj", CQTensor), ("down_proj", CQTensor),
                ("shared_gate_proj", CQTensor), ("shared_up_proj", CQTensor),
                ("shared_down_proj", CQTensor), ("shared_expert_gate", CQTensor),
                ("shared_intermediate", ctypes.c_int32)]


# Every symbol include/riallm_cuda.h declares: name -> (restype, argtypes).
_i32, _u32, _u64, _vp = ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_void_p
_pp = ctypes.POINTER(ctypes.c_void_p)
SIGNATURES = {
    "riallm_cuda_abi_version": (_i32, []),
    "riallm_cuda_ctx_create": (_i32, [_i32, _pp]),
    "riallm_cuda_ctx_destroy": (_i32, [_vp]),
    "riallm_cuda_last_error": (ctypes.c_char_p, [_vp]),
    "riallm_cuda_alloc": (_i32, [_vp, _u64, _pp]),
    "riallm_cuda_free": (_i32, [_vp, _vp]),
    "riallm_cuda_host_alloc_pinned": (_i32, [_vp, _u64, _pp]),
    "riallm_cuda_host_free_pinned": (_i32, [_vp, _vp]),
    "riallm_cuda_memcpy_h2d_async": (_i32, [_vp, _vp, _vp, _u64, _vp]),
    "riallm_cuda_memcpy_d2h_async": (_i32, [_vp, _vp, _vp, _u64, _vp]),
    "riallm_cuda_stream_synchronize": (_i32, [_vp, _vp]),
    "riallm_cuda_ctx_set_wait_limit": (_i32, [_vp, _u64]),
    "riallm_cuda_ep_unique_id": (_i32, [_vp]),
    "riallm_cuda_ep_init": (_i32, [_vp, _vp, _i32, _i32]),
    "riallm_cuda_ep_destroy": (_i32, [_vp]),
    "riallm_cuda_ep_async_error": (_i32, [_vp]),
    "riallm_cuda_moe_forward_ep_a2a": (_i32, [_vp, ctypes.POINTER(CMoeWeights), _vp, _vp, _i32, _i32, _i32,
                                              _i32, _i32, _u32, _vp]),
    "riallm_ep_exchange_plan": (_i32, [_i32, _i32, _vp, _vp, _vp, _vp]),
    "riallm_cuda_ep_peer_init": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32]),
    "riallm_cuda_moe_forward_ep_peer": (_i32, [_vp, ctypes.POINTER(CMoeWeights), _vp, _vp, _i32, _i32, _i32,
                                               _i32, _i32, _u32, _vp]),
    "riallm_cuda_event_create": (_i32, [_vp, _pp]),
    "riallm_cuda_event_destroy": (_i32, [_vp, _vp]),
    "riallm_cuda_event_record": (_i32, [_vp, _vp, _vp]),
    "riallm_cuda_stream_wait_event": (_i32, [_vp, _vp, _vp]),
    "riallm_cuda_event_synchronize": (_i32, [_vp, _vp]),
    "riallm_cuda_ctx_expire_next_wait": (_i32, [_vp]),
    "riallm_cuda_memory_stats": (_i32, [_vp, ctypes.POINTER(_u64), ctypes.POINTER(_u64)]),
    "riallm_quant_num_blocks": (_u64, [_i32, _u64]),
    "riallm_quant_data_bytes": (_u64, [_i32, _u64]),
    "riallm_cuda_quantize": (_i32, [_vp, _i32, _vp, _u64, _vp, _vp, _vp, _vp]),
    "riallm_cuda_dequantize": (_i32, [_vp, ctypes.POINTER(CQTensor), _i32, _vp, _i32, _vp]),
    "riallm_cuda_moe_forward": (_i32, [_vp, ctypes.POINTER(CMoeWeights), _vp, _vp, _i32, _i32, _i32,
                                       _i32, _i32, _i32, _u32, _vp]),
    "riallm_cuda_moe_reserve": (_i32, [_vp, _i32, _i32, _i32, _i32, _i32, _i32]),
    "riallm_cuda_moe_route": (_i32, [_vp, ctypes.POINTER(CQTensor), _vp, _i32, _i32, _i32, _i32, _i32,
                                     _vp, _vp, _vp, _vp, _vp, _vp]),
    "riallm_cuda_profile_enable": (_i32, [_vp, _i32]),
    "riallm_cuda_profile_read": (_i32, [_vp, ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_u64)]),
    "riallm_cuda_launch_count": (_u64, [_vp]),
    "riallm_cuda_moe_forward_noalloc": (_i32, [ctypes.POINTER(CMoeWeights), _vp, _vp, _i32, _i32, _i32,
                                               _i32, _i32, _u32, _vp]),
    "riallm_cuda_moe_forward_noalloc_sync": (_i32, [_vp]),
    "riallm_cuda_moe_forward_ep": (_i32, [_vp, ctypes.POINTER(CMoeWeights), _vp, _vp, _i32, _i32, _i32,
                                          _i32, _i32, _i32, _i32, _vp]),
    "riallm_cuda_streamer_create": (_i32, [_vp, _i32, _u64, _vp, ctypes.POINTER(_vp)]),
    "riallm_cuda_streamer_destroy": (_i32, [_vp]),
    "riallm_cuda_streamer_prefetch": (_i32, [_vp, _i32, _vp, _u64]),
    "riallm_cuda_streamer_prefetch_ranges": (_i32, [_vp, _i32, _vp, _vp, _vp, _i32]),
    "riallm_cuda_streamer_acquire": (_i32, [_vp, _i32, _vp, ctypes.POINTER(_vp)]),
    "riallm_cuda_streamer_release": (_i32, [_vp, _i32, _vp]),
    "riallm_cuda_streamer_stats": (_i32, [_vp, ctypes.POINTER(_u64), ctypes.POINTER(_u64),
                                          ctypes.POINTER(ctypes.c_double)]),
    "riallm_cuda_rmsnorm": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, ctypes.c_float, _vp]),
    "riallm_cuda_rope_kv_append": (_i32, [_vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp,
                                          _i32, _vp]),
    "riallm_cuda_attention": (_i32, [_vp, _vp, _vp, _vp, _vp, _i32, _i32, _i32, _i32, _i32, _i32, _vp, _vp]),
    "riallm_cuda_linear_bf16": (_i32, [_vp, _vp, _vp, _vp, _i32, _i32, _i32, _vp]),
}

PHASES = ("route", "gather", "gate_up", "down", "shared", "combine", "dispatch", "return")

_lib: Optional[ctypes.CDLL] = None


def lib() -> ctypes.CDLL:
    """Loads libriallm_cuda.so (built in-tree by riallm_b200.build). Raises
    when it is missing: there is no fallback path."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RiallmError(f"{LIB_PATH} is missing; build it with `python -m riallm_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        if L.riallm_cuda_abi_version() != 1:
            raise RiallmError("libriallm_cuda ABI version mismatch")
        _lib = L
    return _lib


# ------------------------------------------------------------ config.rs

class CompressionType(enum.IntEnum):
    """src/config.rs:323-346."""
    None_ = 0
    FourBit = 1
    EightBit = 2

    @staticmethod
    def from_str(s: str) -> "CompressionType":
        if s in ("none", ""):
            return CompressionType.None_
        if s == "4bit":
            return CompressionType.FourBit
        if s == "8bit":
            return CompressionType.EightBit
        raise ConfigError(f"Invalid compression type: {s}. Use 'none', '4bit', or '8bit'")


@dataclass(frozen=True)
class DeviceSpec:
    """src/config.rs:349-372: Cpu, Cuda(id) or Metal."""
    kind: str = "cuda"
    id: int = 0

    @staticmethod
    def Cuda(i: int = 0) -> "DeviceSpec":
        return DeviceSpec("cuda", i)

    @staticmethod
    def Cpu() -> "DeviceSpec":
        return DeviceSpec("cpu", 0)

    def is_cuda(self) -> bool:
        return self.kind == "cuda"

    def device_id(self) -> Optional[int]:
        return self.id if self.is_cuda() else None


@dataclass
class ModelOptions:
    """src/config.rs:376-411, same defaults."""
    compression: CompressionType = CompressionType.None_
    device: DeviceSpec = field(default_factory=lambda: DeviceSpec.Cuda(0))
    max_seq_len: Optional[int] = None
    profiling_mode: bool = False
    prefetch_layers: bool = True
    prefetch_buffer_size: int = 2
    dtype: str = "float16"


# --------------------------------------------------------------- context

def _check(status: int, ctx_ptr=None) -> None:
    if status == 0:
        return
    msg = ""
    if ctx_ptr:
        raw = lib().riallm_cuda_last_error(ctx_ptr)
        msg = raw.decode() if raw else ""
    raise _STATUS.get(status, RiallmError)(msg or f"riallm_cuda status {status}")


class Context:
    """One riallm_ctx per CUDA device (include/riallm_cuda.h)."""

    _by_device: Dict[int, "Context"] = {}

    def __init__(self, device: int = 0):
        L = lib()
        p = ctypes.c_void_p()
        _check(L.riallm_cuda_ctx_create(device, ctypes.byref(p)))
        self.ptr = p
        self.device = device

    @classmethod
    def get(cls, device: int) -> "Context":
        if device not in cls._by_device:
            cls._by_device[device] = Context(device)
        return cls._by_device[device]

    def check(self, status: int) -> None:
        _check(status, self.ptr)

    def synchronize(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        s = (stream or torch.cuda.current_stream(self.device)).cuda_stream
        self.check(lib().riallm_cuda_stream_synchronize(self.ptr, s))

    def set_wait_limit(self, wait_ns: int) -> None:
        """Bound of a kernel's wait for other CTAs' published work (0: 1 s)."""
        self.check(lib().riallm_cuda_ctx_set_wait_limit(self.ptr, int(wait_ns)))

    def expire_next_wait(self) -> None:
        """Test hook: the next MoE call's split-tile owners wait for a count
        that is never reached; synchronize() then raises TimeoutError_."""
        self.check(lib().riallm_cuda_ctx_expire_next_wait(self.ptr))

    def reserve(self, T: int, H: int, I: int, E: int, k: int, dtype: torch.dtype) -> None:
        self.check(lib().riallm_cuda_moe_reserve(self.ptr, T, H, I, E, k, _act_dtype(dtype)))

    def profile(self, enable: bool) -> None:
        self.check(lib().riallm_cuda_profile_enable(self.ptr, 1 if enable else 0))

    def profile_read(self):
        """(dict phase -> accumulated device ms since the last read, calls)."""
        ms = (ctypes.c_float * len(PHASES))()
        calls = ctypes.c_uint64()
        self.check(lib().riallm_cuda_profile_read(self.ptr, ms, ctypes.byref(calls)))
        return dict(zip(PHASES, list(ms))), calls.value

    def launch_count(self) -> int:
        return int(lib().riallm_cuda_launch_count(self.ptr))

    def close(self) -> None:
        if self.ptr:
            lib().riallm_cuda_ctx_destroy(self.ptr)
            self.ptr = None
            if Context._by_device.get(self.device) is self:
                del Context._by_device[self.device]


def _stream_ptr(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def _act_dtype(dtype: torch.dtype) -> int:
    if dtype == torch.bfloat16:
        return 1
    if dtype == torch.float32:
        return 0
    raise ConfigError(f"activation dtype {dtype} unsupported (bf16 or float32)")


# -------------------------------------------------------- quantization.rs

@dataclass
class QuantizedTensor:
    """src/quantization.rs:12-30, with device-resident buffers."""
    data: torch.Tensor         # uint8 codes (float32 values when qtype is None_)
    shape: tuple
    qtype: CompressionType
    scales: torch.Tensor       # float32
    zero_points: torch.Tensor  # float32
    block_size: int

    @property
    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= int(d)
        return n

    def as_c(self) -> CQTensor:
        return CQTensor(int(self.qtype), int(self.block_size), self.data.data_ptr(),
                        self.scales.data_ptr() if self.scales.numel() else None,
                        self.zero_points.data_ptr() if self.zero_points.numel() else None,
                        self.numel, self.scales.numel(), self.zero_points.numel())

    def dequantize(self, dtype: torch.dtype = torch.float32, codebook: bool = False) -> torch.Tensor:
        """QuantizedTensor::dequantize (src/quantization.rs:34-95); codebook=True
        decodes NF4 with its table instead (see riallm_dequant_mode)."""
        if self.qtype == CompressionType.None_:
            raise QuantizationError("Tensor is not quantized")
        ctx = Context.get(self.data.device.index or 0)
        out = torch.empty(self.numel, dtype=dtype, device=self.data.device)
        c = self.as_c()
        ctx.check(lib().riallm_cuda_dequantize(ctx.ptr, ctypes.byref(c), 1 if codebook else 0,
                                               out.data_ptr(), _act_dtype(dtype), _stream_ptr(out)))
        return out.view(*self.shape) if self.shape else out

    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size() + 4 * (self.scales.numel() + self.zero_points.numel())

    def expert_slice(self, e_begin: int, e_count: int) -> "QuantizedTensor":
        """Experts [e_begin, e_begin + e_count) of a quantized [E, ...] expert
        tensor, as views (no copy). Blocks never straddle experts, so the
        slice is a contiguous range of codes, scales and zero points; the
        parameters of the block after the slice ride along, because the
        reference's NF4 decode gives the last element of every block the
        next block's scale and zero (src/quantization.rs:55-72), and for the
        slice's last block that block belongs to the next expert."""
        if self.qtype == CompressionType.None_:
            raise QuantizationError("expert_slice expects a quantized tensor")
        E = int(self.shape[0])
        if e_begin < 0 or e_count <= 0 or e_begin + e_count > E:
            raise ConfigError(f"expert range [{e_begin}, {e_begin + e_count}) outside [0, {E})")
        per = self.numel // E
        bpe = per // self.block_size
        if per % self.block_size:
            raise QuantizationError("expert size is not a whole number of quantization blocks")
        bytes_per = per // 2 if self.qtype == CompressionType.FourBit else per
        b0, b1 = e_begin * bpe, (e_begin + e_count) * bpe
        extra = 1 if b1 < self.scales.numel() else 0
        return QuantizedTensor(self.data[e_begin * bytes_per:(e_begin + e_count) * bytes_per],
                               (e_count,) + tuple(self.shape[1:]), self.qtype,
                               self.scales[b0:b1 + extra], self.zero_points[b0:b1 + extra], self.block_size)


def quantize_tensor(tensor: torch.Tensor, compression: CompressionType) -> QuantizedTensor:
    """src/quantization.rs:99-107 (NF4 :111-176, 8-bit :199-245), on the GPU,
    bit-identical to the reference's host loops."""
    compression = CompressionType(compression)
    if compression == CompressionType.None_:
        raise QuantizationError("No compression specified")
    if not tensor.is_cuda:
        raise ConfigError("quantize_tensor expects a CUDA tensor")
    src = tensor.detach().to(torch.float32).contiguous().reshape(-1)
    n = src.numel()
    L = lib()
    nb = L.riallm_quant_num_blocks(int(compression), n)
    data = torch.empty(L.riallm_quant_data_bytes(int(compression), n), dtype=torch.uint8, device=src.device)
    scales = torch.empty(nb, dtype=torch.float32, device=src.device)
    zeros = torch.empty(nb, dtype=torch.float32, device=src.device)
    ctx = Context.get(src.device.index or 0)
    ctx.check(L.riallm_cuda_quantize(ctx.ptr, int(compression), src.data_ptr(), n, data.data_ptr(),
                                     scales.data_ptr(), zeros.data_ptr(), _stream_ptr(src)))
    return QuantizedTensor(data, tuple(tensor.shape), compression, scales, zeros,
                           64 if compression == CompressionType.FourBit else 128)


def _plain(t: torch.Tensor) -> QuantizedTensor:
    f = t.detach().to(torch.float32).contiguous()
    empty = torch.empty(0, dtype=torch.float32, device=f.device)
    return QuantizedTensor(f.reshape(-1), tuple(t.shape), CompressionType.None_, empty, empty, 0)


def compress_layer_state_dict(state_dict: Mapping[str, torch.Tensor], compression: CompressionType):
    """src/quantization.rs:278-312: tensors with >= 4096 elements are
    quantized, the rest kept. Returns (compressed, metadata) like the
    reference; here `metadata` maps names to device QuantizedTensors."""
    compression = CompressionType(compression)
    if compression == CompressionType.None_:
        return dict(state_dict), {}
    compressed, metadata = {}, {}
    for name, t in state_dict.items():
        if t.numel() < 4096:
            compressed[name] = t
            continue
        qt = quantize_tensor(t, compression)
        metadata[name] = qt
        compressed[name] = qt.data
    return compressed, metadata


def dequantize_layer_state_dict(state_dict: Mapping[str, torch.Tensor],
                                quant_metadata: Mapping[str, QuantizedTensor]):
    """src/quantization.rs:248-275."""
    out = {name: qt.dequantize(torch.float32) for name, qt in quant_metadata.items()}
    for name, t in state_dict.items():
        if name not in quant_metadata:
            out[name] = t
    return out


# ---------------------------------------------------------------- model.rs

_MOE_NAMES = ("mlp.gate.weight", "mlp.experts.gate_up_proj", "mlp.experts.down_proj")
_SHARED_NAMES = ("mlp.shared_expert.gate_proj.weight", "mlp.shared_expert.up_proj.weight",
                 "mlp.shared_expert.down_proj.weight", "mlp.shared_expert_gate.weight")

TensorLike = Union[torch.Tensor, QuantizedTensor]


def _as_q(t: TensorLike) -> QuantizedTensor:
    return t if isinstance(t, QuantizedTensor) else _plain(t)


def _get(tensors: Mapping[str, TensorLike], name: str) -> QuantizedTensor:
    if name not in tensors:
        raise ModelLoadingError(f"Tensor not found: {name}")  # src/model.rs:1311-1315
    return _as_q(tensors[name])


def _weights(tensors: Mapping[str, TensorLike]):
    keep = []
    gate, gu, down = (_get(tensors, n) for n in _MOE_NAMES)
    keep += [gate, gu, down]
    w = CMoeWeights()
    w.gate, w.gate_up_proj, w.down_proj = gate.as_c(), gu.as_c(), down.as_c()
    if _SHARED_NAMES[0] in tensors:
        sg, su, sd, sgate = (_get(tensors, n) for n in _SHARED_NAMES)
        keep += [sg, su, sd, sgate]
        w.shared_gate_proj, w.shared_up_proj = sg.as_c(), su.as_c()
        w.shared_down_proj, w.shared_expert_gate = sd.as_c(), sgate.as_c()
        w.shared_intermediate = int(sg.shape[0])
    return w, keep, gu


def apply_moe(tensors: Mapping[str, TensorLike], hidden: torch.Tensor, num_experts_per_tok: int,
              num_experts: int, out: Optional[torch.Tensor] = None, add_to_out: bool = False,
              ctx: Optional[Context] = None) -> torch.Tensor:
    """apply_qwen3_5_moe (src/model.rs:751-818) on the GPU.

    tensors: "mlp.gate.weight" [E,H], "mlp.experts.gate_up_proj" [E,2I,H],
    "mlp.experts.down_proj" [E,H,I] (+ optional shared expert tensors), each a
    QuantizedTensor (expert tensors must be) or a float tensor. hidden is
    [B,S,H] or [T,H], bf16 or float32. Returns the block output in hidden's
    shape and dtype (out += output when add_to_out)."""
    if not hidden.is_cuda:
        raise ConfigError("hidden must be a CUDA tensor")
    w, keep, gu = _weights(tensors)
    shape = hidden.shape
    H = int(shape[-1])
    flat = hidden.reshape(-1, H).contiguous()
    T = flat.shape[0]
    E = int(num_experts)
    k = int(num_experts_per_tok)
    I = int(gu.shape[1]) // 2 if len(gu.shape) == 3 else gu.numel // (2 * E * H)
    if out is None:
        out = torch.empty_like(flat)
        add_to_out = False
    ctx = ctx or Context.get(hidden.device.index or 0)
    ctx.check(lib().riallm_cuda_moe_forward(ctx.ptr, ctypes.byref(w), flat.data_ptr(), out.data_ptr(),
                                            T, H, I, E, k, _act_dtype(hidden.dtype),
                                            1 if add_to_out else 0, _stream_ptr(flat)))
    del keep
    return out.view(shape)


def apply_moe_ep_partial(tensors: Mapping[str, TensorLike], hidden: torch.Tensor, num_experts_per_tok: int,
                         num_experts: int, e_begin: int, e_local: int,
                         ctx: Optional[Context] = None) -> torch.Tensor:
    """One expert-parallel rank's share of the MoE block (no counterpart in
    the reference, which has no multi-GPU path): hidden [T,H] bf16 holds the
    tokens of every rank, "mlp.gate.weight" the full router, the expert
    tensors only experts [e_begin, e_begin + e_local) (see
    QuantizedTensor.expert_slice). Returns float32 [T,H]: per token, the
    routing-weighted sum of its owned experts' outputs in expert-ascending
    order; the sum of all ranks' partials is the block output."""
    if not hidden.is_cuda or hidden.dtype != torch.bfloat16:
        raise ConfigError("hidden must be a bf16 CUDA tensor")
    w, keep, gu = _weights(tensors)
    H = int(hidden.shape[-1])
    flat = hidden.reshape(-1, H).contiguous()
    T = flat.shape[0]
    I = int(gu.shape[1]) // 2 if len(gu.shape) == 3 else gu.numel // (2 * int(e_local) * H)
    partial = torch.empty((T, H), dtype=torch.float32, device=flat.device)
    ctx = ctx or Context.get(hidden.device.index or 0)
    ctx.check(lib().riallm_cuda_moe_forward_ep(ctx.ptr, ctypes.byref(w), flat.data_ptr(), partial.data_ptr(),
                                               T, H, I, int(num_experts), int(num_experts_per_tok),
                                               int(e_begin), int(e_local), _stream_ptr(flat)))
    del keep
    return partial


def route(gate: TensorLike, hidden: torch.Tensor, num_experts_per_tok: int, num_experts: int,
          ctx: Optional[Context] = None):
    """Router + bucketing only (src/model.rs:762-789). Returns
    (topk_idx int32 [T,k], topk_w float32 [T,k], counts [E], offsets [E+1],
    perm_pair [T*k])."""
    g = _as_q(gate)
    H = int(hidden.shape[-1])
    flat = hidden.reshape(-1, H).contiguous()
    T, E, k = flat.shape[0], int(num_experts), int(num_experts_per_tok)
    dev = flat.device
    idx = torch.empty((T, k), dtype=torch.int32, device=dev)
    tw = torch.empty((T, k), dtype=torch.float32, device=dev)
    counts = torch.empty(E, dtype=torch.int32, device=dev)
    offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(T * k, dtype=torch.int32, device=dev)
    ctx = ctx or Context.get(dev.index or 0)
    c = g.as_c()
    ctx.check(lib().riallm_cuda_moe_route(ctx.ptr, ctypes.byref(c), flat.data_ptr(), T, H, E, k,
                                          _act_dtype(flat.dtype), idx.data_ptr(), tw.data_ptr(),
                                          counts.data_ptr(), offsets.data_ptr(), perm.data_ptr(),
                                          _stream_ptr(flat)))
    return idx, tw, counts, offsets, perm


def __getattr__(name: str):
    """AutoModel / ModelConfig (src/auto_model.rs, src/config.rs) live in
    riallm_b200.auto_model and are loaded on first use."""
    if name in ("AutoModel", "ModelConfig"):
        from . import auto_model
        return getattr(auto_model, name)
    raise AttributeError(f"module 'riallm_b200' has no attribute {name!r}")
