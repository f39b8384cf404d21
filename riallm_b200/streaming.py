"""Layer streaming: quantized layer weights kept in pinned host memory and
copied into a ring of device slots ahead of use.

riallm moves each layer's tensors to the device with synchronous copies on
every forward (`load_layer_to_device`, src/model.rs:1131-1201;
`move_tensors_to_device`, src/memory.rs:113-125); its
`ModelOptions.prefetch_layers` / `prefetch_buffer_size`
(src/config.rs:389-393) are not acted on. `LayerStreamer` acts on them: each
layer is packed once into one host blob, and the library's streamer
(riallm_cuda_streamer_*) copies blob i into device slot i % depth on a copy
stream, ordered by events against the compute stream, so the copies of the
next layers overlap the compute of the current one.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Dict, Mapping, Optional, Sequence

import torch

from . import CompressionType, ConfigError, Context, ModelOptions, QuantizedTensor, TensorLike, lib

ALIGN = 256


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


@dataclass
class _Entry:
    kind: str          # "q" (QuantizedTensor) or "t" (plain tensor)
    shape: tuple
    dtype: torch.dtype
    qtype: int
    block_size: int
    parts: tuple       # ((offset, nbytes), ...) data[, scales, zeros]


class PackedLayer:
    """One layer's tensors in a single host blob (every part 256-byte
    aligned), pinned through the library when `pinned`."""

    def __init__(self, tensors: Mapping[str, TensorLike], pinned: bool = True, ctx: Optional[Context] = None):
        self.index: Dict[str, _Entry] = {}
        layout = []
        off = 0
        for name, t in tensors.items():
            if isinstance(t, QuantizedTensor):
                parts = []
                for part in (t.data, t.scales, t.zero_points):
                    nb = part.numel() * part.element_size()
                    parts.append((off, nb))
                    layout.append((off, part))
                    off = _align(off + nb)
                self.index[name] = _Entry("q", tuple(t.shape), t.data.dtype, int(t.qtype), int(t.block_size),
                                          tuple(parts))
            else:
                nb = t.numel() * t.element_size()
                self.index[name] = _Entry("t", tuple(t.shape), t.dtype, 0, 0, ((off, nb),))
                layout.append((off, t))
                off = _align(off + nb)
        self.nbytes = max(off, ALIGN)
        self._ctx = ctx
        self._hptr = None
        if pinned:
            self._ctx = ctx or Context.get(0)
            p = ctypes.c_void_p()
            self._ctx.check(lib().riallm_cuda_host_alloc_pinned(self._ctx.ptr, self.nbytes, ctypes.byref(p)))
            self._hptr = p.value
            buf = (ctypes.c_uint8 * self.nbytes).from_address(self._hptr)
            self.blob = torch.frombuffer(buf, dtype=torch.uint8)
        else:
            self.blob = torch.empty(self.nbytes, dtype=torch.uint8)
        for o, t in layout:
            src = t.detach().contiguous().reshape(-1).cpu()
            nb = src.numel() * src.element_size()
            self.blob[o:o + nb].copy_(src.view(torch.uint8))

    def data_ptr(self) -> int:
        return self.blob.data_ptr()

    def views(self, buf: torch.Tensor) -> Dict[str, TensorLike]:
        """The layer's tensors as views of `buf` (the blob's bytes, host or
        device)."""
        out: Dict[str, TensorLike] = {}
        for name, e in self.index.items():
            if e.kind == "q":
                (od, nd), (os_, ns), (oz, nz) = e.parts
                out[name] = QuantizedTensor(buf[od:od + nd], e.shape, CompressionType(e.qtype),
                                            buf[os_:os_ + ns].view(torch.float32),
                                            buf[oz:oz + nz].view(torch.float32), e.block_size)
            else:
                (o, n), = e.parts
                out[name] = buf[o:o + n].view(e.dtype).view(e.shape)
        return out

    def expert_ranges(self, experts: Sequence[int], names: Sequence[str] = ("mlp.experts.gate_up_proj",
                                                                              "mlp.experts.down_proj")):
        """(offsets, sizes) of the blob bytes that experts `experts` of the
        quantized [E, ...] tensors `names` occupy: each expert's codes, and
        its scales and zero points plus the first of the next expert's (the
        NF4 decode gives element 63 of a block the next block's parameters,
        and the next block of an expert's last row is the next expert's
        first)."""
        offs, sizes = [], []
        for name in names:
            e = self.index[name]
            if e.kind != "q":
                raise ConfigError(f"{name} is not a quantized tensor")
            (od, nd), (os_, ns), (oz, nz) = e.parts
            E = int(e.shape[0])
            per_d, per_p = nd // E, (ns // 4) // E  # bytes of codes, parameters (f32) per expert
            for x in sorted(set(int(v) for v in experts)):
                if not 0 <= x < E:
                    raise ConfigError(f"expert {x} outside [0, {E})")
                offs.append(od + x * per_d)
                sizes.append(per_d)
                extra = 1 if (x + 1) * per_p < ns // 4 else 0
                for o in (os_, oz):
                    offs.append(o + 4 * x * per_p)
                    sizes.append(4 * (per_p + extra))
        return offs, sizes

    def tensor(self, name: str, device) -> TensorLike:
        """One of the layer's tensors copied to `device` (its own memory)."""
        t = self.views(self.blob)[name]
        if isinstance(t, QuantizedTensor):
            return QuantizedTensor(t.data.to(device), t.shape, t.qtype, t.scales.to(device), t.zero_points.to(device),
                                   t.block_size)
        return t.to(device)

    def close(self):
        if self._hptr is not None:
            self.blob = None
            self._ctx.check(lib().riallm_cuda_host_free_pinned(self._ctx.ptr, self._hptr))
            self._hptr = None


class LayerStreamer:
    """Streams packed layers through `depth` device slots (depth =
    ModelOptions.prefetch_buffer_size). Usage per forward:

        s.prefetch(0) ... s.prefetch(depth - 1)
        for i: t = s.acquire(i); <kernels on t>; s.release(i); s.prefetch(i + depth)

    or s.run(fn, n) which does exactly that."""

    def __init__(self, layers: Sequence[PackedLayer], depth: int = 2, device: int = 0, routed: bool = False):
        """routed: decode steps copy only the experts the step's batch routes
        to (prefetch_experts, after routing with a device-resident router);
        prefills and the plain prefetch copy whole layers."""
        if depth < 1:
            raise ConfigError("prefetch_buffer_size must be at least 1")
        self.layers = list(layers)
        self.depth = int(depth)
        self.routed = bool(routed)
        self.ctx = Context.get(device)
        self.slot_bytes = _align(max(l.nbytes for l in self.layers))
        self.slots = torch.empty(self.depth * self.slot_bytes, dtype=torch.uint8, device=torch.device("cuda", device))
        h = ctypes.c_void_p()
        self.ctx.check(lib().riallm_cuda_streamer_create(self.ctx.ptr, self.depth, self.slot_bytes,
                                                          self.slots.data_ptr(), ctypes.byref(h)))
        self.h = h.value

    @classmethod
    def from_options(cls, layers: Sequence[PackedLayer], options: ModelOptions, device: int = 0,
                     routed: bool = False):
        return cls(layers, options.prefetch_buffer_size if options.prefetch_layers else 1, device, routed)

    def prefetch(self, i: int):
        if 0 <= i < len(self.layers):
            L = lib()
            rc = L.riallm_cuda_streamer_prefetch(self.h, i, self.layers[i].data_ptr(), self.layers[i].nbytes)
            self.ctx.check(rc)

    def prefetch_experts(self, i: int, experts: Sequence[int]):
        """Copies into layer i's slot only the bytes of experts `experts`
        (PackedLayer.expert_ranges); the slot's router and other experts are
        left as they are, so the caller routes with a resident router and
        runs only these experts."""
        offs, sizes = self.layers[i].expert_ranges(experts)
        n = len(offs)
        o = (ctypes.c_uint64 * max(n, 1))(*offs)
        z = (ctypes.c_uint64 * max(n, 1))(*sizes)
        self.ctx.check(lib().riallm_cuda_streamer_prefetch_ranges(self.h, i, self.layers[i].data_ptr(), o, z, n))

    def acquire(self, i: int, stream: Optional[torch.cuda.Stream] = None) -> Dict[str, TensorLike]:
        st = (stream or torch.cuda.current_stream()).cuda_stream
        p = ctypes.c_void_p()
        self.ctx.check(lib().riallm_cuda_streamer_acquire(self.h, i, st, ctypes.byref(p)))
        slot = i % self.depth
        base = slot * self.slot_bytes
        assert p.value == self.slots.data_ptr() + base
        return self.layers[i].views(self.slots[base:base + self.slot_bytes])

    def release(self, i: int, stream: Optional[torch.cuda.Stream] = None):
        st = (stream or torch.cuda.current_stream()).cuda_stream
        self.ctx.check(lib().riallm_cuda_streamer_release(self.h, i, st))

    def run(self, fn: Callable[[int, Dict[str, TensorLike]], None], n: Optional[int] = None,
            stream: Optional[torch.cuda.Stream] = None):
        n = len(self.layers) if n is None else n
        for i in range(min(self.depth, n)):
            self.prefetch(i)
        for i in range(n):
            t = self.acquire(i, stream)
            fn(i, t)
            self.release(i, stream)
            self.prefetch(i + self.depth)

    def stats(self) -> dict:
        b, c, ms = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_double()
        self.ctx.check(lib().riallm_cuda_streamer_stats(self.h, ctypes.byref(b), ctypes.byref(c), ctypes.byref(ms)))
        gbs = b.value / (ms.value / 1000.0) / 1e9 if ms.value > 0 else 0.0
        return {"bytes": b.value, "copies": c.value, "copy_ms": ms.value, "h2d_gbs": gbs}

    def close(self):
        if self.h:
            lib().riallm_cuda_streamer_destroy(self.h)
            self.h = None
