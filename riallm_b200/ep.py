"""Expert-parallel MoE block across the ranks of one node.

No counterpart in the reference (riallm runs on one device). Rank r of W
owns the experts [r E/W, (r+1) E/W). Each step:

  1. all-gather the W ranks' tokens (every rank then holds all W*T tokens);
  2. every rank routes all tokens over all E experts (the router weight is
     replicated, so every rank computes the same routing) and runs only its
     own experts, producing float32 partial sums per token, expert-ascending
     (riallm_cuda_moe_forward_ep);
  3. reduce-scatter the partials: rank r receives the summed block output of
     its own T tokens, which it rounds to the activation dtype.

The exchange volume per rank is (W-1)/W of the gathered tokens plus of the
float32 partials; there is no host synchronisation, so a step can be
captured in a CUDA graph. With NCCL both collectives run over NVLink
(NVSwitch reduces in the switch where NCCL enables NVLS).

`ops` computes step 2. The default runs the library on the GPU; tests pass
a CPU implementation to check the orchestration with gloo ranks.
"""
from __future__ import annotations

import datetime
from typing import Callable, Mapping, Optional

import torch
import torch.distributed as dist

from . import ConfigError, RiallmError, TensorLike, apply_moe_ep_partial
from . import _weights as _weights_of


class RankFailureError(RiallmError):
    """A peer rank stopped taking part in the expert-parallel steps (it
    exited, crashed or hangs). Raised on the surviving ranks on the host,
    before any of the failed step's collectives or kernels are launched when
    a PeerWatch is in use, or when a collective of the step fails or times
    out. `ranks` lists the peers known to be missing (empty if unknown)."""

    def __init__(self, msg: str, ranks=()):
        super().__init__(msg)
        self.ranks = tuple(ranks)


class PeerWatch:
    """Host-side liveness check between expert-parallel steps.

    Before step n each rank posts the key `<prefix>/<rank>/<n>` to the
    process group's key-value store and waits, at most `timeout_s` seconds,
    for every peer's key of the same step. A rank that has left (between
    steps, with none of its kernels or collectives in flight) therefore
    stops the others on the host, with the missing ranks named, instead of
    leaving them blocked inside a collective. Each rank deletes its own key
    of step n - 2, so the store stays small."""

    def __init__(self, store, rank: int, world: int, timeout_s: float = 5.0, prefix: str = "riallm/ep/step"):
        self.store, self.rank, self.world = store, int(rank), int(world)
        self.timeout = datetime.timedelta(seconds=float(timeout_s))
        self.prefix = prefix
        self.n = 0

    def _key(self, r: int, n: int) -> str:
        return f"{self.prefix}/{r}/{n}"

    def step(self) -> None:
        n = self.n
        self.store.set(self._key(self.rank, n), "1")
        peers = [self._key(r, n) for r in range(self.world) if r != self.rank]
        try:
            if peers:
                self.store.wait(peers, self.timeout)
        except Exception as exc:  # the store's timeout error type differs by store and version
            missing = [r for r in range(self.world) if r != self.rank and not self.store.check([self._key(r, n)])]
            raise RankFailureError(f"expert-parallel step {n}: rank(s) {missing} did not arrive within "
                                   f"{self.timeout.total_seconds():g} s ({exc})", missing) from None
        if n >= 2:
            try:
                self.store.delete_key(self._key(self.rank, n - 2))
            except Exception:
                pass
        self.n += 1

PartialFn = Callable[[torch.Tensor, int, int], torch.Tensor]


def expert_range(num_experts: int, rank: int, world: int) -> tuple:
    """(e_begin, e_local) of `rank`: contiguous, equal shares."""
    if world <= 0 or num_experts % world:
        raise ConfigError(f"{num_experts} experts do not split evenly over {world} ranks")
    e_local = num_experts // world
    return rank * e_local, e_local


class ExpertParallelMoE:
    """One rank's handle on an expert-parallel MoE block.

    tensors: this rank's weights: the full router "mlp.gate.weight" [E,H] and
    the owned experts' "mlp.experts.gate_up_proj" / "mlp.experts.down_proj"
    (QuantizedTensor.expert_slice of the full tensors). forward(x) takes this
    rank's tokens [T,H] (every rank the same T) and returns their block
    output.
    """

    def __init__(self, tensors: Optional[Mapping[str, TensorLike]], num_experts: int, top_k: int,
                 group: Optional[dist.ProcessGroup] = None, ops: Optional[PartialFn] = None,
                 watch: Optional[PeerWatch] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.E = int(num_experts)
        self.k = int(top_k)
        self.e_begin, self.e_local = expert_range(self.E, self.rank, self.world)
        self.tensors = tensors
        self.ops = ops
        # gloo has no reduce-scatter: it all-reduces and keeps its own slice.
        self.backend = dist.get_backend(group)
        self.watch = watch

    def forward(self, x: torch.Tensor, tensors: Optional[Mapping[str, TensorLike]] = None,
                add_to: Optional[torch.Tensor] = None, ctx=None) -> torch.Tensor:
        """x: this rank's tokens [T,H]. tensors: this call's weights (default:
        the ones given at construction), so one handle serves every layer of
        a model. With add_to (a [T,H] tensor of x's dtype), the block output
        is added to it in float32 and rounded once, in place (what
        apply_moe(..., add_to_out=True) does on one GPU), and add_to is
        returned. ctx: the library context of the expert kernels."""
        if self.watch is not None:
            self.watch.step()
        tensors = self.tensors if tensors is None else tensors
        try:
            y = self._forward(x, tensors, ctx)
        except RiallmError:
            raise
        except RuntimeError as exc:
            # A collective that failed or timed out (a peer left during the
            # step, or the process group's timeout expired).
            raise RankFailureError(f"expert-parallel collective failed: {exc}") from exc
        if add_to is not None:
            add_to.copy_(add_to.float().add_(y))
            return add_to
        return y.to(x.dtype)

    def _forward(self, x: torch.Tensor, tensors, ctx) -> torch.Tensor:
        T, H = x.shape
        W = self.world
        x = x.contiguous()
        x_all = torch.empty((W * T, H), dtype=x.dtype, device=x.device)
        if self.backend == "gloo":
            parts = [torch.empty_like(x) for _ in range(W)]
            dist.all_gather(parts, x, group=self.group)
            x_all = torch.cat(parts, 0)
        else:
            dist.all_gather_into_tensor(x_all, x, group=self.group)
        if self.ops is not None:
            partial = self.ops(x_all, self.e_begin, self.e_local)
        else:
            partial = apply_moe_ep_partial(tensors, x_all, self.k, self.E, self.e_begin, self.e_local, ctx=ctx)
        if self.backend == "gloo":
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
            out = partial[self.rank * T:(self.rank + 1) * T]
        else:
            out = torch.empty((T, H), dtype=partial.dtype, device=partial.device)
            dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=self.group)
        return out

    __call__ = forward


class ExpertParallelA2A:
    """One rank's expert-parallel MoE block with the token all-to-all inside
    the library (riallm_cuda_ep_init + riallm_cuda_moe_forward_ep_a2a).

    tensors: the full router "mlp.gate.weight" [E,H] and this rank's experts'
    "mlp.experts.gate_up_proj" / "mlp.experts.down_proj" (expert_slice of the
    full tensors, experts [r E/W, (r+1) E/W)). Rank 0 makes the NCCL id and
    the process group carries it to the other ranks; the library then builds
    its own communicator on a context of its own. forward(x) takes this
    rank's bf16 tokens [T,H] (the same T on every rank) and returns their
    block output. A PeerWatch, when given, checks the peers on the host
    before every step, and the communicator's asynchronous error state is
    polled after it: a failed or vanished peer raises RankFailureError."""

    def __init__(self, tensors: Mapping[str, TensorLike], num_experts: int, top_k: int,
                 group: Optional[dist.ProcessGroup] = None, device: Optional[int] = None,
                 watch: Optional[PeerWatch] = None, transport: str = "nccl", max_tokens: int = 0):
        """transport "nccl": NCCL point-to-point moves the rows (one host
        synchronisation per call for the message sizes). "peer": the
        library's kernels store the rows into the peers' IPC-mapped buffers
        (riallm_cuda_ep_peer_init, for calls of up to max_tokens tokens; no
        host synchronisation, graph-capturable)."""
        import ctypes
        from . import Context, lib
        if transport not in ("nccl", "peer"):
            raise ConfigError(f"unknown transport {transport!r}")
        if transport == "peer" and max_tokens < 1:
            raise ConfigError("the peer transport needs max_tokens >= 1")
        self.transport = transport
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.E, self.k = int(num_experts), int(top_k)
        self.e_begin, self.e_local = expert_range(self.E, self.rank, self.world)
        self.tensors = tensors
        self.watch = watch
        dev = torch.cuda.current_device() if device is None else int(device)
        self.ctx = Context(dev)
        buf = (ctypes.c_uint8 * 128)()
        if self.rank == 0:
            self.ctx.check(lib().riallm_cuda_ep_unique_id(buf))
        obj = [bytes(buf)]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(obj[0])
        self.ctx.check(lib().riallm_cuda_ep_init(self.ctx.ptr, uid, self.rank, self.world))
        if transport == "peer":
            _, _, gu = _weights_of(tensors)
            H, I = int(gu.shape[2]), int(gu.shape[1]) // 2
            self.ctx.reserve(int(max_tokens), H, I, self.E, self.k, torch.bfloat16)
            self.ctx.check(lib().riallm_cuda_ep_peer_init(self.ctx.ptr, int(max_tokens), H, I, self.E, self.k))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        import ctypes
        from . import _stream_ptr, _weights, lib
        if self.watch is not None:
            self.watch.step()
        if x.dtype != torch.bfloat16 or not x.is_cuda:
            raise ConfigError("expert-parallel calls take bf16 CUDA tokens")
        x = x.contiguous()
        T, H = x.shape
        w, keep, gu = _weights(self.tensors)
        I = int(gu.shape[1]) // 2
        out = torch.empty_like(x)
        fwd = (lib().riallm_cuda_moe_forward_ep_peer if self.transport == "peer"
               else lib().riallm_cuda_moe_forward_ep_a2a)
        self.ctx.check(fwd(self.ctx.ptr, ctypes.byref(w), x.data_ptr(), out.data_ptr(), T, H, I, self.E, self.k, 0,
                           _stream_ptr(x)))
        rc = lib().riallm_cuda_ep_async_error(self.ctx.ptr)
        if rc != 0:
            raise RankFailureError(lib().riallm_cuda_last_error(self.ctx.ptr).decode())
        del keep
        return out

    __call__ = forward

    def close(self):
        from . import lib
        if self.ctx is not None:
            torch.cuda.synchronize()
            lib().riallm_cuda_ep_destroy(self.ctx.ptr)
            self.ctx.close()
            self.ctx = None
