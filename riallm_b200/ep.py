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

from typing import Callable, Mapping, Optional

import torch
import torch.distributed as dist

from . import ConfigError, TensorLike, apply_moe_ep_partial

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

    def __init__(self, tensors: Mapping[str, TensorLike], num_experts: int, top_k: int,
                 group: Optional[dist.ProcessGroup] = None, ops: Optional[PartialFn] = None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.E = int(num_experts)
        self.k = int(top_k)
        self.e_begin, self.e_local = expert_range(self.E, self.rank, self.world)
        self.tensors = tensors
        self.ops = ops or self._gpu_partial
        # gloo has no reduce-scatter: it all-reduces and keeps its own slice.
        self.backend = dist.get_backend(group)

    def _gpu_partial(self, x_all: torch.Tensor, e_begin: int, e_local: int) -> torch.Tensor:
        return apply_moe_ep_partial(self.tensors, x_all, self.k, self.E, e_begin, e_local)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
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
        partial = self.ops(x_all, self.e_begin, self.e_local)
        if self.backend == "gloo":
            dist.all_reduce(partial, op=dist.ReduceOp.SUM, group=self.group)
            out = partial[self.rank * T:(self.rank + 1) * T]
        else:
            out = torch.empty((T, H), dtype=partial.dtype, device=partial.device)
            dist.reduce_scatter_tensor(out, partial, op=dist.ReduceOp.SUM, group=self.group)
        return out.to(x.dtype)

    __call__ = forward
