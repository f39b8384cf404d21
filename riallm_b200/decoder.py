"""A small Mixtral-style decoder around the MoE block, for end-to-end
checks and decode tokens/s.

Layer skeleton as riallm's (src/model.rs:491-528): RMSNorm
(src/model.rs:456-468) -> attention (q/k/v projections, rotate-half RoPE
with inv_freq = theta^(-i/d) (src/model.rs:1002-1071), grouped-query heads
repeated as in repeat_heads (src/model.rs:1317-1328), causal mask, softmax,
o projection) -> residual -> RMSNorm -> MoE block -> residual; a final
RMSNorm and the LM head give the logits. The MoE tensors (router gate and
experts) of at least 4096 elements are quantized (compress_layer_state_dict's
rule, src/quantization.rs:291-295) and stay quantized for the MoE block;
attention, embedding and LM-head weights are bf16 (quantized ones are
dequantized once at load with riallm_cuda_dequantize).

riallm's NF4 reconstruction is (code - block mean) * block absmax with the
code index 0..15 rather than the table value (src/quantization.rs:45-70), so a
dequantized weight sits near 7.5 * absmax: positive and nearly constant. The
synthetic expert weights are therefore drawn with a small standard deviation
(4e-4) that keeps the block's output at the residual stream's scale, and the
RMSNorm weight in front of the block alternates +1/-1 so that the block's
own near-constant output, added to the residual, does not reach the next
block as a large common component.

Arithmetic (bf16 activations): projections are bf16 GEMMs with float32
accumulation rounded to bf16; RMSNorm, RoPE, the attention scores, softmax
and the weighted sum of values run in float32 and round to bf16; the MoE
block adds its output to the residual in float32 and rounds once
(RIALLM_MOE_ADD_TO_OUT). The attention and norms are plain torch ops: the
hot path this library owns is the MoE block.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional

import torch

from . import CompressionType, QuantizedTensor, apply_moe, quantize_tensor


@dataclass
class DecoderConfig:
    layers: int = 2
    hidden: int = 1024
    heads: int = 8
    kv_heads: int = 2
    head_dim: int = 128
    eps: float = 1e-5
    theta: float = 1e6
    vocab: int = 32000
    experts: int = 8
    top_k: int = 2
    intermediate: int = 2816


def synthetic_weights(cfg: DecoderConfig, seed: int = 0, device: str = "cuda",
                      expert_std: float = 4e-4) -> Dict[str, torch.Tensor]:
    """float32 weights from a seeded torch generator on `device` in a fixed
    order: N(0, 0.02), the expert tensors N(0, expert_std); RMSNorm weights
    are 1.0 except the one in front of the MoE block, which alternates +1/-1."""
    g = torch.Generator(device=device).manual_seed(seed)
    H, I, E = cfg.hidden, cfg.intermediate, cfg.experts
    kvd = cfg.kv_heads * cfg.head_dim

    def n(*shape, std=0.02):
        return torch.empty(shape, device=device).normal_(0.0, std, generator=g)
    w = {"model.embed_tokens.weight": n(cfg.vocab, H)}
    for l in range(cfg.layers):
        p = f"model.layers.{l}."
        w[p + "input_layernorm.weight"] = torch.ones(H, device=device)
        w[p + "self_attn.q_proj.weight"] = n(cfg.heads * cfg.head_dim, H)
        w[p + "self_attn.k_proj.weight"] = n(kvd, H)
        w[p + "self_attn.v_proj.weight"] = n(kvd, H)
        w[p + "self_attn.o_proj.weight"] = n(H, cfg.heads * cfg.head_dim)
        alt = torch.ones(H, device=device)
        alt[1::2] = -1.0
        w[p + "post_attention_layernorm.weight"] = alt
        w[p + "mlp.gate.weight"] = n(E, H)
        w[p + "mlp.experts.gate_up_proj"] = n(E, 2 * I, H, std=expert_std)
        w[p + "mlp.experts.down_proj"] = n(E, H, I, std=expert_std)
    w["model.norm.weight"] = torch.ones(H, device=device)
    w["lm_head.weight"] = n(cfg.vocab, H)
    return w


def quantize_weights(w: Dict[str, torch.Tensor],
                     compression: CompressionType = CompressionType.FourBit) -> Dict[str, object]:
    """Quantizes the MoE tensors (names containing ".mlp.") of at least 4096
    elements; the rest are returned unchanged."""
    return {k: (quantize_tensor(v, compression) if ".mlp." in k and v.numel() >= 4096 else v)
            for k, v in w.items()}


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """src/model.rs:456-468, float32 inside, rounded to x's dtype."""
    xf = x.float()
    var = (xf * xf).sum(-1, keepdim=True) / x.shape[-1]
    return (xf * torch.rsqrt(var + eps) * w.float()).to(x.dtype)


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    inv = torch.tensor([1.0 / theta ** (i / head_dim) for i in range(0, head_dim, 2)], dtype=torch.float32,
                       device=positions.device)
    freqs = positions.float()[:, None] * inv[None, :]
    return torch.cos(freqs), torch.sin(freqs)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [heads, seq, d]; rotate-half (src/model.rs:1044-1071)."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)


class TinyDecoder:
    def __init__(self, cfg: DecoderConfig, qweights: Dict[str, object]):
        self.cfg = cfg
        self.w: Dict[str, object] = {}
        for k, v in qweights.items():
            if ".mlp." in k or k.endswith("layernorm.weight") or k == "model.norm.weight":
                self.w[k] = v
            elif isinstance(v, QuantizedTensor):
                self.w[k] = v.dequantize(torch.bfloat16)
            else:
                self.w[k] = v.to(torch.bfloat16)
        self.cache: List[Optional[tuple]] = [None] * cfg.layers

    def reset(self):
        self.cache = [None] * self.cfg.layers

    def _attention(self, l: int, x: torch.Tensor, pos0: int) -> torch.Tensor:
        c, p = self.cfg, f"model.layers.{l}.self_attn."
        T = x.shape[0]
        q = (x @ self.w[p + "q_proj.weight"].t()).view(T, c.heads, c.head_dim).transpose(0, 1)
        k = (x @ self.w[p + "k_proj.weight"].t()).view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        v = (x @ self.w[p + "v_proj.weight"].t()).view(T, c.kv_heads, c.head_dim).transpose(0, 1)
        cos, sin = rope_tables(torch.arange(pos0, pos0 + T, device=x.device), c.head_dim, c.theta)
        q, k = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
        if self.cache[l] is not None:
            k = torch.cat([self.cache[l][0], k], 1)
            v = torch.cat([self.cache[l][1], v], 1)
        self.cache[l] = (k, v)
        rep = c.heads // c.kv_heads
        kr = k.repeat_interleave(rep, 0).float()
        vr = v.repeat_interleave(rep, 0).float()
        s = (q.float() @ kr.transpose(1, 2)) * (1.0 / math.sqrt(c.head_dim))
        S = kr.shape[1]
        mask = torch.arange(S, device=x.device)[None, :] > (torch.arange(T, device=x.device)[:, None] + pos0)
        s = s.masked_fill(mask[None], float("-inf"))
        o = (torch.softmax(s, -1) @ vr).to(x.dtype).transpose(0, 1).reshape(T, c.heads * c.head_dim)
        return o @ self.w[p + "o_proj.weight"].t()

    def forward(self, ids: torch.Tensor, pos0: int) -> torch.Tensor:
        """ids [T] -> logits [T, V] float32, appending to the KV cache."""
        c = self.cfg
        h = self.w["model.embed_tokens.weight"][ids]
        for l in range(c.layers):
            p = f"model.layers.{l}."
            h = h + self._attention(l, rms_norm(h, self.w[p + "input_layernorm.weight"], c.eps), pos0)
            n2 = rms_norm(h, self.w[p + "post_attention_layernorm.weight"], c.eps)
            moe = {"mlp.gate.weight": self.w[p + "mlp.gate.weight"],
                   "mlp.experts.gate_up_proj": self.w[p + "mlp.experts.gate_up_proj"],
                   "mlp.experts.down_proj": self.w[p + "mlp.experts.down_proj"]}
            h = apply_moe(moe, n2, c.top_k, c.experts, out=h, add_to_out=True)
        h = rms_norm(h, self.w["model.norm.weight"], c.eps)
        return (h @ self.w["lm_head.weight"].t()).float()

    def generate(self, prompt: torch.Tensor, new_tokens: int, keep_logits: bool = False):
        """Greedy: prefill the prompt, then one token per step. Returns the
        new token ids, and with keep_logits also each step's last-position
        logits [new_tokens, V] (float32, on the device)."""
        self.reset()
        logits = self.forward(prompt, 0)[-1]
        out, kept = [int(torch.argmax(logits).item())], [logits]
        pos = prompt.numel()
        for _ in range(new_tokens - 1):
            logits = self.forward(torch.tensor([out[-1]], device=prompt.device), pos)[-1]
            pos += 1
            out.append(int(torch.argmax(logits).item()))
            kept.append(logits)
        return (out, torch.stack(kept)) if keep_logits else out
