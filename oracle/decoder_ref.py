"""ORACLE (test infrastructure only; never shipped or measured): a numpy
restatement of the small decoder in riallm_b200/decoder.py, used to check
its logits and greedy tokens.

It follows riallm's layer skeleton (src/model.rs:491-528), RMSNorm
(src/model.rs:456-468), rotate-half RoPE with inv_freq = theta^(-i/d)
(src/model.rs:1002-1071), attention (src/model.rs:912-1000) with grouped
query heads repeated as repeat_heads does (src/model.rs:1317-1328; the
reference's attention does not call it, so its grouped-query path is broken)
and the MoE block of riallm_oracle.c. Rounding points mirror the GPU decoder's: bf16 weights and
activations (float32 attention and embedding weights rounded to bf16 as
the GPU decoder loads them), projections accumulated in float64 and rounded to bf16, norms,
RoPE and attention in float64 rounded to bf16, the MoE output added to the
residual in float32 and rounded once, logits in float64 from the bf16
final hidden state. Parity unpinned: the reference cannot run here.
"""
from __future__ import annotations

import math

import numpy as np

from . import oracle as O


def bf(a):
    return O.bf16_bits_to_f32(O.f32_to_bf16_bits(np.asarray(a, np.float32)))


def _dq(q, shape):
    return bf(O.dequantize(q)).reshape(shape)


class DecoderRef:
    """qw: name -> oracle QTensor (NF4) or float32 array (small tensors);
    shapes: name -> shape of every QTensor."""

    def __init__(self, cfg, qw, shapes):
        self.c = cfg
        self.w = {}
        self.q = {k: (v if isinstance(v, O.QTensor) or ".mlp." not in k else O.quantize(v, O.NONE))
                  for k, v in qw.items()}
        for k, v in qw.items():
            if ".mlp." in k:
                continue
            if isinstance(v, O.QTensor):
                self.w[k] = _dq(v, shapes[k]).astype(np.float64)
            elif "norm" in k:
                self.w[k] = np.asarray(v, np.float64)
            else:
                self.w[k] = bf(v).astype(np.float64)
        self.cache = [None] * cfg.layers

    def reset(self):
        self.cache = [None] * self.c.layers

    def _norm(self, x, w):
        x64 = x.astype(np.float64)
        var = (x64 * x64).sum(-1, keepdims=True) / x.shape[-1]
        return bf(x64 / np.sqrt(var + self.c.eps) * w)

    def _rope(self, x, pos):
        d = self.c.head_dim
        inv = np.array([1.0 / self.c.theta ** (i / d) for i in range(0, d, 2)], np.float32)
        f = (np.asarray(pos, np.float32)[:, None] * inv[None, :]).astype(np.float32)
        cos, sin = np.cos(f).astype(np.float64), np.sin(f).astype(np.float64)
        half = d // 2
        x1, x2 = x[..., :half].astype(np.float64), x[..., half:].astype(np.float64)
        return bf(np.concatenate([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1))

    def _attn(self, l, x, pos0):
        c, p = self.c, f"model.layers.{l}.self_attn."
        T = x.shape[0]
        xd = x.astype(np.float64)
        q = bf(xd @ self.w[p + "q_proj.weight"].T).reshape(T, c.heads, c.head_dim).transpose(1, 0, 2)
        k = bf(xd @ self.w[p + "k_proj.weight"].T).reshape(T, c.kv_heads, c.head_dim).transpose(1, 0, 2)
        v = bf(xd @ self.w[p + "v_proj.weight"].T).reshape(T, c.kv_heads, c.head_dim).transpose(1, 0, 2)
        pos = np.arange(pos0, pos0 + T)
        q, k = self._rope(q, pos), self._rope(k, pos)
        if self.cache[l] is not None:
            k = np.concatenate([self.cache[l][0], k], 1)
            v = np.concatenate([self.cache[l][1], v], 1)
        self.cache[l] = (k, v)
        rep = c.heads // c.kv_heads
        kr = np.repeat(k, rep, 0).astype(np.float64)
        vr = np.repeat(v, rep, 0).astype(np.float64)
        s = (q.astype(np.float64) @ kr.transpose(0, 2, 1)) / math.sqrt(c.head_dim)
        S = kr.shape[1]
        mask = np.arange(S)[None, :] > (np.arange(T)[:, None] + pos0)
        s = np.where(mask[None], -np.inf, s)
        s = s - s.max(-1, keepdims=True)
        pr = np.exp(s)
        pr = pr / pr.sum(-1, keepdims=True)
        o = bf(pr @ vr).transpose(1, 0, 2).reshape(T, c.heads * c.head_dim)
        return bf(o.astype(np.float64) @ self.w[p + "o_proj.weight"].T)

    def forward(self, ids, pos0, last_only=False):
        c = self.c
        h = self.w["model.embed_tokens.weight"][np.asarray(ids)].astype(np.float32)
        for l in range(c.layers):
            p = f"model.layers.{l}."
            h = bf(h.astype(np.float64) + self._attn(l, self._norm(h, self.w[p + "input_layernorm.weight"]), pos0))
            n2 = self._norm(h, self.w[p + "post_attention_layernorm.weight"])
            w = O.MoeWeights(self.q[p + "mlp.gate.weight"], self.q[p + "mlp.experts.gate_up_proj"],
                             self.q[p + "mlp.experts.down_proj"])
            T = n2.shape[0]
            moe, _, _, _ = O.moe_forward(w, O.f32_to_bf16_bits(n2), T, c.hidden, c.intermediate, c.experts, c.top_k)
            h = bf(moe + h)
        h = self._norm(h, self.w["model.norm.weight"])
        if last_only:
            h = h[-1:]
        return h.astype(np.float64) @ self.w["lm_head.weight"].T
