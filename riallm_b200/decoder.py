"""A Mixtral-style decoder around the MoE block, for end-to-end checks and
decode tokens/s, with a device-resident bf16 KV cache.

Layer skeleton as riallm's (src/model.rs:491-528): RMSNorm
(src/model.rs:456-468) -> attention (q/k/v projections, rotate-half RoPE
with inv_freq = theta^(-i/d) (src/model.rs:1002-1071), grouped-query heads
sharing a KV head as in repeat_heads (src/model.rs:1317-1328), causal mask,
softmax, o projection) -> residual -> RMSNorm -> MoE block -> residual; a
final RMSNorm and the LM head give the logits.

Kernels: RMSNorm (with the residual add fused), RoPE + KV-cache append and
the attention are this library's (riallm_cuda_rmsnorm,
riallm_cuda_rope_kv_append, riallm_cuda_attention); the MoE block is
riallm_cuda_moe_forward adding into the residual stream (bf16, rounded
once); the q/k/v (one fused weight), o and LM-head projections are bf16
with float32 accumulation: riallm_cuda_linear_bf16 (the weight streamed
once) for single-row decode steps, cuBLAS GEMMs otherwise. Positions live in a device array, so
one decode step (all layers, LM head and the greedy argmax) is captured
once in a CUDA graph and replayed per token.

The MoE tensors (router gate and experts) of at least 4096 elements are
quantized (compress_layer_state_dict's rule, src/quantization.rs:291-295)
and stay quantized; attention, embedding and LM-head weights are bf16
(quantized ones are dequantized once at load).

riallm's NF4 reconstruction is (code - block mean) * block absmax with the
code index 0..15 rather than the table value (src/quantization.rs:45-70), so
a dequantized weight sits near 7.5 * absmax: positive and nearly constant.
The synthetic expert weights are therefore drawn with a small standard
deviation (4e-4) that keeps the block's output at the residual stream's
scale, and the RMSNorm weight in front of the block alternates +1/-1 so
that the block's own near-constant output, added to the residual, does not
reach the next block as a large common component (which would also route
every token to the same experts).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict

import torch

from . import (CompressionType, ConfigError, Context, QuantizedTensor, apply_moe, lib, quantize_tensor, route)


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

    @classmethod
    def mixtral_8x7b(cls) -> "DecoderConfig":
        return cls(layers=32, hidden=4096, heads=32, kv_heads=8, head_dim=128, eps=1e-5, theta=1e6,
                   vocab=32000, experts=8, top_k=2, intermediate=14336)


def _layer_weights(cfg: DecoderConfig, l: int, n, device, alt_norm: bool = True) -> Dict[str, torch.Tensor]:
    H, I, E = cfg.hidden, cfg.intermediate, cfg.experts
    kvd = cfg.kv_heads * cfg.head_dim
    p = f"model.layers.{l}."
    alt = torch.ones(H, device=device)
    if alt_norm:
        alt[1::2] = -1.0
    return {p + "input_layernorm.weight": torch.ones(H, device=device),
            p + "self_attn.q_proj.weight": n(cfg.heads * cfg.head_dim, H),
            p + "self_attn.k_proj.weight": n(kvd, H),
            p + "self_attn.v_proj.weight": n(kvd, H),
            p + "self_attn.o_proj.weight": n(H, cfg.heads * cfg.head_dim),
            p + "post_attention_layernorm.weight": alt,
            p + "mlp.gate.weight": n(E, H),
            p + "mlp.experts.gate_up_proj": n(E, 2 * I, H, std=None),
            p + "mlp.experts.down_proj": n(E, H, I, std=None)}


def _normal(device, seed, expert_std):
    g = torch.Generator(device=device).manual_seed(seed)

    def n(*shape, std=0.02):
        return torch.empty(shape, device=device).normal_(0.0, expert_std if std is None else std, generator=g)
    return n


def synthetic_weights(cfg: DecoderConfig, seed: int = 0, device: str = "cuda",
                      expert_std: float = 4e-4, alt_norm: bool = True) -> Dict[str, torch.Tensor]:
    """float32 weights from a seeded torch generator on `device` in a fixed
    order: N(0, 0.02), the expert tensors N(0, expert_std); RMSNorm weights
    are 1.0 except the one in front of the MoE block, which alternates +1/-1
    when alt_norm is set. expert_std=0.02 with alt_norm=False is the tiny
    configuration exactly as specified (every weight N(0, 0.02), unit norms)."""
    n = _normal(device, seed, expert_std)
    w = {"model.embed_tokens.weight": n(cfg.vocab, cfg.hidden)}
    for l in range(cfg.layers):
        w.update(_layer_weights(cfg, l, n, device, alt_norm))
    w["model.norm.weight"] = torch.ones(cfg.hidden, device=device)
    w["lm_head.weight"] = n(cfg.vocab, cfg.hidden)
    return w


def quantize_weights(w: Dict[str, torch.Tensor],
                     compression: CompressionType = CompressionType.FourBit) -> Dict[str, object]:
    """Quantizes the MoE tensors (names containing ".mlp.") of at least 4096
    elements; the rest are returned unchanged."""
    return {k: (quantize_tensor(v, compression) if ".mlp." in k and v.numel() >= 4096 else v)
            for k, v in w.items()}


def synthetic_model(cfg: DecoderConfig, seed: int = 0, device: str = "cuda", expert_std: float = 4e-4,
                    compression: CompressionType = CompressionType.FourBit) -> Dict[str, object]:
    """synthetic_weights + quantize_weights one layer at a time (the same
    values, in the same generator order), with the dense weights cast to
    bf16 as they are made, so that a full-size model never exists in
    float32."""
    n = _normal(device, seed, expert_std)

    def keep(k, v):
        if ".mlp." in k and v.numel() >= 4096:
            return quantize_tensor(v, compression)
        return v if "norm" in k else v.to(torch.bfloat16)
    out = {"model.embed_tokens.weight": n(cfg.vocab, cfg.hidden).to(torch.bfloat16)}
    for l in range(cfg.layers):
        for k, v in _layer_weights(cfg, l, n, device).items():
            out[k] = keep(k, v)
            del v
    out["model.norm.weight"] = torch.ones(cfg.hidden, device=device)
    out["lm_head.weight"] = n(cfg.vocab, cfg.hidden).to(torch.bfloat16)
    return out


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """src/model.rs:456-468 in torch (float32 inside, rounded to x's dtype);
    the decoder itself uses riallm_cuda_rmsnorm."""
    xf = x.float()
    var = (xf * xf).sum(-1, keepdim=True) / x.shape[-1]
    return (xf * torch.rsqrt(var + eps) * w.float()).to(x.dtype)


def inv_freq(head_dim: int, theta: float, device=None) -> torch.Tensor:
    """theta^(-i/d) for even i < d, computed in double and stored as float32."""
    return torch.tensor([1.0 / theta ** (i / head_dim) for i in range(0, head_dim, 2)], dtype=torch.float32,
                        device=device)


def rope_tables(positions: torch.Tensor, head_dim: int, theta: float):
    freqs = positions.float()[:, None] * inv_freq(head_dim, theta, positions.device)[None, :]
    return torch.cos(freqs), torch.sin(freqs)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [heads, seq, d]; rotate-half (src/model.rs:1044-1071), in torch."""
    half = x.shape[-1] // 2
    xf = x.float()
    x1, x2 = xf[..., :half], xf[..., half:]
    return torch.cat([x1 * cos - x2 * sin, x2 * cos + x1 * sin], -1).to(x.dtype)


def _bf16(v) -> torch.Tensor:
    if isinstance(v, QuantizedTensor):
        return v.dequantize(torch.bfloat16).reshape(v.shape)
    return v.to(torch.bfloat16).contiguous()


class Decoder:
    """Greedy decoding of up to `max_batch` sequences of equal length with a
    KV cache of `max_seq` positions per sequence."""

    def __init__(self, cfg: DecoderConfig, qweights: Dict[str, object], max_batch: int = 1,
                 max_seq: int = 2048, device: int = 0, streamer=None, ep=None):
        """streamer: a LayerStreamer over the layers' MoE tensors (router
        gate and experts, one PackedLayer per layer, in layer order); they
        are then not taken from qweights but copied from pinned host memory
        into the streamer's device slots ahead of each layer on every forward
        (ModelOptions.prefetch_layers). Such a decoder runs its decode steps
        eagerly (the copies are host-driven, so there is no decode graph).

        ep: an ExpertParallelMoE handle (riallm_b200.ep; one process per GPU,
        every rank running its own batch of sequences through its own
        Decoder in lockstep). qweights then holds this rank's experts of
        every layer (QuantizedTensor.expert_slice) and the full router; the
        attention, norms, embedding and LM head are replicated. Each MoE
        block all-gathers the ranks' tokens, runs the local experts and
        reduce-scatters the partial sums (NCCL collectives, which the decode
        graph captures)."""
        if streamer is not None and ep is not None:
            raise ConfigError("layer streaming and expert parallelism do not combine")
        c = self.cfg = cfg
        if c.heads % c.kv_heads or c.heads // c.kv_heads not in (1, 2, 4, 6, 8) or c.head_dim not in (64, 128):
            raise ConfigError("need heads / kv_heads in {1, 2, 4, 6, 8} and head_dim 64 or 128")
        self.dev = torch.device("cuda", device)
        # Two contexts of its own: prefill calls grow `ctx`'s MoE scratch
        # arena as needed, while the decode graphs use `ctx_step`, reserved
        # once for max_batch tokens, whose arena therefore never moves.
        self.ctx = Context(device)
        self.ctx_step = Context(device)
        self.ep = ep
        step_tokens = max_batch * (ep.world if ep is not None else 1)
        self.ctx_step.reserve(step_tokens, c.hidden, c.intermediate, c.experts, c.top_k, torch.bfloat16)
        self.embed = _bf16(qweights["model.embed_tokens.weight"])
        self.lm_head = _bf16(qweights["lm_head.weight"])
        self.final_norm = qweights["model.norm.weight"].float().contiguous()
        self.layers = []
        for l in range(c.layers):
            p = f"model.layers.{l}."
            self.layers.append({
                "in_norm": qweights[p + "input_layernorm.weight"].float().contiguous(),
                "post_norm": qweights[p + "post_attention_layernorm.weight"].float().contiguous(),
                "wqkv": torch.cat([_bf16(qweights[p + f"self_attn.{n}_proj.weight"]) for n in "qkv"], 0),
                "wo": _bf16(qweights[p + "self_attn.o_proj.weight"]),
                "moe": None if streamer is not None else {
                    k: qweights[p + k] for k in ("mlp.gate.weight", "mlp.experts.gate_up_proj",
                                                 "mlp.experts.down_proj")},
            })
        self.streamer = streamer
        if streamer is not None and len(streamer.layers) != c.layers:
            raise ConfigError(f"streamer holds {len(streamer.layers)} layers, the model {c.layers}")
        # A routed streamer's decode steps route with device-resident routers
        # (E x H per layer, small) and then copy only the routed experts.
        self.gates = ([pl.tensor("mlp.gate.weight", self.dev) for pl in streamer.layers]
                      if streamer is not None and streamer.routed else None)
        self.max_batch, self.max_seq = max_batch, max_seq
        shape = (max_batch, c.kv_heads, max_seq, c.head_dim)
        self.k_cache = [torch.zeros(shape, dtype=torch.bfloat16, device=self.dev) for _ in range(c.layers)]
        self.v_cache = [torch.zeros(shape, dtype=torch.bfloat16, device=self.dev) for _ in range(c.layers)]
        self.inv_freq = inv_freq(c.head_dim, c.theta, self.dev)
        self.pos = torch.zeros(max_batch, dtype=torch.int32, device=self.dev)
        self.length = 0
        self._graphs: Dict[int, tuple] = {}

    def reset(self):
        self.pos.zero_()
        self.length = 0

    # ------------------------------------------------------------ kernels
    def _st(self):
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _norm(self, x, w, out, delta=None):
        self.ctx.check(lib().riallm_cuda_rmsnorm(self.ctx.ptr, x.data_ptr(),
                                                 delta.data_ptr() if delta is not None else None,
                                                 w.data_ptr(), out.data_ptr(), x.shape[0], x.shape[1],
                                                 self.cfg.eps, self._st()))

    def _linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """x [M, K] · wᵀ (w [N, K]) in bf16: riallm_cuda_linear_bf16 (weight
        streamed once; faster than cuBLAS at one row) for a single row,
        cuBLAS otherwise (faster from two rows on)."""
        M, K = x.shape
        if M > 1 or K % 256:
            return x @ w.t()
        y = torch.empty(M, w.shape[0], dtype=torch.bfloat16, device=self.dev)
        self.ctx.check(lib().riallm_cuda_linear_bf16(self.ctx.ptr, x.data_ptr(), w.data_ptr(), y.data_ptr(), M,
                                                     w.shape[0], K, self._st()))
        return y

    def _forward(self, ids: torch.Tensor, experts_used: list = None) -> torch.Tensor:
        """ids [B, T] on the device -> last-position logits [B, V] float32.
        Appends T positions to every sequence (pos += T on the device).
        With experts_used (a list), the number of distinct experts each
        layer's MoE block routes to is appended to it (an extra router pass;
        eager use only)."""
        c, B, T = self.cfg, ids.shape[0], ids.shape[1]
        moe_ctx = self.ctx_step if T == 1 else self.ctx
        nh, nkv, d = c.heads, c.kv_heads, c.head_dim
        h = self.embed.index_select(0, ids.reshape(-1))          # [B*T, H] residual stream
        n = torch.empty_like(h)
        q = torch.empty(B * T, nh * d, dtype=torch.bfloat16, device=self.dev)
        att = torch.empty_like(q)
        L = lib()
        st = self.streamer
        routed = st is not None and st.routed and T == 1
        if st is not None and not routed:
            for i in range(min(st.depth, c.layers)):
                st.prefetch(i)
        for i, layer in enumerate(self.layers):
            self._norm(h, layer["in_norm"], n)
            qkv = self._linear(n, layer["wqkv"])
            kc, vc = self.k_cache[i], self.v_cache[i]
            self.ctx.check(L.riallm_cuda_rope_kv_append(self.ctx.ptr, qkv.data_ptr(), self.pos.data_ptr(), B, T,
                                                        nh, nkv, d, self.inv_freq.data_ptr(), q.data_ptr(),
                                                        kc.data_ptr(), vc.data_ptr(), self.max_seq, self._st()))
            self.ctx.check(L.riallm_cuda_attention(self.ctx.ptr, q.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                                   self.pos.data_ptr(), B, T, nh, nkv, d, self.max_seq,
                                                   att.data_ptr(), self._st()))
            o = self._linear(att, layer["wo"])
            self._norm(h, layer["post_norm"], n, delta=o)         # h += o; n = norm(h)
            if st is None:
                moe = layer["moe"]
            elif routed:
                # The experts this step's tokens route to (one host
                # synchronisation), copied alone into the layer's slot.
                counts = route(self.gates[i], n, c.top_k, c.experts, ctx=moe_ctx)[2]
                st.prefetch_experts(i, torch.nonzero(counts > 0).flatten().tolist())
                moe = dict(st.acquire(i))
                moe["mlp.gate.weight"] = self.gates[i]
            else:
                moe = st.acquire(i)
            if experts_used is not None:
                counts = route(moe["mlp.gate.weight"], n, c.top_k, c.experts, ctx=moe_ctx)[2]
                experts_used.append(int((counts > 0).sum().item()))
            if self.ep is not None:
                self.ep.forward(n, tensors=moe, add_to=h, ctx=moe_ctx)
            else:
                apply_moe(moe, n, c.top_k, c.experts, out=h, add_to_out=True, ctx=moe_ctx)
            if st is not None:
                st.release(i)
                if not routed:
                    st.prefetch(i + st.depth)
        self.pos[:B].add_(T)
        last = h.view(B, T, -1)[:, -1].contiguous()
        nl = torch.empty_like(last)
        self._norm(last, self.final_norm, nl)
        return self._linear(nl, self.lm_head).float()

    def _advance(self, B: int, T: int):
        if B > self.max_batch:
            raise ConfigError(f"batch {B} > max_batch {self.max_batch}")
        if self.length + T > self.max_seq:
            raise ConfigError(f"sequence length {self.length + T} > max_seq {self.max_seq}")
        self.length += T

    def forward(self, ids: torch.Tensor) -> torch.Tensor:
        """ids [B, T] (or [T] for one sequence) -> last-position logits [B, V]."""
        if ids.dim() == 1:
            ids = ids[None]
        ids = ids.to(self.dev)
        self._advance(ids.shape[0], ids.shape[1])
        return self._forward(ids)

    # ------------------------------------------------------------ decoding
    def _decode_graph(self, B: int):
        """A CUDA graph of one decode step for B sequences: reads ids [B, 1],
        writes logits [B, V] and the greedy next ids [B]."""
        if B in self._graphs:
            return self._graphs[B]
        ids = torch.zeros(B, 1, dtype=torch.long, device=self.dev)
        saved = self.pos.clone()
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(side):
            # Warm-up outside the capture sizes the MoE scratch arena and
            # cuBLAS workspaces; what it writes to the caches is overwritten
            # when the restored positions are decoded for real.
            for _ in range(2):
                self._forward(ids)
                self.pos.copy_(saved)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            logits = self._forward(ids)
            nxt = torch.argmax(logits, -1)
        self.pos.copy_(saved)
        self._graphs[B] = (g, ids, logits, nxt)
        return self._graphs[B]

    def generate(self, prompt: torch.Tensor, new_tokens: int, keep_logits: bool = False,
                 use_graph: bool = True):
        """Greedy decoding: prefill the prompt [B, T] (or [T]), then one token
        per step. Returns the new ids [B, new_tokens] (a list for a 1-D
        prompt) and, with keep_logits, each step's logits [B, new_tokens, V]."""
        one = prompt.dim() == 1
        if one:
            prompt = prompt[None]
        B = prompt.shape[0]
        self.reset()
        logits = self.forward(prompt)
        tok = torch.argmax(logits, -1)
        toks, kept = [tok], ([logits] if keep_logits else [])
        step = self._decode_graph(B) if use_graph and new_tokens > 1 and self.streamer is None else None
        for _ in range(new_tokens - 1):
            self._advance(B, 1)
            if step is not None:
                g, ids, lg, nxt = step
                ids.copy_(tok.view(B, 1))
                g.replay()
                logits, tok = lg, nxt.clone()
            else:
                logits = self._forward(tok.view(B, 1))
                tok = torch.argmax(logits, -1)
            toks.append(tok)
            if keep_logits:
                kept.append(logits.clone())
        out = torch.stack(toks, 1)
        res = out[0].tolist() if one else out
        if keep_logits:
            lk = torch.stack(kept, 1)
            return res, (lk[0] if one else lk)
        return res

    def decode_forced(self, ids: torch.Tensor) -> None:
        """Decode steps fed given ids (teacher forcing): ids [S, B, 1] on the
        device, one graph replay per step after a prefill; the logits and
        greedy ids of each step are computed and dropped. Measures the decode
        step with a chosen continuation."""
        S, B = ids.shape[0], ids.shape[1]
        if self.streamer is not None:
            for i in range(S):
                self._advance(B, 1)
                self._forward(ids[i])
            return
        g, buf, _, _ = self._decode_graph(B)
        for i in range(S):
            self._advance(B, 1)
            buf.copy_(ids[i])
            g.replay()

    def experts_per_layer(self, ids: torch.Tensor) -> list:
        """One eager decode step of ids [B, 1] that also counts, per layer,
        the distinct experts its MoE block routes to."""
        used = []
        self._advance(ids.shape[0], ids.shape[1])
        self._forward(ids.to(self.dev), experts_used=used)
        return used

    def close(self):
        self._graphs.clear()
        torch.cuda.synchronize(self.dev)
        for ctx in (self.ctx, self.ctx_step):
            ctx.close()


# The small-config decoder of the end-to-end tests.
TinyDecoder = Decoder
