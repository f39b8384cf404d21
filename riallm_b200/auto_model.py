"""AutoModel.from_pretrained: a Mixtral-architecture checkpoint directory to
a decoding model whose MoE blocks run on this library.

Reference behaviour followed (paths inside the riallm crate):
  * AutoModel::from_pretrained (src/auto_model.rs:82-128): a local path is
    required ("Model not found locally: ..." otherwise); config.json is read;
    the architecture comes from model_type; options default to
    ModelOptions::default();
  * ModelConfig::from_path / from_value (src/config.rs:58-204): the same
    fields, the same fallbacks (text_config, intermediate_size /
    moe_intermediate_size / shared_expert_intermediate_size,
    max_position_embeddings / seq_length, rms_norm_eps / layer_norm_epsilon,
    rope_theta or rope_parameters.rope_theta) and the same error messages;
  * generate (src/model.rs:1223-1270): greedy, temperature and top_p are
    accepted and unused, the returned ids are the prompt followed by the new
    tokens.

What differs, by design: riallm looks for Mixtral's FFN under
`mlp.gate_proj` and fails on `block_sparse_moe` (its model path has no
Mixtral MoE); here the Mixtral expert tensors are mapped onto the fused
layout of the MoE block (riallm_b200.loader). CompressionType FourBit /
EightBit quantizes the MoE block's tensors with the reference's rule
(tensors of >= 4096 elements, src/quantization.rs:291-295) through an
on-disk quantized-shard cache; attention, embedding and LM-head weights stay
in the checkpoint's precision as bf16. The expert GEMMs need quantized
weights, so CompressionType::None is refused, as is a CPU device (there is
no CPU path). ModelOptions.prefetch_layers streams every layer's MoE
tensors from pinned host memory through prefetch_buffer_size device slots
on each forward; without it all layers stay resident in HBM.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence

import torch

from . import CompressionType, ConfigError, ModelLoadingError, ModelOptions, QuantizedTensor


def _config_value(value: dict, key: str):
    tc = value.get("text_config")
    if isinstance(tc, dict) and key in tc:
        return tc[key]
    return value.get(key)


def _opt_usize(value: dict, key: str) -> Optional[int]:
    v = _config_value(value, key)
    if isinstance(v, bool) or not isinstance(v, int) or v < 0:
        return None
    return int(v)


def _usize(value: dict, key: str) -> int:
    v = _opt_usize(value, key)
    if v is None:
        raise ConfigError(f"Missing integer field: {key}")
    return v


def _usize_any(value: dict, keys: Sequence[str]) -> int:
    for k in keys:
        v = _opt_usize(value, k)
        if v is not None:
            return v
    raise ConfigError(f"Missing integer field; expected one of: {', '.join(keys)}")


def _opt_f32(value: dict, key: str) -> Optional[float]:
    v = _config_value(value, key)
    if isinstance(v, bool) or not isinstance(v, (int, float)):
        return None
    return float(v)


def _f32_any(value: dict, keys: Sequence[str]) -> float:
    for k in keys:
        v = _opt_f32(value, k)
        if v is not None:
            return v
    raise ConfigError(f"Missing float field; expected one of: {', '.join(keys)}")


@dataclass
class ModelConfig:
    """src/config.rs:11-54 (ModelConfig), parsed as from_value does."""
    model_type: str
    model_path: str
    vocab_size: int
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: Optional[int]
    intermediate_size: int
    max_position_embeddings: int
    rms_norm_eps: float
    rope_theta: Optional[float]
    sliding_window: Optional[int]
    split_path: Optional[str] = None
    extra: Dict[str, Any] = field(default_factory=dict)

    @classmethod
    def from_path(cls, model_path: str) -> "ModelConfig":
        cfg = os.path.join(model_path, "config.json")
        if not os.path.exists(cfg):
            raise ConfigError(f"config.json not found in {model_path!r}")
        with open(cfg) as f:
            try:
                value = json.load(f)
            except ValueError as exc:
                raise ConfigError(f"invalid config.json in {model_path!r}: {exc}") from None
        return cls.from_value(value, model_path)

    @classmethod
    def from_value(cls, value: dict, model_path: str) -> "ModelConfig":
        mt = value.get("model_type")
        if not isinstance(mt, str):
            mt = _config_value(value, "model_type")
        if not isinstance(mt, str):
            raise ConfigError("Missing string field: model_type")
        rope = _opt_f32(value, "rope_theta")
        if rope is None:
            rp = _config_value(value, "rope_parameters")
            if isinstance(rp, dict) and isinstance(rp.get("rope_theta"), (int, float)):
                rope = float(rp["rope_theta"])
        extra = dict(value)
        if isinstance(value.get("text_config"), dict):
            for k, v in value["text_config"].items():
                extra.setdefault(k, v)
        return cls(model_type=mt, model_path=model_path,
                   vocab_size=_usize(value, "vocab_size"),
                   hidden_size=_usize(value, "hidden_size"),
                   num_hidden_layers=_usize(value, "num_hidden_layers"),
                   num_attention_heads=_usize(value, "num_attention_heads"),
                   num_key_value_heads=_opt_usize(value, "num_key_value_heads"),
                   intermediate_size=_usize_any(value, ["intermediate_size", "moe_intermediate_size",
                                                        "shared_expert_intermediate_size"]),
                   max_position_embeddings=_usize_any(value, ["max_position_embeddings", "seq_length"]),
                   rms_norm_eps=_f32_any(value, ["rms_norm_eps", "layer_norm_epsilon"]),
                   rope_theta=rope, sliding_window=_opt_usize(value, "sliding_window"), extra=extra)

    def get_num_key_value_heads(self) -> int:
        return self.num_key_value_heads if self.num_key_value_heads is not None else self.num_attention_heads

    def uses_gqa(self) -> bool:
        return self.num_key_value_heads is not None and self.num_key_value_heads != self.num_attention_heads

    def is_qwen3_5_moe(self) -> bool:
        return "qwen3_5_moe" in self.model_type.lower()

    def head_dim(self) -> int:
        hd = self.extra.get("head_dim")
        return int(hd) if isinstance(hd, int) and hd > 0 else self.hidden_size // self.num_attention_heads

    def num_experts(self) -> int:
        for k in ("num_local_experts", "num_experts"):
            v = self.extra.get(k)
            if isinstance(v, int) and v > 0:
                return v
        raise ConfigError("Missing integer field; expected one of: num_local_experts, num_experts")

    def num_experts_per_tok(self) -> int:
        v = self.extra.get("num_experts_per_tok")
        if isinstance(v, int) and v > 0:
            return v
        raise ConfigError("Missing integer field: num_experts_per_tok")


def _is_mixtral(model_type: str) -> bool:
    return model_type.lower() in ("mixtral", "mixtralforcausallm")


class MoeCausalLM:
    """The loaded model (AirLLMBaseModel's role, src/model.rs:41-191): a
    Decoder over this library's kernels, greedy generation."""

    def __init__(self, config: ModelConfig, options: ModelOptions, decoder, streamer=None, packed=None):
        self.config = config
        self.options = options
        self.decoder = decoder
        self.streamer = streamer
        self._packed = packed or []

    @property
    def device(self) -> torch.device:
        return self.decoder.dev

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Prefill of input_ids [B, T] (or [T]) from an empty cache; returns
        the last position's logits [B, V] (float32)."""
        self.decoder.reset()
        return self.decoder.forward(torch.as_tensor(input_ids).to(self.device))

    def generate(self, input_ids, max_new_tokens: int, temperature: float = 1.0,
                 top_p: Optional[float] = None) -> List[int]:
        """src/model.rs:1223-1270: greedy decoding of max_new_tokens tokens
        after the prompt; temperature and top_p are unused there and here.
        Returns the prompt ids followed by the new ones."""
        ids = torch.as_tensor(input_ids).reshape(-1).to(torch.long)
        if max_new_tokens <= 0:
            return ids.tolist()
        new = self.decoder.generate(ids.to(self.device), int(max_new_tokens))
        return ids.tolist() + [int(t) for t in new]

    def stream_stats(self) -> Optional[dict]:
        return self.streamer.stats() if self.streamer is not None else None

    def close(self):
        self.decoder.close()
        if self.streamer is not None:
            self.streamer.close()
        for pl in self._packed:
            pl.close()


class AutoModel:
    """src/auto_model.rs:82-128."""

    @staticmethod
    def from_pretrained(model_id: str, options: Optional[ModelOptions] = None,
                        cache_dir: Optional[str] = None, max_batch: int = 1,
                        max_seq: Optional[int] = None, routed_streaming: bool = False) -> MoeCausalLM:
        """Loads a local Mixtral-architecture checkpoint directory
        (config.json plus safetensors shards). routed_streaming (with
        ModelOptions.prefetch_layers; no counterpart in the reference): decode
        steps copy only the experts their batch routes to, after routing with
        device-resident routers. cache_dir holds the quantized
        per-layer shards (default: <model_id>/riallm_quantized); max_seq
        defaults to ModelOptions.max_seq_len, else the config's
        max_position_embeddings capped at 4096."""
        from . import Context
        from .decoder import Decoder, DecoderConfig
        from .loader import CheckpointIndex, QuantizedShardCache, mixtral_moe_layer
        from .streaming import LayerStreamer, PackedLayer

        options = options or ModelOptions()
        if not os.path.exists(model_id):
            raise ModelLoadingError(f"Model not found locally: '{model_id}'. HuggingFace download not yet implemented.")
        config = ModelConfig.from_path(model_id)
        if not _is_mixtral(config.model_type):
            raise ConfigError(f"unsupported model_type {config.model_type!r}: this engine loads Mixtral-architecture "
                              "MoE checkpoints")
        comp = CompressionType(options.compression)
        if comp == CompressionType.None_:
            raise ConfigError("the MoE kernels take FourBit or EightBit expert weights; set ModelOptions.compression")
        if not options.device.is_cuda():
            raise ConfigError("only DeviceSpec::Cuda is supported: there is no CPU path")
        dev = options.device.device_id() or 0
        E, k = config.num_experts(), config.num_experts_per_tok()
        cfg = DecoderConfig(layers=config.num_hidden_layers, hidden=config.hidden_size,
                            heads=config.num_attention_heads, kv_heads=config.get_num_key_value_heads(),
                            head_dim=config.head_dim(), eps=config.rms_norm_eps,
                            theta=config.rope_theta if config.rope_theta is not None else 10000.0,
                            vocab=config.vocab_size, experts=E, top_k=k, intermediate=config.intermediate_size)
        if max_seq is None:
            max_seq = options.max_seq_len or min(config.max_position_embeddings, 4096)
        ckpt = CheckpointIndex(model_id)
        cache = QuantizedShardCache(cache_dir or os.path.join(model_id, "riallm_quantized"), comp)
        device = torch.device("cuda", dev)

        def dense(name):
            return ckpt.get([name])[name].to(device)

        weights: Dict[str, object] = {"model.embed_tokens.weight": dense("model.embed_tokens.weight").to(torch.bfloat16),
                                      "model.norm.weight": dense("model.norm.weight").float(),
                                      "lm_head.weight": dense("lm_head.weight").to(torch.bfloat16)}
        moe_layers = []
        for l in range(cfg.layers):
            p = f"model.layers.{l}."
            for n in ("input_layernorm.weight", "post_attention_layernorm.weight"):
                weights[p + n] = dense(p + n).float()
            for n in ("q", "k", "v", "o"):
                weights[p + f"self_attn.{n}_proj.weight"] = dense(p + f"self_attn.{n}_proj.weight").to(torch.bfloat16)
            moe = cache.layer(l, lambda l=l: mixtral_moe_layer(ckpt, l, E))
            moe_layers.append(moe)
        streamer, packed = None, None
        if options.prefetch_layers:
            ctx = Context.get(dev)
            packed = [PackedLayer(m, pinned=True, ctx=ctx) for m in moe_layers]
            streamer = LayerStreamer.from_options(packed, options, dev, routed=routed_streaming)
        else:
            for l, moe in enumerate(moe_layers):
                for name, t in moe.items():
                    weights[f"model.layers.{l}.{name}"] = _to_device(t, device)
        decoder = Decoder(cfg, weights, max_batch=max_batch, max_seq=max_seq, device=dev, streamer=streamer)
        return MoeCausalLM(config, options, decoder, streamer, packed)


def _to_device(t, device):
    if isinstance(t, QuantizedTensor):
        return QuantizedTensor(t.data.to(device), tuple(t.shape), t.qtype, t.scales.to(device),
                               t.zero_points.to(device), t.block_size)
    return t.to(device)
