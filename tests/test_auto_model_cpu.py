"""ModelConfig parsing and AutoModel.from_pretrained's argument checks on
the CPU (src/config.rs:58-204, src/auto_model.rs:82-128)."""
import json

import pytest

import riallm_b200 as rb
from riallm_b200.auto_model import AutoModel, ModelConfig

MIXTRAL = {"model_type": "mixtral", "vocab_size": 32000, "hidden_size": 4096, "num_hidden_layers": 32,
           "num_attention_heads": 32, "num_key_value_heads": 8, "intermediate_size": 14336,
           "max_position_embeddings": 32768, "rms_norm_eps": 1e-5, "rope_theta": 1e6,
           "num_local_experts": 8, "num_experts_per_tok": 2, "sliding_window": None}


def test_config_fields_and_fallbacks(tmp_path):
    c = ModelConfig.from_value(MIXTRAL, str(tmp_path))
    assert (c.hidden_size, c.num_hidden_layers, c.get_num_key_value_heads(), c.head_dim()) == (4096, 32, 8, 128)
    assert c.uses_gqa() and not c.is_qwen3_5_moe()
    assert (c.num_experts(), c.num_experts_per_tok(), c.rope_theta, c.sliding_window) == (8, 2, 1e6, None)
    # text_config nesting, the alternative field names and rope_parameters
    v = {"model_type": "qwen3_5_moe", "text_config": {
        "vocab_size": 10, "hidden_size": 64, "num_hidden_layers": 2, "num_attention_heads": 4,
        "moe_intermediate_size": 32, "seq_length": 128, "layer_norm_epsilon": 1e-6,
        "rope_parameters": {"rope_theta": 5e5}, "num_experts": 16, "num_experts_per_tok": 4}}
    q = ModelConfig.from_value(v, "x")
    assert (q.intermediate_size, q.max_position_embeddings, q.rms_norm_eps, q.rope_theta) == (32, 128, 1e-6, 5e5)
    assert q.get_num_key_value_heads() == 4 and not q.uses_gqa() and q.is_qwen3_5_moe()
    assert q.num_experts() == 16
    bad = dict(MIXTRAL)
    del bad["hidden_size"]
    with pytest.raises(rb.ConfigError, match="Missing integer field: hidden_size"):
        ModelConfig.from_value(bad, "x")
    bad = dict(MIXTRAL)
    del bad["model_type"]
    with pytest.raises(rb.ConfigError, match="Missing string field: model_type"):
        ModelConfig.from_value(bad, "x")
    bad = dict(MIXTRAL)
    del bad["intermediate_size"]
    with pytest.raises(rb.ConfigError, match="expected one of: intermediate_size"):
        ModelConfig.from_value(bad, "x")
    with pytest.raises(rb.ConfigError, match="config.json not found"):
        ModelConfig.from_path(str(tmp_path))


def test_from_pretrained_argument_checks(tmp_path):
    with pytest.raises(rb.ModelLoadingError, match="Model not found locally"):
        AutoModel.from_pretrained(str(tmp_path / "nope"))
    (tmp_path / "config.json").write_text(json.dumps(MIXTRAL))
    with pytest.raises(rb.ConfigError, match="FourBit or EightBit"):
        AutoModel.from_pretrained(str(tmp_path), rb.ModelOptions())
    with pytest.raises(rb.ConfigError, match="no CPU path"):
        AutoModel.from_pretrained(str(tmp_path), rb.ModelOptions(compression=rb.CompressionType.FourBit,
                                                                 device=rb.DeviceSpec.Cpu()))
    llama = dict(MIXTRAL, model_type="llama")
    (tmp_path / "config.json").write_text(json.dumps(llama))
    with pytest.raises(rb.ConfigError, match="unsupported model_type"):
        AutoModel.from_pretrained(str(tmp_path), rb.ModelOptions(compression=rb.CompressionType.FourBit))
    assert rb.AutoModel is AutoModel
