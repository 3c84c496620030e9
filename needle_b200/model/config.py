"""Model configuration, field-for-field compatible with needle's ``ModelConfig``.

Mirrors ``needle/model/config.py:9-65``: the same dataclass fields, the same
derived ``head_dim = hidden_size // num_attention_heads`` (``:28-29``) and the
same ``from_pretrained`` / ``_from_dict`` parsing of a HuggingFace
``config.json``.  ``PRESETS`` adds the architectures the benchmarks run, with
random weights (no checkpoints are needed or downloaded).
"""
from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path


@dataclass
class ModelConfig:
    model_type: str = "llama"
    hidden_size: int = 4096
    num_hidden_layers: int = 32
    num_attention_heads: int = 32
    num_key_value_heads: int = 32
    intermediate_size: int = 11008
    vocab_size: int = 32000
    max_position_embeddings: int = 4096
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    hidden_act: str = "silu"
    # Not a needle field: needle ties lm_head to the embedding only when a
    # checkpoint lacks lm_head.weight (needle/model/loader.py:138-143); the
    # synthetic weight generator uses this flag to decide whether to emit it.
    tie_word_embeddings: bool = False

    head_dim: int = field(init=False)

    def __post_init__(self):
        self.head_dim = self.hidden_size // self.num_attention_heads

    @property
    def num_kv_heads(self) -> int:
        return self.num_key_value_heads

    @property
    def is_gqa(self) -> bool:
        return self.num_key_value_heads != self.num_attention_heads

    @classmethod
    def from_pretrained(cls, model_path: str) -> "ModelConfig":
        config_path = Path(model_path) / "config.json"
        if not config_path.exists():
            raise FileNotFoundError(f"config.json not found in {model_path}")
        with open(config_path) as f:
            return cls._from_dict(json.load(f))

    @classmethod
    def _from_dict(cls, cfg: dict) -> "ModelConfig":
        return cls(
            model_type=cfg.get("model_type", "llama"),
            hidden_size=cfg.get("hidden_size", 4096),
            num_hidden_layers=cfg.get("num_hidden_layers", 32),
            num_attention_heads=cfg.get("num_attention_heads", 32),
            num_key_value_heads=cfg.get("num_key_value_heads", cfg.get("num_attention_heads", 32)),
            intermediate_size=cfg.get("intermediate_size", 11008),
            vocab_size=cfg.get("vocab_size", 32000),
            max_position_embeddings=cfg.get("max_position_embeddings", 4096),
            rms_norm_eps=cfg.get("rms_norm_eps", 1e-5),
            rope_theta=cfg.get("rope_theta", 10000.0),
            hidden_act=cfg.get("hidden_act", "silu"),
            tie_word_embeddings=cfg.get("tie_word_embeddings", False),
        )


PRESETS = {
    # Qwen2-0.5B shape: 24 layers, hidden 896, 14 q / 2 kv heads (D=64).
    "qwen2-0.5b": dict(model_type="qwen2", hidden_size=896, num_hidden_layers=24,
                       num_attention_heads=14, num_key_value_heads=2,
                       intermediate_size=4864, vocab_size=151936,
                       max_position_embeddings=4096, rms_norm_eps=1e-6,
                       rope_theta=1e6, tie_word_embeddings=True),
    # Llama-3-8B shape: 32 layers, hidden 4096, 32 q / 8 kv heads (D=128).
    "llama3-8b": dict(model_type="llama", hidden_size=4096, num_hidden_layers=32,
                      num_attention_heads=32, num_key_value_heads=8,
                      intermediate_size=14336, vocab_size=128256,
                      max_position_embeddings=8192, rms_norm_eps=1e-5,
                      rope_theta=5e5),
    # Qwen2-72B shape: 80 layers, hidden 8192, 64 q / 8 kv heads (D=128).
    "qwen2-72b": dict(model_type="qwen2", hidden_size=8192, num_hidden_layers=80,
                      num_attention_heads=64, num_key_value_heads=8,
                      intermediate_size=29568, vocab_size=152064,
                      max_position_embeddings=32768, rms_norm_eps=1e-6,
                      rope_theta=1e6),
}


def preset(name: str, **overrides) -> ModelConfig:
    """A ``ModelConfig`` for one of ``PRESETS``, with optional field overrides."""
    kw = dict(PRESETS[name])
    kw.update(overrides)
    return ModelConfig(**kw)
