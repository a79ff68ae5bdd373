"""Llama-family architecture configs (the benchmarked shapes, plus the reference's model)."""
from __future__ import annotations

from dataclasses import dataclass, field, replace
from typing import Optional

__all__ = ["LlamaConfig", "PRESETS", "get_config"]


@dataclass(frozen=True)
class LlamaConfig:
    name: str
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    vocab_size: int
    head_dim: int = 128
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: Optional[dict] = field(default=None, hash=False, compare=False)
    max_position: int = 8192
    tie_word_embeddings: bool = False

    def with_layers(self, n: int) -> "LlamaConfig":
        return replace(self, num_layers=n)

    @classmethod
    def from_hf_dict(cls, d: dict, name: str = "hf") -> "LlamaConfig":
        """From a Hugging Face Llama ``config.json`` (or ``LlamaConfig.to_dict()``)."""
        heads = d["num_attention_heads"]
        return cls(name=name, hidden_size=d["hidden_size"], intermediate_size=d["intermediate_size"],
                   num_layers=d["num_hidden_layers"], num_heads=heads,
                   num_kv_heads=d.get("num_key_value_heads") or heads, vocab_size=d["vocab_size"],
                   head_dim=d.get("head_dim") or d["hidden_size"] // heads, rms_eps=d.get("rms_norm_eps", 1e-5),
                   rope_theta=d.get("rope_theta", 10000.0), rope_scaling=d.get("rope_scaling"),
                   max_position=d.get("max_position_embeddings", 8192),
                   tie_word_embeddings=bool(d.get("tie_word_embeddings", False)))

    def to_hf_dict(self) -> dict:
        """A Hugging Face ``LlamaForCausalLM`` config.json for this architecture."""
        return {"architectures": ["LlamaForCausalLM"], "model_type": "llama", "hidden_size": self.hidden_size,
                "intermediate_size": self.intermediate_size, "num_hidden_layers": self.num_layers,
                "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
                "vocab_size": self.vocab_size, "head_dim": self.head_dim, "rms_norm_eps": self.rms_eps,
                "rope_theta": self.rope_theta, "rope_scaling": self.rope_scaling,
                "max_position_embeddings": self.max_position, "tie_word_embeddings": self.tie_word_embeddings,
                "hidden_act": "silu", "torch_dtype": "bfloat16"}


PRESETS = {
    # prefill benchmark: Llama-2-7B (MHA, SwiGLU 11008, vocab 32000)
    "llama2-7b": LlamaConfig("llama2-7b", 4096, 11008, 32, 32, 32, 32000, rope_theta=10000.0, max_position=4096),
    # decode benchmark: Llama-3-8B (GQA 32/8, SwiGLU 14336, vocab 128256)
    "llama3-8b": LlamaConfig("llama3-8b", 4096, 14336, 32, 32, 8, 128256, rope_theta=500000.0, max_position=8192),
    # prefill + decode benchmark at TP 8: Llama-3-70B (GQA 64/8, SwiGLU 28672)
    "llama3-70b": LlamaConfig("llama3-70b", 8192, 28672, 80, 64, 8, 128256, rope_theta=500000.0, max_position=8192),
    # The reference's model (main.py:190): Llama-3.2-3B-Instruct
    "llama3.2-3b": LlamaConfig("llama3.2-3b", 3072, 8192, 28, 24, 8, 128256, rope_theta=500000.0,
                               rope_scaling={"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0,
                                             "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
                               max_position=8192, tie_word_embeddings=True),
    # small shapes for tests
    "tiny": LlamaConfig("tiny", 1024, 2048, 2, 8, 4, 1024, head_dim=128, max_position=2048),
    "tiny-hd64": LlamaConfig("tiny-hd64", 512, 1024, 2, 8, 4, 1024, head_dim=64, max_position=2048),
    "tiny-mha": LlamaConfig("tiny-mha", 1024, 2048, 2, 8, 8, 2048, head_dim=128, max_position=2048),
}


def get_config(name: str) -> LlamaConfig:
    try:
        return PRESETS[name]
    except KeyError:
        raise KeyError(f"unknown model {name!r}; choose from {sorted(PRESETS)}") from None
