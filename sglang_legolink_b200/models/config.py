"""Model configuration for the Qwen2 / Qwen2.5 / Qwen3 dense families.

The reference serves only ``Qwen2ForCausalLM`` (reference
``patched_sglang_files/python/sglang/srt/models/qwen2.py:465-558``); Qwen3 adds
per-head RMSNorm on Q and K before RoPE and drops the QKV bias.  The config is
read from an HF ``config.json`` (same keys as transformers) or built from one
of the named presets used by the benchmarks.
"""

from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field, replace
from typing import Any, Optional


@dataclass(frozen=True)
class ModelConfig:
    arch: str = "qwen2"  # "qwen2" | "qwen3"
    hidden_size: int = 256
    num_layers: int = 2
    num_heads: int = 4
    num_kv_heads: int = 2
    head_dim: int = 64
    intermediate_size: int = 512
    vocab_size: int = 1024
    rope_theta: float = 1_000_000.0
    rms_norm_eps: float = 1e-6
    tie_word_embeddings: bool = False
    max_position_embeddings: int = 32768
    qkv_bias: bool = True
    qk_norm: bool = False
    name: str = "tiny-qwen2"
    extra: dict = field(default_factory=dict, compare=False, hash=False)

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def qkv_size(self) -> int:
        return self.q_size + 2 * self.kv_size

    @property
    def rotary_dim(self) -> int:
        return self.head_dim

    def num_params(self) -> int:
        h, i, v, l = self.hidden_size, self.intermediate_size, self.vocab_size, self.num_layers
        per_layer = h * self.qkv_size + self.q_size * h + 3 * h * i + 2 * h
        if self.qkv_bias:
            per_layer += self.qkv_size
        if self.qk_norm:
            per_layer += 2 * self.head_dim
        emb = v * h * (1 if self.tie_word_embeddings else 2)
        return l * per_layer + emb + h

    def fingerprint(self) -> str:
        """Stable identity of the architecture (keys registry compatibility)."""
        import hashlib

        d = asdict(self)
        d.pop("extra", None)
        d.pop("name", None)
        return hashlib.sha256(json.dumps(d, sort_keys=True).encode()).hexdigest()[:16]

    def with_(self, **kw: Any) -> "ModelConfig":
        return replace(self, **kw)

    @staticmethod
    def from_hf_dict(d: dict, name: Optional[str] = None) -> "ModelConfig":
        archs = d.get("architectures") or []
        arch = "qwen3" if (d.get("model_type") == "qwen3" or any("Qwen3" in a for a in archs)) else "qwen2"
        heads = int(d["num_attention_heads"])
        hidden = int(d["hidden_size"])
        head_dim = int(d.get("head_dim") or hidden // heads)
        return ModelConfig(
            arch=arch,
            hidden_size=hidden,
            num_layers=int(d["num_hidden_layers"]),
            num_heads=heads,
            num_kv_heads=int(d.get("num_key_value_heads", heads)),
            head_dim=head_dim,
            intermediate_size=int(d["intermediate_size"]),
            vocab_size=int(d["vocab_size"]),
            rope_theta=float(d.get("rope_theta", 10000.0)),
            rms_norm_eps=float(d.get("rms_norm_eps", 1e-6)),
            tie_word_embeddings=bool(d.get("tie_word_embeddings", False)),
            max_position_embeddings=int(d.get("max_position_embeddings", 32768)),
            qkv_bias=bool(d.get("attention_bias", arch == "qwen2")) if arch == "qwen3" else True,
            qk_norm=arch == "qwen3",
            name=name or d.get("_name_or_path", arch),
        )

    @staticmethod
    def from_pretrained(path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json"), encoding="utf-8") as f:
            return ModelConfig.from_hf_dict(json.load(f), name=os.path.basename(path.rstrip("/")))

    def to_hf_dict(self) -> dict:
        return {
            "architectures": ["Qwen3ForCausalLM" if self.arch == "qwen3" else "Qwen2ForCausalLM"],
            "model_type": self.arch,
            "hidden_size": self.hidden_size,
            "num_hidden_layers": self.num_layers,
            "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads,
            "head_dim": self.head_dim,
            "intermediate_size": self.intermediate_size,
            "vocab_size": self.vocab_size,
            "rope_theta": self.rope_theta,
            "rms_norm_eps": self.rms_norm_eps,
            "tie_word_embeddings": self.tie_word_embeddings,
            "max_position_embeddings": self.max_position_embeddings,
            "attention_bias": self.qkv_bias,
            "torch_dtype": "bfloat16",
        }


#: Shapes named by the benchmark configurations (random-init weights).
PRESETS: dict[str, ModelConfig] = {
    # CPU fake-runtime config: 2 layers, hidden 256, 4 Q / 2 KV heads, head_dim 64.
    "tiny-qwen2": ModelConfig(),
    "qwen2.5-7b": ModelConfig(
        arch="qwen2", hidden_size=3584, num_layers=28, num_heads=28, num_kv_heads=4,
        head_dim=128, intermediate_size=18944, vocab_size=152064, rope_theta=1e6,
        name="qwen2.5-7b",
    ),
    "qwen3-32b": ModelConfig(
        arch="qwen3", hidden_size=5120, num_layers=64, num_heads=64, num_kv_heads=8,
        head_dim=128, intermediate_size=25600, vocab_size=151936, rope_theta=1e6,
        qkv_bias=False, qk_norm=True, name="qwen3-32b",
    ),
    # Small GPU test shape with production head_dim.
    "small-qwen2": ModelConfig(
        arch="qwen2", hidden_size=512, num_layers=2, num_heads=4, num_kv_heads=2,
        head_dim=128, intermediate_size=1024, vocab_size=2048, rope_theta=1e6,
        name="small-qwen2",
    ),
    "small-qwen3": ModelConfig(
        arch="qwen3", hidden_size=512, num_layers=2, num_heads=4, num_kv_heads=2,
        head_dim=128, intermediate_size=1024, vocab_size=2048, rope_theta=1e6,
        qkv_bias=False, qk_norm=True, name="small-qwen3",
    ),
}


def get_config(name_or_path: str) -> ModelConfig:
    if name_or_path in PRESETS:
        return PRESETS[name_or_path]
    if os.path.isdir(name_or_path):
        return ModelConfig.from_pretrained(name_or_path)
    raise KeyError(f"unknown model preset or path: {name_or_path}")
