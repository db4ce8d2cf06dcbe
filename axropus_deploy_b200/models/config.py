"""Model architectures the framework serves (random-init weights of the real shapes)."""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Optional

LLAMA3_ROPE_SCALING = {"factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                       "original_max_position_embeddings": 8192}


@dataclass(frozen=True)
class ModelConfig:
    name: str
    num_layers: int
    hidden: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 500000.0
    rope_scaling: Optional[Dict] = None
    rms_eps: float = 1e-5
    num_experts: int = 0
    top_k: int = 0
    max_position: int = 131072

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def kv_bytes_per_token(self, elem_bytes: float = 2.0) -> float:
        return self.num_layers * 2 * self.num_kv_heads * self.head_dim * elem_bytes

    def param_count(self) -> int:
        attn = self.hidden * (self.q_size + 2 * self.kv_size) + self.q_size * self.hidden
        mlp = 3 * self.hidden * self.ffn * max(1, self.num_experts) + (self.hidden * self.num_experts)
        return self.num_layers * (attn + mlp + 2 * self.hidden) + 2 * self.vocab * self.hidden + self.hidden


PRESETS: Dict[str, ModelConfig] = {
    "llama3-8b": ModelConfig("llama3-8b", 32, 4096, 32, 8, 128, 14336, 128256, 500000.0, LLAMA3_ROPE_SCALING),
    "llama3-70b": ModelConfig("llama3-70b", 80, 8192, 64, 8, 128, 28672, 128256, 500000.0, LLAMA3_ROPE_SCALING),
    "mixtral-8x7b": ModelConfig("mixtral-8x7b", 32, 4096, 32, 8, 128, 14336, 32000, 1000000.0, None,
                                num_experts=8, top_k=2, max_position=32768),
    # CPU plumbing shape of BASELINE config 1 (2 layers, 4 KV heads, head_dim 64)
    "tiny": ModelConfig("tiny", 2, 256, 8, 4, 64, 512, 32000, 10000.0, None, max_position=4096),
    # small GPU-friendly shapes (head_dim 128, which the prefill/rope kernels need)
    "tiny128": ModelConfig("tiny128", 2, 512, 8, 2, 128, 1024, 32000, 500000.0, LLAMA3_ROPE_SCALING,
                           max_position=16384),
    "tiny-moe": ModelConfig("tiny-moe", 2, 512, 8, 2, 128, 512, 32000, 1000000.0, None, num_experts=4, top_k=2,
                            max_position=16384),
}


def get_config(name: str) -> ModelConfig:
    try:
        return PRESETS[name]
    except KeyError:
        raise KeyError(f"unknown model {name!r}; presets: {sorted(PRESETS)}") from None
