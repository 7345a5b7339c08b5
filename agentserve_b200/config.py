"""Model geometry: the reference's ModelConfig fields (agentserve/model/config.py:10-30).

Any object with these attributes works (the reference's own ModelConfig included):
hidden_dim, n_heads, n_kv_heads, n_layers, vocab_size, max_seq_len, rms_norm_eps,
rope_theta, intermediate_size and the derived head_dim.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass
class ModelConfig:
    hidden_dim: int
    n_heads: int
    n_kv_heads: int
    n_layers: int
    vocab_size: int
    max_seq_len: int
    rms_norm_eps: float = 1e-5
    rope_theta: float = 500000.0
    intermediate_size: int = 0

    def __post_init__(self):
        if self.intermediate_size == 0:  # config.py:21-25: 8/3 * hidden rounded up to 256
            raw = int(8 / 3 * self.hidden_dim)
            self.intermediate_size = (raw + 255) // 256 * 256

    @property
    def head_dim(self) -> int:
        return self.hidden_dim // self.n_heads


# config.py:34-44
TinyConfig = ModelConfig(hidden_dim=64, n_heads=4, n_kv_heads=2, n_layers=2, vocab_size=256,
                         max_seq_len=512, intermediate_size=128, rms_norm_eps=1e-5,
                         rope_theta=10000.0)
# config.py:47-56 (Llama-3.2-1B)
Llama32_1B = ModelConfig(hidden_dim=2048, n_heads=32, n_kv_heads=8, n_layers=16,
                         vocab_size=128256, max_seq_len=131072, rope_theta=500000.0,
                         intermediate_size=8192)
# config.py:59-68 (Llama-3.2-3B)
Llama32_3B = ModelConfig(hidden_dim=3072, n_heads=24, n_kv_heads=8, n_layers=28,
                         vocab_size=128256, max_seq_len=131072, rope_theta=500000.0,
                         intermediate_size=8192)
# config.py:71-80 (Llama-3-8B geometry; the reference caps max_seq_len at 8192)
Llama32_8B = ModelConfig(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=32,
                         vocab_size=128256, max_seq_len=8192, rope_theta=500000.0,
                         intermediate_size=14336)


def llama_8b_long(max_seq_len: int = 33024) -> ModelConfig:
    """8B geometry with a RoPE table long enough for 32K-token contexts plus 256 decode
    steps (the reference's Llama32_8B stops at 8192)."""
    return ModelConfig(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=32,
                       vocab_size=128256, max_seq_len=max_seq_len, rope_theta=500000.0,
                       intermediate_size=14336)
