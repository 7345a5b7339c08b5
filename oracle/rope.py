"""Rotate-half RoPE restated from agentserve/model/llama.py:63-99."""

from __future__ import annotations

import torch


def precompute_rope_freqs(head_dim: int, max_seq_len: int, theta: float = 10000.0) -> torch.Tensor:
    """llama.py:63-77: table [max_seq_len, head_dim] = cos(p * f_i) || sin(p * f_i),
    f_i = 1 / theta^(2i/D), all in fp32."""
    inv_freq = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    pos = torch.arange(max_seq_len, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    return torch.cat([freqs.cos(), freqs.sin()], dim=-1)


def apply_rope(x: torch.Tensor, cos_sin: torch.Tensor) -> torch.Tensor:
    """llama.py:80-99: x [T, heads, D], cos_sin [T, D].  Halves (not interleaved pairs)
    are rotated: (x1, x2) -> (x1 c - x2 s, x2 c + x1 s), computed in the promoted type
    of x and the table (fp32 for an fp32 table) and cast back to x.dtype."""
    d = x.shape[-1] // 2
    x1, x2 = x[..., :d], x[..., d:]
    c = cos_sin[:, :d].unsqueeze(1)
    s = cos_sin[:, d:].unsqueeze(1)
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], dim=-1).to(x.dtype)
