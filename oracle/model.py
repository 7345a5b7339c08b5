"""Llama decoder restated from agentserve/model/llama.py (test infrastructure only).

Same parameter names and shapes as the reference LlamaModel (llama.py:245-262), so
state dicts move between the reference, this oracle and the B200 model.  The three
methods the engine calls are restated op for op:

  forward              llama.py:478-520 (prefill, optionally over a cached prefix)
  forward_decode_batch llama.py:265-376 (padded per-request KV lists)
  forward_decode_paged llama.py:379-475 (KV in an allocator's kv_pool)

`config` is duck-typed: hidden_dim, n_heads, n_kv_heads, n_layers, vocab_size,
max_seq_len, rms_norm_eps, rope_theta, intermediate_size, head_dim
(agentserve/model/config.py:10-30).
"""

from __future__ import annotations

import torch
import torch.nn as nn
import torch.nn.functional as F

from .attention import (decode_attention_padded, decode_attention_prepadded, flatten_decode_output,
                        prefill_attention)
from .rope import apply_rope, precompute_rope_freqs


class RMSNorm(nn.Module):
    """llama.py:39-56: fp32 rms, cast back, then scale by the weight."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (xf * r).to(x.dtype) * self.weight


class Attn(nn.Module):
    def __init__(self, c):
        super().__init__()
        H, Kh, D = c.n_heads, c.n_kv_heads, c.head_dim
        self.q_proj = nn.Linear(c.hidden_dim, H * D, bias=False)
        self.k_proj = nn.Linear(c.hidden_dim, Kh * D, bias=False)
        self.v_proj = nn.Linear(c.hidden_dim, Kh * D, bias=False)
        self.o_proj = nn.Linear(H * D, c.hidden_dim, bias=False)


class MLP(nn.Module):
    """llama.py:193-211 SwiGLU."""

    def __init__(self, c):
        super().__init__()
        self.gate_proj = nn.Linear(c.hidden_dim, c.intermediate_size, bias=False)
        self.up_proj = nn.Linear(c.hidden_dim, c.intermediate_size, bias=False)
        self.down_proj = nn.Linear(c.intermediate_size, c.hidden_dim, bias=False)

    def forward(self, x):
        return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))


class Layer(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.attn_norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.attn = Attn(c)
        self.ffn_norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.ffn = MLP(c)


class OracleLlama(nn.Module):
    def __init__(self, config):
        super().__init__()
        c = self.config = config
        self.embed = nn.Embedding(c.vocab_size, c.hidden_dim)
        self.layers = nn.ModuleList([Layer(c) for _ in range(c.n_layers)])
        self.norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.lm_head = nn.Linear(c.hidden_dim, c.vocab_size, bias=False)
        self.register_buffer("rope_table",
                             precompute_rope_freqs(c.head_dim, c.max_seq_len, c.rope_theta),
                             persistent=False)

    def _qkv(self, layer, h, n):
        c = self.config
        a = layer.attn
        return (a.q_proj(h).view(n, c.n_heads, c.head_dim),
                a.k_proj(h).view(n, c.n_kv_heads, c.head_dim),
                a.v_proj(h).view(n, c.n_kv_heads, c.head_dim))

    @torch.inference_mode()
    def forward(self, token_ids, kv_cache=None, position_offset: int = 0):
        """llama.py:478-520 with LlamaAttention.forward (llama.py:128-186) inlined."""
        dev = self.embed.weight.device
        if not isinstance(token_ids, torch.Tensor):
            token_ids = torch.tensor(token_ids, dtype=torch.long, device=dev)
        token_ids = token_ids.to(dev)
        T = token_ids.shape[0]
        x = self.embed(token_ids)
        cs = self.rope_table[torch.arange(position_offset, position_offset + T, device=dev)]
        new_cache = []
        for i, layer in enumerate(self.layers):
            h = layer.attn_norm(x)
            q, k, v = self._qkv(layer, h, T)
            q = apply_rope(q, cs)
            k = apply_rope(k, cs)
            if kv_cache is not None:
                k = torch.cat([kv_cache[i][0], k], dim=0)
                v = torch.cat([kv_cache[i][1], v], dim=0)
            new_cache.append((k, v))
            x = x + layer.attn.o_proj(prefill_attention(q, k, v))
            x = x + layer.ffn(layer.ffn_norm(x))
        return self.lm_head(self.norm(x)), new_cache

    @torch.inference_mode()
    def forward_decode_batch(self, last_token_ids, kv_caches, position_offsets):
        """llama.py:265-376."""
        B = len(last_token_ids)
        c = self.config
        if B == 0:
            return torch.zeros(0, c.vocab_size), []
        dev = self.rope_table.device
        x = self.embed(torch.tensor(last_token_ids, dtype=torch.long, device=dev))
        cs = self.rope_table[torch.tensor(position_offsets, dtype=torch.long, device=dev)]
        new = [[] for _ in range(B)]
        for li, layer in enumerate(self.layers):
            kh = [kv_caches[b][li][0] for b in range(B)]
            vh = [kv_caches[b][li][1] for b in range(B)]
            h = layer.attn_norm(x)
            q, kn, vn = self._qkv(layer, h, B)
            q = apply_rope(q, cs)
            kn = apply_rope(kn, cs)
            x = x + layer.attn.o_proj(flatten_decode_output(decode_attention_padded(q, kh, vh, kn, vn)))
            x = x + layer.ffn(layer.ffn_norm(x))
            # llama.py:327-328 appends the new token after the padding (column max_len)
            # and llama.py:370-372 keeps k_full[b, :L+1]: a sequence shorter than the
            # batch maximum stores a padding (zero) row in place of its new token.
            max_len = max(int(k.shape[0]) for k in kh)
            for b in range(B):
                L = int(kh[b].shape[0])
                kb = kn[b:b + 1] if L == max_len else torch.zeros_like(kn[b:b + 1])
                vb = vn[b:b + 1] if L == max_len else torch.zeros_like(vn[b:b + 1])
                new[b].append((torch.cat([kh[b].to(x.dtype), kb], 0),
                               torch.cat([vh[b].to(x.dtype), vb], 0)))
        return self.lm_head(self.norm(x)), new

    @torch.inference_mode()
    def forward_decode_paged(self, last_token_ids, seq_lens, position_offsets, allocator,
                             request_ids):
        """llama.py:379-475: gather history from the pool, write the new token's K/V
        (write_kv_decode), attend over history + new token."""
        B = len(last_token_ids)
        c = self.config
        if B == 0:
            return torch.zeros(0, c.vocab_size), None
        dev = self.rope_table.device
        x = self.embed(torch.tensor(last_token_ids, dtype=torch.long, device=dev))
        cs = self.rope_table[torch.tensor(position_offsets, dtype=torch.long, device=dev)]
        Kh, D = c.n_kv_heads, c.head_dim
        max_len = max(seq_lens)
        for li, layer in enumerate(self.layers):
            # llama.py:421-426: the history of every sequence gathered into zero padding,
            # one sequence at a time, before the projections
            kp = x.new_zeros(B, max_len, Kh, D)
            vp = x.new_zeros(B, max_len, Kh, D)
            for b, (rid, L) in enumerate(zip(request_ids, seq_lens)):
                k_b, v_b = allocator.gather_kv(rid, L, li)
                kp[b, :L] = k_b.to(dtype=x.dtype, device=dev)
                vp[b, :L] = v_b.to(dtype=x.dtype, device=dev)
            h = layer.attn_norm(x)
            q, kn, vn = self._qkv(layer, h, B)
            q = apply_rope(q, cs)
            kn = apply_rope(kn, cs)
            for b, (rid, L) in enumerate(zip(request_ids, seq_lens)):
                allocator.write_kv_decode(rid, L, li, kn[b], vn[b])
            attn = decode_attention_prepadded(q, kp, vp, kn, vn, seq_lens)
            x = x + layer.attn.o_proj(flatten_decode_output(attn))
            x = x + layer.ffn(layer.ffn_norm(x))
        return self.lm_head(self.norm(x)), None


def greedy(logits):
    """sampling.py:46-58 at temperature <= 1e-6: fp32 upcast, NaN -> 0, +inf -> 1e4,
    -inf -> -1e4, argmax (first maximum)."""
    lf = torch.nan_to_num(logits.float(), nan=0.0, posinf=1e4, neginf=-1e4)
    return lf.argmax(dim=-1)
