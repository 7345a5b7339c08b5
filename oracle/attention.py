"""Attention restated from agentserve/model/llama.py (prefill :128-186, decode :303-361
and :419-469).  torch's CPU scaled_dot_product_attention is called exactly where the
reference calls it; the GQA expansion, padding and masks are rebuilt the same way."""

from __future__ import annotations

from typing import List, Sequence

import torch
import torch.nn.functional as F

from .paged import gather_kv


def _expand_kv(x: torch.Tensor, n_heads: int) -> torch.Tensor:
    """llama.py:446-452: [B, S, Kh, D] -> [B, S, H, D], query head h reads KV head
    h // (H / Kh)."""
    B, S, Kh, D = x.shape
    g = n_heads // Kh
    if g == 1:
        return x
    return x.unsqueeze(3).expand(B, S, Kh, g, D).reshape(B, S, n_heads, D)


def decode_attention_padded(q: torch.Tensor, k_hist: List[torch.Tensor],
                            v_hist: List[torch.Tensor], k_new: torch.Tensor,
                            v_new: torch.Tensor) -> torch.Tensor:
    """One decode step as llama.py:303-361 / :419-469 compute it.

    q [B, H, D] (RoPE applied); k_hist[b]/v_hist[b] [L_b, Kh, D] cached history;
    k_new/v_new [B, Kh, D] the new token.  Returns the SDPA output [B, H, D] in
    q.dtype (flatten_decode_output gives the reference's [B, H*D] view).
    """
    B, H, D = q.shape
    Kh = k_new.shape[1]
    lens = [int(k.shape[0]) for k in k_hist]
    max_len = max(lens)
    kp = q.new_zeros(B, max_len, Kh, D)
    vp = q.new_zeros(B, max_len, Kh, D)
    for b in range(B):
        kp[b, :lens[b]] = k_hist[b].to(q.dtype)
        vp[b, :lens[b]] = v_hist[b].to(q.dtype)
    return decode_attention_prepadded(q, kp, vp, k_new, v_new, lens)


def decode_attention_prepadded(q: torch.Tensor, kp: torch.Tensor, vp: torch.Tensor,
                               k_new: torch.Tensor, v_new: torch.Tensor,
                               lens: Sequence[int]) -> torch.Tensor:
    """The rest of one decode step once the history is padded into kp/vp
    [B, max_len, Kh, D] (llama.py:441-469): append the new token, expand the KV heads,
    mask the padding columns, SDPA.  Returns [B, H, D]."""
    B, H, D = q.shape
    lens = [int(L) for L in lens]
    max_len = kp.shape[1]
    k_full = torch.cat([kp, k_new.unsqueeze(1)], dim=1)
    v_full = torch.cat([vp, v_new.unsqueeze(1)], dim=1)
    total = max_len + 1
    k4 = _expand_kv(k_full, H).transpose(1, 2)
    v4 = _expand_kv(v_full, H).transpose(1, 2)
    mask = None
    if min(lens) < max_len:  # llama.py:350-358: pad columns -> -inf
        lt = torch.tensor(lens, device=q.device)
        col = torch.arange(total, device=q.device)
        is_pad = (col[None, :] >= lt[:, None]) & (col[None, :] < max_len)
        mask = q.new_zeros(B, 1, 1, total)
        mask.masked_fill_(is_pad[:, None, None, :], float("-inf"))
    out = F.scaled_dot_product_attention(q.unsqueeze(2), k4, v4, attn_mask=mask)
    return out.squeeze(2)


def flatten_decode_output(o: torch.Tensor) -> torch.Tensor:
    """llama.py:362 / :470: the decode paths flatten the SDPA output [B, H, D] with
    `.transpose(1, 2).reshape(B, H*D)`, i.e. dim-major (element (h, d) lands at
    d*H + h) before o_proj.  Prefill (llama.py:184) flattens head-major instead."""
    B, H, D = o.shape
    return o.transpose(1, 2).reshape(B, H * D)


def decode_attention_from_pool(q: torch.Tensor, k_plane: torch.Tensor, v_plane: torch.Tensor,
                               block_tables: List[List[int]],
                               seq_lens_k: Sequence[int]) -> torch.Tensor:
    """Decode attention when the new token is already in the pool (the order the
    reference's paged path uses: write_kv_decode at llama.py:437-439, then attention
    over the history plus that token).  seq_lens_k[b] = cached tokens + 1.

    Planes are [NB, BS, Kh, D].  The history is gathered with gather_kv
    (cache.py:158-189) and the last token split off as the "new" one.
    """
    ks, vs, kn, vn = [], [], [], []
    for b, L in enumerate(seq_lens_k):
        k = gather_kv(k_plane, block_tables[b], int(L))
        v = gather_kv(v_plane, block_tables[b], int(L))
        ks.append(k[:-1])
        vs.append(v[:-1])
        kn.append(k[-1])
        vn.append(v[-1])
    return decode_attention_padded(q, ks, vs, torch.stack(kn), torch.stack(vn))


def prefill_attention(q: torch.Tensor, k_all: torch.Tensor, v_all: torch.Tensor) -> torch.Tensor:
    """llama.py:146-184 for one sequence: q [T, H, D] of the new tokens, k_all/v_all
    [P+T, Kh, D] = cached prefix followed by the new tokens.  The prefix is attended
    freely, the new tokens causally (mask of llama.py:171-180).  Returns [T, H*D]."""
    T, H, D = q.shape
    T_total, Kh, _ = k_all.shape
    g = H // Kh
    k = k_all
    v = v_all
    if g > 1:
        k = k.unsqueeze(2).expand(-1, -1, g, -1).reshape(T_total, H, D)
        v = v.unsqueeze(2).expand(-1, -1, g, -1).reshape(T_total, H, D)
    qh, kh, vh = q.transpose(0, 1), k.transpose(0, 1), v.transpose(0, 1)
    mask = None
    if T > 1:
        offset = T_total - T
        mask = torch.zeros(T, T_total, device=q.device, dtype=q.dtype)
        causal = torch.triu(torch.full((T, T), float("-inf"), device=q.device, dtype=q.dtype),
                            diagonal=1)
        mask[:, offset:] = causal
        mask = mask.unsqueeze(0)
    out = F.scaled_dot_product_attention(qh, kh, vh, attn_mask=mask)
    return out.transpose(0, 1).reshape(T, H * D)


def prefill_attention_from_pool(q: torch.Tensor, k_plane: torch.Tensor, v_plane: torch.Tensor,
                                block_tables: List[List[int]], cu_seqlens_q: Sequence[int],
                                seq_lens_k: Sequence[int]) -> torch.Tensor:
    """Varlen form of prefill_attention: sequence r's new tokens are q rows
    cu[r]..cu[r+1]-1 and its first seq_lens_k[r] tokens are in the pool."""
    outs = []
    for r in range(len(seq_lens_k)):
        a, b = int(cu_seqlens_q[r]), int(cu_seqlens_q[r + 1])
        if b == a:
            continue
        k = gather_kv(k_plane, block_tables[r], int(seq_lens_k[r]))
        v = gather_kv(v_plane, block_tables[r], int(seq_lens_k[r]))
        outs.append(prefill_attention(q[a:b], k, v))
    return torch.cat(outs, dim=0)
