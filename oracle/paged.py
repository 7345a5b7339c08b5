"""Paged-KV bookkeeping restated from the reference (integer work, bit-exact).

Sources (krishs0404/agentserve):
  agentserve/engine/cache.py:33-119   BlockAllocator (free deque, ref counts, MemoryError)
  agentserve/engine/cache.py:125-156  write_kv_prefill / write_kv_decode slot arithmetic
  agentserve/engine/cache.py:158-189  gather_kv
  agentserve/engine/engine.py:349-357 decode positions / seq_lens
  agentserve/engine/engine.py:296-308 prefill from num_cached_tokens
"""

from __future__ import annotations

from collections import deque
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch


def blocks_needed(num_tokens: int, block_size: int) -> int:
    """cache.py:117-119 — ceil division."""
    return (num_tokens + block_size - 1) // block_size


def slot_of(block_ids: Sequence[int], pos: int, block_size: int) -> int:
    """cache.py:137-138 / 153-154 — block_ids[pos // bs] * bs + pos % bs."""
    return int(block_ids[pos // block_size]) * block_size + pos % block_size


def pack_decode(block_tables: List[List[int]], seq_lens: Sequence[int], block_size: int = 16):
    """Decode packing.  engine.py:350,356: position == seq_len == tokens cached before
    this step; the new token's K/V goes to that position (llama.py:437-439), and the
    attention then sees seq_len + 1 keys (llama.py:442-444)."""
    B = len(seq_lens)
    positions = np.asarray(seq_lens, dtype=np.int64)
    slots = np.array([slot_of(block_tables[b], int(seq_lens[b]), block_size) for b in range(B)],
                     dtype=np.int64)
    seq_lens_k = positions.astype(np.int32) + 1
    cu = np.arange(B + 1, dtype=np.int32)
    return positions, slots, seq_lens_k, cu


def pack_prefill(block_tables: List[List[int]], num_cached: Sequence[int],
                 num_new: Sequence[int], block_size: int = 16):
    """Varlen prefill packing.  engine.py:299-307 processes tokens from
    num_cached_tokens at position offset num_cached_tokens; cache.py:136-140 places
    token `tok` at block_ids[tok // bs], offset tok % bs."""
    R = len(num_new)
    cu = np.zeros(R + 1, dtype=np.int32)
    cu[1:] = np.cumsum(np.asarray(num_new, dtype=np.int64)).astype(np.int32)
    positions, slots = [], []
    for r in range(R):
        for i in range(int(num_new[r])):
            p = int(num_cached[r]) + i
            positions.append(p)
            slots.append(slot_of(block_tables[r], p, block_size))
    seq_lens_k = (np.asarray(num_cached, dtype=np.int64) + np.asarray(num_new, dtype=np.int64))
    return (cu, np.asarray(positions, dtype=np.int64), np.asarray(slots, dtype=np.int64),
            seq_lens_k.astype(np.int32))


def write_kv(k_plane: torch.Tensor, v_plane: torch.Tensor, block_ids: Sequence[int],
             first_pos: int, k: torch.Tensor, v: torch.Tensor) -> None:
    """cache.py:125-156 — per-token index_put of k/v [T, Kh, D] into planes
    [NB, BS, Kh, D] starting at position first_pos."""
    bs = k_plane.shape[1]
    for i in range(k.shape[0]):
        pos = first_pos + i
        b = int(block_ids[pos // bs])
        o = pos % bs
        k_plane[b, o] = k[i]
        v_plane[b, o] = v[i]


def gather_kv(plane: torch.Tensor, block_ids: Sequence[int], seq_len: int) -> torch.Tensor:
    """cache.py:158-189 — first seq_len tokens of a request, concatenated in order."""
    bs = plane.shape[1]
    n_full, rem = divmod(seq_len, bs)
    parts = [plane[int(block_ids[i])] for i in range(n_full)]
    if rem:
        parts.append(plane[int(block_ids[n_full]), :rem])
    if not parts:
        return plane.new_zeros(0, *plane.shape[2:])
    return torch.cat(parts, dim=0)


class OracleBlockAllocator:
    """cache.py:33-119 restated: FIFO free list, per-request block lists, MemoryError on
    exhaustion, optional physical pool kv_pool[2, L, NB, BS, Kh, D] (cache.py:60-66)."""

    def __init__(self, num_blocks: int, block_size: int = 16, num_layers: int = 1,
                 num_kv_heads: int = 1, head_dim: int = 64, allocate_tensor: bool = False,
                 dtype: torch.dtype = torch.float32, device: str | torch.device = "cpu"):
        self.num_blocks = num_blocks
        self.block_size = block_size
        self._ref = [0] * num_blocks
        self._free: deque[int] = deque(range(num_blocks))
        self._used: set[int] = set()
        self._request_blocks: Dict[str, List[int]] = {}
        self.kv_pool: Optional[torch.Tensor] = None
        if allocate_tensor:
            self.kv_pool = torch.zeros(2, num_layers, num_blocks, block_size, num_kv_heads,
                                       head_dim, dtype=dtype, device=device)

    def num_free_blocks(self) -> int:
        return len(self._free)

    def num_used_blocks(self) -> int:
        return len(self._used)

    def can_allocate(self, n: int = 1) -> bool:
        return len(self._free) >= n

    def allocate(self, request_id: str, num_blocks: int = 1) -> List[int]:
        if not self.can_allocate(num_blocks):
            raise MemoryError(f"Out of KV-cache blocks: need {num_blocks}, have {len(self._free)}")
        out = []
        for _ in range(num_blocks):
            b = self._free.popleft()
            self._ref[b] = 1
            self._used.add(b)
            out.append(b)
        self._request_blocks.setdefault(request_id, []).extend(out)
        return out

    def assign(self, request_id: str, block_ids: Sequence[int]) -> None:
        """Test helper: give a request an explicit (e.g. permuted) block list."""
        for b in block_ids:
            self._free.remove(b)
            self._ref[b] = 1
            self._used.add(b)
        self._request_blocks.setdefault(request_id, []).extend(int(b) for b in block_ids)

    def free(self, request_id: str) -> None:
        for b in self._request_blocks.pop(request_id, []):
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._used.discard(b)
                self._free.append(b)

    def blocks_for(self, request_id: str) -> List[int]:
        return list(self._request_blocks.get(request_id, []))

    def blocks_needed(self, num_tokens: int) -> int:
        return blocks_needed(num_tokens, self.block_size)

    def write_kv_prefill(self, request_id: str, layer: int, k: torch.Tensor, v: torch.Tensor):
        write_kv(self.kv_pool[0, layer], self.kv_pool[1, layer],
                 self._request_blocks[request_id], 0, k, v)

    def write_kv_decode(self, request_id: str, token_pos: int, layer: int, k: torch.Tensor,
                        v: torch.Tensor):
        write_kv(self.kv_pool[0, layer], self.kv_pool[1, layer],
                 self._request_blocks[request_id], token_pos, k[None], v[None])

    def gather_kv(self, request_id: str, seq_len: int, layer: int):
        ids = self._request_blocks[request_id]
        return (gather_kv(self.kv_pool[0, layer], ids, seq_len),
                gather_kv(self.kv_pool[1, layer], ids, seq_len))
