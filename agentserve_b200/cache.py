"""Device-resident paged KV allocator with the reference BlockAllocator's interface.

Host bookkeeping is the reference's (agentserve/engine/cache.py:33-119): a FIFO
free list, per-request block lists, ref counts, MemoryError on exhaustion.  What
changes is where the data lives:

* kv_pool [2, L, NB, 16, Kh, D] is allocated on the GPU in the model dtype
  (the reference engine forces fp16 after allocating on the host, engine.py:169-170);
* every live request owns a row of a device int32 block table
  [max_seqs, max_blocks_per_seq], updated only when blocks are allocated, so a
  decode step packs its batch on the device with no per-step host rebuild;
* write_kv_prefill / write_kv_decode / gather_kv are kernels (as_rope_reshape_and_cache
  without rotation, as_block_copy) instead of per-token index_put loops and
  per-block torch.cat (cache.py:125-189).
"""

from __future__ import annotations

from collections import deque
from typing import Dict, List, Optional, Sequence

import torch

from . import ops


class DeviceBlockAllocator:
    def __init__(self, num_blocks: int, block_size: int = 16, num_layers: int = 1,
                 num_kv_heads: int = 1, head_dim: int = 64, allocate_tensor: bool = True,
                 dtype: torch.dtype = torch.bfloat16, device: str | torch.device | None = None,
                 max_seqs: int = 256, max_blocks_per_seq: Optional[int] = None):
        if block_size != ops.BLOCK_SIZE:
            raise ValueError("the sm_100a kernels use 16-token blocks (block_size=16)")
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        # host bookkeeping (cache.py:54-58)
        self._ref = [0] * num_blocks
        self._free: deque[int] = deque(range(num_blocks))
        self._used: set[int] = set()
        self._request_blocks: Dict[str, List[int]] = {}
        # device block-table rows
        self.max_seqs = max_seqs
        self.max_blocks_per_seq = max_blocks_per_seq or num_blocks
        self._rows: Dict[str, int] = {}
        self._free_rows: deque[int] = deque(range(max_seqs))
        self.block_tables = torch.zeros(max_seqs, self.max_blocks_per_seq, dtype=torch.int32,
                                        device=self.device)
        self.kv_pool: Optional[torch.Tensor] = None
        if allocate_tensor:
            self.kv_pool = torch.zeros(2, num_layers, num_blocks, block_size, num_kv_heads,
                                       head_dim, dtype=dtype, device=self.device)

    # ------------------------------------------------------------------ bookkeeping
    def num_free_blocks(self) -> int:
        return len(self._free)

    def num_used_blocks(self) -> int:
        return len(self._used)

    def memory_usage(self) -> float:
        return self.num_used_blocks() / self.num_blocks

    def can_allocate(self, num_blocks_needed: int = 1) -> bool:
        return len(self._free) >= num_blocks_needed

    def allocate(self, request_id: str, num_blocks: int = 1) -> List[int]:
        """cache.py:85-101, plus the device table row of the request."""
        if not self.can_allocate(num_blocks):
            raise MemoryError(f"Out of KV-cache blocks: need {num_blocks}, have {len(self._free)}")
        have = len(self._request_blocks.get(request_id, []))
        if have + num_blocks > self.max_blocks_per_seq:
            raise MemoryError(f"request {request_id} would hold {have + num_blocks} blocks; "
                              f"the device table row holds {self.max_blocks_per_seq}")
        row = self._rows.get(request_id)
        if row is None:
            if not self._free_rows:
                raise MemoryError(f"no free block-table row (max_seqs={self.max_seqs})")
            row = self._free_rows.popleft()
            self._rows[request_id] = row
        out = []
        for _ in range(num_blocks):
            b = self._free.popleft()
            self._ref[b] = 1
            self._used.add(b)
            out.append(b)
        self._request_blocks.setdefault(request_id, []).extend(out)
        if out:
            self.block_tables[row, have:have + len(out)].copy_(self._host_ints(out, torch.int32),
                                                               non_blocking=True)
        return out

    def _host_ints(self, vals, dtype) -> torch.Tensor:
        t = torch.tensor(vals, dtype=dtype)
        return t.pin_memory() if self.device.type == "cuda" else t

    def free(self, request_id: str) -> None:
        """cache.py:103-111, plus releasing the device table row."""
        for b in self._request_blocks.pop(request_id, []):
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._used.discard(b)
                self._free.append(b)
        row = self._rows.pop(request_id, None)
        if row is not None:
            self._free_rows.append(row)

    # ------------------------------------------------------------------ prefix sharing
    def _check_live(self, block_ids: Sequence[int]) -> List[int]:
        ids = [int(b) for b in block_ids]
        for b in ids:
            if not (0 <= b < self.num_blocks) or self._ref[b] <= 0:
                raise ValueError(f"block {b} is not allocated")
        return ids

    def retain_blocks(self, block_ids: Sequence[int]) -> None:
        """Take a reference on live blocks (a prefix-cache entry keeping a finished
        request's prefix blocks), using the reference's per-block ref count
        (Block.ref_count, cache.py:24-30)."""
        for b in self._check_live(block_ids):
            self._ref[b] += 1

    def release_blocks(self, block_ids: Sequence[int]) -> None:
        """Drop references taken by retain_blocks; a block whose count reaches zero
        returns to the free list (in this order, like free())."""
        for b in self._check_live(block_ids):
            self._ref[b] -= 1
            if self._ref[b] == 0:
                self._used.discard(b)
                self._free.append(b)

    def share_blocks(self, request_id: str, block_ids: Sequence[int]) -> None:
        """Zero-copy prefix hit: the request's block list (and its device table row)
        starts with these live blocks, shared with their other holders, instead of a
        fresh copy of their K/V (engine.py:274-281 seeds a clone).  Shared blocks are
        read in place by the attention kernels; new tokens must land in blocks of the
        request's own, so share only full blocks (a block-aligned prefix match, as
        prefix_cache.py:110-183 makes) and allocate() the rest afterwards."""
        ids = self._check_live(block_ids)
        if self._request_blocks.get(request_id):
            raise ValueError(f"request {request_id} already holds blocks; share the prefix first")
        if len(ids) > self.max_blocks_per_seq:
            raise MemoryError(f"request {request_id} would hold {len(ids)} blocks; "
                              f"the device table row holds {self.max_blocks_per_seq}")
        row = self._rows.get(request_id)
        if row is None:
            if not self._free_rows:
                raise MemoryError(f"no free block-table row (max_seqs={self.max_seqs})")
            row = self._free_rows.popleft()
            self._rows[request_id] = row
        for b in ids:
            self._ref[b] += 1
        self._request_blocks[request_id] = list(ids)
        if ids:
            self.block_tables[row, :len(ids)].copy_(self._host_ints(ids, torch.int32),
                                                    non_blocking=True)

    def ref_count(self, block_id: int) -> int:
        return self._ref[block_id]

    def num_free_rows(self) -> int:
        return len(self._free_rows)

    def can_admit(self, num_blocks: int, shared: int = 0) -> bool:
        """True if a new request holding `shared` shared blocks plus `num_blocks` blocks
        of its own fits: free blocks, a free table row and the row's width."""
        return (len(self._free) >= num_blocks and bool(self._free_rows)
                and shared + num_blocks <= self.max_blocks_per_seq)

    _PAD_ID = "\x00pad"

    def scratch_row(self) -> int:
        """Table row of a one-block scratch sequence (taken once, never freed): padding
        rows of a bucketed decode batch write their dummy token there."""
        row = self._rows.get(self._PAD_ID)
        if row is None:
            self.allocate(self._PAD_ID, 1)
            row = self._rows[self._PAD_ID]
        return row

    def blocks_for(self, request_id: str) -> List[int]:
        return list(self._request_blocks.get(request_id, []))

    def blocks_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.block_size - 1) // self.block_size

    def row_of(self, request_id: str) -> int:
        return self._rows[request_id]

    def rows_for(self, request_ids: Sequence[str]) -> List[int]:
        return [self._rows[r] for r in request_ids]

    # ------------------------------------------------------------------ planes
    def k_plane(self, layer: int) -> torch.Tensor:
        return self.kv_pool[0, layer]

    def v_plane(self, layer: int) -> torch.Tensor:
        return self.kv_pool[1, layer]

    def _slots(self, request_id: str, first_pos: int, n: int) -> torch.Tensor:
        ids = self._request_blocks[request_id]
        bs = self.block_size
        s = [ids[p // bs] * bs + p % bs for p in range(first_pos, first_pos + n)]
        return self._host_ints(s, torch.int64).to(self.device, non_blocking=True)

    # ------------------------------------------------------------------ KV data
    def write_kv_prefill(self, request_id: str, layer: int, k: torch.Tensor,
                         v: torch.Tensor) -> None:
        """cache.py:125-140 as one kernel launch: k, v [T, Kh, D] to positions 0..T-1."""
        assert self.kv_pool is not None, "kv_pool not allocated (pass allocate_tensor=True)"
        T = k.shape[0]
        if T == 0:
            return
        ops.rope_reshape_and_cache(None, k.to(self.dtype).contiguous(),
                                   v.to(self.dtype).contiguous(), None,
                                   self._slots(request_id, 0, T), None, self.k_plane(layer),
                                   self.v_plane(layer))

    def write_kv_decode(self, request_id: str, token_pos: int, layer: int, k: torch.Tensor,
                        v: torch.Tensor) -> None:
        """cache.py:142-156: one token's k, v [Kh, D] to position token_pos."""
        assert self.kv_pool is not None
        ops.rope_reshape_and_cache(None, k.to(self.dtype).reshape(1, *k.shape[-2:]).contiguous(),
                                   v.to(self.dtype).reshape(1, *v.shape[-2:]).contiguous(), None,
                                   self._slots(request_id, token_pos, 1), None,
                                   self.k_plane(layer), self.v_plane(layer))

    def _block_ids(self, request_id: str, n: int) -> torch.Tensor:
        ids = self._request_blocks[request_id][:n]
        return self._host_ints(ids, torch.int32).to(self.device, non_blocking=True)

    def gather_blocks(self, request_id: str, n_blocks: int) -> torch.Tensor:
        """All layers' K and V of the request's first n_blocks blocks as one contiguous
        tensor [2, L, n_blocks, 16, Kh, D] (one kernel; the prefix-cache payload)."""
        assert self.kv_pool is not None
        out = torch.empty(2, self.num_layers, n_blocks, self.block_size, self.num_kv_heads,
                          self.head_dim, dtype=self.dtype, device=self.device)
        if n_blocks == 0:
            return out
        bpb = self.block_size * self.num_kv_heads * self.head_dim * self.kv_pool.element_size()
        ops.block_copy(out, self.kv_pool, self._block_ids(request_id, n_blocks), None, bpb,
                       2 * self.num_layers, self.num_blocks * bpb, n_blocks * bpb,
                       self.num_blocks, n_blocks)
        return out

    def seed_blocks(self, request_id: str, payload: torch.Tensor) -> None:
        """Copy a [2, L, n, 16, Kh, D] payload into the request's first n blocks (prefix
        cache hit, engine.py:274-281, without going through the host)."""
        assert self.kv_pool is not None
        n = payload.shape[2]
        if n == 0:
            return
        bpb = self.block_size * self.num_kv_heads * self.head_dim * self.kv_pool.element_size()
        src_ids = torch.arange(n, dtype=torch.int32, device=self.device)
        ops.block_copy(self.kv_pool, payload.contiguous(), src_ids, self._block_ids(request_id, n),
                       bpb, 2 * self.num_layers, n * bpb, self.num_blocks * bpb, n,
                       self.num_blocks)

    def gather_kv(self, request_id: str, seq_len: int, layer: int):
        """cache.py:158-189: contiguous [seq_len, Kh, D] K and V of one layer."""
        assert self.kv_pool is not None
        n = self.blocks_needed(seq_len)
        Kh, D = self.num_kv_heads, self.head_dim
        if n == 0:
            z = torch.zeros(0, Kh, D, dtype=self.dtype, device=self.device)
            return z, z
        out = torch.empty(2, n, self.block_size, Kh, D, dtype=self.dtype, device=self.device)
        bpb = self.block_size * Kh * D * self.kv_pool.element_size()
        plane_stride = self.num_layers * self.num_blocks * bpb  # K plane -> V plane
        src = self.kv_pool[0, layer]
        ops.block_copy(out, src, self._block_ids(request_id, n), None, bpb, 2, plane_stride,
                       n * bpb, self.num_blocks, n)
        return (out[0].view(n * self.block_size, Kh, D)[:seq_len],
                out[1].view(n * self.block_size, Kh, D)[:seq_len])
