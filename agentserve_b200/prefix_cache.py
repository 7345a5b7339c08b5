"""Prefix cache whose payload is the KV blocks themselves (zero copy).

Matching and eviction are AgentServe's (agentserve/engine/prefix_cache.py:62-211):
complete 16-token blocks are hashed in a chain (each block's hash covers every block
before it), an entry is keyed by the chained hash of its last block, a lookup walks a
prompt's block hashes from the longest down and verifies the tokens of the first hit,
and eviction takes the entry with the lowest (reuse_count, last_access_step).

What differs is the payload.  The reference stores a clone of every layer's K/V of
the prefix (engine.py:338-345; about 470 MB for a 14,336-token prefix of the 1B
model in bf16) and seeds a hit by handing those tensors to the forward pass.  Here an
entry holds the ids of the pool blocks that already contain that K/V: storing takes a
reference on them (DeviceBlockAllocator.retain_blocks), a hit shares them with the new
request (share_blocks) so its prefill reads them in place, and eviction drops the
reference (release_blocks).  No K/V byte moves.
"""

from __future__ import annotations

import hashlib
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np


@dataclass
class PrefixEntry:
    token_ids: List[int]
    block_ids: List[int]
    kv_tensors: Optional[list] = None  # always None here: the blocks are the payload
    reuse_count: int = 0
    last_access_step: int = 0


@dataclass
class PrefixCacheStats:
    hits: int = 0
    misses: int = 0
    evictions: int = 0
    tokens_saved: int = 0

    @property
    def hit_rate(self) -> float:
        total = self.hits + self.misses
        return self.hits / total if total else 0.0


def block_hash(tokens: Sequence[int], prev: int = 0) -> int:
    """64-bit chained hash of one block: blake2b over the previous hash (8 bytes, little
    endian) and the token ids (4 bytes each, little endian), prefix_cache.py:62-68."""
    return _chain(np.asarray(tokens, dtype="<u4").tobytes(), len(tokens), prev)[-1]


def _chain(token_bytes: bytes, block_size: int, prev: int = 0) -> List[int]:
    """Chained hashes of consecutive blocks of block_size 4-byte token ids."""
    step = 4 * block_size
    out = []
    for start in range(0, len(token_bytes) // step * step, step):
        h = hashlib.blake2b(prev.to_bytes(8, "little"), digest_size=8)
        h.update(token_bytes[start:start + step])
        prev = int.from_bytes(h.digest(), "little")
        out.append(prev)
    return out


class PrefixCache:
    def __init__(self, block_size: int = 16, max_entries: int = 1024, allocator=None):
        """allocator: the DeviceBlockAllocator whose blocks the entries point at
        (retained on store, released on eviction); None keeps ids only."""
        self.block_size = block_size
        self.max_entries = max_entries
        self.allocator = allocator
        self.stats = PrefixCacheStats()
        self._step = 0
        self._cache: Dict[int, PrefixEntry] = {}
        self._token_to_hash: Dict[tuple, int] = {}
        self._memo: Dict[bytes, List[int]] = {}

    def _block_hashes(self, token_ids: Sequence[int]) -> List[int]:
        """Chained hashes of every complete block (prefix_cache.py:94-104).  The last
        few prompts' hashes are memoised (an admission peeks and then looks up)."""
        n = len(token_ids) // self.block_size * self.block_size
        key = np.asarray(token_ids[:n], dtype="<u4").tobytes()
        hashes = self._memo.get(key)
        if hashes is None:
            hashes = _chain(key, self.block_size)
            self._memo[key] = hashes
            if len(self._memo) > 8:
                self._memo.pop(next(iter(self._memo)))
        return hashes

    def store(self, token_ids: Sequence[int], block_ids: Sequence[int],
              kv_tensors: Optional[list] = None) -> bool:
        """Cache a computed prefix of complete blocks whose K/V sit in block_ids
        (prefix_cache.py:110-149).  A prefix already cached only gets its counters
        bumped; otherwise the lowest-ranked entry is evicted when the cache is full.
        Returns True when a new entry now holds these blocks."""
        hashes = self._block_hashes(token_ids)
        if not hashes:
            return False
        key = hashes[-1]
        entry = self._cache.get(key)
        if entry is not None:
            entry.reuse_count += 1
            entry.last_access_step = self._step
            return False
        if len(self._cache) >= self.max_entries:
            self._evict_lfu(1)
        ids = [int(b) for b in block_ids[:len(hashes)]]
        if self.allocator is not None:
            self.allocator.retain_blocks(ids)
        self._cache[key] = PrefixEntry(list(token_ids), ids, None, 1, self._step)
        self._token_to_hash[tuple(token_ids)] = key
        return True

    def peek_longest_prefix(self, token_ids: Sequence[int]) -> Tuple[int, List[int]]:
        """find_longest_prefix without counting it (no stats, no reuse bump): what a
        lookup would return now, for sizing an admission before making it."""
        hashes = self._block_hashes(token_ids)
        for i in range(len(hashes) - 1, -1, -1):
            entry = self._cache.get(hashes[i])
            n = (i + 1) * self.block_size
            if entry is not None and entry.token_ids == list(token_ids[:n]):
                return n, list(entry.block_ids)
        return 0, []

    def find_longest_prefix(self, token_ids: Sequence[int]) -> Tuple[int, List[int], None]:
        """(matched tokens, block ids, None) for the longest cached prefix, or
        (0, [], None) (prefix_cache.py:151-183)."""
        self._step += 1
        hashes = self._block_hashes(token_ids)
        for i in range(len(hashes) - 1, -1, -1):
            entry = self._cache.get(hashes[i])
            if entry is None:
                continue
            n = (i + 1) * self.block_size
            if entry.token_ids == list(token_ids[:n]):
                entry.reuse_count += 1
                entry.last_access_step = self._step
                self.stats.hits += 1
                self.stats.tokens_saved += n
                return n, list(entry.block_ids), None
        self.stats.misses += 1
        return 0, [], None

    def _evict_lfu(self, n: int, keep_tokens: Optional[Sequence[int]] = None) -> None:
        ranked = sorted(self._cache.items(),
                        key=lambda kv: (kv[1].reuse_count, kv[1].last_access_step))
        if keep_tokens is not None:
            keep = list(keep_tokens)
            ranked = [kv for kv in ranked if kv[1].token_ids != keep]
        for key, entry in ranked[:n]:
            del self._cache[key]
            self._token_to_hash.pop(tuple(entry.token_ids), None)
            if self.allocator is not None:
                self.allocator.release_blocks(entry.block_ids)
            self.stats.evictions += 1

    def evict_lfu(self, n: int = 1, keep_tokens: Optional[Sequence[int]] = None) -> None:
        """Evict the n lowest-ranked entries (never the one cached for keep_tokens)."""
        self._evict_lfu(n, keep_tokens)

    def size(self) -> int:
        return len(self._cache)

    def clear(self) -> None:
        if self.allocator is not None:
            for entry in self._cache.values():
                self.allocator.release_blocks(entry.block_ids)
        self._cache.clear()
        self._token_to_hash.clear()
