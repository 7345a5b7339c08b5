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
from collections import OrderedDict
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
        # recently hashed prompts (token list, chained hashes), keyed by their first
        # block: a prompt that starts like one of them resumes its chain (multi-turn
        # sessions and a shared system prefix rehash only their new blocks)
        self._memo: "OrderedDict[tuple, Tuple[List[int], List[int]]]" = OrderedDict()

    def block_hashes(self, token_ids: Sequence[int]) -> List[int]:
        """Chained hashes of every complete block (prefix_cache.py:94-104).  A caller
        that looks a prompt up several times (peek, find, then store a prefix of it)
        can compute them once and pass them as `hashes`; the last few prompts' hashes
        are also memoised."""
        bs = self.block_size
        nb = len(token_ids) // bs
        if nb == 0:
            return []
        toks = list(token_ids)
        key = tuple(toks[:bs])
        done, hashes = 0, []
        hit = self._memo.get(key)
        if hit is not None:
            old, old_h = hit
            # longest common prefix in whole blocks: 64 blocks at a time, then block
            # by block inside the first chunk that differs
            m = min(nb, len(old_h))
            k = 0
            while k + 64 <= m and toks[k * bs:(k + 64) * bs] == old[k * bs:(k + 64) * bs]:
                k += 64
            while k < m and toks[k * bs:(k + 1) * bs] == old[k * bs:(k + 1) * bs]:
                k += 1
            done, hashes = k, old_h[:k]
        if done < nb:
            prev = hashes[-1] if hashes else 0
            tail = np.asarray(toks[done * bs:nb * bs], dtype="<u4").tobytes()
            hashes = hashes + _chain(tail, bs, prev)
        self._memo[key] = (toks, hashes)
        self._memo.move_to_end(key)
        if len(self._memo) > 64:
            self._memo.popitem(last=False)
        return hashes

    _block_hashes = block_hashes

    def _hashes(self, token_ids: Sequence[int], hashes: Optional[Sequence[int]]) -> Sequence[int]:
        if hashes is None:
            return self.block_hashes(token_ids)
        return hashes[:len(token_ids) // self.block_size]

    def store(self, token_ids: Sequence[int], block_ids: Sequence[int],
              kv_tensors: Optional[list] = None,
              hashes: Optional[Sequence[int]] = None) -> bool:
        """Cache a computed prefix of complete blocks whose K/V sit in block_ids
        (prefix_cache.py:110-149).  A prefix already cached only gets its counters
        bumped; otherwise the lowest-ranked entry is evicted when the cache is full.
        Returns True when a new entry now holds these blocks.  hashes: block_hashes()
        of token_ids or of a longer prompt it begins (computed here if omitted)."""
        hashes = self._hashes(token_ids, hashes)
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
        return True

    def peek_longest_prefix(self, token_ids: Sequence[int],
                            hashes: Optional[Sequence[int]] = None) -> Tuple[int, List[int]]:
        """find_longest_prefix without counting it (no stats, no reuse bump): what a
        lookup would return now, for sizing an admission before making it."""
        hashes = self._hashes(token_ids, hashes)
        for i in range(len(hashes) - 1, -1, -1):
            entry = self._cache.get(hashes[i])
            n = (i + 1) * self.block_size
            if entry is not None and entry.token_ids == list(token_ids[:n]):
                return n, list(entry.block_ids)
        return 0, []

    def find_longest_prefix(self, token_ids: Sequence[int],
                            hashes: Optional[Sequence[int]] = None
                            ) -> Tuple[int, List[int], None]:
        """(matched tokens, block ids, None) for the longest cached prefix, or
        (0, [], None) (prefix_cache.py:151-183)."""
        self._step += 1
        hashes = self._hashes(token_ids, hashes)
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
