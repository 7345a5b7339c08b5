"""Continuous-batching engine on the B200 attention step, with AgentServe's Engine
surface (agentserve/engine/engine.py:67-399): submit / submit_many / step /
run_until_done / generate, `metrics` (EngineMetrics), `completed_requests`,
`scheduler`, `allocator`, `prefix_cache`, `model`.

One step is the reference's (engine.py:217-252): admit new requests (classify, look
up the prefix cache, allocate KV blocks), prefill the scheduler's prefill batch,
decode every decoding request by one token, free finished requests.  The scheduler
and its policies, request lifecycle and metrics behave as AgentServe's.  What runs
underneath is the device path:

* the prefill batch is ONE varlen forward (B200LlamaModel.forward_prefill_paged)
  writing every new token's K/V into its request's pool blocks, instead of one
  forward per request plus a per-token Python write loop (engine.py:228-229,
  311-315); the first tokens of all of them come back in one copy;
* the decode step replays a captured graph (pack, 16 layers, lm_head, greedy) and
  returns all next tokens in one copy, instead of a per-request sample().item()
  (engine.py:379-383);
* a prefix-cache hit shares the cached blocks with the new request (zero copy) and
  its prefill attends over them in place; the reference clones every layer's prefix
  K/V into the cache (engine.py:338-345) and, in its paged mode, drops them
  (engine.py:311-316: kv_cache is None after a paged prefill, so `store` keeps no
  K/V and a later hit prefills its suffix without the prefix);
* a request whose blocks do not fit waits in the admission queue (oldest first),
  after the least-used prefix-cache entries have been evicted to make room; the
  reference admits it without blocks (engine.py:286-289), which only its CPU mock
  model survives.

Sampling is greedy (temperature 0, sampling.py:46-58); other temperatures are
rejected.  The difficulty classifier and output-length predictor of AgentServe are
optional collaborators: pass objects with `classify(prompt)` (returning .level.value,
.priority, .estimated_output_tokens) and `predict(prompt)` / `update(prompt, n)`;
without them the request's own difficulty, priority and estimate are used.
"""

from __future__ import annotations

import time
from collections import deque
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import torch

from .cache import DeviceBlockAllocator
from .model import B200LlamaModel
from .prefix_cache import PrefixCache
from .scheduler import Scheduler


@dataclass
class EngineMetrics:
    """engine.py:42-64."""
    total_requests: int = 0
    completed_requests: int = 0
    total_prompt_tokens: int = 0
    total_output_tokens: int = 0
    prefix_cache_hits: int = 0
    prefix_cache_misses: int = 0
    prefix_tokens_saved: int = 0
    steps: int = 0
    wall_time: float = 0.0
    difficulty_counts: Dict[str, int] = field(
        default_factory=lambda: {"easy": 0, "medium": 0, "hard": 0})

    @property
    def throughput_tokens_per_sec(self) -> float:
        if self.wall_time <= 0:
            return 0.0
        return (self.total_prompt_tokens + self.total_output_tokens) / self.wall_time

    @property
    def prefix_hit_rate(self) -> float:
        total = self.prefix_cache_hits + self.prefix_cache_misses
        return self.prefix_cache_hits / total if total > 0 else 0.0


class _Speculation:
    """A decode step queued for `batch` before its inputs were confirmed."""

    def __init__(self, batch: List, expect_out: List[int], handle):
        self.batch, self.expect_out, self.handle = batch, expect_out, handle

    def positions_of(self, batch: List) -> Optional[List[int]]:
        """Row of each request of `batch` in the speculated step, or None if the step
        does not apply: `batch` must be the speculated requests in the same order
        (some may have finished), each with exactly the expected number of outputs."""
        idx = {id(r): i for i, r in enumerate(self.batch)}
        rows = []
        for r in batch:
            i = idx.get(id(r))
            if i is None or r.num_output_tokens != self.expect_out[i] or (rows and i <= rows[-1]):
                return None
            rows.append(i)
        return rows


class B200Engine:
    def __init__(self, config, *, model: Optional[B200LlamaModel] = None,
                 dtype: torch.dtype = torch.bfloat16, device: str = "cuda",
                 agent_aware: bool = True, max_batch_size: int = 8,
                 max_prefill_per_step: int = 4, num_cache_blocks: int = 256,
                 block_size: int = 16, eos_token_id: int = 2,
                 max_prefix_cache_entries: int = 512, temperature: float = 0.0,
                 top_p: float = 1.0, top_k: int = 0, enable_priority: bool = True,
                 enable_overflow: bool = True, enable_preemption: bool = True,
                 scheduler_policy=None, use_relative_batching: bool = False,
                 use_combined_batching: bool = False, classifier=None, predictor=None,
                 scheduler=None, max_seqs: int = 1024,
                 max_blocks_per_seq: Optional[int] = None):
        if temperature > 1e-6:
            raise ValueError("B200Engine samples greedily (temperature 0); "
                             f"temperature={temperature} is not supported")
        self.config = config
        self.eos_token_id = eos_token_id
        self.temperature, self.top_p, self.top_k = temperature, top_p, top_k
        self.model = model if model is not None else B200LlamaModel(config, dtype=dtype,
                                                                    device=device)
        self.device = self.model.device
        dtype = self.model.dtype
        # decode batches come in many (batch size, block bucket) shapes: keep their
        # captured graphs instead of recapturing as the batch grows and shrinks
        if hasattr(self.model, "max_decode_graphs"):
            self.model.max_decode_graphs = max(self.model.max_decode_graphs, 64)
        self.scheduler = scheduler if scheduler is not None else Scheduler(
            max_batch_size=max_batch_size, max_prefill_per_step=max_prefill_per_step,
            baseline_mode=not agent_aware, enable_priority=enable_priority,
            enable_overflow=enable_overflow, enable_preemption=enable_preemption,
            policy=scheduler_policy, use_relative_batching=use_relative_batching,
            use_combined_batching=use_combined_batching)
        self.use_relative_batching = use_relative_batching
        self.use_combined_batching = use_combined_batching
        if max_blocks_per_seq is None:
            max_blocks_per_seq = min(num_cache_blocks,
                                     -(-config.max_seq_len // block_size))
        self.allocator = DeviceBlockAllocator(
            num_blocks=num_cache_blocks, block_size=block_size, num_layers=config.n_layers,
            num_kv_heads=self.model.Kh, head_dim=config.head_dim, dtype=dtype,
            device=self.device, max_seqs=max_seqs, max_blocks_per_seq=max_blocks_per_seq)
        self.prefix_cache = PrefixCache(block_size=block_size,
                                        max_entries=max_prefix_cache_entries,
                                        allocator=self.allocator)
        self.classifier = classifier
        self.predictor = predictor
        self.metrics = EngineMetrics()
        self.completed_requests: List = []
        self._incoming: deque = deque()
        # leading tokens of a request whose blocks are shared (a prefix-cache hit, or
        # its own prefix stored in the cache): never rewritten, not even when the
        # request is preempted and prefilled again
        self._frozen: Dict[str, int] = {}
        self._hashes: Dict[str, tuple] = {}  # request id -> (prompt list, its block hashes)
        # queue the next decode step before reading this one's tokens (see _decode)
        self.speculative_decode: bool = True
        self._spec: Optional[_Speculation] = None
        self.spec_stats = {"queued": 0, "used": 0}

    # ------------------------------------------------------------------ submission
    def submit(self, request) -> None:
        self._incoming.append(request)

    def submit_many(self, requests) -> None:
        for r in requests:
            self.submit(r)

    def run_until_done(self, max_steps: int = 10_000) -> List:
        start = time.monotonic()
        for _ in range(max_steps):
            if self._is_idle():
                break
            self.step()
        self.metrics.wall_time = time.monotonic() - start
        return self.completed_requests

    def generate(self, requests, max_steps: int = 10_000) -> List:
        self.submit_many(requests)
        return self.run_until_done(max_steps=max_steps)

    def _is_idle(self) -> bool:
        return not self._incoming and self.scheduler.is_finished()

    # ------------------------------------------------------------------ one step
    def step(self) -> List:
        self.metrics.steps += 1
        self._ingest_incoming()
        batch = self.scheduler.get_prefill_batch()
        if batch:
            self._prefill(batch)
        decode = self.scheduler.get_decode_batch()
        if decode:
            self._decode(decode)
        else:
            self._spec = None
        done = self.scheduler.pop_completed()
        for req in done:
            self._release(req)
            self.metrics.completed_requests += 1
            self.metrics.total_output_tokens += req.num_output_tokens
            self.metrics.difficulty_counts[req.difficulty] = (
                self.metrics.difficulty_counts.get(req.difficulty, 0) + 1)
            self.completed_requests.append(req)
            if self.predictor is not None and req.num_output_tokens > 0:
                self.predictor.update(req.prompt, req.num_output_tokens)
        return done

    def _release(self, req) -> None:
        self.allocator.free(req.request_id)
        self._frozen.pop(req.request_id, None)
        self._hashes.pop(req.request_id, None)

    def _prompt_hashes(self, req) -> List[int]:
        """The prompt's chained block hashes, computed once per request (admission
        peeks, then looks up, and the prefill stores a prefix of the same prompt)."""
        h = self._hashes.get(req.request_id)
        if h is None or h[0] is not req.token_ids:
            h = self._hashes[req.request_id] = (req.token_ids,
                                                self.prefix_cache.block_hashes(req.token_ids))
        return h[1]

    # ------------------------------------------------------------------ admission
    def _classify(self, req) -> None:
        """engine.py:263-272."""
        if self.classifier is not None:
            diff = self.classifier.classify(req.prompt)
            req.difficulty = diff.level.value
            req.priority = diff.priority
            req.estimated_output_tokens = diff.estimated_output_tokens
        if self.predictor is not None and (self.use_relative_batching
                                           or self.use_combined_batching):
            req.estimated_output_tokens = int(self.predictor.predict(req.prompt))

    def _fits(self, req, shared_blocks: int) -> bool:
        need = self.allocator.blocks_needed(len(req.token_ids) + req.max_tokens) - shared_blocks
        return self.allocator.can_admit(max(need, 0), shared_blocks)

    def _ingest_incoming(self) -> None:
        """engine.py:258-294, admitting a request only when its blocks fit."""
        while self._incoming:
            req = self._incoming[0]
            hashes = self._prompt_hashes(req)
            matched, ids = self.prefix_cache.peek_longest_prefix(req.token_ids, hashes=hashes)
            if not self._fits(req, len(ids)):
                keep = req.token_ids[:matched] if matched else None
                while self.prefix_cache.size() > (1 if matched else 0) and \
                        not self._fits(req, len(ids)):
                    self.prefix_cache.evict_lfu(1, keep_tokens=keep)
                if not self._fits(req, len(ids)):
                    if self.scheduler.is_finished():  # nothing running will free blocks
                        need = self.allocator.blocks_needed(len(req.token_ids) + req.max_tokens)
                        raise MemoryError(
                            f"request {req.request_id} needs {need} KV-cache blocks "
                            f"({len(ids)} shared) or a free table row; the pool has "
                            f"{self.allocator.num_free_blocks()} free of "
                            f"{self.allocator.num_blocks}")
                    return  # wait for running requests to finish
            self._incoming.popleft()
            self._classify(req)
            matched, ids, _ = self.prefix_cache.find_longest_prefix(req.token_ids, hashes=hashes)
            req.num_cached_tokens = matched
            if matched > 0:
                self.metrics.prefix_cache_hits += 1
                self.metrics.prefix_tokens_saved += matched
                self.allocator.share_blocks(req.request_id, ids)
                self._frozen[req.request_id] = matched
            else:
                self.metrics.prefix_cache_misses += 1
            need = self.allocator.blocks_needed(len(req.token_ids) + req.max_tokens) - len(ids)
            self.allocator.allocate(req.request_id, max(need, 0))
            req.block_ids = self.allocator.blocks_for(req.request_id)
            self.metrics.total_requests += 1
            self.metrics.total_prompt_tokens += req.num_prompt_tokens
            self.scheduler.add(req)

    # ------------------------------------------------------------------ prefill
    def _prefill(self, batch: List) -> None:
        """engine.py:296-345 for the whole prefill batch in one forward."""
        bs = self.allocator.block_size
        for req in batch:
            # a preempted request restarts from 0 (scheduler.py:425-435) but keeps its
            # blocks: the shared / cached ones already hold its prefix K/V
            frozen = self._frozen.get(req.request_id, 0)
            if req.num_cached_tokens < frozen:
                req.num_cached_tokens = frozen
        first = self.model.prefill_paged_greedy([r.token_ids for r in batch],
                                                [r.num_cached_tokens for r in batch],
                                                self.allocator, [r.request_id for r in batch])
        for req, tok in zip(batch, first):
            req.num_cached_tokens = len(req.token_ids)
            self.scheduler.on_prefill_complete(req)
            req.output_token_ids.append(tok)
            if req.num_output_tokens >= req.max_tokens or tok == self.eos_token_id:
                req.mark_done()
                self.scheduler.decoding.remove(req)
                self.scheduler.completed.append(req)
            n = len(req.token_ids) // bs * bs
            if n > 0:
                ids = self.allocator.blocks_for(req.request_id)[:n // bs]
                if self.prefix_cache.store(req.token_ids[:n], ids,
                                           hashes=self._prompt_hashes(req)):
                    self._frozen[req.request_id] = max(self._frozen.get(req.request_id, 0), n)

    # ------------------------------------------------------------------ decode
    def _decode(self, batch: List) -> None:
        """engine.py:347-384: every decoding request advances one token.

        With speculative_decode (and a model that can queue steps), the next step of
        the same batch is queued on the device before this step's tokens are read back,
        fed by this step's output tokens on the device; the host's bookkeeping then
        overlaps the GPU instead of alternating with it.  It is used at the next step
        only if that step's decode batch is the same requests in the same order with
        exactly one more token each (requests that finished in between are dropped
        from it); otherwise it is discarded: its only effect was writing K/V for
        positions the real step rewrites, or in blocks of finished requests.  Tokens
        and scheduling decisions are the same either way."""
        spec, self._spec = self._spec, None
        rids = [r.request_id for r in batch]
        seq_lens = [r.num_cached_tokens + r.num_output_tokens - 1 for r in batch]
        launch = getattr(self.model, "decode_paged_greedy_launch", None)
        pick = spec.positions_of(batch) if spec is not None else None
        if pick is not None:
            handle, take = spec.handle, pick
            self.spec_stats["used"] += 1
        elif launch is not None:
            last = [r.output_token_ids[-1] for r in batch]
            handle, take = launch(last, seq_lens, self.allocator, rids), None
        else:  # a model with only the blocking call
            nxt = self.model.decode_paged_greedy([r.output_token_ids[-1] for r in batch],
                                                 seq_lens, self.allocator, rids)
            for req, tok in zip(batch, nxt):
                self.scheduler.on_decode_step(req, tok, self.eos_token_id)
            return
        # queue the next step now if it will most likely be this batch again; the
        # device feed needs this step's rows to be exactly the batch (a used
        # speculation with finished requests dropped has extra rows)
        same_rows = take is None or len(take) == len(spec.batch)
        if same_rows and self.speculative_decode and self._worth_speculating(batch):
            nxt_h = launch(None, [x + 1 for x in seq_lens], self.allocator, rids,
                           feed_from=handle)
            self._spec = _Speculation(list(batch), [r.num_output_tokens + 1 for r in batch],
                                      nxt_h)
            self.spec_stats["queued"] += 1
        toks = handle.result()
        if take is not None:
            toks = [toks[i] for i in take]
        for req, tok in zip(batch, toks):
            self.scheduler.on_decode_step(req, tok, self.eos_token_id)

    def _worth_speculating(self, batch: List) -> bool:
        """The next decode batch is likely this one again: nobody reaches max_tokens
        with this step's token, no request waits to be admitted, and no prefill can
        start (nothing pending, or the batch is at its cap)."""
        if self._incoming:
            return False
        if any(r.num_output_tokens + 1 >= r.max_tokens for r in batch):
            return False
        sch = self.scheduler
        return len(sch.decoding) >= sch.max_batch_size or not sch.pending
