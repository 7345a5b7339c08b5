"""Continuous-batching scheduler with AgentServe's agent-aware policies
(agentserve/engine/scheduler.py:54-447), the caller of the attention step.

Decisions are the reference's, step for step, so the B200 engine admits, batches and
preempts exactly the requests AgentServe's engine would; tests pin them against the
reference's own scheduler traces.  Modes:

* baseline (or enable_priority=False): one FIFO;
* agent-aware: one FIFO per priority (easy, medium, hard); an easy request may push
  the decode batch to the soft cap max_batch_size * overflow_factor; when every decode
  slot holds a hard request and an easy one waits, the hard request with the fewest
  output tokens (fewer than preempt_after_tokens) is sent back to the front of its
  queue and re-prefilled later;
* policy: a SchedulerPolicy orders one sorted pending list;
* relative batching: admit the window of requests (sorted by predicted output length)
  with the smallest variance minus an age credit;
* combined: priority tiers, relative batching inside each tier.
"""

from __future__ import annotations

import bisect
import statistics
import time
from collections import deque
from typing import List, Optional

from .request import RequestStatus

_AGE_WEIGHT = 0.15  # credit per second of waiting in the relative-batching score


def _tightest_window(candidates: list, n: int) -> list:
    """n requests whose predicted output lengths cluster most tightly, older requests
    breaking ties (scheduler.py:274-324, 357-378): windows of the length-sorted list
    scored by variance - 0.15 * (summed age); the first lowest score wins."""
    ordered = sorted(candidates, key=lambda r: r.estimated_output_tokens)
    best, best_score = ordered[:n], float("inf")
    now = time.monotonic()
    for i in range(len(ordered) - n + 1):
        window = ordered[i:i + n]
        lens = [r.estimated_output_tokens for r in window]
        var = statistics.variance(lens) if len(lens) > 1 else 0.0
        score = var - _AGE_WEIGHT * sum(now - r.arrival_time for r in window)
        if score < best_score:
            best, best_score = window, score
    return best


class Scheduler:
    def __init__(self, max_batch_size: int = 8, max_prefill_per_step: int = 4,
                 overflow_factor: float = 1.25, preempt_after_tokens: int = 10,
                 baseline_mode: bool = False, enable_priority: bool = True,
                 enable_overflow: bool = True, enable_preemption: bool = True,
                 policy=None, use_relative_batching: bool = False,
                 use_combined_batching: bool = False):
        self.max_batch_size = max_batch_size
        self.max_prefill_per_step = max_prefill_per_step
        self.overflow_factor = overflow_factor
        self.preempt_after_tokens = preempt_after_tokens
        self.baseline_mode = baseline_mode
        self.enable_priority = enable_priority and not baseline_mode
        self.enable_overflow = enable_overflow and not baseline_mode
        self.enable_preemption = enable_preemption and not baseline_mode
        self.soft_cap = int(max_batch_size * overflow_factor)
        self.use_relative_batching = use_relative_batching
        self.use_combined_batching = use_combined_batching
        self.policy = policy

        self._flat: List = []           # relative batching
        self._sorted: list = []         # policy: (key, arrival sequence, request)
        self._seq = 0
        self._tiers = (deque(), deque(), deque())  # easy, medium, hard
        self._fifo: deque = deque()     # baseline / priority disabled
        self.decoding: List = []
        self.completed: List = []

    # ------------------------------------------------------------------ queue views
    def _mode(self) -> str:
        if self.use_relative_batching:
            return "relative"
        if self.policy is not None:
            return "policy"
        if self.baseline_mode or not self.enable_priority:
            return "fifo"
        return "tiers"

    @property
    def pending(self) -> deque:
        mode = self._mode()
        if mode == "relative":
            return deque(self._flat)
        if mode == "policy":
            return deque(item[2] for item in self._sorted)
        if mode == "fifo":
            return deque(self._fifo)
        out = deque()
        for q in self._tiers:
            out.extend(q)
        return out

    def add(self, request) -> None:
        request.status = RequestStatus.PENDING
        mode = self._mode()
        if mode == "relative":
            self._flat.append(request)
        elif mode == "policy":
            bisect.insort(self._sorted, (self.policy.priority_key(request), self._seq, request))
            self._seq += 1
        elif mode == "fifo":
            self._fifo.append(request)
        else:
            self._tiers[request.priority].append(request)

    def _has_pending(self) -> bool:
        mode = self._mode()
        if mode == "relative":
            return bool(self._flat)
        if mode == "policy":
            return bool(self._sorted)
        if mode == "fifo":
            return bool(self._fifo)
        return any(self._tiers)

    def is_finished(self) -> bool:
        return not self._has_pending() and not self.decoding

    def _peek(self):
        mode = self._mode()
        if mode == "relative":
            return self._flat[0] if self._flat else None
        if mode == "policy":
            return self._sorted[0][2] if self._sorted else None
        if mode == "fifo":
            return self._fifo[0] if self._fifo else None
        for q in self._tiers:
            if q:
                return q[0]
        return None

    def _pop(self):
        if self.policy is not None:
            return self._sorted.pop(0)[2]
        if self.baseline_mode or not self.enable_priority:
            return self._fifo.popleft()
        for q in self._tiers:
            if q:
                return q.popleft()
        raise RuntimeError("no pending request to pop")

    # ------------------------------------------------------------------ batches
    def get_prefill_batch(self) -> List:
        """Requests to prefill this step (scheduler.py:174-204)."""
        if self.use_relative_batching:
            return self._prefill_relative()
        if self.use_combined_batching:
            return self._prefill_combined()
        if self._peek() is None:
            return []
        if self.enable_preemption:
            self._maybe_preempt()
        batch: List = []
        while len(batch) < self.max_prefill_per_step:
            cand = self._peek()
            if cand is None:
                break
            easy = cand.priority == 0
            cap = self.soft_cap if (self.enable_overflow and easy) else self.max_batch_size
            if len(self.decoding) + len(batch) >= cap:
                break
            req = self._pop()
            req.mark_prefill_start()
            batch.append(req)
        return batch

    def _prefill_relative(self) -> List:
        if not self._flat:
            return []
        slots = max(0, self.max_batch_size - len(self.decoding))
        n = min(self.max_prefill_per_step, slots, len(self._flat))
        if n == 0:
            return []
        chosen = _tightest_window(self._flat, n)
        ids = {id(r) for r in chosen}
        self._flat = [r for r in self._flat if id(r) not in ids]
        for r in chosen:
            r.mark_prefill_start()
        return chosen

    def _prefill_combined(self) -> List:
        slots = max(0, self.max_batch_size - len(self.decoding))
        if slots == 0:
            return []
        n = min(self.max_prefill_per_step, slots)
        if self.enable_preemption:
            self._maybe_preempt()
        batch: List = []
        for q in self._tiers:
            if len(batch) >= n or not q:
                continue
            cands = list(q)
            chosen = cands if len(cands) <= n - len(batch) else _tightest_window(
                cands, n - len(batch))
            for r in chosen:
                q.remove(r)
                r.mark_prefill_start()
                batch.append(r)
        return batch

    def get_decode_batch(self) -> List:
        return list(self.decoding)

    def on_prefill_complete(self, request) -> None:
        request.mark_first_token()
        self.decoding.append(request)

    def on_decode_step(self, request, token_id: int, eos_token_id: int = 1) -> bool:
        """Append one token; True when the request is done (scheduler.py:215-234)."""
        request.output_token_ids.append(token_id)
        done = len(request.output_token_ids) >= request.max_tokens or token_id == eos_token_id
        if done:
            request.mark_done()
            self.decoding.remove(request)
            self.completed.append(request)
            if self.policy is not None:
                self.policy.on_request_complete(request)
        return done

    def pop_completed(self) -> List:
        done = list(self.completed)
        self.completed.clear()
        return done

    # ------------------------------------------------------------------ preemption
    def _maybe_preempt(self) -> None:
        """An easy request waits and every decode slot is taken: send back the hard
        request with the fewest output tokens, if it has fewer than
        preempt_after_tokens (scheduler.py:406-423)."""
        if not self._tiers[0] or len(self.decoding) < self.max_batch_size:
            return
        hard = [r for r in self.decoding
                if r.priority == 2 and r.num_output_tokens < self.preempt_after_tokens]
        if hard:
            self._preempt(min(hard, key=lambda r: r.num_output_tokens))

    def _preempt(self, request) -> None:
        """Back to the front of its tier with its output discarded; it is prefilled
        again from scratch (scheduler.py:425-435)."""
        self.decoding.remove(request)
        request.status = RequestStatus.PENDING
        request.output_token_ids.clear()
        request.kv_cache = None
        request.num_cached_tokens = 0
        request.first_token_time = 0.0
        self._tiers[request.priority].appendleft(request)

    def stats(self) -> dict:
        return {"pending": len(self.pending), "decoding": len(self.decoding),
                "completed_this_epoch": len(self.completed), "baseline_mode": self.baseline_mode}
