"""Seeded request streams for the engine-level fixtures, and the harness that drives an
engine through them.

Used by tests/golden/make_engine_golden.py (which runs AgentServe's own Engine) and by
the tests (which run agentserve_b200.B200Engine), so both sides see the same requests,
arrival steps, classifier / predictor stubs and follow-up turns.

* Scheduler traces use a deterministic stand-in model: the next token is a function of
  the whole token history, so the decisions of both engines (which requests prefill,
  decode and finish at every step; prefix hits; metrics) can be compared exactly.
* Token scenarios use the real model (random-init N(0, 0.02) weights) in fp32.
"""

from __future__ import annotations

import math
from types import SimpleNamespace
from typing import Callable, Dict, List, Optional

import numpy as np
import torch

CLASSES = {"easy": (0, 20), "medium": (1, 100), "hard": (2, 256)}
VOCAB_FAKE = 1000


# --------------------------------------------------------------------------- stubs
class ClassStub:
    """Difficulty classifier stand-in: the class is the first word of the prompt."""

    def classify(self, prompt: str):
        name = prompt.split()[0]
        prio, est = CLASSES[name]
        return SimpleNamespace(level=SimpleNamespace(value=name), priority=prio,
                               estimated_output_tokens=est)


class PredictorStub:
    """Output-length predictor stand-in: class estimate plus a per-request offset
    (the prompt's second word), no learning."""

    def predict(self, prompt: str) -> float:
        words = prompt.split()
        return CLASSES[words[0]][1] + int(words[1])

    def update(self, prompt: str, n: int) -> None:
        pass


def history_token(history: List[int]) -> int:
    """Next token of the stand-in model: a fixed function of the whole history."""
    acc = 0
    for i, t in enumerate(history):
        acc = (acc * 31 + (i + 1) * int(t)) % 1_000_003
    return (acc + 7919 * len(history)) % VOCAB_FAKE


class HistoryModelForReference:
    """The stand-in model behind AgentServe's Engine (its non-paged interface,
    llama.py:265-376, 478-520).  Its "KV cache" is one layer holding the token history
    as a [len, 1] tensor, so prefix-cache clones and seeds carry the history along."""

    def __init__(self, vocab: int = VOCAB_FAKE):
        self.vocab = vocab

    def _logits(self, hist: List[int]) -> torch.Tensor:
        x = torch.zeros(1, self.vocab)
        x[0, history_token(hist)] = 1.0
        return x

    def forward(self, token_ids, kv_cache=None, position_offset: int = 0):
        prev = [] if kv_cache is None else [int(t) for t in kv_cache[0][0][:, 0].tolist()]
        hist = prev + [int(t) for t in token_ids]
        kv = torch.tensor(hist, dtype=torch.float32).view(-1, 1)
        return self._logits(hist), [(kv, kv.clone())]

    def forward_decode_batch(self, last_token_ids, kv_caches, position_offsets):
        logits, new = [], []
        for last, kv in zip(last_token_ids, kv_caches):
            hist = [int(t) for t in kv[0][0][:, 0].tolist()] + [int(last)]
            t = torch.tensor(hist, dtype=torch.float32).view(-1, 1)
            logits.append(self._logits(hist))
            new.append([(t, t.clone())])
        return torch.cat(logits), new


class _Handle:
    def __init__(self, tokens: List[int]):
        self.tokens = tokens

    def result(self) -> List[int]:
        return list(self.tokens)


class HistoryModelForB200:
    """The same stand-in behind agentserve_b200.B200Engine (its greedy paged methods),
    on the CPU.  A request's history is kept by position, like a KV cache: a decode step
    at position s writes its input token at s and forgets anything after it, so a step
    the engine queued ahead and then discarded leaves no trace."""

    def __init__(self, n_layers: int = 1):
        self.device = torch.device("cpu")
        self.dtype = torch.float32
        self.Kh = 1
        self.hist: Dict[str, List[int]] = {}

    def prefill_paged_greedy(self, token_ids, num_cached, allocator, request_ids):
        out = []
        for toks, c, rid in zip(token_ids, num_cached, request_ids):
            h = list(toks) if c < len(toks) else list(toks) + [toks[-1]]
            self.hist[rid] = h
            out.append(history_token(h))
        return out

    def decode_paged_greedy_launch(self, last_token_ids, seq_lens, allocator, request_ids,
                                   feed_from=None):
        if feed_from is not None:
            last_token_ids = feed_from.tokens
        out = []
        for last, s, rid in zip(last_token_ids, seq_lens, request_ids):
            h = self.hist[rid][:s] + [int(last)]
            self.hist[rid] = h
            out.append(history_token(h))
        return _Handle(out)

    def decode_paged_greedy(self, last_token_ids, seq_lens, allocator, request_ids):
        return self.decode_paged_greedy_launch(last_token_ids, seq_lens, allocator,
                                               request_ids).result()


# --------------------------------------------------------------------------- streams
def _lognormal(rng, median, sigma, lo, hi):
    return int(np.clip(round(rng.lognormal(math.log(median), sigma)), lo, hi))


def mixed_stream(seed: int, spec: List[tuple], vocab: int) -> List[dict]:
    """spec rows: (class, count, prompt median, (out lo, out hi), arrival step)."""
    rng = np.random.default_rng(seed)
    out = []
    for cls, count, med, (olo, ohi), step in spec:
        for _ in range(count):
            n = _lognormal(rng, med, 0.5, 4, 4 * med)
            out.append(dict(rid=f"q{len(out)}", cls=cls, step=step,
                            jitter=int(rng.integers(0, 17)),
                            tokens=rng.integers(3, vocab, n).tolist(),
                            max_tokens=int(rng.integers(olo, ohi + 1))))
    return out


# (name, engine kwargs, stream spec) of the stand-in-model trace scenarios
TRACE_SCENARIOS = {
    "priority_overflow_preemption": (
        dict(max_batch_size=4, max_prefill_per_step=2),
        [("hard", 4, 30, (30, 40), 0), ("easy", 6, 12, (3, 8), 3), ("medium", 4, 20, (10, 16), 5),
         ("easy", 3, 12, (3, 8), 20)]),
    "combined_batching": (
        dict(max_batch_size=6, max_prefill_per_step=3, use_combined_batching=True),
        [("easy", 18, 30, (3, 8), 0), ("medium", 9, 60, (8, 20), 0), ("hard", 3, 100, (20, 40), 0),
         ("easy", 4, 30, (3, 8), 10)]),
    "relative_batching": (
        dict(max_batch_size=5, max_prefill_per_step=2, use_relative_batching=True),
        [("easy", 8, 30, (3, 8), 0), ("medium", 8, 60, (8, 20), 0), ("hard", 4, 100, (20, 30), 0)]),
    "baseline_fifo": (
        dict(max_batch_size=3, max_prefill_per_step=2, agent_aware=False),
        [("hard", 3, 40, (10, 20), 0), ("easy", 6, 20, (3, 8), 0), ("medium", 3, 30, (6, 12), 2)]),
    "priority_policy": (
        dict(max_batch_size=3, max_prefill_per_step=2, policy="priority"),
        [("hard", 3, 40, (10, 20), 0), ("easy", 6, 20, (3, 8), 0), ("medium", 3, 30, (6, 12), 2)]),
    "trajectory_progress_policy": (
        dict(max_batch_size=3, max_prefill_per_step=2, policy="trajectory_progress"),
        [("medium", 10, 30, (4, 12), 0)]),
}

# multi-turn sessions over one shared prefix (the prefix-cache workload in miniature)
MULTI_TURN = dict(seed=7, prefix_len=96, sessions=5, turns=3, suffix_median=20,
                  out_range=(4, 12))


def multi_turn_plan(vocab: int, prefix_len: int, sessions: int, turns: int, suffix_median: int,
                    out_range, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    prefix = rng.integers(3, vocab, prefix_len).tolist()
    suffixes = [[rng.integers(3, vocab, _lognormal(rng, suffix_median, 0.5, 4, 4 * suffix_median)
                              ).tolist() for _ in range(turns)] for _ in range(sessions)]
    outs = [[int(rng.integers(out_range[0], out_range[1] + 1)) for _ in range(turns)]
            for _ in range(sessions)]
    return dict(prefix=prefix, suffixes=suffixes, outs=outs)


# --------------------------------------------------------------------------- harness
def _policy(name: Optional[str], mod):
    if name is None:
        return None
    return {"priority": mod.PriorityPolicy, "fifo": mod.FifoPolicy,
            "trajectory_progress": mod.TrajectoryProgressPolicy}[name]()


def make_request(Request, d: dict, index: int):
    """One request of a stream (class word, predictor offset word, token ids)."""
    r = Request(prompt=f"{d['cls']} {d['jitter']} request", token_ids=list(d["tokens"]),
                max_tokens=d["max_tokens"], request_id=d["rid"])
    r.arrival_time = 1000.0 + 0.001 * index
    if "step_index" in d:
        r.step_index, r.total_steps = d["step_index"], d["total_steps"]
    r.estimated_output_tokens = CLASSES[d["cls"]][1] + d["jitter"]
    return r


def record_batches(engine) -> dict:
    """Wrap the engine's scheduler so every prefill / decode batch it hands out is
    recorded (works for any scheduler with AgentServe's method names)."""
    log = {"prefill": [], "decode": []}
    sch = engine.scheduler
    gp, gd = sch.get_prefill_batch, sch.get_decode_batch

    def get_prefill_batch():
        b = gp()
        log["prefill"].append([r.request_id for r in b])
        return b

    def get_decode_batch():
        b = gd()
        log["decode"].append([r.request_id for r in b])
        return b

    sch.get_prefill_batch, sch.get_decode_batch = get_prefill_batch, get_decode_batch
    return log


def run_stream(engine, Request, stream: List[dict], max_steps: int = 2000) -> dict:
    """Submit each request at its arrival step and step the engine until idle.
    Returns the per-step trace, the output tokens and the metrics."""
    log = record_batches(engine)
    completed, by_step = [], {}
    for i, d in enumerate(stream):
        by_step.setdefault(d["step"], []).append((i, d))
    last_arrival = max(by_step) if by_step else 0
    for step in range(max_steps):
        for i, d in by_step.get(step, []):
            engine.submit(make_request(Request, d, i))
        if step > last_arrival and not engine._incoming and engine.scheduler.is_finished():
            break
        completed.append([r.request_id for r in engine.step()])
    return _result(engine, log, completed)


def run_multi_turn(engine, Request, plan: dict, warm: bool = True, max_steps: int = 4000) -> dict:
    """Sessions over a shared prefix: turn t of session s is submitted once turn t-1
    finished; its prompt is the previous prompt + its output + a new suffix.  With
    warm=True a prefix-only request (one output token) goes first so that first turns
    hit the cache on the shared prefix."""
    log = record_batches(engine)
    completed, outputs = [], {}
    S, T = len(plan["suffixes"]), len(plan["suffixes"][0])
    prompts = {}
    n_sub = 0

    def submit(rid, tokens, max_tokens, cls="medium"):
        nonlocal n_sub
        d = dict(rid=rid, cls=cls, jitter=0, tokens=tokens, max_tokens=max_tokens, step=0)
        engine.submit(make_request(Request, d, n_sub))
        n_sub += 1

    pending_first = True
    if warm:
        submit("warm", plan["prefix"], 1)
    for step in range(max_steps):
        if pending_first and (not warm or "warm" in outputs):
            for s in range(S):
                prompts[(s, 0)] = plan["prefix"] + plan["suffixes"][s][0]
                submit(f"s{s}t0", prompts[(s, 0)], plan["outs"][s][0])
            pending_first = False
        if not pending_first and not engine._incoming and engine.scheduler.is_finished():
            break
        done = engine.step()
        completed.append([r.request_id for r in done])
        for r in done:
            outputs[r.request_id] = list(r.output_token_ids)
            if r.request_id == "warm":
                continue
            s, t = (int(x) for x in r.request_id[1:].split("t"))
            if t + 1 < T:
                p = prompts[(s, t)] + list(r.output_token_ids) + plan["suffixes"][s][t + 1]
                prompts[(s, t + 1)] = p
                submit(f"s{s}t{t + 1}", p, plan["outs"][s][t + 1])
    return _result(engine, log, completed)


def _result(engine, log, completed) -> dict:
    m = engine.metrics
    outs = {r.request_id: list(r.output_token_ids) for r in engine.completed_requests}
    return dict(prefill=log["prefill"], decode=log["decode"], completed=completed, outputs=outs,
                metrics=dict(total_requests=m.total_requests,
                             completed_requests=m.completed_requests,
                             total_prompt_tokens=m.total_prompt_tokens,
                             total_output_tokens=m.total_output_tokens,
                             prefix_cache_hits=m.prefix_cache_hits,
                             prefix_cache_misses=m.prefix_cache_misses,
                             prefix_tokens_saved=m.prefix_tokens_saved, steps=m.steps,
                             difficulty_counts=dict(m.difficulty_counts)))


def trace_stream(name: str) -> List[dict]:
    _, spec = TRACE_SCENARIOS[name]
    stream = mixed_stream(sum(map(ord, name)), spec, VOCAB_FAKE)
    if name == "trajectory_progress_policy":
        for i, d in enumerate(stream):
            d["step_index"], d["total_steps"] = i % 4, 4
    return stream


def engine_kwargs(name: str, policies_module) -> dict:
    kw = dict(TRACE_SCENARIOS[name][0])
    kw["scheduler_policy"] = _policy(kw.pop("policy", None), policies_module)
    return kw


# --------------------------------------------------------------------------- real model
# The 1B attention geometry (32 query / 8 KV heads, head_dim 64, theta 5e5) with two
# layers, a small FFN and vocabulary, fp32.
TOKEN_MODEL = dict(hidden_dim=2048, n_heads=32, n_kv_heads=8, n_layers=2, vocab_size=512,
                   max_seq_len=2048, intermediate_size=1024, rms_norm_eps=1e-5,
                   rope_theta=500000.0)
TOKEN_SEED = 0

# mixed ragged prefill + decode (the mixed workload in miniature): under combined
# batching, and under agent-aware priority with overflow and preemption (hard requests
# first, easy ones arriving while they decode: the youngest hard one is sent back).
# Combined batching never preempts: scheduler.py:337-339 returns before
# _maybe_preempt whenever the decode batch is full, the only case it would act on.
TOKEN_MIXED = dict(
    seed=21, engine=dict(max_batch_size=4, max_prefill_per_step=2, use_combined_batching=True),
    spec=[("hard", 4, 120, (24, 40), 0), ("easy", 6, 40, (4, 10), 3),
          ("medium", 4, 80, (12, 24), 6)])
TOKEN_PREEMPT = dict(seed=22, engine=dict(max_batch_size=4, max_prefill_per_step=2),
                     spec=TOKEN_MIXED["spec"])
TOKEN_MULTI_TURN = dict(seed=8, prefix_len=160, sessions=4, turns=3, suffix_median=24,
                        out_range=(6, 14))


def token_mixed_stream(spec: dict = TOKEN_MIXED) -> List[dict]:
    return mixed_stream(spec["seed"], spec["spec"], TOKEN_MODEL["vocab_size"])


def token_multi_turn_plan() -> dict:
    c = TOKEN_MULTI_TURN
    return multi_turn_plan(TOKEN_MODEL["vocab_size"], c["prefix_len"], c["sessions"], c["turns"],
                           c["suffix_median"], c["out_range"], c["seed"])


def margins_of(logits: torch.Tensor) -> List[float]:
    """Top-1 minus top-2 logit of each row (how safe a greedy choice is)."""
    top = torch.topk(logits.float(), 2, dim=-1).values
    return (top[:, 0] - top[:, 1]).tolist()
