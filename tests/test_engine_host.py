"""Host side of the B200 engine (no GPU): its Scheduler, policies, PrefixCache and step
loop against AgentServe's own Engine.

tests/golden/engine_golden.json holds, for each scheduling mode (agent-aware priority
with overflow and preemption, combined and relative batching, baseline FIFO, the
priority and trajectory-progress policies, multi-turn sessions over a shared prefix),
what the reference Engine.step loop did with a stand-in model whose next token is a
fixed function of the token history: the prefill batch, decode batch and completed
requests of every step, each request's output and the EngineMetrics.  B200Engine runs
the same streams with the same stand-in on the CPU and must make the same decisions.
"""

import json
from pathlib import Path

import pytest
import torch

from agentserve_b200 import policies as P
from agentserve_b200.config import ModelConfig
from agentserve_b200.engine import B200Engine
from agentserve_b200.prefix_cache import PrefixCache, block_hash
from agentserve_b200.request import Request
from agentserve_b200.scheduler import Scheduler
from tests.golden import engine_scenarios as E

GOLDEN = json.loads((Path(__file__).parent / "golden" / "engine_golden.json").read_text())
FAKE_CFG = ModelConfig(hidden_dim=64, n_heads=4, n_kv_heads=2, n_layers=1, vocab_size=E.VOCAB_FAKE,
                       max_seq_len=4096, intermediate_size=128)


def fake_engine(num_cache_blocks=8192, **kw):
    return B200Engine(FAKE_CFG, model=E.HistoryModelForB200(), num_cache_blocks=num_cache_blocks,
                      eos_token_id=-1, classifier=E.ClassStub(), predictor=E.PredictorStub(),
                      **kw)


def assert_same_run(got, want):
    assert got["prefill"] == want["prefill"]
    assert got["decode"] == want["decode"]
    assert got["completed"] == want["completed"]
    assert got["outputs"] == want["outputs"]
    assert got["metrics"] == want["metrics"]


@pytest.mark.parametrize("name", list(E.TRACE_SCENARIOS))
def test_engine_step_loop_matches_reference_trace(name):
    eng = fake_engine(**E.engine_kwargs(name, P))
    got = E.run_stream(eng, Request, E.trace_stream(name))
    assert_same_run(got, GOLDEN["traces"][name])
    # every block is back: requests freed, nothing cached (no complete-block prompt
    # was stored twice) beyond what the prefix cache still holds
    held = sum(len(e.block_ids) for e in eng.prefix_cache._cache.values())
    assert eng.allocator.num_used_blocks() <= held


def test_multi_turn_prefix_hits_match_reference():
    eng = fake_engine(max_batch_size=3, max_prefill_per_step=2)
    c = E.MULTI_TURN
    plan = E.multi_turn_plan(E.VOCAB_FAKE, c["prefix_len"], c["sessions"], c["turns"],
                             c["suffix_median"], c["out_range"], c["seed"])
    got = E.run_multi_turn(eng, Request, plan)
    want = GOLDEN["traces"]["multi_turn_prefix_cache"]
    assert_same_run(got, want)
    assert want["metrics"]["prefix_cache_hits"] == 15
    assert eng.metrics.prefix_hit_rate == pytest.approx(15 / 16)


def test_preempted_request_keeps_shared_prefix_blocks():
    """A hard request on a cached prefix, preempted by an easy one, is prefilled
    again only past the blocks it shares (they are never rewritten)."""
    eng = fake_engine(max_batch_size=1, max_prefill_per_step=1)
    prefix = list(range(3, 3 + 32))
    warm = Request(prompt="hard 0 x", token_ids=prefix, max_tokens=1, request_id="warm")
    eng.generate([warm])
    hard = Request(prompt="hard 0 x", token_ids=prefix + [7, 8, 9], max_tokens=20,
                   request_id="h")
    eng.submit(hard)
    eng.step()
    eng.step()
    shared = eng.allocator.blocks_for("h")[:2]
    assert all(eng.allocator.ref_count(b) >= 2 for b in shared)
    easy = Request(prompt="easy 0 x", token_ids=[5, 6, 7], max_tokens=2, request_id="e")
    eng.submit(easy)
    calls = []
    pf = eng.model.prefill_paged_greedy

    def spy(toks, cached, alloc, rids):
        calls.append(dict(zip(rids, cached)))
        return pf(toks, cached, alloc, rids)

    eng.model.prefill_paged_greedy = spy
    eng.run_until_done()
    assert {"e": 0} in calls and {"h": 32} in calls  # re-prefill starts past the prefix
    assert len(hard.output_token_ids) == 20


def test_admission_waits_for_blocks_instead_of_skipping_allocation():
    """engine.py:286-289 admits a request without blocks when the pool is short (only
    its CPU mock model survives that).  B200Engine keeps it queued until running
    requests free enough blocks, and every request still completes."""
    stream = E.trace_stream("combined_batching")
    need = max(-(-(len(d["tokens"]) + d["max_tokens"]) // 16) for d in stream)
    eng = fake_engine(num_cache_blocks=need + 8, max_batch_size=6, max_prefill_per_step=3,
                      use_combined_batching=True)
    got = E.run_stream(eng, Request, stream, max_steps=5000)
    assert sorted(got["outputs"]) == sorted(GOLDEN["traces"]["combined_batching"]["outputs"])
    for rid, toks in got["outputs"].items():  # same tokens whatever the schedule
        assert toks == GOLDEN["traces"]["combined_batching"]["outputs"][rid]
    assert not eng._incoming and eng.scheduler.is_finished()


def test_request_that_can_never_fit_raises_memory_error():
    eng = fake_engine(num_cache_blocks=4)
    eng.submit(Request(prompt="easy 0 x", token_ids=list(range(100)), max_tokens=10))
    with pytest.raises(MemoryError):
        eng.step()


def test_admission_evicts_cold_prefix_entries_to_make_room():
    eng = fake_engine(num_cache_blocks=12, max_batch_size=2)
    a = Request(prompt="easy 0 x", token_ids=list(range(3, 3 + 64)), max_tokens=2,
                request_id="a")
    eng.generate([a])
    assert eng.prefix_cache.size() == 1 and eng.allocator.num_used_blocks() == 4
    b = Request(prompt="easy 0 x", token_ids=list(range(500, 500 + 150)), max_tokens=2,
                request_id="b")
    eng.generate([b])  # needs 10 of 12 blocks: the cached entry is evicted
    assert b.is_done and eng.prefix_cache.stats.evictions == 1


def test_greedy_only():
    with pytest.raises(ValueError):
        B200Engine(FAKE_CFG, model=E.HistoryModelForB200(), temperature=0.7)


# ----------------------------------------------------------------------- prefix cache
def test_prefix_cache_hash_and_matching():
    # chained blake2b of (previous hash, 4-byte little-endian ids), prefix_cache.py:62-68
    h1 = block_hash(list(range(16)))
    assert h1 == block_hash(list(range(16)), 0)
    assert block_hash(list(range(16)), h1) != h1
    pc = PrefixCache(block_size=4, max_entries=2)
    pc.store([1, 2, 3, 4, 5, 6, 7, 8], [10, 11, 99])
    assert pc._cache[pc._block_hashes([1, 2, 3, 4, 5, 6, 7, 8])[-1]].block_ids == [10, 11]
    assert pc.peek_longest_prefix([1, 2, 3, 4, 5, 6, 7, 8, 9]) == (8, [10, 11])
    assert pc.stats.hits == 0  # a peek is not counted
    assert pc.find_longest_prefix([1, 2, 3, 4, 5, 6, 7, 8, 9]) == (8, [10, 11], None)
    assert pc.find_longest_prefix([1, 2, 3, 4, 0, 0, 0, 0]) == (0, [], None)  # only final keys
    assert (pc.stats.hits, pc.stats.misses) == (1, 1)
    pc.store([9, 9, 9, 9], [5])
    pc.store([8, 8, 8, 8], [6])  # full: the lowest (reuse, last access) entry goes
    assert pc.stats.evictions == 1 and pc.size() == 2
    assert pc.peek_longest_prefix([1, 2, 3, 4, 5, 6, 7, 8])[0] == 8  # reused entry kept


def _plain_chain(tokens, bs=16):
    hs, prev = [], 0
    for i in range(len(tokens) // bs):
        prev = block_hash(tokens[i * bs:(i + 1) * bs], prev)
        hs.append(prev)
    return hs


def test_block_hashes_resume_the_chain_of_a_recent_prompt_exactly():
    """A prompt that begins like a recently hashed one reuses that chain up to the
    longest common block-aligned prefix and hashes the rest: the result must equal the
    chain computed from scratch (extensions, shared prefixes, a first difference inside
    a 64-block chunk or at its edge, prompts shorter than a block, memo eviction)."""
    rng = torch.Generator().manual_seed(0)
    rand = lambda n: torch.randint(3, 50000, (n,), generator=rng).tolist()  # noqa: E731
    pc = PrefixCache(block_size=16)
    base = rand(16 * 200 + 5)
    cases = [base, base + rand(40), base[:16 * 64] + rand(100), base[:16 * 64 + 7] + rand(50),
             base[:16 * 63] + rand(16), base[:16 * 130 + 3], base[:10], base[:16],
             rand(16 * 70) + base, base + rand(16 * 3)]
    for t in cases:
        assert pc.block_hashes(t) == _plain_chain(t), len(t)
    for i in range(80):  # more first blocks than the memo holds
        t = rand(16 * 3 + i)
        assert pc.block_hashes(t) == _plain_chain(t)
    assert pc.block_hashes(base + [1] * 16) == _plain_chain(base + [1] * 16)


def test_precomputed_hashes_give_the_same_lookups_and_entries():
    toks = list(range(1000, 1000 + 16 * 12 + 3))
    a, b = PrefixCache(), PrefixCache()
    hs = a.block_hashes(toks)
    assert a.store(toks[:16 * 8], list(range(8)), hashes=hs) == b.store(toks[:16 * 8], list(range(8)))
    assert a.peek_longest_prefix(toks, hashes=hs) == b.peek_longest_prefix(toks) == (128, list(range(8)))
    assert a.find_longest_prefix(toks, hashes=hs) == b.find_longest_prefix(toks)
    assert set(a._cache) == set(b._cache)


def test_scheduler_modes_basic():
    s = Scheduler(max_batch_size=2, max_prefill_per_step=2)
    reqs = [Request(prompt="x", token_ids=[1], max_tokens=3, priority=p) for p in (2, 0, 1)]
    for r in reqs:
        s.add(r)
    assert [r.priority for r in s.pending] == [0, 1, 2]
    b = s.get_prefill_batch()
    assert [r.priority for r in b] == [0, 1]
    for r in b:
        s.on_prefill_complete(r)
    assert s.get_prefill_batch() == []  # at capacity, hard request waits
    s2 = Scheduler(policy=P.FifoPolicy())
    for r in reqs:
        s2.add(r)
    assert s2.pending[0] is reqs[0] or s2.pending[0].arrival_time <= reqs[0].arrival_time


def test_deadline_policy_orders_urgent_first():
    pol = P.TrajectoryDeadlinePolicy(estimated_tps=50.0)
    late = Request(prompt="x", token_ids=[1], deadline=0.0)
    easy = Request(prompt="x", token_ids=[1], deadline=float("inf"))
    assert pol.priority_key(late) < pol.priority_key(easy)


def test_cpu_fake_engine_uses_no_gpu():
    eng = fake_engine()
    assert eng.allocator.kv_pool.device.type == "cpu"
    assert not torch.cuda.is_initialized()


@pytest.mark.parametrize("name", ["priority_overflow_preemption", "combined_batching"])
def test_queued_next_step_changes_nothing(name):
    """The engine queues the next decode step before reading this one's tokens when the
    batch will likely be the same; the decisions and outputs are the reference's either
    way, and the queued steps are used (or discarded when a preemption changes the
    batch)."""
    runs = {}
    for spec in (True, False):
        eng = fake_engine(**E.engine_kwargs(name, P))
        eng.speculative_decode = spec
        runs[spec] = (E.run_stream(eng, Request, E.trace_stream(name)), dict(eng.spec_stats))
    assert_same_run(runs[True][0], runs[False][0])
    assert_same_run(runs[True][0], GOLDEN["traces"][name])
    queued, used = runs[True][1]["queued"], runs[True][1]["used"]
    assert used > 0.5 * runs[True][0]["metrics"]["steps"] and used <= queued
    assert runs[False][1] == {"queued": 0, "used": 0}
