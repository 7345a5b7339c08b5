"""Generate tests/golden/engine_golden.json by running AgentServe's own Engine.

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_engine_golden.py --reference PATH

PATH is a checkout of krishs0404/agentserve (or set AGENTSERVE_REFERENCE).  Written:

* "traces": for each scheduler scenario of engine_scenarios.TRACE_SCENARIOS and the
  multi-turn prefix-cache scenario, the reference Engine.step loop (engine.py:217-252)
  with its Scheduler, policies and PrefixCache, driving the stand-in history model:
  per step the prefill batch, the decode batch and the completed requests, every
  request's output tokens and the EngineMetrics;
* "tokens": the reference Engine with its own LlamaModel (fp32, random-init N(0, 0.02)
  weights from oracle.weights, greedy) on two real-model scenarios: mixed ragged
  prefill + decode under combined batching with preemption (paged mode,
  forward_decode_paged; the pool is kept fp32 instead of the fp16 cast of
  engine.py:169-170), and multi-turn sessions over a shared prefix (the non-paged mode,
  whose prefix hits seed the cached K/V, run one request at a time so the zero-append
  of forward_decode_batch, llama.py:327, 372, never applies); each request's output
  tokens and the smallest top-1 / top-2 logit margin of every greedy choice.  The
  mixed stream also runs under agent-aware priority with preemption ("preempt").

The tests never import the reference; they compare agentserve_b200.B200Engine with
this file.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.weights import init_weights_  # noqa: E402
from tests.golden import engine_scenarios as E  # noqa: E402

OUT = HERE / "engine_golden.json"


def import_reference(path: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, path)
    from agentserve.engine import policies
    from agentserve.engine.engine import Engine
    from agentserve.engine.request import Request
    from agentserve.model.config import ModelConfig
    return Engine, Request, ModelConfig, policies


def fake_engine(Engine, ModelConfig, kw):
    cfg = ModelConfig(hidden_dim=64, n_heads=4, n_kv_heads=2, n_layers=1, vocab_size=E.VOCAB_FAKE,
                      max_seq_len=4096, intermediate_size=128)
    eng = Engine(config=cfg, use_mock=True, num_cache_blocks=8192, eos_token_id=-1,
                 temperature=0.0, **kw)
    eng.model = E.HistoryModelForReference()
    eng.classifier = E.ClassStub()
    eng.predictor = E.PredictorStub()
    return eng


def gen_traces(Engine, Request, ModelConfig, policies) -> dict:
    out = {}
    for name in E.TRACE_SCENARIOS:
        eng = fake_engine(Engine, ModelConfig, E.engine_kwargs(name, policies))
        out[name] = E.run_stream(eng, Request, E.trace_stream(name))
    eng = fake_engine(Engine, ModelConfig, dict(max_batch_size=3, max_prefill_per_step=2))
    c = E.MULTI_TURN
    plan = E.multi_turn_plan(E.VOCAB_FAKE, c["prefix_len"], c["sessions"], c["turns"],
                             c["suffix_median"], c["out_range"], c["seed"])
    out["multi_turn_prefix_cache"] = E.run_multi_turn(eng, Request, plan)
    return out


def real_engine(Engine, ModelConfig, paged: bool, kw):
    cfg = ModelConfig(**E.TOKEN_MODEL)
    # device=None: engine.py:110-113 picks "cpu" here (passing it explicitly trips
    # the local `import torch` of engine.py:111 at :118)
    eng = Engine(config=cfg, use_mock=False, device=None, use_paged_kv=paged,
                 num_cache_blocks=2048, eos_token_id=-1, temperature=0.0, **kw)
    init_weights_(eng.model, seed=E.TOKEN_SEED)
    if paged:
        eng.allocator.kv_pool = eng.allocator.kv_pool.float()
    eng.classifier = E.ClassStub()
    eng.predictor = E.PredictorStub()
    margins = []
    sample = eng._sample

    def _sample(logits):
        margins.extend(E.margins_of(logits))
        return sample(logits)

    eng._sample = _sample
    return eng, margins


def gen_tokens(Engine, Request, ModelConfig) -> dict:
    out = {}
    for name, spec in (("mixed", E.TOKEN_MIXED), ("preempt", E.TOKEN_PREEMPT)):
        eng, margins = real_engine(Engine, ModelConfig, True, spec["engine"])
        with torch.no_grad():
            res = E.run_stream(eng, Request, E.token_mixed_stream(spec))
        out[name] = dict(outputs=res["outputs"], metrics=res["metrics"],
                         prefills=sum(len(b) for b in res["prefill"]), min_margin=min(margins))
    eng, margins = real_engine(Engine, ModelConfig, False,
                               dict(max_batch_size=1, max_prefill_per_step=1))
    with torch.no_grad():
        res = E.run_multi_turn(eng, Request, E.token_multi_turn_plan())
    out["multi_turn"] = dict(outputs=res["outputs"], metrics=res["metrics"],
                             min_margin=min(margins))
    return out


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AGENTSERVE_REFERENCE"),
                    help="checkout of krishs0404/agentserve (or $AGENTSERVE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set AGENTSERVE_REFERENCE")
    Engine, Request, ModelConfig, policies = import_reference(args.reference)
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.time()
    data = dict(traces=gen_traces(Engine, Request, ModelConfig, policies))
    t1 = time.time()
    data["tokens"] = gen_tokens(Engine, Request, ModelConfig)
    OUT.write_text(json.dumps(data, separators=(",", ":")))
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes; traces {t1 - t0:.1f}s, "
          f"tokens {time.time() - t1:.1f}s)")
    for k, v in data["tokens"].items():
        print(k, "min margin", v["min_margin"], "metrics", v["metrics"])


if __name__ == "__main__":
    main()
