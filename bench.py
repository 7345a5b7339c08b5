"""Decode throughput of the B200 attention step on the continuous-batching decode
workload (Llama-3.2-1B architecture, bf16, 64 sequences per GPU, contexts
U{128..4096}, 16-token paged blocks, greedy decoding).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 is launched by torchrun: one replica per GPU (request-partitioned, weak
scaling, no collective on the data path; a MAX all-reduce of the timings only).

One JSON line on rank 0:
  value         tokens/s of K graph-replayed decode steps, inputs resident in HBM;
  e2e           tokens/s through the reference-facing call
                model.forward_decode_paged(host lists ...) + greedy + device->host read;
  roofline      the paged decode attention kernel, timed alone with CUDA events;
  per_rank      each rank's step time and host-core affinity;
  strong        (N > 1) the same 64 sequences split over the N GPUs;
  config5       the 8B geometry at N GPUs: request-partitioned replicas, and (N > 1)
                KV-head tensor parallelism with one NCCL all-reduce per layer;
  prefill       the varlen prefill kernel alone on the prefix-cache workload's shape;
  config1       (N = 1) the single decode-attention op of the reference's CPU case,
                on the host (mean of 50) and on the GPU at batch 8 / 64 / 256;
  engine        (N = 1) the mixed-request and prefix-cache-session workloads through
                B200Engine;
  cpu_baseline  (N = 1) the oracle port of the reference's forward_decode_paged on the
                host cores, on the same 64 sequences.
"""

from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import torch

REPO = Path(__file__).resolve().parent
METRIC = "decode tok/s at 1/2/4/8 B200 + paged-attention achieved HBM GB/s"
WORKLOADS = {
    "1b": ("continuous-batching decode step, Llama-3.2-1B architecture (16 layers, hidden "
           "2048, 32/8 heads, head_dim 64, FFN 8192, vocab 128256), bf16, random-init "
           "N(0,0.02), {batch} sequences per GPU, contexts U{{{lo}..{hi}}}, 16-token blocks, "
           "greedy"),
    "8b": ("8B-geometry decode step (32 layers, hidden 4096, 32/8 heads, head_dim 128, FFN "
           "14336, vocab 128256), bf16, random-init N(0,0.02), {batch} sequences per GPU "
           "(request-partitioned replicas; 8 GPUs x 32 = the 256-sequence configuration), "
           "contexts U{{{lo}..{hi}}}, 16-token blocks, greedy"),
}
MODEL_DEFAULTS = {"1b": dict(batch=64, ctx_min=128, ctx_max=4096, layers=16, cpu_sample_seqs=64),
                  "8b": dict(batch=32, ctx_min=1024, ctx_max=32768, layers=32, cpu_sample_seqs=2)}


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--model", default="1b", choices=["1b", "8b"])
    ap.add_argument("--batch", type=int, default=None)
    ap.add_argument("--ctx-min", type=int, default=None)
    ap.add_argument("--ctx-max", type=int, default=None)
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--cpu-sample-seqs", type=int, default=None)
    ap.add_argument("--cpu-sample-steps", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--no-config1", action="store_true")
    ap.add_argument("--no-config5", action="store_true")
    ap.add_argument("--no-strong", action="store_true")
    ap.add_argument("--no-engine", action="store_true",
                    help="skip the engine workloads (mixed requests, prefix-cache sessions)")
    ap.add_argument("--engine-sessions", type=int, default=256)
    ap.add_argument("--engine-turns", type=int, default=4)
    ap.add_argument("--config5-steps", type=int, default=20)
    ap.add_argument("--blocks-per-split", type=int, default=0)
    ap.add_argument("--tp", action="store_true",
                    help="KV-head tensor parallelism over all ranks instead of replicas")
    ap.add_argument("--layers", type=int, default=None, help=argparse.SUPPRESS)
    args = ap.parse_args()
    for k, v in MODEL_DEFAULTS[args.model].items():
        if getattr(args, k) is None:
            setattr(args, k, v)
    return args


def dist_env():
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def config_8b(layers: int = 32):
    from agentserve_b200.config import ModelConfig
    return ModelConfig(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=layers,
                       vocab_size=128256, max_seq_len=33024 + 1024, rope_theta=500000.0,
                       intermediate_size=14336)


def model_config(args):
    from agentserve_b200.config import ModelConfig
    if args.model == "8b":
        return config_8b(args.layers)
    # the RoPE table covers the prefix-cache workload's longest prompts (~20K tokens)
    return ModelConfig(hidden_dim=2048, n_heads=32, n_kv_heads=8, n_layers=args.layers,
                       vocab_size=128256, max_seq_len=24576, rope_theta=500000.0,
                       intermediate_size=8192)


def workload(args) -> str:
    return WORKLOADS[args.model].format(batch=args.batch, lo=args.ctx_min, hi=args.ctx_max)


def context_lengths(batch, lo, hi, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (batch,), generator=g).tolist()


def line_config(args, world: int, tp: int) -> dict:
    """The `config` object of both arms' JSON lines (identical for the same N)."""
    cfg = model_config(args)
    B = args.batch * tp
    lens = context_lengths(B, args.ctx_min, args.ctx_max, 0)
    kv_gb = cfg.n_layers * decode_attention_bytes([L + 1 for L in lens], cfg.n_heads // tp,
                                                  cfg.n_kv_heads // tp, cfg.head_dim, 2) / 1e9
    H, hid, inter, V = cfg.n_heads, cfg.hidden_dim, cfg.intermediate_size, cfg.vocab_size
    w_gb = 2 * (2 * V * hid + cfg.n_layers * (2 * hid * H * cfg.head_dim // tp
                + 2 * hid * cfg.n_kv_heads * cfg.head_dim // tp + 3 * hid * inter)) / 1e9
    return {"workload": workload(args), "global_batch": B * (world // tp),
            "seq_len": f"{args.ctx_min}-{args.ctx_max} context + decode",
            "parallelism": (f"KV-head tensor parallel over {world} GPUs, one NCCL all-reduce "
                            f"per layer after o_proj, MLP replicated" if tp > 1 else
                            f"{world} request-partitioned replicas, no collective"),
            "cuda_graph": True, "blocks_per_split": args.blocks_per_split,
            "l2": (f"inputs larger than L2 every step (~{kv_gb:.1f} GB KV + ~{w_gb:.1f} GB "
                   f"weights per GPU)"),
            "kv": "context KV synthesised N(0,1) into the pool"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.idx = gpu_index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [r.split(",") for r in out.strip().splitlines() if r.count(",") >= 8]
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ------------------------------------------------------------------ CPU baseline
def _cpu_model_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return ""


def cpu_baseline(args, steps: int, warmup: int, seqs: int):
    """The oracle port of the reference's forward_decode_paged (llama.py:379-475: per
    layer and sequence gather_kv into zero padding, projections, RoPE, write_kv_decode,
    GQA expansion, masked SDPA, the same order of torch CPU operations) on the host
    cores, fp32, all threads: `seqs` of the workload's sequences (the same context
    lengths as the GPU run), `steps` timed decode steps after `warmup` untimed ones."""
    sys.path.insert(0, str(REPO))
    from oracle.model import OracleLlama
    from oracle.paged import OracleBlockAllocator
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = model_config(args)
    m = OracleLlama(cfg)
    g = torch.Generator().manual_seed(1234)
    with torch.no_grad():
        for p in m.parameters():
            if p.dim() == 2:
                p.normal_(0.0, 0.02, generator=g)
    m.eval()
    lens = context_lengths(args.batch, args.ctx_min, args.ctx_max, 0)[:seqs]
    total = steps + warmup + 1
    nb = sum((L + total + 15) // 16 for L in lens)
    a = OracleBlockAllocator(nb, 16, cfg.n_layers, cfg.n_kv_heads, cfg.head_dim,
                             allocate_tensor=True)
    a.kv_pool.normal_(0.0, 1.0, generator=g)
    rids = [f"c{i}" for i in range(len(lens))]
    for r, L in zip(rids, lens):
        a.allocate(r, (L + total + 15) // 16)
    last = torch.randint(3, cfg.vocab_size, (len(lens),), generator=g).tolist()
    cur = list(lens)
    t0 = 0.0
    for i in range(warmup + steps):
        if i == warmup:
            t0 = time.perf_counter()
        lg, _ = m.forward_decode_paged(last, cur, cur, a, rids)
        last = lg.float().argmax(-1).tolist()
        cur = [x + 1 for x in cur]
    dt = time.perf_counter() - t0
    return {"value": len(lens) * steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"oracle port of forward_decode_paged, fp32, {len(lens)} of the "
                       f"{args.batch} sequences (contexts {min(lens)}-{max(lens)}), {steps} timed "
                       f"step(s) after {warmup} warm-up, full {cfg.n_layers}-layer geometry, "
                       f"CPU {_cpu_model_name()}"),
            "seconds": dt}


def config1_inputs(batch: int, seed: int = 0, num_blocks: int = 512):
    """The single-op decode case: `batch` sequences with cached lengths U{17..1024}
    (torch.randint(17, 1025), seed 0), 16-token blocks from a random permutation of the
    pool (512 blocks, or as many as the batch needs), H=32 / Kh=8 / D=64, q and the pool
    N(0,1) fp32; the new token is already in the pool, so each sequence sees L+1 keys."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(17, 1025, (batch,), generator=g).tolist()
    need = sum((L + 1 + 15) // 16 for L in lens)
    num_blocks = max(num_blocks, need)
    perm = torch.randperm(num_blocks, generator=g)
    tables, off = [], 0
    for L in lens:
        n = (L + 1 + 15) // 16
        tables.append(perm[off:off + n].tolist())
        off += n
    q = torch.randn(batch, 32, 64, generator=g)
    kp = torch.randn(num_blocks, 16, 8, 64, generator=g)
    vp = torch.randn(num_blocks, 16, 8, 64, generator=g)
    return q, kp, vp, tables, [L + 1 for L in lens]


def config1_cpu(warmup: int = 3, reps: int = 50):
    """The attention section of the reference's forward_decode_paged on the CPU
    (gather_kv -> pad -> GQA expand -> masked SDPA, llama.py:421-469, as the oracle
    port restates it), fp32, batch 8: ms per op (mean of `reps` after `warmup`) and
    algorithmic GB/s."""
    sys.path.insert(0, str(REPO))
    from oracle import attention as OA
    torch.set_num_threads(os.cpu_count() or 1)
    q, kp, vp, tables, lk = config1_inputs(8)
    for _ in range(warmup):
        OA.decode_attention_from_pool(q, kp, vp, tables, lk)
    t0 = time.perf_counter()
    for _ in range(reps):
        OA.decode_attention_from_pool(q, kp, vp, tables, lk)
    ms = (time.perf_counter() - t0) / reps * 1e3
    nbytes = decode_attention_bytes(lk, 32, 8, 64, 4)
    return {"ms_per_op": ms, "gb_s": nbytes / (ms / 1e3) / 1e9, "algorithmic_bytes": nbytes,
            "cores": os.cpu_count() or 1, "kind": "port", "reps": reps, "warmup": warmup}


def config1_gpu(dev, reps: int = 20):
    """The same op on the GPU (as_paged_decode_attention): fp32 at batch 8 (the case
    itself) and bf16 at batch 8 / 64 / 256 with the same length distribution.  Each
    launch is timed alone with CUDA events after a 256 MB write that evicts L2, so the
    KV comes from HBM as it would in a step."""
    from agentserve_b200 import ops
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = {}
    for dtype, batches in ((torch.float32, (8,)), (torch.bfloat16, (8, 64, 256))):
        for B in batches:
            q, kp, vp, tables, lk = config1_inputs(B)
            q, kp, vp = q.to(dev, dtype), kp.to(dev, dtype), vp.to(dev, dtype)
            w = max(len(t) for t in tables)
            bt = torch.zeros(B, w, dtype=torch.int32)
            for i, t in enumerate(tables):
                bt[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
            bt = bt.to(dev)
            lkt = torch.tensor(lk, dtype=torch.int32, device=dev)
            ws = ops.new_decode_workspace(B, 32, 8, 64, w, 0, dev)
            o = torch.empty(B, 32 * 64, dtype=dtype, device=dev)
            for _ in range(3):
                ops.paged_decode_attention(q, kp, vp, bt, lkt, 0.125, 0, ws, out=o)
            tot = 0.0
            for _ in range(reps):
                flush.zero_()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                ops.paged_decode_attention(q, kp, vp, bt, lkt, 0.125, 0, ws, out=o)
                e1.record()
                torch.cuda.synchronize()
                tot += e0.elapsed_time(e1)
            ms = tot / reps
            nbytes = decode_attention_bytes(lk, 32, 8, 64, 4 if dtype == torch.float32 else 2)
            tag = f"{'fp32' if dtype == torch.float32 else 'bf16'}_b{B}"
            out[tag] = {"us_per_op": ms * 1e3, "gb_s": nbytes / (ms / 1e3) / 1e9,
                        "algorithmic_bytes": nbytes, "keys": sum(lk)}
    return out


# ------------------------------------------------------------------ helpers
def decode_attention_bytes(seq_lens_k, H, Kh, D, elem):
    """Algorithmic bytes of one paged decode attention launch: K+V of every visible
    token, q in, out, and the block-table entries read."""
    kv = sum(seq_lens_k) * Kh * D * 2 * elem
    qo = 2 * len(seq_lens_k) * H * D * elem
    bt = 4 * sum((L + 15) // 16 for L in seq_lens_k)
    return kv + qo + bt


def load_traffic():
    p = REPO / "profiles" / "decode_attention_config2_traffic.json"
    if not p.exists():
        return None
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return None


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d["hbm_gbs"]), "measured"
        except (OSError, ValueError, KeyError):
            pass
    return 6650.0, "fallback"


def prefill_flops(num_cached, num_new, H, D):
    """Algorithmic FLOPs of varlen prefill attention: QK^T and PV over the visible
    (query, key) pairs only, 2 FLOPs per MAC: 4*H*D*sum(T*P + T(T+1)/2)."""
    return sum(4 * H * D * (T * P + T * (T + 1) // 2) for P, T in zip(num_cached, num_new))


def measure_prefill(dev, reps: int = 10, D: int = 64):
    """The prefix-cache workload's prefill shape (a 14,336-token cached prefix plus a
    600-token suffix, 32/8 heads of head_dim D: 64 is the Llama-3.2-1B geometry, 128 the
    8B one, bf16), as the reference runs it (one request per call) and as a varlen batch
    of 8 such requests, on the varlen prefill kernel alone; CUDA events around `reps`
    launches."""
    from agentserve_b200 import ops
    H, Kh = 32, 8
    res = {}
    for tag, R in (("1x", 1), ("8x", 8)):
        num_cached, num_new = [14336] * R, [600] * R
        lens = [c + n for c, n in zip(num_cached, num_new)]
        nb = [(L + 15) // 16 for L in lens]
        NB = sum(nb)
        g = torch.Generator(device=dev).manual_seed(5)
        kp = torch.randn(NB, 16, Kh, D, device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
        vp = torch.randn(NB, 16, Kh, D, device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
        q = torch.randn(sum(num_new), H, D, device=dev, generator=g, dtype=torch.float32).to(torch.bfloat16)
        bt = torch.zeros(R, max(nb), dtype=torch.int32)
        perm = torch.randperm(NB, generator=torch.Generator().manual_seed(6))
        off = 0
        for i, n in enumerate(nb):
            bt[i, :n] = perm[off:off + n].to(torch.int32)
            off += n
        bt = bt.to(dev)
        cu = torch.tensor([0] + list(torch.cumsum(torch.tensor(num_new), 0).tolist()),
                          dtype=torch.int32, device=dev)
        lk = torch.tensor(lens, dtype=torch.int32, device=dev)
        out = torch.empty(sum(num_new), H * D, device=dev, dtype=torch.bfloat16)
        need = ops.prefill_workspace_bytes(R, max(num_new), H, Kh, D, bt.shape[1])
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=dev)
        for _ in range(2):
            ops.varlen_prefill_attention(q, kp, vp, bt, cu, lk, max(num_new), D ** -0.5, out=out,
                                         workspace=ws)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            ops.varlen_prefill_attention(q, kp, vp, bt, cu, lk, max(num_new), D ** -0.5, out=out,
                                         workspace=ws)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / reps
        fl = prefill_flops(num_cached, num_new, H, D)
        res[tag] = {"ms": ms, "tflops": fl / (ms / 1e3) / 1e12, "flops": fl}
    return res


def measured_bf16_peak():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except (OSError, ValueError, KeyError):
            pass
    return 1590.0, "fallback"


# ------------------------------------------------------------------ engine workloads
class _Classes:
    """Synthetic request classes for the engine workloads: the prompt text's first word
    is the class (the engine's difficulty classifier hook), its second the predicted
    output length (the output-length predictor hook)."""
    EST = {"easy": (0, 20), "medium": (1, 100), "hard": (2, 256)}

    def classify(self, prompt):
        from types import SimpleNamespace
        name = prompt.split()[0]
        prio, est = self.EST[name]
        return SimpleNamespace(level=SimpleNamespace(value=name), priority=prio,
                               estimated_output_tokens=est)

    def predict(self, prompt):
        return float(prompt.split()[1])

    def update(self, prompt, n):
        pass


def _lognormal_len(rng, median, lo=16, hi=4096, sigma=0.5):
    import numpy as np
    return int(np.clip(round(rng.lognormal(math.log(median), sigma)), lo, hi))


def _prefill_timer(eng):
    """Wrap the engine model's batched prefill to time it (host clock around the call,
    which ends with the first tokens' device-to-host copy) and add up the attention
    FLOPs of every prefill batch (4*H*D*(T*P + T(T+1)/2) per request)."""
    st = {"s": 0.0, "attn_flops": 0, "new_tokens": 0, "calls": 0}
    m = eng.model
    inner = m.prefill_paged_greedy
    H, D = m.H, m.D

    def timed(token_ids, num_cached, allocator, request_ids):
        t0 = time.perf_counter()
        out = inner(token_ids, num_cached, allocator, request_ids)
        st["s"] += time.perf_counter() - t0
        for toks, c in zip(token_ids, num_cached):
            T = max(1, len(toks) - c)
            st["attn_flops"] += 4 * H * D * (T * c + T * (T + 1) // 2) * m.config.n_layers
            st["new_tokens"] += T
        st["calls"] += 1
        return out

    m.prefill_paged_greedy = timed
    return st


def _engine_summary(eng, wall, pst, extra):
    met = eng.metrics
    lat = {}
    for cls in ("easy", "medium", "hard"):
        rs = [r for r in eng.completed_requests if r.difficulty == cls]
        if rs:
            lat[cls] = {"n": len(rs), "mean_latency_s": statistics.mean(r.latency for r in rs),
                        "mean_ttft_s": statistics.mean(r.ttft for r in rs)}
    out = {"wall_s": wall, "steps": met.steps, "requests": met.completed_requests,
           "queued_decode_steps": dict(getattr(eng, "spec_stats", {})),
           "prompt_tokens": met.total_prompt_tokens, "output_tokens": met.total_output_tokens,
           "output_tok_s": met.total_output_tokens / wall,
           "engine_throughput_tok_s": (met.total_prompt_tokens + met.total_output_tokens) / wall,
           "prefill": {"seconds": pst["s"], "calls": pst["calls"], "new_tokens": pst["new_tokens"],
                       "attention_flops": pst["attn_flops"],
                       "attention_tflops_over_prefill_time":
                           pst["attn_flops"] / max(pst["s"], 1e-9) / 1e12},
           "per_class": lat}
    out.update(extra)
    return out


def _reset_engine(eng) -> None:
    """Between the warm-up and the timed run on one engine: drop the cached prefixes
    (their blocks return to the pool) and start the counters afresh."""
    from agentserve_b200 import EngineMetrics
    eng.prefix_cache.clear()
    eng.metrics = EngineMetrics()
    eng.completed_requests = []
    eng.spec_stats = {"queued": 0, "used": 0}


def _mixed_requests(seed: int, tag: str):
    import numpy as np
    from agentserve_b200 import Request
    rng = np.random.default_rng(seed)
    spec = [("easy", 64, 300, (10, 30)), ("medium", 27, 800, (100, 300)),
            ("hard", 9, 1500, (500, 1000))]
    reqs = []
    for cls, n, med, (lo, hi) in spec:
        for _ in range(n):
            L = _lognormal_len(rng, med)
            out = int(rng.integers(lo, hi + 1))
            est = _Classes.EST[cls][1] + int(rng.integers(0, 17))
            reqs.append(Request(prompt=f"{cls} {est} synthetic agent call",
                                token_ids=rng.integers(3, 128000, L).tolist(), max_tokens=out,
                                request_id=f"{tag}{len(reqs)}"))
    return reqs


def engine_mixed(args, dev, model):
    """Mixed ragged prefill + decode: 100 agent requests at t=0 (64 easy: prompts
    lognormal median 300, outputs U[10,30]; 27 medium: 800, U[100,300]; 9 hard: 1500,
    U[500,1000]; sigma 0.5, clipped to [16, 4096]), batch cap 32, overflow 1.25,
    priority + relative (combined) batching, EOS off, through B200Engine.  One untimed
    run of a differently seeded stream of the same shape warms the engine (cuBLAS
    algorithm choices, the decode graphs of each batch and block bucket); then the
    timed run."""
    from agentserve_b200 import B200Engine
    warm, reqs = _mixed_requests(100, "w"), _mixed_requests(0, "m")
    blocks = max(sum(-(-(len(r.token_ids) + r.max_tokens) // 16) for r in rs)
                 for rs in (warm, reqs)) + 64
    eng = B200Engine(model.config, model=model, max_batch_size=32, max_prefill_per_step=4,
                     num_cache_blocks=blocks, eos_token_id=-1, use_combined_batching=True,
                     classifier=_Classes(), predictor=_Classes(), max_seqs=256)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.generate(warm, max_steps=100_000)
    torch.cuda.synchronize()
    cold = time.perf_counter() - t0
    _reset_engine(eng)
    pst = _prefill_timer(eng)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.generate(reqs, max_steps=100_000)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    del model.prefill_paged_greedy
    res = _engine_summary(eng, wall, pst, {
        "workload": "100 synthetic agent requests at t=0 (64 easy / 27 medium / 9 hard, "
                    "prompts lognormal medians 300 / 800 / 1500, outputs U[10,30] / "
                    "U[100,300] / U[500,1000]), batch cap 32, overflow 1.25, priority + "
                    "relative batching, greedy, EOS off",
        "timing": "host wall clock around engine.generate (every step ends with its tokens "
                  "copied to the host), after one untimed run of another stream of the "
                  "same shape on the same engine",
        "first_run_wall_s": cold})
    del eng
    return res


def engine_decode(args, dev, model, steps: int, warmup: int, ranks=None, rank: int = 0):
    """The decode workload through B200Engine.step: this GPU's 64 sequences (contexts
    U{128..4096}, random token ids) are admitted and prefilled by the engine (untimed),
    then `warmup` and `steps` engine steps decode all 64 at once, each step staging the
    batch's positions and table rows in one pinned host-to-device copy and ending with
    its tokens on the host (the engine queues the next step on the device before it
    reads them).  With several ranks: barrier on both sides, the slowest rank's time."""
    import numpy as np
    from agentserve_b200 import B200Engine, Request
    lens = context_lengths(args.batch, args.ctx_min, args.ctx_max, seed=rank)
    rng = np.random.default_rng(3 + rank)
    n_out = warmup + steps + 32  # nobody finishes inside the timed steps
    reqs = [Request(prompt="medium 100 decode", token_ids=rng.integers(3, 128000, L).tolist(),
                    max_tokens=n_out, request_id=f"d{i}") for i, L in enumerate(lens)]
    blocks = sum(-(-(L + n_out) // 16) for L in lens) + 64
    eng = B200Engine(model.config, model=model, max_batch_size=args.batch,
                     max_prefill_per_step=16, num_cache_blocks=blocks, eos_token_id=-1,
                     max_seqs=args.batch + 8, max_blocks_per_seq=-(-(max(lens) + n_out) // 16))
    eng.submit_many(reqs)
    while len(eng.scheduler.decoding) < len(reqs):
        eng.step()
    for _ in range(warmup):
        eng.step()
    if ranks is not None:
        ranks.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out0 = sum(r.num_output_tokens for r in reqs)
    for _ in range(steps):
        eng.step()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    made = sum(r.num_output_tokens for r in reqs) - out0
    world = 1
    if ranks is not None:
        ranks.barrier()
        wall = ranks.max(wall)
        world = ranks.world
    res = {"value": world * made / wall, "unit": "tok/s", "steps": steps,
           "sequences": world * len(reqs), "ms_per_step": wall / steps * 1e3,
           "h2d_bytes_per_step": 3 * 4 * len(reqs), "d2h_bytes_per_step": 8 * len(reqs),
           "queued_decode_steps": dict(eng.spec_stats),
           "api": "B200Engine.step (scheduler, bookkeeping, one pinned copy of positions "
                  "and table rows in, the tokens out, every step)"}
    model.release_decode_graphs()
    del eng
    return res


def _session_plan(seed: int, sessions: int, turns: int):
    import numpy as np
    rng = np.random.default_rng(seed)
    prefix = rng.integers(3, 128000, 14336).tolist()
    suffix = [[rng.integers(3, 128000, _lognormal_len(rng, 600)).tolist() for _ in range(turns)]
              for _ in range(sessions)]
    outs = [[int(rng.integers(32, 513)) for _ in range(turns)] for _ in range(sessions)]
    return prefix, suffix, outs


def _run_sessions(eng, plan, tag: str) -> None:
    """A prefix-only request first, then every session's turns, turn t+1 submitted
    when turn t finishes (its prompt: turn t's prompt + output + the next suffix)."""
    from agentserve_b200 import Request
    prefix, suffix, outs = plan
    turns = len(suffix[0])
    prompts = {}

    def req(rid, toks, n):
        return Request(prompt="medium 100 session turn", token_ids=toks, max_tokens=n,
                       request_id=rid)

    eng.generate([req(f"{tag}warm", prefix, 1)])
    for s in range(len(suffix)):
        prompts[(s, 0)] = prefix + suffix[s][0]
        eng.submit(req(f"{tag}{s}t0", prompts[(s, 0)], outs[s][0]))
    while eng._incoming or not eng.scheduler.is_finished():
        for r in eng.step():
            s, t = (int(x) for x in r.request_id[len(tag):].split("t"))
            if t + 1 < turns:
                p = prompts[(s, t)] + list(r.output_token_ids) + suffix[s][t + 1]
                prompts[(s, t + 1)] = p
                eng.submit(req(f"{tag}{s}t{t + 1}", p, outs[s][t + 1]))


def engine_prefix(args, dev, model, sessions: int, turns: int):
    """Prefix-cache-heavy multi-turn: `sessions` sessions share a 14,336-token random
    prefix; turn t's prompt is the previous prompt + its output + a new suffix
    (lognormal median 600, clipped to 4096); outputs U[32,512].  One prefix-only
    request warms the cache first.  Batch cap 64; prefix hits share the cached
    blocks in place.  An untimed run of 32 sessions x 2 turns on another prefix warms
    the engine first."""
    from agentserve_b200 import B200Engine
    plan = _session_plan(1, sessions, turns)
    warm = _session_plan(2, min(sessions, 32), min(turns, 2))
    longest = 14336 + turns * (4096 + 512)
    suffix, outs = plan[1], plan[2]
    per_turn = [sum(len(suffix[s][t]) + outs[s][t] for s in range(sessions)) for t in range(turns)]
    blocks = 896 + 2 * sum(-(-p // 16) for p in per_turn) + 64 * sessions + 256
    eng = B200Engine(model.config, model=model, max_batch_size=64, max_prefill_per_step=4,
                     num_cache_blocks=blocks, eos_token_id=-1,
                     max_prefix_cache_entries=4 * sessions * turns + 16,
                     max_seqs=2 * sessions + 8, max_blocks_per_seq=-(-longest // 16))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _run_sessions(eng, warm, "w")
    torch.cuda.synchronize()
    cold = time.perf_counter() - t0
    _reset_engine(eng)
    pst = _prefill_timer(eng)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _run_sessions(eng, plan, "s")
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    del model.prefill_paged_greedy
    res = _engine_summary(eng, wall, pst, {
        "workload": (f"{sessions} sessions x {turns} turns sharing a 14,336-token prefix; "
                     "per-turn suffix lognormal median 600 (clip 4096), outputs U[32,512]; "
                     "one prefix-only warm-up request; batch cap 64; greedy, EOS off"),
        "prefix_hit_rate": eng.metrics.prefix_hit_rate,
        "prefix_tokens_saved": eng.metrics.prefix_tokens_saved,
        "timing": "host wall clock from the prefix-only request to the last turn, after an "
                  "untimed run of 32 sessions x 2 turns on another prefix, same engine",
        "warm_up_run_wall_s": cold})
    del eng
    return res


# ------------------------------------------------------------------ decode runs
class Ranks:
    """Barriers and cross-rank reductions (no-ops on one GPU)."""

    def __init__(self, world: int, dev):
        self.world, self.dev = world, dev

    def barrier(self):
        if self.world > 1:
            torch.distributed.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=self.dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    def gather(self, obj) -> list:
        if self.world == 1:
            return [obj]
        out = [None] * self.world
        torch.distributed.all_gather_object(out, obj)
        return out


def build_model(cfg, dev, tp: int, rank: int, group=None):
    """Random-init N(0, 0.02) weights of the architecture, seeded; under KV-head TP the
    sharded projections get per-rank seeds and everything else the same seed on every
    rank (as replicated weights must be)."""
    from agentserve_b200 import B200LlamaModel
    model = B200LlamaModel(cfg, dtype=torch.bfloat16, device=dev, tp_size=tp,
                           tp_rank=rank if tp > 1 else 0, tp_group=group)
    sharded = ("q_proj", "k_proj", "v_proj", "o_proj")
    with torch.no_grad():
        for i, (n, p) in enumerate(model.named_parameters()):
            if p.dim() == 2:
                own = tp > 1 and any(k in n for k in sharded)
                g = torch.Generator(device=dev).manual_seed(
                    1000 + i + (rank if (tp == 1 or own) else 0) * 100003)
                p.normal_(0.0, 0.02, generator=g)
    model.eval()
    model.fuse_projections_()
    return model


class DecodeRun:
    """One decode batch resident on this GPU: its pool (context KV synthesised
    N(0,1)), block tables and a self-advancing captured decode step."""

    def __init__(self, model, lens, horizon: int, bps: int, seed: int,
                 token_seed: int | None = None):
        from agentserve_b200 import DeviceBlockAllocator
        cfg = model.config
        dev = model.device
        self.model, self.lens, self.bps = model, list(lens), bps
        self.B = len(lens)
        nblk = [(L + horizon + 15) // 16 for L in lens]
        self.alloc = DeviceBlockAllocator(sum(nblk), 16, cfg.n_layers, model.Kh, cfg.head_dim,
                                          dtype=torch.bfloat16, device=dev, max_seqs=self.B,
                                          max_blocks_per_seq=max(nblk))
        gen = torch.Generator(device=dev).manual_seed(77 + seed)
        self.alloc.kv_pool.normal_(0.0, 1.0, generator=gen)
        self.rids = [f"s{i}" for i in range(self.B)]
        for r, n in zip(self.rids, nblk):
            self.alloc.allocate(r, n)
        self.rows = self.alloc.rows_for(self.rids)
        self.max_blocks = max(nblk)
        # under KV-head TP every rank must feed the same tokens (token_seed shared)
        ts = seed if token_seed is None else token_seed
        self.tokens0 = torch.randint(3, cfg.vocab_size, (self.B,),
                                     generator=torch.Generator().manual_seed(7 + ts)).tolist()
        self.cur = list(lens)
        self.last = self.tokens0
        self.graph = None

    def timed_steps(self, ranks: Ranks, steps: int, warmup: int, clocks=None) -> float:
        """K replays of the captured step (CUDA events on the launching stream, barrier
        and synchronize on both sides); returns this rank's milliseconds."""
        from agentserve_b200 import DecodeGraph
        self.graph = DecodeGraph(self.model, self.alloc, self.B, self.max_blocks, self.bps,
                                 advance=True)
        self.graph.capture(self.last, self.cur, self.rows)
        for _ in range(warmup):
            self.graph.replay()
        torch.cuda.synchronize()
        if clocks is not None:
            clocks.start()
        ranks.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            self.graph.replay()
        e1.record()
        torch.cuda.synchronize()
        ranks.barrier()
        ms = e0.elapsed_time(e1)
        self.cur = [L + warmup + steps for L in self.cur]
        self.last = self.graph.next_tokens.cpu().tolist()
        self.graph.release()
        self.graph = None
        return ms

    def e2e_steps(self, ranks: Ranks, steps: int) -> float:
        """`steps` decode steps through forward_decode_paged(host lists) + greedy + a
        device-to-host read of the tokens, host wall clock; returns seconds."""
        from agentserve_b200 import greedy
        m = self.model
        for _ in range(2):  # captures forward_decode_paged's graph for this batch
            lg, _ = m.forward_decode_paged(self.last, self.cur, self.cur, self.alloc, self.rids)
            self.last = greedy(lg).cpu().tolist()
            self.cur = [x + 1 for x in self.cur]
        ranks.barrier()
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(steps):
            lg, _ = m.forward_decode_paged(self.last, self.cur, self.cur, self.alloc, self.rids)
            self.last = greedy(lg).cpu().tolist()
            self.cur = [x + 1 for x in self.cur]
        torch.cuda.synchronize()
        return time.perf_counter() - t0

    def attention_alone(self, reps_per_layer: int = 3) -> dict:
        """The paged decode attention kernel alone: consecutive launches cycle through
        the layers' planes so none reuses L2; mean launch time and algorithmic bytes."""
        from agentserve_b200 import ops
        m, cfg, dev = self.model, self.model.config, self.model.device
        seq_lens = torch.tensor(self.cur, dtype=torch.int32, device=dev)
        rows_t = torch.tensor(self.rows, dtype=torch.int32, device=dev)
        pk = ops.pack_decode(self.alloc.block_tables, seq_lens, rows_t, self.max_blocks)
        q = torch.randn(self.B, m.H, cfg.head_dim, device=dev, dtype=torch.bfloat16)
        ws = ops.new_decode_workspace(self.B, m.H, m.Kh, cfg.head_dim, self.max_blocks,
                                      self.bps, dev)
        out = torch.empty(self.B, m.H * cfg.head_dim, device=dev, dtype=torch.bfloat16)
        L = cfg.n_layers
        for li in range(L):
            ops.paged_decode_attention(q, self.alloc.k_plane(li), self.alloc.v_plane(li),
                                       pk.block_tables, pk.seq_lens_k, m.scale, self.bps, ws,
                                       out=out)
        torch.cuda.synchronize()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record()
        for i in range(reps_per_layer * L):
            li = i % L
            ops.paged_decode_attention(q, self.alloc.k_plane(li), self.alloc.v_plane(li),
                                       pk.block_tables, pk.seq_lens_k, m.scale, self.bps, ws,
                                       out=out)
        a1.record()
        torch.cuda.synchronize()
        ms = a0.elapsed_time(a1) / (reps_per_layer * L)
        lk = [x + 1 for x in self.cur]
        nbytes = decode_attention_bytes(lk, m.H, m.Kh, cfg.head_dim, 2)
        return {"launch_ms": ms, "algorithmic_bytes_per_launch": nbytes,
                "achieved_gb_s": nbytes / (ms / 1e3) / 1e9}

    def free(self):
        if self.graph is not None:
            self.graph.release()
        self.graph = None
        self.alloc = None


def _gpu_local_cores(index: int) -> set:
    """Host cores NVML reports as close to CUDA device `index` (a read-only query)."""
    import pynvml
    pr = torch.cuda.get_device_properties(index)
    h = pynvml.nvmlDeviceGetHandleByPciBusId(
        f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0")
    words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
    return {64 * w + b for w, word in enumerate(words) for b in range(64) if word >> b & 1}


def pin_rank_cores(local_rank: int, local_world: int) -> None:
    """One process per GPU: give this rank its own slice of the host cores close to its
    GPU (the GPUs sharing a set of close cores split it evenly), so the ranks' host
    threads neither share cores nor cross sockets.  Skipped when that information is not
    available or a slice would have fewer than 2 cores."""
    if local_world <= 1:
        return
    try:
        import pynvml
        pynvml.nvmlInit()
        allowed = os.sched_getaffinity(0)
        sets = [frozenset(_gpu_local_cores(i) & allowed) for i in range(local_world)]
        mine = sets[local_rank] or frozenset(allowed)
        peers = [r for r in range(local_world) if (sets[r] or frozenset(allowed)) == mine]
        cores = sorted(mine)
        chunk = len(cores) // len(peers)
        if chunk < 2:
            return
        k = peers.index(local_rank)
        part = cores[k * chunk:(k + 1) * chunk]
        os.sched_setaffinity(0, part)
        torch.set_num_threads(len(part))
    except Exception as e:  # noqa: BLE001 - pinning is an optimisation only
        print(f"rank {local_rank}: host-core pinning skipped ({e!r})", file=sys.stderr)


def affinity() -> dict:
    try:
        cores = sorted(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return {}
    return {"cores": len(cores), "first": cores[0], "last": cores[-1]}


def allreduce_ms(ranks: Ranks, B: int, hidden: int, dev, reps: int = 50) -> float:
    """One NCCL all-reduce of the [B, hidden] bf16 o_proj output, timed alone."""
    t = torch.randn(B, hidden, device=dev, dtype=torch.bfloat16)
    for _ in range(5):
        torch.distributed.all_reduce(t)
    torch.cuda.synchronize()
    ranks.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        torch.distributed.all_reduce(t)
    e1.record()
    torch.cuda.synchronize()
    return ranks.max(e0.elapsed_time(e1) / reps)


def config5(args, dev, ranks: Ranks, rank: int, world: int) -> dict:
    """The 8B geometry (32 layers, hidden 4096, 32/8 heads, head_dim 128, FFN 14336),
    contexts U{1024..32768}: (a) request-partitioned replicas, 32 sequences per GPU
    (8 GPUs x 32 = the 256-sequence configuration); (b) for N > 1, KV-head tensor
    parallelism over the N GPUs with one NCCL all-reduce of the [B, 4096] o_proj output
    per layer, on min(256, 32 N) sequences (each GPU holds Kh/N KV heads of every
    sequence: the same per-GPU KV as a replica)."""
    cfg = config_8b()
    steps, warm = args.config5_steps, 3
    res = {"workload": ("8B geometry, bf16, random-init N(0,0.02), contexts U{1024..32768}, "
                        "16-token blocks, greedy, CUDA-graph steps")}
    model = build_model(cfg, dev, 1, rank)
    run = DecodeRun(model, context_lengths(32, 1024, 32768, seed=500 + rank), warm + steps + 4,
                    0, seed=500 + rank)
    ms = ranks.max(run.timed_steps(ranks, steps, warm))
    note_status("config5 replica steps")
    att = run.attention_alone(reps_per_layer=1)
    note_status("config5 replica attention")
    res["replicas"] = {"sequences_per_gpu": 32, "n_gpus": world,
                       "value": world * 32 * steps / (ms / 1e3), "unit": "tok/s",
                       "ms_per_step": ms / steps,
                       "attention_gb_s": att["achieved_gb_s"],
                       "attention_frac": att["achieved_gb_s"] / measured_peaks()[0]}
    run.free()
    del run, model
    gc.collect()
    torch.cuda.empty_cache()
    if world > 1:
        B = min(256, 32 * world)
        model = build_model(cfg, dev, world, rank, group=torch.distributed.group.WORLD)
        run = DecodeRun(model, context_lengths(B, 1024, 32768, seed=600), warm + steps + 4, 0,
                        seed=600 + rank, token_seed=600)
        ms = ranks.max(run.timed_steps(ranks, steps, warm))
        note_status("config5 tensor-parallel steps")
        att = run.attention_alone(reps_per_layer=1)
        ar = allreduce_ms(ranks, B, cfg.hidden_dim, dev)
        step_ms = ms / steps
        res["tensor_parallel"] = {
            "sequences": B, "n_gpus": world, "kv_heads_per_gpu": cfg.n_kv_heads // world,
            "value": B * steps / (ms / 1e3), "unit": "tok/s", "ms_per_step": step_ms,
            "attention_gb_s_per_gpu": att["achieved_gb_s"],
            "attention_frac": att["achieved_gb_s"] / measured_peaks()[0],
            "allreduce_ms_alone": ar,
            "allreduce_share_of_step": cfg.n_layers * ar / step_ms,
            "collective": f"NCCL all-reduce (sum, bf16) of [{B}, {cfg.hidden_dim}] after "
                          f"o_proj, {cfg.n_layers} per step, captured in the step's graph"}
        model.release_decode_graphs()
        run.free()
        del run, model
        gc.collect()
        torch.cuda.empty_cache()
    return res


# ------------------------------------------------------------------ main arms
def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    cb = cpu_baseline(args, steps=max(1, min(args.steps, args.cpu_sample_steps)),
                      warmup=min(args.warmup, 1), seqs=args.cpu_sample_seqs)
    tp = world if args.tp else 1
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": line_config(args, world, tp),
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def _optional(name: str, fn):
    """Run one of the line's supplementary measurements; a failure there is reported in
    its place (and on stderr) instead of losing the headline line."""
    try:
        return fn()
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        import traceback
        traceback.print_exc()
        print(f"{name} failed: {e!r}", file=sys.stderr, flush=True)
        return {"error": f"{type(e).__name__}: {e}"}


_STATUS = {"bits": 0}


def note_status(tag: str) -> int:
    """Read and clear this rank's device status word (bit 4: a bounded wait ran out);
    report a non-zero word on stderr with the section it follows; accumulate it."""
    from agentserve_b200 import ops
    bits = ops.device_status(clear=True)
    if bits:
        print(f"rank {os.environ.get('RANK', '0')}: device status bits {bits} after {tag}",
              file=sys.stderr, flush=True)
    _STATUS["bits"] |= bits
    return bits


def launches_per_step(model, cfg, batch: int) -> int:
    """The library's kernel launches in one graphed decode step: pack + first RMSNorm +
    greedy argmax (+ lm_head on the small-batch kernel), and per layer the RoPE/cache +
    attention launch (two without the fusion), 2 x add+RMSNorm, and either QKV, o_proj,
    gate/up+SwiGLU and down on the small-batch kernel or SwiGLU alone (cuBLAS
    projections)."""
    small = model.small_batch_linear and batch <= model.small_batch_max_rows
    per_layer = (1 if model.fused_rope_decode else 2) + 2 + (4 if small else 1)
    return 3 + (1 if small else 0) + per_layer * cfg.n_layers


def run_b200(args):
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    pin_rank_cores(local_rank, int(os.environ.get("LOCAL_WORLD_SIZE", world)))
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                             device_id=dev)
    from agentserve_b200 import ops
    ranks = Ranks(world, dev)
    cfg = model_config(args)
    tp = world if args.tp else 1
    # replicas: every rank decodes its own `batch` sequences; KV-head TP: all ranks
    # decode the same batch * world sequences, each holding 1/world of the KV heads
    B = args.batch * tp
    group = torch.distributed.group.WORLD if tp > 1 else None
    model = build_model(cfg, dev, tp, rank, group)
    lens = context_lengths(B, args.ctx_min, args.ctx_max, seed=rank if tp == 1 else 0)
    horizon = args.warmup + args.steps + args.e2e_steps + 4
    run = DecodeRun(model, lens, horizon, args.blocks_per_split, seed=rank if tp == 1 else 0)

    # ---------------- device-resident decode steps (CUDA graph, self-advancing)
    clocks = ClockSampler(local_rank)
    my_ms = run.timed_steps(ranks, args.steps, args.warmup, clocks=clocks)
    clk = clocks.stop()
    ms = ranks.max(my_ms)
    value = (world // tp) * B * args.steps / (ms / 1e3)
    per_rank = ranks.gather({"rank": rank, "ms_per_step": my_ms / args.steps,
                             "affinity": affinity()})

    # ---------------- end to end through forward_decode_paged with host lists
    e2e_n = max(1, args.e2e_steps - 2)
    e2e_s = ranks.max(run.e2e_steps(ranks, e2e_n))
    e2e_call = (world // tp) * B * e2e_n / e2e_s

    # ---------------- paged decode attention kernel alone (roofline)
    note_status("the timed decode steps and the end-to-end model calls")
    att = run.attention_alone()
    peak, peak_kind = measured_peaks()
    note_status("the attention-alone launches")
    model.release_decode_graphs()
    run.free()
    del run
    gc.collect()
    torch.cuda.empty_cache()

    # ---------------- end to end through B200Engine.step (every rank its own engine)
    e2e_engine = None
    if tp == 1 and args.model == "1b" and not args.no_engine:
        def e2e_engine_run():
            # the first engine of the process runs ~2% slower per step throughout (seen
            # with either projection path): an untimed run on another engine goes first
            engine_decode(args, dev, model, 5, 3, ranks, rank)
            return engine_decode(args, dev, model, max(args.steps, 20), max(args.warmup, 3),
                                 ranks, rank)
        e2e_engine = _optional("e2e engine", e2e_engine_run)
        note_status("the engine end-to-end steps")
    if e2e_engine is not None and "error" not in e2e_engine:
        e2e = {"value": e2e_engine["value"], "unit": "tok/s",
               "api": "B200Engine.step on the same 64 sequences per GPU (scheduler, "
                      "bookkeeping, greedy, one pinned copy of positions and table rows in "
                      "and the tokens out every step; the next step queued on the device "
                      "before the host reads this one's tokens; after an untimed run on "
                      "another engine of the same model)",
               "h2d_bytes_per_step": e2e_engine["h2d_bytes_per_step"] * (world // tp),
               "d2h_bytes_per_step": e2e_engine["d2h_bytes_per_step"] * (world // tp),
               "ms_per_step": e2e_engine["ms_per_step"],
               "queued_decode_steps": e2e_engine["queued_decode_steps"]}
    else:
        e2e = None
    e2e_model_call = {"value": e2e_call, "unit": "tok/s",
                      "api": "B200LlamaModel.forward_decode_paged(host lists) + greedy + .cpu()",
                      # one pinned int32 [3, B] copy in (tokens, lengths, table rows),
                      # the greedy int64 tokens out
                      "h2d_bytes_per_step": 3 * B * 4, "d2h_bytes_per_step": B * 8}
    if e2e is None:
        e2e = e2e_model_call

    # ---------------- the same 64 sequences split over the N GPUs (strong scaling)
    def strong_scaling():
        all_lens = context_lengths(args.batch, args.ctx_min, args.ctx_max, seed=0)
        mine = all_lens[rank::world]
        srun = DecodeRun(model, mine, args.warmup + args.steps + 4, args.blocks_per_split,
                         seed=900 + rank)
        s_ms = srun.timed_steps(ranks, args.steps, args.warmup)
        s_max = ranks.max(s_ms)
        res = {"sequences_total": args.batch, "sequences_per_gpu": len(mine),
               "value": args.batch * args.steps / (s_max / 1e3), "unit": "tok/s",
               "ms_per_step": s_max / args.steps,
               "per_rank_ms_per_step": [x / args.steps for x in ranks.gather(s_ms)],
               "note": "strong scaling: total work fixed at the 64 sequences of one GPU's "
                       "workload, split round-robin over the N GPUs"}
        srun.free()
        model.release_decode_graphs()
        gc.collect()
        torch.cuda.empty_cache()
        return res

    strong = None
    if world > 1 and tp == 1 and not args.no_strong:
        strong = _optional("strong", strong_scaling)
        note_status("the strong-scaling steps")

    # ---------------- 8B geometry: replicas, and KV-head TP over the N GPUs
    c5 = None
    if args.model == "1b" and tp == 1 and not args.no_config5:
        c5 = _optional("config5", lambda: config5(args, dev, ranks, rank, world))
        note_status("config5")

    pf = pf128 = c1 = engines = None
    if rank == 0 and world == 1 and tp == 1:
        if not args.no_prefill:
            pf = _optional("prefill", lambda: {"64": measure_prefill(dev),
                                               "128": measure_prefill(dev, D=128)})
            if "error" not in pf:
                pf, pf128 = pf["64"], pf["128"]
            else:
                pf = None
        if not args.no_config1:
            c1 = _optional("config1", lambda: {
                "cpu": config1_cpu(), "gpu": config1_gpu(dev),
                "case": "one paged decode-attention op: 8 sequences, cached lengths "
                        "U{17..1024} (seed 0), 512-block pool, 32/8 heads, head_dim 64, "
                        "fp32; the GPU also at batch 64 / 256 and in bf16"})
        if not args.no_engine and args.model == "1b":
            engines = {"mixed_requests": _optional("engine", lambda: engine_mixed(args, dev, model)),
                       "prefix_cache_sessions": _optional("engine", lambda: engine_prefix(
                           args, dev, model, args.engine_sessions, args.engine_turns))}
        note_status("prefill, config1 and the engine workloads")

    status_per_rank = ranks.gather(_STATUS["bits"])
    status_all = 0
    for b_ in status_per_rank:
        status_all |= b_
    ranks.barrier()
    if rank == 0:
        traffic = load_traffic() if args.model == "1b" else None
        traffic_launch = None
        if traffic:
            traffic_launch = (traffic["dram_bytes_per_launch"] * att["algorithmic_bytes_per_launch"]
                              / traffic["algorithmic_bytes_captured"])
        bf16_peak, bf16_kind = measured_bf16_peak()
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": line_config(args, world, tp),
            "roofline": {"kernel": f"paged_decode_attention (bf16, D={cfg.head_dim}, GQA "
                                   f"{model.H // model.Kh}, {model.Kh} KV heads per GPU)",
                         "bound": "hbm", "achieved": att["achieved_gb_s"], "peak": peak,
                         "unit": "GB/s", "frac": att["achieved_gb_s"] / peak,
                         "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": att["algorithmic_bytes_per_launch"],
                         "launch_ms": att["launch_ms"], "traffic": traffic_launch,
                         "traffic_source": (traffic or {}).get("source")},
            "e2e": e2e,
            "e2e_model_call": e2e_model_call,
            "gpu_launches": args.steps * launches_per_step(model, cfg, B),
            "per_rank": per_rank,
            "strong": strong,
            "config5": c5,
            "prefill": None if pf is None else {
                "kernel": "varlen prefill attention, tcgen05 + TMEM (bf16, D=64, GQA 4)",
                "shape": "prefix 14336 + 600 new tokens per request (prefix-cache workload)",
                "roofline": {"bound": "tensor", "achieved": pf["8x"]["tflops"],
                             "peak": bf16_peak, "unit": "TFLOP/s",
                             "frac": pf["8x"]["tflops"] / bf16_peak,
                             "peak_source": bf16_kind + " bf16_tflops (burst)"},
                "one_request": pf["1x"], "eight_requests": pf["8x"],
                "head_dim_128": {"note": "same shape with the 8B geometry's head_dim 128 "
                                         "(32/8 heads)", "one_request": pf128["1x"],
                                 "eight_requests": pf128["8x"],
                                 "frac": pf128["8x"]["tflops"] / bf16_peak}},
            "config1": c1,
            "engine": engines,
            "clocks": clk, "device_status": status_all,
            "device_status_per_rank": status_per_rank,
        }
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline(args, steps=args.cpu_sample_steps, warmup=1,
                              seqs=args.cpu_sample_seqs)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    model.release_decode_graphs()  # they may hold this group's all-reduce
    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
