"""Decode throughput of the B200 attention step on the continuous-batching decode
workload (Llama-3.2-1B architecture, bf16, 64 sequences per GPU, contexts
U{128..4096}, 16-token paged blocks, greedy decoding).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 is launched by torchrun: one replica per GPU (request-partitioned, weak
scaling, no collective on the data path; a MAX all-reduce of the timings only).

One JSON line on rank 0:
  value        tokens/s of K graph-replayed decode steps, inputs resident in HBM;
  e2e          tokens/s through the reference-facing call
               model.forward_decode_paged(host lists ...) + greedy + device->host read;
  roofline     the paged decode attention kernel, timed alone with CUDA events;
  cpu_baseline the oracle port of the reference's forward_decode_paged on host cores.
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
MODEL_DEFAULTS = {"1b": dict(batch=64, ctx_min=128, ctx_max=4096, layers=16, cpu_sample_seqs=8),
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
    ap.add_argument("--cpu-sample-steps", type=int, default=2)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true")
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


def model_config(args):
    from agentserve_b200.config import ModelConfig
    if args.model == "8b":
        return ModelConfig(hidden_dim=4096, n_heads=32, n_kv_heads=8, n_layers=args.layers,
                           vocab_size=128256, max_seq_len=33024 + 1024, rope_theta=500000.0,
                           intermediate_size=14336)
    return ModelConfig(hidden_dim=2048, n_heads=32, n_kv_heads=8, n_layers=args.layers,
                       vocab_size=128256, max_seq_len=8192, rope_theta=500000.0,
                       intermediate_size=8192)


def workload(args) -> str:
    return WORKLOADS[args.model].format(batch=args.batch, lo=args.ctx_min, hi=args.ctx_max)


def context_lengths(batch, lo, hi, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randint(lo, hi + 1, (batch,), generator=g).tolist()


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
def cpu_baseline(args, steps: int, warmup: int, seqs: int):
    """The oracle port of the reference's forward_decode_paged (llama.py:379-475) on the
    host cores, fp32, all threads: `seqs` of the workload's sequences, `steps` timed
    decode steps after `warmup` untimed ones."""
    sys.path.insert(0, str(REPO))
    from oracle.model import OracleLlama
    from oracle.paged import OracleBlockAllocator
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = model_config(args)
    m = OracleLlama(cfg)
    g = torch.Generator().manual_seed(1234)
    with torch.no_grad():
        for n, p in m.named_parameters():
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
    cpu_model = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu_model = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return {"value": len(lens) * steps / dt, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"oracle port of forward_decode_paged, fp32, {len(lens)} of the "
                       f"{args.batch} sequences (contexts {min(lens)}-{max(lens)}), {steps} timed "
                       f"steps after {warmup} warm-up, full {cfg.n_layers}-layer geometry, "
                       f"CPU {cpu_model}"),
            "seconds": dt}


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


# ------------------------------------------------------------------ main arms
def run_reference(args):
    rank, _, world = dist_env()
    if rank != 0:
        return
    cb = cpu_baseline(args, steps=max(1, min(args.steps, args.cpu_sample_steps)),
                      warmup=min(args.warmup, 1), seqs=args.cpu_sample_seqs)
    line = {"impl": "reference", "metric": METRIC, "value": cb["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": workload(args),
                                            "sample": cb["sample"]},
            "cpu_baseline": {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": cb["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_b200(args):
    rank, local_rank, world = dist_env()
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    from agentserve_b200 import B200LlamaModel, DecodeGraph, DeviceBlockAllocator, greedy, ops

    cfg = model_config(args)
    tp = world if args.tp else 1
    # replicas: every rank decodes its own `batch` sequences; KV-head TP: all ranks
    # decode the same batch * world sequences, each holding 1/world of the KV heads
    B = args.batch * tp
    model = B200LlamaModel(cfg, dtype=torch.bfloat16, device=dev, tp_size=tp,
                           tp_rank=rank if tp > 1 else 0)
    sharded = ("q_proj", "k_proj", "v_proj", "o_proj")
    with torch.no_grad():
        for i, (n, p) in enumerate(model.named_parameters()):
            if p.dim() == 2:
                own = tp > 1 and any(k in n for k in sharded)
                g = torch.Generator(device=dev).manual_seed(
                    1000 + i + (rank if (tp == 1 or own) else 0) * 100003)
                p.normal_(0.0, 0.02, generator=g)
    gen = torch.Generator(device=dev).manual_seed(77 + (rank if tp == 1 else 0))
    model.eval()
    model.fuse_projections_()

    lens = context_lengths(B, args.ctx_min, args.ctx_max, seed=rank if tp == 1 else 0)
    horizon = args.warmup + args.steps + args.e2e_steps + 4
    nblk = [(L + horizon + 15) // 16 for L in lens]
    alloc = DeviceBlockAllocator(sum(nblk), 16, cfg.n_layers, model.Kh, cfg.head_dim,
                                 dtype=torch.bfloat16, device=dev, max_seqs=B,
                                 max_blocks_per_seq=max(nblk))
    alloc.kv_pool.normal_(0.0, 1.0, generator=gen)  # synthesised context KV
    rids = [f"s{i}" for i in range(B)]
    for r, n in zip(rids, nblk):
        alloc.allocate(r, n)
    rows = alloc.rows_for(rids)
    max_blocks = max(nblk)
    bps = args.blocks_per_split  # 0: balanced persistent partition
    model.decode_blocks_per_split = bps
    tokens0 = torch.randint(3, cfg.vocab_size, (B,),
                            generator=torch.Generator().manual_seed(7 + (rank if tp == 1 else 0)))

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-resident decode steps (CUDA graph, self-advancing)
    graph = DecodeGraph(model, alloc, B, max_blocks, bps, advance=True)
    graph.capture(tokens0.tolist(), lens, rows)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    clocks = ClockSampler(local_rank)
    clocks.start()
    barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1))
    value = (world // tp) * B * args.steps / (ms / 1e3)

    # ---------------- end to end through forward_decode_paged with host lists
    cur = [L + args.warmup + args.steps for L in lens]
    last = graph.next_tokens.cpu().tolist()
    graph.release()
    del graph
    torch.cuda.synchronize()
    e2e_steps = max(3, args.e2e_steps)
    for _ in range(2):  # capture forward_decode_paged's graph for this batch
        lg, _ = model.forward_decode_paged(last, cur, cur, alloc, rids)
        last = greedy(lg).cpu().tolist()
        cur = [x + 1 for x in cur]
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps - 2):
        lg, _ = model.forward_decode_paged(last, cur, cur, alloc, rids)
        last = greedy(lg).cpu().tolist()
        cur = [x + 1 for x in cur]
    torch.cuda.synchronize()
    e2e_s = max_over_ranks(time.perf_counter() - t0)
    e2e_value = (world // tp) * B * (e2e_steps - 2) / e2e_s

    # ---------------- paged decode attention kernel alone (roofline)
    seq_lens = torch.tensor(cur, dtype=torch.int32, device=dev)
    rows_t = torch.tensor(rows, dtype=torch.int32, device=dev)
    pk = ops.pack_decode(alloc.block_tables, seq_lens, rows_t, max_blocks)
    q = torch.randn(B, model.H, cfg.head_dim, device=dev, dtype=torch.bfloat16)
    ws = ops.new_decode_workspace(B, model.H, model.Kh, cfg.head_dim, max_blocks, bps, dev)
    out = torch.empty(B, model.H * cfg.head_dim, device=dev, dtype=torch.bfloat16)
    reps = 3 * cfg.n_layers
    for li in range(cfg.n_layers):  # warm
        ops.paged_decode_attention(q, alloc.k_plane(li), alloc.v_plane(li), pk.block_tables,
                                   pk.seq_lens_k, model.scale, bps, ws, out=out)
    torch.cuda.synchronize()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for i in range(reps):  # consecutive launches read different layers' planes (> L2)
        li = i % cfg.n_layers
        ops.paged_decode_attention(q, alloc.k_plane(li), alloc.v_plane(li), pk.block_tables,
                                   pk.seq_lens_k, model.scale, bps, ws, out=out)
    a1.record()
    torch.cuda.synchronize()
    attn_ms = a0.elapsed_time(a1) / reps
    lk = [x + 1 for x in cur]
    abytes = decode_attention_bytes(lk, model.H, model.Kh, cfg.head_dim, 2)
    achieved = abytes / (attn_ms / 1e3) / 1e9
    peak, peak_kind = measured_peaks()
    pf = measure_prefill(dev) if not args.no_prefill and tp == 1 else None
    pf128 = measure_prefill(dev, D=128) if not args.no_prefill and tp == 1 else None
    bits = ops.device_status(clear=True)

    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        kv_gb = cfg.n_layers * decode_attention_bytes(lk, model.H, model.Kh,
                                                      cfg.head_dim, 2) / 1e9
        w_gb = sum(p.numel() for p in model.parameters()) * 2 / 1e9
        traffic = load_traffic() if args.model == "1b" else None
        traffic_launch = None
        if traffic:
            traffic_launch = (traffic["dram_bytes_per_launch"] * abytes
                              / traffic["algorithmic_bytes_captured"])
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": {"workload": workload(args), "global_batch": B * (world // tp),
                       "seq_len": f"{args.ctx_min}-{args.ctx_max} context + decode",
                       "parallelism": (f"KV-head tensor parallel over {world} GPUs, one NCCL "
                                       f"all-reduce per layer after o_proj, MLP replicated"
                                       if tp > 1 else
                                       f"{world} request-partitioned replicas, no collective"),
                       "cuda_graph": True, "blocks_per_split": bps,
                       "l2": (f"inputs larger than L2 every step (~{kv_gb:.1f} GB KV + "
                              f"~{w_gb:.1f} GB weights)"),
                       "kv": "context KV synthesised N(0,1) into the pool"},
            "roofline": {"kernel": f"paged_decode_attention (bf16, D={cfg.head_dim}, GQA "
                                   f"{model.H // model.Kh}, {model.Kh} KV heads per GPU)",
                         "bound": "hbm",
                         "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": f"{peak_kind} hbm_gbs",
                         "algorithmic_bytes_per_launch": abytes, "launch_ms": attn_ms,
                         "traffic": traffic_launch,
                         "traffic_source": (traffic or {}).get("source")},
            "e2e": {"value": e2e_value, "unit": "tok/s", "api": "B200LlamaModel.forward_decode_paged"
                    "(host lists) + greedy + .cpu()",
                    # one pinned int32 [3, B] copy in (tokens, lengths, table rows),
                    # the greedy int64 tokens out
                    "h2d_bytes_per_step": 3 * B * 4, "d2h_bytes_per_step": B * 8},
            # per step: pack + first RMSNorm + greedy argmax + per layer (RoPE/cache,
            # attention, 2 x add+RMSNorm, SwiGLU); the projections and lm_head are cuBLAS
            "gpu_launches": args.steps * (3 + 5 * cfg.n_layers),
            "prefill": None if pf is None else {
                "kernel": "varlen prefill attention, tcgen05 + TMEM (bf16, D=64, GQA 4)",
                "shape": "prefix 14336 + 600 new tokens per request (prefix-cache workload)",
                "roofline": {"bound": "tensor", "achieved": pf["8x"]["tflops"],
                             "peak": measured_bf16_peak()[0], "unit": "TFLOP/s",
                             "frac": pf["8x"]["tflops"] / measured_bf16_peak()[0],
                             "peak_source": measured_bf16_peak()[1] + " bf16_tflops (burst)"},
                "one_request": pf["1x"], "eight_requests": pf["8x"],
                "head_dim_128": {"note": "same shape with the 8B geometry's head_dim 128 "
                                         "(32/8 heads)", "one_request": pf128["1x"],
                                 "eight_requests": pf128["8x"],
                                 "frac": pf128["8x"]["tflops"] / measured_bf16_peak()[0]}},
            "clocks": clk, "device_status": bits,
        }
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline(args, steps=args.cpu_sample_steps, warmup=1,
                              seqs=args.cpu_sample_seqs)
            line["cpu_baseline"] = {k: cb[k] for k in ("value", "unit", "cores", "kind", "sample")}
        print(json.dumps(line), flush=True)
    model.release_decode_graphs()  # they captured this group's all-reduce
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
