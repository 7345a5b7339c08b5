"""KV-head tensor parallelism on two GPUs over NCCL (runs only where two GPUs are
visible): B200LlamaModel(tp_size=2) built from shard_state_dict() must give the logits
of the unsharded model on the same inputs, for a batched paged prefill and three
graphed decode steps, with the reference decode's dim-major flatten and with the
head-major one.  Each rank holds half the KV heads (and their query heads) of every
sequence; o_proj's partial outputs are summed by one all-reduce per layer.

fp32 is compared at 1e-4 (the all-reduce only reorders fp32 sums), bf16 at 2e-2
absolute on logits of magnitude ~1 (bf16 rounding of the partial sums)."""

import os
import socket
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

CFG = dict(hidden_dim=1024, n_heads=8, n_kv_heads=4, n_layers=2, vocab_size=1000,
           max_seq_len=4096, intermediate_size=1024, rope_theta=500000.0)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out_dir: str, dtype_name: str, compat: bool):
    import datetime

    import torch.distributed as dist

    from agentserve_b200 import B200LlamaModel, DeviceBlockAllocator, greedy
    from agentserve_b200.config import ModelConfig
    from agentserve_b200.model import shard_state_dict
    from oracle.weights import init_weights_

    torch.backends.cuda.matmul.allow_tf32 = False
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    dtype = getattr(torch, dtype_name)
    cfg = ModelConfig(**CFG)
    full = B200LlamaModel(cfg, dtype=dtype, device=dev, reference_compat=compat)
    init_weights_(full, seed=3)
    full.eval()
    part = B200LlamaModel(cfg, dtype=dtype, device=dev, reference_compat=compat, tp_size=world,
                          tp_rank=rank, tp_group=dist.group.WORLD)
    part.load_state_dict(shard_state_dict(full.state_dict(), cfg, world, rank, compat))
    part.eval()

    g = torch.Generator().manual_seed(11)
    prompts = [torch.randint(3, cfg.vocab_size, (n,), generator=g).tolist()
               for n in (37, 300, 129, 16)]
    diffs = []

    def pool(model):
        a = DeviceBlockAllocator(256, 16, cfg.n_layers, model.Kh, cfg.head_dim, dtype=dtype,
                                 device=dev, max_seqs=8)
        for i, p in enumerate(prompts):
            a.allocate(f"r{i}", a.blocks_needed(len(p) + 8))
        return a

    af, ap = pool(full), pool(part)
    rids = [f"r{i}" for i in range(len(prompts))]
    lf = full.forward_prefill_paged(prompts, [0] * 4, af, rids)
    lp = part.forward_prefill_paged(prompts, [0] * 4, ap, rids)
    diffs.append((lf.float() - lp.float()).abs().max().item())
    last = greedy(lf).tolist()
    lens = [len(p) for p in prompts]
    for _ in range(3):
        lf, _ = full.forward_decode_paged(last, lens, lens, af, rids)
        lp, _ = part.forward_decode_paged(last, lens, lens, ap, rids)
        diffs.append((lf.float() - lp.float()).abs().max().item())
        last = greedy(lf).tolist()
        lens = [x + 1 for x in lens]
    torch.cuda.synchronize()
    part.release_decode_graphs()
    full.release_decode_graphs()
    with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
        f.write(" ".join(f"{d:.6g}" for d in diffs))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("dtype_name,compat,tol", [("float32", True, 1e-4),
                                                   ("float32", False, 1e-4),
                                                   ("bfloat16", True, 2e-2)])
def test_kv_head_tensor_parallel_matches_unsharded(dtype_name, compat, tol):
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_worker, args=(2, _free_port(), d, dtype_name, compat), nprocs=2, join=True)
        for r in range(2):
            diffs = [float(x) for x in open(os.path.join(d, f"rank{r}.txt")).read().split()]
            assert len(diffs) == 4
            assert max(diffs) <= tol, diffs
