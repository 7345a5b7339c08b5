"""Seeded input recipes shared by the golden generator and the tests.

Each function rebuilds the same inputs from fixed seeds, so fixtures only need to
store outputs (plus a sha256 of large inputs to detect generator drift).
"""

from __future__ import annotations

import torch

DECODE_STEPS = 3

# Model geometries for the end-to-end goldens (fields of ModelConfig,
# agentserve/model/config.py:10-30).  "tiny" is the reference's TinyConfig
# (config.py:34-44); "l1b2" keeps the Llama-3.2-1B attention geometry (32 query
# heads, 8 KV heads, head_dim 64, theta 5e5) with 2 layers, a small FFN and vocab.
MODEL_CONFIGS = {
    "tiny": dict(hidden_dim=64, n_heads=4, n_kv_heads=2, n_layers=2, vocab_size=256,
                 max_seq_len=512, intermediate_size=128, rms_norm_eps=1e-5,
                 rope_theta=10000.0),
    "l1b2": dict(hidden_dim=2048, n_heads=32, n_kv_heads=8, n_layers=2, vocab_size=512,
                 max_seq_len=2048, intermediate_size=1024, rms_norm_eps=1e-5,
                 rope_theta=500000.0),
}


def rope_inputs():
    g = torch.Generator().manual_seed(11)
    pos = torch.tensor([0, 1, 17, 1000, 2047])
    x32 = torch.randn(5, 4, 64, generator=g)
    return pos, x32, x32.to(torch.bfloat16)


def cache_inputs():
    g = torch.Generator().manual_seed(12)
    kC = torch.randn(2, 37, 2, 16, generator=g)
    vC = torch.randn(2, 37, 2, 16, generator=g)
    kd = torch.randn(2, 2, 16, generator=g)
    vd = torch.randn(2, 2, 16, generator=g)
    return kC, vC, kd, vd


def decode_cfg1_inputs(batch: int = 8, num_blocks: int = 512, seed: int = 0):
    """Config 1: B=8 sequences, cached lengths U{17..1024}, 16-token blocks taken from a
    random permutation of a 512-block pool, H=32 / Kh=8 / D=64, q/k/v ~ N(0,1) fp32."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(17, 1025, (batch,), generator=g)
    perm = torch.randperm(num_blocks, generator=g)
    tables, off = [], 0
    for L in lens.tolist():
        n = (L + 1 + 15) // 16  # history + the new token
        tables.append(perm[off:off + n].tolist())
        off += n
    q = torch.randn(batch, 32, 64, generator=g)
    kpool = torch.randn(num_blocks, 16, 8, 64, generator=g)
    vpool = torch.randn(num_blocks, 16, 8, 64, generator=g)
    kn = torch.randn(batch, 8, 64, generator=g)
    vn = torch.randn(batch, 8, 64, generator=g)
    return dict(lens=lens.tolist(), tables=tables, q=q, kpool=kpool, vpool=vpool, kn=kn, vn=vn)


def model_scenario(tag: str, cfg):
    g = torch.Generator().manual_seed(100 + len(tag))
    V = cfg.vocab_size
    prompt = torch.randint(3, V, (37,), generator=g).tolist()
    batch_prompts = [torch.randint(3, V, (n,), generator=g).tolist() for n in (4, 6, 5, 19)]
    return dict(prompt=prompt, batch_prompts=batch_prompts)


def greedy_logits():
    """Seeded logits for greedy sampling (sampling.py:46-58): NaN, +-inf, a tie, an
    all -inf row and values past the 1e4 the reference maps +inf to.  Returns the fp32
    logits and their bf16 rounding."""
    g = torch.Generator().manual_seed(21)
    x = torch.randn(6, 3000, generator=g) * 4
    x[0, 11] = float("nan")
    x[0, 1200] = float("inf")
    x[1, :] = -float("inf")
    x[2, 5] = x[2, 2999] = x[2].max() + 2.0
    x[3, 7] = 2.0e4            # finite and above +inf's replacement (1e4)
    x[3, 8] = float("inf")
    x[4, :] = float("nan")     # all NaN -> all 0 -> index 0
    return x, x.to(torch.bfloat16)
