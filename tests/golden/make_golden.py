"""Generate the golden fixtures in tests/golden/ by running the reference itself.

Run in a container where the reference (krishs0404/agentserve) is checked out:

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py [--reference PATH]

PATH (or $AGENTSERVE_REFERENCE) is a checkout of the reference.  Every array
written here comes from the reference's own code (BlockAllocator, apply_rope,
precompute_rope_freqs, LlamaModel.forward / forward_decode_batch /
forward_decode_paged, sample at temperature 0), on seeded inputs that the tests regenerate.  Large inputs
are not stored: the tests rebuild them from the same seeds and check the stored
sha256 of their bytes first.  The tests never import the reference.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from oracle.weights import init_weights_  # noqa: E402
from tests.golden import scenarios as S  # noqa: E402


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()


def import_reference(path: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, path)
    import agentserve.engine.cache as cache  # noqa: F401
    import agentserve.model.config as config  # noqa: F401
    import agentserve.model.llama as llama  # noqa: F401
    return cache, config, llama


def gen_greedy(path: str, out):
    """The reference's sampler at temperature 0 (sampling.py:46-58)."""
    import agentserve.engine.sampling as sampling
    x32, xbf = S.greedy_logits()
    out["greedy_tokens_f32"] = sampling.sample(x32, temperature=0.0).numpy()
    out["greedy_tokens_bf16"] = sampling.sample(xbf, temperature=0.0).numpy()


def gen_rope(llama, out):
    table = llama.precompute_rope_freqs(64, 2048, 500000.0)
    pos, x32, xbf = S.rope_inputs()
    cs = table[pos]
    out["rope_table_sha"] = np.array(sha(table))
    out["rope_rows"] = table[pos].numpy()
    out["rope_pos"] = pos.numpy()
    out["rope_out_f32"] = llama.apply_rope(x32, cs).numpy()
    out["rope_out_bf16"] = llama.apply_rope(xbf, cs).view(torch.int16).numpy()
    tiny = llama.precompute_rope_freqs(16, 512, 10000.0)
    out["rope_tiny_sha"] = np.array(sha(tiny))


def gen_cache(cache, out):
    """BlockAllocator bookkeeping + write_kv_prefill/decode + gather_kv on a small pool."""
    a = cache.BlockAllocator(num_blocks=32, block_size=16, num_layers=2, num_kv_heads=2,
                             head_dim=16, allocate_tensor=True)
    a.allocate("A", 3)
    a.allocate("B", 2)
    a.free("A")
    a.allocate("C", 4)  # churn: C reuses A's blocks after the untouched tail
    a.allocate("B", 1)
    kC, vC, kdec, vdec = S.cache_inputs()
    for layer in range(2):
        a.write_kv_prefill("C", layer, kC[layer], vC[layer])
        a.write_kv_decode("C", 37, layer, kdec[layer], vdec[layer])
    out["cache_bt_B"] = np.array(a.blocks_for("B"), dtype=np.int32)
    out["cache_bt_C"] = np.array(a.blocks_for("C"), dtype=np.int32)
    out["cache_free_after"] = np.array(list(a._free), dtype=np.int32)
    out["cache_pool"] = a.kv_pool.numpy()
    k0, v0 = a.gather_kv("C", 38, 1)
    out["cache_gather_k"] = k0.numpy()
    out["cache_gather_v"] = v0.numpy()
    out["cache_blocks_needed"] = np.array([a.blocks_needed(n) for n in (0, 1, 15, 16, 17, 33)])


def gen_decode_cfg1(cache, out):
    """Config-1 decode attention: reference gather_kv / write_kv_decode, then the SDPA
    sequence of llama.py:441-470 (pad -> cat new token -> GQA expand -> pad mask)."""
    import torch.nn.functional as F
    inp = S.decode_cfg1_inputs()
    lens, tables, q, kpool, vpool, kn, vn = (inp[k] for k in
                                             ("lens", "tables", "q", "kpool", "vpool", "kn", "vn"))
    out["cfg1_input_sha"] = np.array(sha(torch.cat([q.flatten(), kpool.flatten(),
                                                    vpool.flatten(), kn.flatten(),
                                                    vn.flatten()])))
    B, H, D = q.shape
    Kh = kpool.shape[2]
    a = cache.BlockAllocator(num_blocks=512, block_size=16, num_layers=1, num_kv_heads=Kh,
                             head_dim=D, allocate_tensor=True)
    a.kv_pool[0, 0] = kpool
    a.kv_pool[1, 0] = vpool
    for b in range(B):
        a._request_blocks[str(b)] = list(int(x) for x in tables[b])
    max_len = int(max(lens))
    kp = q.new_zeros(B, max_len, Kh, D)
    vp = q.new_zeros(B, max_len, Kh, D)
    for b in range(B):
        kb, vb = a.gather_kv(str(b), int(lens[b]), 0)
        kp[b, :lens[b]] = kb
        vp[b, :lens[b]] = vb
    for b in range(B):
        a.write_kv_decode(str(b), int(lens[b]), 0, kn[b], vn[b])
    kf = torch.cat([kp, kn.unsqueeze(1)], 1)
    vf = torch.cat([vp, vn.unsqueeze(1)], 1)
    tot = max_len + 1
    g = H // Kh
    ke = kf.unsqueeze(3).expand(B, tot, Kh, g, D).reshape(B, tot, H, D).transpose(1, 2)
    ve = vf.unsqueeze(3).expand(B, tot, Kh, g, D).reshape(B, tot, H, D).transpose(1, 2)
    lt = torch.tensor([int(x) for x in lens])
    col = torch.arange(tot)
    is_pad = (col[None, :] >= lt[:, None]) & (col[None, :] < max_len)
    mask = q.new_zeros(B, 1, 1, tot)
    mask.masked_fill_(is_pad[:, None, None, :], float("-inf"))
    o = F.scaled_dot_product_attention(q.unsqueeze(2), ke, ve, attn_mask=mask)
    out["cfg1_out"] = o.squeeze(2).numpy()
    out["cfg1_pool_after_sha"] = np.array(sha(a.kv_pool))


def gen_models(config_mod, llama, cache, out):
    for tag, cfg_kwargs in S.MODEL_CONFIGS.items():
        cfg = config_mod.ModelConfig(**cfg_kwargs)
        torch.manual_seed(0)
        m = llama.LlamaModel(cfg)
        init_weights_(m, seed=0)
        m.eval()
        sc = S.model_scenario(tag, cfg)
        # prefill of the full prompt
        logits, kv = m.forward(sc["prompt"])
        out[f"{tag}_prefill_logits"] = logits.numpy()
        # prefix-hit prefill: first 32 tokens cached (block-aligned, engine.py:274-281)
        pre = [(k[:32].clone(), v[:32].clone()) for k, v in kv]
        logits2, _ = m.forward(sc["prompt"][32:], kv_cache=pre, position_offset=32)
        out[f"{tag}_prefix_logits"] = logits2.numpy()
        # padded-list decode: prefill each request, then greedy steps
        caches, last, pos = [], [], []
        for p in sc["batch_prompts"]:
            lg, kvp = m.forward(p)
            caches.append(kvp)
            last.append(int(lg[-1].argmax()))
            pos.append(len(p))
        steps = []
        toks = []
        for _ in range(S.DECODE_STEPS):
            lg, caches = m.forward_decode_batch(last, caches, pos)
            steps.append(lg.numpy())
            last = [int(t) for t in lg.argmax(-1)]
            toks.append(last)
            pos = [x + 1 for x in pos]
        out[f"{tag}_batch_logits"] = np.stack(steps)
        out[f"{tag}_batch_tokens"] = np.array(toks, dtype=np.int64)
        # paged decode through the reference allocator (fp32 pool)
        a = cache.BlockAllocator(num_blocks=64, block_size=16, num_layers=cfg.n_layers,
                                 num_kv_heads=cfg.n_kv_heads, head_dim=cfg.head_dim,
                                 allocate_tensor=True)
        rids, last, lens = [], [], []
        for i, p in enumerate(sc["batch_prompts"]):
            rid = f"r{i}"
            a.allocate(rid, a.blocks_needed(len(p) + S.DECODE_STEPS + 1))
            lg, kvp = m.forward(p)
            for li, (k, v) in enumerate(kvp):
                a.write_kv_prefill(rid, li, k, v)
            rids.append(rid)
            last.append(int(lg[-1].argmax()))
            lens.append(len(p))
        steps, toks = [], []
        for _ in range(S.DECODE_STEPS):
            lg, _ = m.forward_decode_paged(last, lens, lens, a, rids)
            steps.append(lg.numpy())
            last = [int(t) for t in lg.argmax(-1)]
            toks.append(last)
            lens = [x + 1 for x in lens]
        out[f"{tag}_paged_logits"] = np.stack(steps)
        out[f"{tag}_paged_tokens"] = np.array(toks, dtype=np.int64)
        bts = [a.blocks_for(r) for r in rids]
        w = max(len(b) for b in bts)
        out[f"{tag}_block_tables"] = np.array([b + [-1] * (w - len(b)) for b in bts],
                                              dtype=np.int32)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("AGENTSERVE_REFERENCE"),
                    help="checkout of krishs0404/agentserve (or $AGENTSERVE_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference PATH or set AGENTSERVE_REFERENCE")
    torch.set_num_threads(min(8, os.cpu_count() or 1))
    cache, config_mod, llama = import_reference(args.reference)
    out: dict = {}
    gen_rope(llama, out)
    gen_cache(cache, out)
    gen_decode_cfg1(cache, out)
    gen_models(config_mod, llama, cache, out)
    gen_greedy(args.reference, out)
    path = HERE / "reference_golden.npz"
    np.savez_compressed(path, **out)
    print(f"wrote {path} ({path.stat().st_size / 1e6:.2f} MB, {len(out)} arrays)")


if __name__ == "__main__":
    main()
