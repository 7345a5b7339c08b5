"""KV-head tensor parallelism, host side, on CPU with two gloo ranks: an attention block
(q/k/v projections, RoPE, decode attention over a ragged history, flatten, o_proj)
computed by two ranks from shard_state_dict() shards and summed with all_reduce equals
the unsharded block, for both the reference's dim-major decode flatten and head-major.
The attention math is the oracle's (torch, CPU); the kernels are not involved."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from agentserve_b200.config import ModelConfig
from agentserve_b200.model import shard_state_dict
from oracle.attention import decode_attention_padded, flatten_decode_output
from oracle.rope import apply_rope, precompute_rope_freqs

CFG = ModelConfig(hidden_dim=128, n_heads=8, n_kv_heads=4, n_layers=1, vocab_size=64,
                  max_seq_len=256, intermediate_size=64, rope_theta=10000.0)


def full_weights():
    g = torch.Generator().manual_seed(3)
    H, Kh, D, hid = CFG.n_heads, CFG.n_kv_heads, CFG.head_dim, CFG.hidden_dim
    return {"layers.0.attn.q_proj.weight": torch.randn(H * D, hid, generator=g) * 0.05,
            "layers.0.attn.k_proj.weight": torch.randn(Kh * D, hid, generator=g) * 0.05,
            "layers.0.attn.v_proj.weight": torch.randn(Kh * D, hid, generator=g) * 0.05,
            "layers.0.attn.o_proj.weight": torch.randn(hid, H * D, generator=g) * 0.05,
            "layers.0.ffn_norm.weight": torch.ones(hid)}


def inputs():
    g = torch.Generator().manual_seed(4)
    B, Kh, D = 3, CFG.n_kv_heads, CFG.head_dim
    x = torch.randn(B, CFG.hidden_dim, generator=g)
    lens = [5, 17, 9]
    kh = [torch.randn(L, Kh, D, generator=g) for L in lens]
    vh = [torch.randn(L, Kh, D, generator=g) for L in lens]
    return x, lens, kh, vh


def attn_block(sd, x, lens, kh, vh, H, Kh, dim_major):
    D = CFG.head_dim
    B = x.shape[0]
    cs = precompute_rope_freqs(D, CFG.max_seq_len, CFG.rope_theta)[torch.tensor(lens)]
    q = apply_rope((x @ sd["layers.0.attn.q_proj.weight"].T).view(B, H, D), cs)
    k = apply_rope((x @ sd["layers.0.attn.k_proj.weight"].T).view(B, Kh, D), cs)
    v = (x @ sd["layers.0.attn.v_proj.weight"].T).view(B, Kh, D)
    o = decode_attention_padded(q, kh, vh, k, v)
    flat = flatten_decode_output(o) if dim_major else o.reshape(B, H * D)
    return flat @ sd["layers.0.attn.o_proj.weight"].T


def _rank(rank, world, port, dim_major, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, lens, kh, vh = inputs()
        sd = shard_state_dict(full_weights(), CFG, world, rank, reference_compat=dim_major)
        Khl = CFG.n_kv_heads // world
        khl = [t[:, rank * Khl:(rank + 1) * Khl].contiguous() for t in kh]
        vhl = [t[:, rank * Khl:(rank + 1) * Khl].contiguous() for t in vh]
        part = attn_block(sd, x, lens, khl, vhl, CFG.n_heads // world, Khl, dim_major)
        dist.all_reduce(part)
        if rank == 0:
            q.put(part)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("dim_major", [True, False])
def test_two_rank_kv_head_tp_equals_unsharded(dim_major):
    x, lens, kh, vh = inputs()
    want = attn_block(full_weights(), x, lens, kh, vh, CFG.n_heads, CFG.n_kv_heads, dim_major)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, dim_major, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-5)


def test_shard_shapes_and_replication():
    sd = shard_state_dict(full_weights(), CFG, 4, 3)
    D = CFG.head_dim
    assert sd["layers.0.attn.q_proj.weight"].shape == (2 * D, CFG.hidden_dim)
    assert sd["layers.0.attn.k_proj.weight"].shape == (1 * D, CFG.hidden_dim)
    assert sd["layers.0.attn.o_proj.weight"].shape == (CFG.hidden_dim, 2 * D)
    assert torch.equal(sd["layers.0.ffn_norm.weight"], full_weights()["layers.0.ffn_norm.weight"])
    with pytest.raises(ValueError):
        shard_state_dict(full_weights(), CFG, 3, 0)


@pytest.mark.parametrize("compat", [True, False])
def test_o_proj_shards_cover_both_flattens(compat):
    """With the reference's flattens, prefill feeds o_proj head-major (llama.py:184) and
    decode dim-major (llama.py:362, 470): the ranks' o_proj (decode) and o_proj_prefill
    shards must each sum back to the unsharded product."""
    H, D, hid = CFG.n_heads, CFG.head_dim, CFG.hidden_dim
    g = torch.Generator().manual_seed(9)
    w = torch.randn(hid, H * D, generator=g)
    o = torch.randn(5, H, D, generator=g)
    full = {"layers.0.attn.o_proj.weight": w}
    want_pre = o.reshape(5, H * D) @ w.T
    want_dec = (o.transpose(1, 2).reshape(5, H * D) if compat else o.reshape(5, H * D)) @ w.T
    got_pre = got_dec = 0
    for r in range(2):
        s = shard_state_dict(full, CFG, 2, r, compat)
        ol = o[:, r * H // 2:(r + 1) * H // 2]
        dec_in = ol.transpose(1, 2).reshape(5, -1) if compat else ol.reshape(5, -1)
        got_dec = got_dec + dec_in @ s["layers.0.attn.o_proj.weight"].T
        wp = s.get("layers.0.attn.o_proj_prefill.weight", s["layers.0.attn.o_proj.weight"])
        got_pre = got_pre + ol.reshape(5, -1) @ wp.T
    torch.testing.assert_close(got_pre, want_pre, rtol=0, atol=1e-4)
    torch.testing.assert_close(got_dec, want_dec, rtol=0, atol=1e-4)
    assert ("layers.0.attn.o_proj_prefill.weight" in shard_state_dict(full, CFG, 2, 0, compat)) \
        == compat
