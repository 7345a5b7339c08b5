"""Parity of every kernel with the oracle, through the C-ABI (ctypes) on a B200.

Bars (from the task's parity contract):
  packing / slot mapping / pool bytes / block copies: bit-exact;
  RoPE (q in place, k into the pool): bit-exact with the reference's fp32 rotate-half;
  attention: fp32 kernel vs fp32 oracle within 1e-5 abs; bf16/fp16 kernel vs fp32
  oracle (on the same bf16/fp16-rounded inputs) within 2e-2 abs.
"""

import math

import numpy as np
import pytest
import torch

from agentserve_b200 import _native as N
from agentserve_b200 import ops
from oracle import attention as OA
from oracle import paged as OP
from oracle import rope as OR
from tests.golden import scenarios as S

pytestmark = pytest.mark.gpu

DEV = "cuda"
ATOL_FP32 = 1e-5
ATOL_LOWP = 2e-2


def make_tables(lens, num_blocks, g, extra_blocks=0):
    """Block lists (from a random permutation of the pool) holding lens[i] tokens."""
    perm = torch.randperm(num_blocks, generator=g).tolist()
    tables, off = [], 0
    for L in lens:
        n = (L + 15) // 16 + extra_blocks
        tables.append(perm[off:off + n])
        off += n
    assert off <= num_blocks
    return tables


def padded(tables, width=None):
    w = width or max(len(t) for t in tables)
    out = torch.zeros(len(tables), w, dtype=torch.int32)
    for i, t in enumerate(tables):
        out[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
    return out


def status_ok():
    bits = ops.device_status(clear=True)
    assert bits == 0, f"device status bits {bits}"


# ---------------------------------------------------------------- packing
def test_pack_decode_bit_exact():
    g = torch.Generator().manual_seed(1)
    lens = [0, 1, 15, 16, 17, 31, 32, 33, 1000, 4095]
    tables = make_tables([L + 1 for L in lens], 2048, g)
    rows = torch.randperm(len(lens) + 5, generator=g)[:len(lens)]
    table_dev = torch.zeros(len(lens) + 5, 300, dtype=torch.int32)
    for i, r in enumerate(rows.tolist()):
        table_dev[r, :len(tables[i])] = torch.tensor(tables[i], dtype=torch.int32)
    pk = ops.pack_decode(table_dev.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV),
                         rows.to(torch.int32).to(DEV), max_blocks=260)
    pos, slots, lk, cu = OP.pack_decode(tables, lens)
    assert pk.positions.cpu().numpy().tolist() == pos.tolist()
    assert pk.slot_mapping.cpu().numpy().tolist() == slots.tolist()
    assert pk.seq_lens_k.cpu().numpy().tolist() == lk.tolist()
    assert pk.cu_seqlens_q.cpu().numpy().tolist() == cu.tolist()
    assert torch.equal(pk.block_tables.cpu(), table_dev[rows][:, :260])
    status_ok()


def test_pack_prefill_bit_exact():
    g = torch.Generator().manual_seed(2)
    num_cached = [0, 32, 37, 0, 14336]
    num_new = [5, 1, 64, 0, 600]
    tables = make_tables([c + n for c, n in zip(num_cached, num_new)], 4096, g)
    bt = padded(tables, 1000)
    total = sum(num_new)
    pk = ops.pack_prefill(bt.to(DEV), torch.tensor(num_cached, dtype=torch.int32, device=DEV),
                          torch.tensor(num_new, dtype=torch.int32, device=DEV), total)
    cu, pos, slots, lk = OP.pack_prefill(tables, num_cached, num_new)
    assert pk.cu_seqlens_q.cpu().tolist() == cu.tolist()
    assert pk.positions.cpu().tolist() == pos.tolist()
    assert pk.slot_mapping.cpu().tolist() == slots.tolist()
    assert pk.seq_lens_k.cpu().tolist() == lk.tolist()
    status_ok()


# ---------------------------------------------------------------- RoPE + cache
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,Kh,D", [(32, 8, 64), (32, 8, 128), (4, 2, 16)])
def test_rope_reshape_and_cache_bit_exact(dtype, H, Kh, D):
    g = torch.Generator().manual_seed(3)
    T, NB = 37, 64
    table = OR.precompute_rope_freqs(D, 4096, 500000.0)
    fused = torch.randn(T, (H + 2 * Kh) * D, generator=g).to(dtype)
    positions = torch.randint(0, 4096, (T,), generator=g)
    slots = torch.randperm(NB * 16, generator=g)[:T]
    slots[5] = -1  # padding token: no cache write
    q, k, v = (fused[:, :H * D].view(T, H, D), fused[:, H * D:(H + Kh) * D].view(T, Kh, D),
               fused[:, (H + Kh) * D:].view(T, Kh, D))
    q_ref = OR.apply_rope(q.clone(), table[positions])
    k_ref = OR.apply_rope(k.clone(), table[positions])
    kc_ref = torch.zeros(NB * 16, Kh, D, dtype=dtype)
    vc_ref = torch.zeros(NB * 16, Kh, D, dtype=dtype)
    keep = slots >= 0
    kc_ref[slots[keep]] = k_ref[keep]
    vc_ref[slots[keep]] = v[keep]

    fd = fused.to(DEV)
    qd = fd[:, :H * D].view(T, H, D)
    kd = fd[:, H * D:(H + Kh) * D].view(T, Kh, D)
    vd = fd[:, (H + Kh) * D:].view(T, Kh, D)
    kc = torch.zeros(NB, 16, Kh, D, dtype=dtype, device=DEV)
    vc = torch.zeros_like(kc)
    k_out = torch.empty(T, Kh, D, dtype=dtype, device=DEV)
    ops.rope_reshape_and_cache(qd, kd, vd, positions.to(DEV), slots.to(DEV), table.to(DEV), kc,
                               vc, k_out=k_out)
    torch.cuda.synchronize()
    assert torch.equal(qd.cpu(), q_ref), "q rotation not bit-exact"
    assert torch.equal(k_out.cpu(), k_ref)
    assert torch.equal(kc.view(-1, Kh, D).cpu(), kc_ref)
    assert torch.equal(vc.view(-1, Kh, D).cpu(), vc_ref)
    status_ok()


def test_reshape_and_cache_without_rotation():
    g = torch.Generator().manual_seed(4)
    T, Kh, D, NB = 21, 8, 64, 16
    k = torch.randn(T, Kh, D, generator=g).to(torch.bfloat16)
    v = torch.randn(T, Kh, D, generator=g).to(torch.bfloat16)
    tables = make_tables([T], NB, g)
    kc = torch.zeros(NB, 16, Kh, D, dtype=torch.bfloat16)
    vc = torch.zeros_like(kc)
    OP.write_kv(kc, vc, tables[0], 0, k, v)
    _, _, slots, _ = OP.pack_prefill(tables, [0], [T])
    kd = torch.zeros(NB, 16, Kh, D, dtype=torch.bfloat16, device=DEV)
    vd = torch.zeros_like(kd)
    ops.rope_reshape_and_cache(None, k.to(DEV), v.to(DEV), None,
                               torch.from_numpy(slots).to(DEV), None, kd, vd)
    assert torch.equal(kd.cpu(), kc) and torch.equal(vd.cpu(), vc)
    status_ok()


# ---------------------------------------------------------------- decode attention
def decode_case(lens, H, Kh, D, dtype, seed, NB=None):
    g = torch.Generator().manual_seed(seed)
    NB = NB or sum((L + 15) // 16 for L in lens) + 8
    tables = make_tables(lens, NB, g)
    kp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype)
    vp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype)
    q = torch.randn(len(lens), H, D, generator=g).to(dtype)
    return tables, kp, vp, q


def run_decode(tables, kp, vp, q, lens, bps, layout=N.AS_LAYOUT_HEAD_MAJOR, ws=None):
    B, H, D = q.shape
    Kh = kp.shape[2]
    bt = padded(tables).to(DEV)
    if ws is None:
        ws = ops.new_decode_workspace(B, H, Kh, D, bt.shape[1], bps, DEV)
    out = ops.paged_decode_attention(q.to(DEV), kp.to(DEV), vp.to(DEV), bt,
                                     torch.tensor(lens, dtype=torch.int32, device=DEV),
                                     1.0 / math.sqrt(D), bps, ws, out_layout=layout)
    torch.cuda.synchronize()
    return out.cpu()


def oracle_decode(tables, kp, vp, q, lens):
    return OA.decode_attention_from_pool(q.float(), kp.float(), vp.float(), tables, lens)


def test_decode_config1_fp32_matches_reference_golden(golden):
    inp = S.decode_cfg1_inputs()
    kp, vp = inp["kpool"].clone(), inp["vpool"].clone()
    for b, L in enumerate(inp["lens"]):
        OP.write_kv(kp, vp, inp["tables"][b], L, inp["kn"][b:b + 1], inp["vn"][b:b + 1])
    lens = [L + 1 for L in inp["lens"]]
    for bps in (8, 64):
        out = run_decode(inp["tables"], kp, vp, inp["q"], lens, bps)
        ref = torch.from_numpy(golden["cfg1_out"]).reshape(8, -1)
        torch.testing.assert_close(out, ref, rtol=0, atol=ATOL_FP32)
    status_ok()


LENS = [1, 15, 16, 17, 100, 257, 1000, 2113, 4096, 33]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bps", [0, 4, 16, 256])
def test_decode_lowp_fast_path(dtype, D, bps):
    H, Kh = 32, 8
    tables, kp, vp, q = decode_case(LENS, H, Kh, D, dtype, seed=D + bps)
    out = run_decode(tables, kp, vp, q, LENS, bps)
    ref = oracle_decode(tables, kp, vp, q, LENS).reshape(len(LENS), -1)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


@pytest.mark.parametrize("H,Kh,D,dtype", [(32, 32, 64, torch.bfloat16), (32, 16, 64, torch.bfloat16),
                                          (8, 1, 128, torch.bfloat16), (4, 2, 16, torch.bfloat16),
                                          (4, 2, 16, torch.float32), (32, 8, 64, torch.float32),
                                          (32, 8, 128, torch.float32), (24, 8, 128, torch.float16),
                                          (64, 4, 64, torch.bfloat16), (15, 3, 64, torch.bfloat16),
                                          (16, 4, 128, torch.float16), (16, 2, 64, torch.bfloat16)])
def test_decode_geometries(H, Kh, D, dtype):
    lens = [1, 16, 17, 300, 1025]
    tables, kp, vp, q = decode_case(lens, H, Kh, D, dtype, seed=H * Kh + D)
    ref = oracle_decode(tables, kp, vp, q, lens).reshape(len(lens), -1)
    atol = ATOL_FP32 if dtype == torch.float32 else ATOL_LOWP
    for bps in (0, 4, 128):
        out = run_decode(tables, kp, vp, q, lens, bps)
        torch.testing.assert_close(out.float(), ref, rtol=0, atol=atol)
    status_ok()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_decode_dim_major_layout(dtype):
    lens = [17, 600, 5]
    H, Kh, D = 32, 8, 64
    tables, kp, vp, q = decode_case(lens, H, Kh, D, dtype, seed=9)
    ref = OA.flatten_decode_output(oracle_decode(tables, kp, vp, q, lens))
    atol = ATOL_FP32 if dtype == torch.float32 else ATOL_LOWP
    for bps in (0, 8):
        out = run_decode(tables, kp, vp, q, lens, bps, layout=N.AS_LAYOUT_DIM_MAJOR)
        torch.testing.assert_close(out.float(), ref, rtol=0, atol=atol)
    status_ok()


def test_decode_workspace_shared_across_batch_sizes():
    H, Kh, D = 32, 8, 64
    ws = ops.DecodeWorkspace(H, Kh, D, DEV)
    for i, lens in enumerate([[700, 3], [900] * 12, [1200, 50, 2000], [4000] * 20, [64]]):
        tables, kp, vp, q = decode_case(lens, H, Kh, D, torch.bfloat16, seed=40 + i)
        bt_w = max(len(t) for t in tables)
        for bps in (8, 0):
            buf = ws.get(len(lens), bt_w, bps)
            out = run_decode(tables, kp, vp, q, lens, bps, ws=buf)
            ref = oracle_decode(tables, kp, vp, q, lens).reshape(len(lens), -1)
            torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


@pytest.mark.parametrize("D", [64, 128])
def test_decode_balanced_large_batch_with_empty_sequences(D):
    """Balanced partition over 300 sequences of mixed lengths (1 .. 3000 tokens, some
    empty: those get a zero row), run twice on one workspace."""
    g = torch.Generator().manual_seed(D)
    lens = torch.randint(1, 3000, (300,), generator=g).tolist()
    for i in (0, 7, 150, 299):
        lens[i] = 0
    H, Kh = 32, 8
    nz = [L for L in lens]
    tables, kp, vp, q = decode_case([max(L, 1) for L in nz], H, Kh, D, torch.bfloat16, seed=D + 1)
    ws = ops.new_decode_workspace(len(lens), H, Kh, D, max(len(t) for t in tables), 0, DEV)
    for _ in range(2):
        out = run_decode(tables, kp, vp, q, lens, 0, ws=ws)
        nonempty = [i for i, L in enumerate(lens) if L > 0]
        ref = oracle_decode([tables[i] for i in nonempty], kp, vp, q[nonempty],
                            [lens[i] for i in nonempty]).reshape(len(nonempty), -1)
        torch.testing.assert_close(out[nonempty].float(), ref, rtol=0, atol=ATOL_LOWP)
        empty = [i for i, L in enumerate(lens) if L == 0]
        assert torch.count_nonzero(out[empty]) == 0
    status_ok()


def test_decode_bad_block_id_is_flagged_not_faulted():
    lens = [40, 40]
    tables, kp, vp, q = decode_case(lens, 32, 8, 64, torch.bfloat16, seed=5)
    tables[1][1] = 10_000_000  # outside the pool: the kernel clamps and flags it
    run_decode(tables, kp, vp, q, lens, 8)
    bits = ops.device_status(clear=True)
    assert bits & 1
    assert ops.device_status(clear=True) == 0


# ---------------------------------------------------------------- prefill attention
def prefill_case(num_cached, num_new, H, Kh, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    lens = [c + n for c, n in zip(num_cached, num_new)]
    NB = sum((L + 15) // 16 for L in lens) + 4
    tables = make_tables(lens, NB, g)
    kp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype)
    vp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype)
    q = torch.randn(sum(num_new), H, D, generator=g).to(dtype)
    cu = np.concatenate([[0], np.cumsum(num_new)]).astype(np.int32)
    return tables, kp, vp, q, cu, lens


def run_prefill(tables, kp, vp, q, cu, lens):
    D = q.shape[2]
    bt = padded(tables).to(DEV)
    num_new = np.diff(cu)
    out = ops.varlen_prefill_attention(q.to(DEV), kp.to(DEV), vp.to(DEV), bt,
                                       torch.from_numpy(cu).to(DEV),
                                       torch.tensor(lens, dtype=torch.int32, device=DEV),
                                       int(num_new.max()), 1.0 / math.sqrt(D))
    torch.cuda.synchronize()
    return out.cpu()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("H,Kh,D", [(32, 8, 64), (32, 8, 128), (4, 2, 16)])
def test_prefill_vs_oracle(dtype, H, Kh, D):
    num_cached = [0, 32, 37, 0, 160]
    num_new = [1, 17, 64, 130, 200]
    tables, kp, vp, q, cu, lens = prefill_case(num_cached, num_new, H, Kh, D, dtype, seed=D)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    atol = ATOL_FP32 if dtype == torch.float32 else ATOL_LOWP
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=atol)
    status_ok()


def test_prefill_long_prefix_bf16():
    """Config-4 shape: a 14,336-token cached prefix plus a 600-token suffix."""
    tables, kp, vp, q, cu, lens = prefill_case([14336], [600], 32, 8, 64, torch.bfloat16, 77)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_consecutive_block_runs(D):
    """Tables whose 8-block KV tiles are runs of consecutive pool ids (loaded as one
    16-block box) mixed with broken runs and a run ending at the last pool block."""
    H, Kh = 32, 8
    num_cached = [300, 1000, 200, 0]
    num_new = [100, 64, 57, 90]
    lens = [c + n for c, n in zip(num_cached, num_new)]
    nb = [(L + 15) // 16 for L in lens]
    NB = sum(nb) + 3
    g = torch.Generator().manual_seed(40 + D)
    tables, off = [], 3  # runs start at an id that is not a multiple of 8
    for n in nb:
        tables.append(list(range(off, off + n)))
        off += n
    tables[1][20], tables[1][21] = tables[1][21], tables[1][20]  # one broken run
    tables[3] = list(range(NB - nb[3], NB))  # last run ends at the pool's last block
    tables[2] = [0, 1, 2] + tables[2][3:]    # blocks 0-2 replace its first ids
    kp = torch.randn(NB, 16, Kh, D, generator=g).to(torch.bfloat16)
    vp = torch.randn(NB, 16, Kh, D, generator=g).to(torch.bfloat16)
    q = torch.randn(sum(num_new), H, D, generator=g).to(torch.bfloat16)
    cu = np.concatenate([[0], np.cumsum(num_new)]).astype(np.int32)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


@pytest.mark.parametrize("num_splits,D", [(2, 64), (3, 64), (5, 64), (8, 64), (16, 64),
                                          (2, 128), (5, 128)])
def test_prefill_split_kv_vs_oracle(num_splits, D):
    """Split-KV prefill (head_dim 64): each query-tile pair's key range divided over
    CTAs and merged; sequences shorter than the split count (empty splits), prefixes
    that end mid-tile and causal tails inside the last splits."""
    num_cached = [3000, 0, 37, 700, 16, 1]
    num_new = [90, 5, 64, 200, 1, 129]
    tables, kp, vp, q, cu, lens = prefill_case(num_cached, num_new, 32, 8, D, torch.bfloat16,
                                               seed=90 + num_splits)
    bt = padded(tables).to(DEV)
    need = ops.prefill_workspace_bytes(len(lens), max(num_new), 32, 8, D, bt.shape[1],
                                       num_splits)
    assert need > 0
    ws = torch.empty(need, dtype=torch.uint8, device=DEV)
    out = ops.varlen_prefill_attention(q.to(DEV), kp.to(DEV), vp.to(DEV), bt,
                                       torch.from_numpy(cu).to(DEV),
                                       torch.tensor(lens, dtype=torch.int32, device=DEV),
                                       max(num_new), D ** -0.5, num_splits=num_splits,
                                       workspace=ws).cpu()
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


def test_prefill_split_kv_auto_one_request_and_workspace_rules():
    """One request with a long cached prefix and a short suffix (8 CTAs unsplit) takes
    an automatic split; forcing a split without enough workspace is an error, while
    the automatic choice falls back to no split."""
    tables, kp, vp, q, cu, lens = prefill_case([30000], [16], 32, 8, 64, torch.bfloat16, 78)
    bt = padded(tables).to(DEV)
    args = (q.to(DEV), kp.to(DEV), vp.to(DEV), bt, torch.from_numpy(cu).to(DEV),
            torch.tensor(lens, dtype=torch.int32, device=DEV), 16, 0.125)
    assert ops.prefill_workspace_bytes(1, 16, 32, 8, 64, bt.shape[1]) > 0  # auto splits here
    auto = ops.varlen_prefill_attention(*args).cpu()
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(auto.float(), ref, rtol=0, atol=ATOL_LOWP)
    small = torch.empty(256, dtype=torch.uint8, device=DEV)
    with pytest.raises(ValueError):
        ops.varlen_prefill_attention(*args, num_splits=4, workspace=small)
    fallback = ops.varlen_prefill_attention(*args, num_splits=0, workspace=small).cpu()
    unsplit = ops.varlen_prefill_attention(*args, num_splits=1).cpu()
    assert torch.equal(fallback, unsplit)
    torch.testing.assert_close(unsplit.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


# ---------------------------------------------------------------- small-batch projections
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,N,K", [(64, 3072, 2048), (1, 2048, 2048), (7, 16384, 2048),
                                   (64, 2048, 8192), (100, 130, 72), (128, 4096, 4096),
                                   (200, 6144, 4096), (256, 512, 1024), (33, 1002, 4096),
                                   (120, 1002, 4096), (128, 1002, 4096)])
def test_linear_small_m_vs_fp32(dtype, M, N, K):
    """as_linear_small_m against an fp32 matmul of the same (rounded) inputs: N not a
    multiple of the 128-row tile (1002: the last split member's rows end mid-vector, and
    odd output rows take the element-wise store), K not a multiple of the 64-wide stage,
    M from 1 to 256, clusters of 1 to 8 K splits, the split partials exchanged by push
    (up to 120 rows here) and by pull (128 rows and more); repeat calls bit-identical
    (splits are summed in member order)."""
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = (torch.randn(M, K, generator=g) * 0.5).to(dtype).to(DEV)
    w = (torch.randn(N, K, generator=g) * 0.05).to(dtype).to(DEV)
    y = ops.linear_small_m(x, w)
    ref = x.float() @ w.float().t()
    tol = 2e-2 * max(1.0, float(ref.abs().max()))
    torch.testing.assert_close(y.float(), ref, rtol=1e-2, atol=tol)
    y2 = ops.linear_small_m(x, w)
    assert torch.equal(y2, y)
    status_ok()


def test_linear_small_m_strided_x_and_out():
    """x as a column slice of a wider buffer and y written into a slice of another."""
    g = torch.Generator().manual_seed(3)
    buf = torch.randn(48, 3072, generator=g).to(torch.bfloat16).to(DEV)
    x = buf[:, 1024:3072]
    w = (torch.randn(2560, 2048, generator=g) * 0.05).to(torch.bfloat16).to(DEV)
    out = torch.zeros(48, 4096, dtype=torch.bfloat16, device=DEV)
    ops.linear_small_m(x, w, out=out[:, 512:3072])
    ref = x.float() @ w.float().t()
    torch.testing.assert_close(out[:, 512:3072].float(), ref, rtol=1e-2, atol=2e-2)
    assert int(out[:, :512].count_nonzero()) == 0 and int(out[:, 3072:].count_nonzero()) == 0
    status_ok()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M,inter,K", [(64, 8192, 2048), (1, 8192, 2048), (7, 192, 2048),
                                       (130, 1024, 200), (256, 512, 1024), (33, 14336, 4096),
                                       (120, 1024, 2048), (128, 1024, 2048)])
def test_linear_small_m_swiglu_vs_fp32(dtype, M, inter, K):
    """Gate/up projection with SwiGLU in the epilogue against silu(g) * u of an fp32
    matmul rounded to the dtype as the two projections' outputs are (llama.py:207-211);
    inter a multiple of 64 (a tile = 64 gate rows + the matching 64 up rows of the
    fused [gate; up] weight), K not a multiple of the 64-wide stage, M from 1 to 256."""
    g = torch.Generator().manual_seed(M * 5 + inter + K)
    x = (torch.randn(M, K, generator=g) * 0.5).to(dtype).to(DEV)
    gu = (torch.randn(2 * inter, K, generator=g) * 0.05).to(dtype).to(DEV)
    y = ops.linear_small_m_swiglu(x, gu)
    assert y.shape == (M, inter)
    proj = (x.float() @ gu.float().t()).to(dtype).float()
    gate, up = proj[:, :inter], proj[:, inter:]
    ref = (torch.nn.functional.silu(gate).to(dtype).float() * up)
    tol = 2e-2 * max(1.0, float(ref.abs().max()))
    torch.testing.assert_close(y.float(), ref, rtol=2e-2, atol=tol)
    status_ok()


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("M", [1, 16, 100, 256])
@pytest.mark.parametrize("K,inter", [(128, 4096), (2048, 4096), (2048, 8192), (4096, 1024)])
def test_linear_small_m_swiglu_bit_exact_vs_projection_then_silu_mul(dtype, M, K, inter):
    """The fused launch splits K the same way as as_linear_small_m on the same weight
    (one fp32 accumulation per split, splits summed in member order; K 128 takes no
    split, the others 2 to 8), so it must equal as_linear_small_m followed by
    as_silu_mul bit for bit; the output may be a row-strided view."""
    g = torch.Generator().manual_seed(11 + M + K + inter)
    x = (torch.randn(M, K, generator=g)).to(dtype).to(DEV)
    gu = (torch.randn(2 * inter, K, generator=g) * 0.2).to(dtype).to(DEV)
    two = ops.silu_mul(ops.linear_small_m(x, gu))
    buf = torch.zeros(M, inter + 256, dtype=dtype, device=DEV)
    y = ops.linear_small_m_swiglu(x, gu, out=buf[:, 128:128 + inter])
    assert torch.equal(y, two)
    assert int(buf[:, :128].count_nonzero()) == 0 and int(buf[:, 128 + inter:].count_nonzero()) == 0
    status_ok()


def test_linear_small_m_swiglu_rejects_bad_arguments():
    xb = torch.randn(8, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # 2*inter not a multiple of 128
        ops.linear_small_m_swiglu(xb, torch.randn(192, 128, device=DEV, dtype=torch.bfloat16))
    with pytest.raises(ValueError):  # dtype mismatch
        ops.linear_small_m_swiglu(xb, torch.randn(256, 128, device=DEV, dtype=torch.float16))
    with pytest.raises(ValueError):  # out of the wrong width
        ops.linear_small_m_swiglu(xb, torch.randn(256, 128, device=DEV, dtype=torch.bfloat16),
                                  out=torch.empty(8, 256, device=DEV, dtype=torch.bfloat16))
    lib = N.load()
    w = torch.randn(256, 128, device=DEV, dtype=torch.bfloat16)
    y = torch.empty(8, 128, device=DEV, dtype=torch.bfloat16)
    s = ops._stream(xb.device)
    assert lib.as_linear_small_m_swiglu(y.data_ptr(), 128, xb.data_ptr(), 128, w.data_ptr(), 8,
                                        96, 128, N.AS_DTYPE_BF16, s) == N.AS_ERR_INVALID_ARG
    assert lib.as_linear_small_m_swiglu(y.data_ptr(), 128, xb.data_ptr(), 128, w.data_ptr(), 300,
                                        128, 128, N.AS_DTYPE_BF16, s) == N.AS_ERR_UNSUPPORTED
    assert lib.as_linear_small_m_swiglu(y.data_ptr(), 128, xb.data_ptr(), 128, w.data_ptr(), 0,
                                        128, 128, N.AS_DTYPE_BF16, s) == N.AS_OK
    status_ok()


# ---------------------------------------------------------------- greedy sampling
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("B,V", [(64, 128256), (3, 1000), (5, 4097), (2, 1), (130, 8192)])
def test_greedy_argmax_matches_reference_sampling(dtype, B, V):
    """as_greedy_argmax equals sampling.py's greedy branch (fp32, nan_to_num(0, 1e4,
    -1e4), first argmax) index for index: NaN, +-inf, ties at two positions, -0/+0,
    rows of -inf only, chunk boundaries."""
    from oracle.model import greedy as oracle_greedy
    g = torch.Generator().manual_seed(B * 31 + V)
    x = torch.randn(B, V, generator=g) * 3
    if V > 10:
        x[0, 7] = float("nan")
        x[0, V // 2] = float("inf")                # -> 1e4: the row maximum
        x[1, :] = -float("inf")                     # all -1e4: first index
        x[2, 3] = x[2, V - 2] = x[2].max() + 1.0    # tie: the first one wins
        if B > 3:
            x[3, :] = 0.0
            x[3, 5] = -0.0                          # -0 and +0 tie: first index (0)
        if B > 4:
            x[4, 4096] = 50.0 if V > 4096 else x[4, 4096 % V]  # max in the second chunk
            x[4, 4095] = 50.0 if V > 4096 else x[4, 4095 % V]  # equal max just before it
    xd = x.to(dtype).to(DEV)
    got = ops.greedy_argmax(xd).cpu()
    want = oracle_greedy(xd).cpu()
    assert torch.equal(got, want)
    # twice in a row on the same (self-resetting) workspace, and on a row-strided view
    wide = torch.zeros(B, V + 24, dtype=dtype, device=DEV)
    wide[:, :V] = xd
    assert torch.equal(ops.greedy_argmax(wide[:, :V]).cpu(), want)
    status_ok()


def test_greedy_argmax_matches_reference_golden(golden):
    """The kernel reproduces the tokens the reference's own sampler chose."""
    x32, xbf = S.greedy_logits()
    assert ops.greedy_argmax(x32.to(DEV)).cpu().tolist() == golden["greedy_tokens_f32"].tolist()
    assert ops.greedy_argmax(xbf.to(DEV)).cpu().tolist() == golden["greedy_tokens_bf16"].tolist()
    status_ok()


# ---------------------------------------------------------------- block copy
def test_block_copy_gather_and_seed_bit_exact():
    g = torch.Generator().manual_seed(6)
    L, NB, Kh, D = 3, 40, 8, 64
    pool = torch.randn(2, L, NB, 16, Kh, D, generator=g).to(torch.bfloat16)
    ids = torch.randperm(NB, generator=g)[:7].to(torch.int32)
    bpb = 16 * Kh * D * 2
    pd = pool.to(DEV)
    out = torch.empty(2, L, 7, 16, Kh, D, dtype=torch.bfloat16, device=DEV)
    ops.block_copy(out, pd, ids.to(DEV), None, bpb, 2 * L, NB * bpb, 7 * bpb, NB, 7)
    assert torch.equal(out.cpu(), pool[:, :, ids.long()])
    # seed the same payload into other blocks and gather again (round trip)
    dst_ids = torch.randperm(NB, generator=g)[:7].to(torch.int32)
    src_ids = torch.arange(7, dtype=torch.int32, device=DEV)
    ops.block_copy(pd, out, src_ids, dst_ids.to(DEV), bpb, 2 * L, 7 * bpb, NB * bpb, 7, NB)
    assert torch.equal(pd[:, :, dst_ids.long()].cpu(), pool[:, :, ids.long()])
    # gather_kv semantics for one layer, 100 tokens
    k = OP.gather_kv(pool[0, 1], ids.tolist(), 100)
    buf = torch.empty(2, 7, 16, Kh, D, dtype=torch.bfloat16, device=DEV)
    ops.block_copy(buf, pool.to(DEV)[0, 1], ids.to(DEV), None, bpb, 2, L * NB * bpb, 7 * bpb, NB, 7)
    assert torch.equal(buf[0].reshape(-1, Kh, D)[:100].cpu(), k)
    status_ok()


def test_block_copy_bad_id_flagged():
    pool = torch.zeros(4, 16, 16, dtype=torch.bfloat16, device=DEV)
    out = torch.empty_like(pool)
    ops.block_copy(out, pool, torch.tensor([0, 9], dtype=torch.int32, device=DEV), None, 512, 1,
                   0, 0, 4, 4)
    assert ops.device_status(clear=True) & 1


# ---------------------------------------------------------------- tensor-core prefill edges
@pytest.mark.parametrize("H,Kh", [(32, 8), (8, 8), (16, 8), (64, 8), (32, 2)])
@pytest.mark.parametrize("D", [64, 128])
def test_prefill_tensor_core_geometries(H, Kh, D):
    """bf16 prefill on the tcgen05 kernel: GQA groups 1..16, new-token counts around the
    query-tile size (128/group tokens), prefixes that are not block- or tile-aligned."""
    tq = 128 // (H // Kh)
    num_new = [1, tq - 1, tq, tq + 1, 3 * tq + 5]
    num_cached = [0, 37, 130, 1, 16]
    tables, kp, vp, q, cu, lens = prefill_case(num_cached, num_new, H, Kh, D, torch.bfloat16,
                                               seed=H * 7 + D)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


def test_prefill_tensor_core_strided_q_and_many_sequences():
    """q as a column slice of a fused QKV buffer (row stride > H*D), 9 sequences."""
    g = torch.Generator().manual_seed(31)
    H, Kh, D = 32, 8, 64
    num_cached = [0, 16, 300, 5, 0, 1000, 77, 128, 2]
    num_new = [40, 1, 200, 33, 129, 64, 7, 300, 31]
    tables, kp, vp, _, cu, lens = prefill_case(num_cached, num_new, H, Kh, D, torch.bfloat16, 32)
    T = int(cu[-1])
    fused = torch.randn(T, (H + 2 * Kh) * D, generator=g).to(torch.bfloat16)
    q = fused[:, :H * D].view(T, H, D)
    bt = padded(tables).to(DEV)
    fd = fused.to(DEV)
    out = ops.varlen_prefill_attention(fd[:, :H * D].view(T, H, D), kp.to(DEV), vp.to(DEV), bt,
                                       torch.from_numpy(cu).to(DEV),
                                       torch.tensor(lens, dtype=torch.int32, device=DEV),
                                       max(num_new), 1.0 / math.sqrt(D))
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float().cpu(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()


# ---------------------------------------------------------------- fused norm / SwiGLU
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("dim", [2048, 4096, 64, 3072])
def test_rmsnorm_and_add_rmsnorm_match_reference_formula(dtype, dim):
    from oracle.model import RMSNorm
    g = torch.Generator().manual_seed(dim)
    rows = 37
    x = torch.randn(rows, dim, generator=g).to(dtype)
    d = torch.randn(rows, dim, generator=g).to(dtype)
    norm = RMSNorm(dim, 1e-5)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(dim, generator=g))
    norm = norm.to(dtype)
    ref = norm(x)
    xs = (x + d)  # residual add rounded to dtype, as `x = x + h` in the reference
    ref2 = norm(xs)
    tol = dict(rtol=0, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    xd, dd, wd = x.to(DEV), d.to(DEV), norm.weight.detach().to(DEV)
    out = ops.rmsnorm(xd, wd, 1e-5)
    torch.testing.assert_close(out.cpu().float(), ref.float(), **tol)
    out2 = ops.add_rmsnorm(xd, dd, wd, 1e-5)
    assert torch.equal(xd.cpu(), xs), "residual sum must be bit-exact"
    torch.testing.assert_close(out2.cpu().float(), ref2.float(), **tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_silu_mul_matches_reference_formula(dtype):
    g = torch.Generator().manual_seed(9)
    gu = (3 * torch.randn(19, 2 * 8192, generator=g)).to(dtype)
    ref = torch.nn.functional.silu(gu[:, :8192]) * gu[:, 8192:]
    out = ops.silu_mul(gu.to(DEV))
    tol = dict(rtol=1e-5, atol=1e-5) if dtype == torch.float32 else dict(rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(out.cpu().float(), ref.float(), **tol)


def test_ops_reject_bad_layouts_with_value_error():
    """Layout and dtype mistakes raise ValueError before any launch (also under -O)."""
    x = torch.randn(4, 64, device=DEV)
    w = torch.ones(64, device=DEV)
    with pytest.raises(ValueError):
        ops.rmsnorm(x.t(), w, 1e-5)                        # non-contiguous rows
    with pytest.raises(ValueError):
        ops.rmsnorm(x, w, 1e-5, out=torch.empty(4, 32, device=DEV))
    with pytest.raises(ValueError):
        ops.add_rmsnorm(x, torch.randn(4, 32, device=DEV), w, 1e-5)
    with pytest.raises(ValueError):
        ops.silu_mul(torch.randn(4, 63, device=DEV))       # odd width
    with pytest.raises(ValueError):
        ops.greedy_argmax(torch.randn(64, 4, device=DEV).t())
    xb = torch.randn(8, 128, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ops.linear_small_m(xb, torch.randn(256, 128, device=DEV, dtype=torch.float16))
    with pytest.raises(ValueError):
        ops.linear_small_m(xb, torch.randn(256, 128, device=DEV, dtype=torch.bfloat16),
                           out=torch.empty(8, 128, device=DEV, dtype=torch.bfloat16))
    status_ok()


# ---------------------------------------------------------------- fused RoPE + decode
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bps", [0, 4])
def test_rope_decode_one_launch_equals_two_launches(dtype, D, bps):
    """as_rope_paged_decode_attention (the new token's RoPE + cache write inside the
    attention launch) leaves the same pool bytes and returns the same output, bit for
    bit, as as_rope_reshape_and_cache followed by as_paged_decode_attention; q, k, v
    are strided column slices of one fused projection output, as in the decode step;
    one slot is negative (skipped) and the output is also checked against the oracle."""
    H, Kh = 32, 8
    g = torch.Generator().manual_seed(D + bps)
    hist = [0, 15, 16, 100, 1000, 2111, 4095, 31]
    lens_k = [L + 1 for L in hist]
    NB = sum((L + 15) // 16 for L in lens_k) + 8
    tables = make_tables(lens_k, NB, g)
    kp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype).to(DEV)
    vp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype).to(DEV)
    B = len(hist)
    qkv = torch.randn(B, (H + 2 * Kh) * D, generator=g).to(dtype).to(DEV)
    table = OR.precompute_rope_freqs(D, 8192, 500000.0).to(DEV)
    pos = torch.tensor(hist, dtype=torch.int64, device=DEV)
    slots = [t[L // 16] * 16 + L % 16 for t, L in zip(tables, hist)]
    slots[3] = -1  # written by neither path
    slot_t = torch.tensor(slots, dtype=torch.int64, device=DEV)
    bt = padded(tables).to(DEV)
    lk = torch.tensor(lens_k, dtype=torch.int32, device=DEV)

    def split(x):
        return (x[:, :H * D].view(B, H, D), x[:, H * D:(H + Kh) * D].view(B, Kh, D),
                x[:, (H + Kh) * D:].view(B, Kh, D))

    ws = ops.new_decode_workspace(B, H, Kh, D, bt.shape[1], bps, DEV)
    kp1, vp1, x1 = kp.clone(), vp.clone(), qkv.clone()
    q, k, v = split(x1)
    ops.rope_reshape_and_cache(q, k, v, pos, slot_t, table, kp1, vp1)
    o1 = ops.paged_decode_attention(q, kp1, vp1, bt, lk, D ** -0.5, bps, ws,
                                    out_layout=N.AS_LAYOUT_DIM_MAJOR)
    kp2, vp2, x2 = kp.clone(), vp.clone(), qkv.clone()
    q, k, v = split(x2)
    o2 = ops.rope_paged_decode_attention(q, k, v, pos, slot_t, table, kp2, vp2, bt, lk,
                                         D ** -0.5, bps, ws, out_layout=N.AS_LAYOUT_DIM_MAJOR)
    torch.cuda.synchronize()
    assert torch.equal(kp1, kp2) and torch.equal(vp1, vp2)
    assert torch.equal(o1, o2)
    assert torch.equal(x2, qkv)  # the projections are left as they were
    ref = OA.flatten_decode_output(OA.decode_attention_from_pool(
        x1[:, :H * D].view(B, H, D).float().cpu(), kp1.float().cpu(), vp1.float().cpu(), tables,
        lens_k))
    torch.testing.assert_close(o2.float().cpu(), ref, rtol=0, atol=ATOL_LOWP)
    status_ok()
