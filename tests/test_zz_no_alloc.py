"""as_paged_decode_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory (their GPU memory belongs to another allocator, or
their serving loop must not reach cudaMalloc).  It keeps its split-K scratch in a
static array inside the library instead of a caller workspace.

Checked here through the C ABI (ctypes): two calls in a row, with different batch
sizes so the second reuses the array the first left behind, each against the
regular entry point on the same inputs and against the oracle (the reference's
gather -> pad -> SDPA restated on the CPU in fp32); with a fixed split and with the
split left to the library (blocks_per_split 0), at head_dim 64 and 128; and a call
whose scratch need exceeds the static array is refused before any GPU work.  The
file is named to run last.
"""

import ctypes
import math

import pytest
import torch

from agentserve_b200 import _native as N
from agentserve_b200 import ops
from oracle import attention as OA

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(lens, H, Kh, D, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    NB = sum((L + 15) // 16 for L in lens) + 4
    perm = torch.randperm(NB, generator=g).tolist()
    width = max((L + 15) // 16 for L in lens)
    bt = torch.zeros(len(lens), width, dtype=torch.int32)
    off = 0
    for i, L in enumerate(lens):
        n = (L + 15) // 16
        bt[i, :n] = torch.tensor(perm[off:off + n], dtype=torch.int32)
        off += n
    kp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype).to(DEV)
    vp = torch.randn(NB, 16, Kh, D, generator=g).to(dtype).to(DEV)
    q = torch.randn(len(lens), H, D, generator=g).to(dtype).to(DEV)
    return q, kp, vp, bt.to(DEV), torch.tensor(lens, dtype=torch.int32, device=DEV)


def _oracle(q, kp, vp, bt, lens, layout):
    tables = [bt[i, :(L + 15) // 16].tolist() for i, L in enumerate(lens)]
    o = OA.decode_attention_from_pool(q.cpu().float(), kp.cpu().float(), vp.cpu().float(),
                                      tables, lens)
    if layout == N.AS_LAYOUT_DIM_MAJOR:
        return OA.flatten_decode_output(o)
    return o.reshape(len(lens), -1)


def _noalloc(q, kp, vp, bt, lk, bps, layout):
    B, H, D = q.shape
    NB, _, Kh, _ = kp.shape
    out = torch.empty(B, H * D, dtype=q.dtype, device=DEV)
    rc = N.load().as_paged_decode_attention_noalloc(
        ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(q.data_ptr()), q.stride(0),
        ctypes.c_void_p(kp.data_ptr()), ctypes.c_void_p(vp.data_ptr()),
        ctypes.c_void_p(bt.data_ptr()), bt.stride(0), ctypes.c_void_p(lk.data_ptr()), B, H, Kh,
        D, 16, NB, bt.shape[1], 1.0 / math.sqrt(D), bps, layout, ops.dtype_code(q.dtype),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    N.check(rc, "as_paged_decode_attention_noalloc")
    return out


def _regular(q, kp, vp, bt, lk, bps, layout):
    B, H, D = q.shape
    ws = ops.new_decode_workspace(B, H, kp.shape[2], D, bt.shape[1], bps, DEV)
    return ops.paged_decode_attention(q, kp, vp, bt, lk, 1.0 / math.sqrt(D), bps, ws,
                                      out_layout=layout)


# (dtype, head_dim, blocks_per_split, tolerance against the fp32 oracle and between the
# two entry points): 1e-5 in fp32, 2e-2 absolute in bf16 / fp16.  blocks_per_split 0
# lets the library choose the split inside the call (the scratch is sized for the
# finest split it may choose).
CASES = [(torch.bfloat16, 64, 8, 2e-2), (torch.float32, 64, 8, 1e-5),
         (torch.bfloat16, 64, 0, 2e-2), (torch.float16, 128, 0, 2e-2),
         (torch.bfloat16, 128, 16, 2e-2)]


@pytest.mark.parametrize("dtype,D,bps,atol", CASES)
def test_noalloc_matches_regular_entry_point_and_oracle_two_calls(dtype, D, bps, atol):
    H, Kh = 32, 8
    calls = [([17, 900, 3, 2048, 160], N.AS_LAYOUT_HEAD_MAJOR),
             ([4096, 1, 700, 33, 1500, 2600, 64, 999, 16, 3000, 250, 1800],
              N.AS_LAYOUT_DIM_MAJOR)]
    for i, (lens, layout) in enumerate(calls):
        q, kp, vp, bt, lk = _case(lens, H, Kh, D, dtype, seed=100 + i + D)
        got = _noalloc(q, kp, vp, bt, lk, bps, layout)
        want = _regular(q, kp, vp, bt, lk, bps, layout)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), rtol=0, atol=atol)
        ref = _oracle(q, kp, vp, bt, lens, layout)
        torch.testing.assert_close(got.float().cpu(), ref, rtol=0, atol=atol)
    assert ops.device_status(clear=True) == 0


def test_noalloc_refuses_calls_beyond_its_static_scratch():
    # 256 sequences x 32 heads x 256 splits x (64 + 2) floats is far above 8 MiB.
    need = ops.decode_workspace_bytes(256, 32, 8, 64, 2048, 8)
    assert need > N.AS_DECODE_NOALLOC_SCRATCH_BYTES
    dummy = torch.zeros(16, dtype=torch.int32, device=DEV)
    p = ctypes.c_void_p(dummy.data_ptr())
    rc = N.load().as_paged_decode_attention_noalloc(
        p, p, 32 * 64, p, p, p, 2048, p, 256, 32, 8, 64, 16, 4096, 2048, 0.125, 8,
        N.AS_LAYOUT_HEAD_MAJOR, N.AS_DTYPE_BF16,
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == N.AS_ERR_WORKSPACE
    assert "static array" in N.last_error()
