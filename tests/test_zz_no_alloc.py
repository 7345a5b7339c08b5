"""as_paged_decode_attention_noalloc: the decode attention entry point for callers
that cannot allocate device memory (their GPU memory belongs to another allocator, or
their serving loop must not reach cudaMalloc).  It keeps its split-K scratch in a
static array inside the library instead of a caller workspace.

Checked here through the C ABI (ctypes): two calls in a row, with different batch
sizes so the second reuses the array the first left behind, each against the
regular entry point on the same inputs; and a call whose scratch need exceeds the
static array is refused before any GPU work.  The file is named to run last.
"""

import ctypes
import math

import pytest
import torch

from agentserve_b200 import _native as N
from agentserve_b200 import ops

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


@pytest.mark.parametrize("dtype,atol", [(torch.bfloat16, 2e-2), (torch.float32, 1e-5)])
def test_noalloc_matches_regular_entry_point_two_calls(dtype, atol):
    H, Kh, D = 32, 8, 64
    calls = [([17, 900, 3, 2048, 160], 8, N.AS_LAYOUT_HEAD_MAJOR),
             ([4096, 1, 700, 33, 1500, 2600, 64, 999, 16, 3000, 250, 1800], 8,
              N.AS_LAYOUT_DIM_MAJOR)]
    for i, (lens, bps, layout) in enumerate(calls):
        q, kp, vp, bt, lk = _case(lens, H, Kh, D, dtype, seed=100 + i)
        got = _noalloc(q, kp, vp, bt, lk, bps, layout)
        want = _regular(q, kp, vp, bt, lk, bps, layout)
        torch.cuda.synchronize()
        torch.testing.assert_close(got.float(), want.float(), rtol=0, atol=atol)
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
