"""Failure detection on the GPU without a fault: bounded waits that run out.

Every mbarrier wait in the attention kernels has a time limit.  Here the limit is cut
to 1 ms (as_set_wait_limit_ns) and the next launch is told to issue none of its loads
(as_debug_starve_next_launch), so its waits run out for real.  The call must come back
(no hang, no trap, the CUDA context stays usable), status bit 4 must be set, and the
next ordinary call (same workspace, so the split-K arrival counters must have been left
at zero) must match the oracle again.
"""

import pytest
import torch

from agentserve_b200 import _native as N
from agentserve_b200 import ops
from oracle import attention as OA
from tests.test_gpu_kernels import (ATOL_LOWP, DEV, LENS, decode_case, padded, prefill_case,
                                    run_decode, run_prefill)

pytestmark = pytest.mark.gpu

WAIT_TIMEOUT_BIT = 4


@pytest.fixture
def short_waits():
    lib = N.load()
    ops.device_status(clear=True)
    prev = lib.as_set_wait_limit_ns(1_000_000)  # 1 ms
    yield lib
    lib.as_set_wait_limit_ns(prev)
    lib.as_debug_starve_next_launch(0)
    ops.device_status(clear=True)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("bps", [0, 4])
def test_decode_wait_that_runs_out_returns_and_next_call_is_correct(short_waits, D, bps):
    lib = short_waits
    tables, kp, vp, q = decode_case(LENS, 32, 8, D, torch.bfloat16, seed=300 + D + bps)
    bt = padded(tables)
    ws = ops.new_decode_workspace(len(LENS), 32, 8, D, bt.shape[1], bps, DEV)
    assert lib.as_debug_starve_next_launch(N.AS_KERNEL_DECODE_ATTENTION) == N.AS_OK
    starved = run_decode(tables, kp, vp, q, LENS, bps, ws=ws)  # synchronises
    assert ops.device_status(clear=True) & WAIT_TIMEOUT_BIT
    # a CTA whose waits ran out contributes nothing: every row comes out zero
    assert torch.count_nonzero(starved) == 0
    lib.as_set_wait_limit_ns(0)
    out = run_decode(tables, kp, vp, q, LENS, bps, ws=ws)
    ref = OA.decode_attention_from_pool(q.float(), kp.float(), vp.float(), tables, LENS)
    torch.testing.assert_close(out.float(), ref.reshape(len(LENS), -1), rtol=0, atol=ATOL_LOWP)
    assert ops.device_status(clear=True) == 0


@pytest.mark.parametrize("D", [64, 128])
def test_prefill_wait_that_runs_out_returns_and_next_call_is_correct(short_waits, D):
    lib = short_waits
    num_cached, num_new = [0, 32, 37, 160], [1, 17, 130, 200]
    tables, kp, vp, q, cu, lens = prefill_case(num_cached, num_new, 32, 8, D, torch.bfloat16,
                                               seed=400 + D)
    assert lib.as_debug_starve_next_launch(N.AS_KERNEL_PREFILL_ATTENTION) == N.AS_OK
    run_prefill(tables, kp, vp, q, cu, lens)  # synchronises; its output is not written
    assert ops.device_status(clear=True) & WAIT_TIMEOUT_BIT
    lib.as_set_wait_limit_ns(0)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    assert ops.device_status(clear=True) == 0


def test_starve_hook_is_consumed_by_one_launch(short_waits):
    lib = short_waits
    lib.as_set_wait_limit_ns(0)
    tables, kp, vp, q = decode_case([100, 700], 32, 8, 64, torch.bfloat16, seed=5)
    assert lib.as_debug_starve_next_launch(N.AS_KERNEL_PREFILL_ATTENTION) == N.AS_OK
    out = run_decode(tables, kp, vp, q, [100, 700], 8)  # a decode launch ignores it
    ref = OA.decode_attention_from_pool(q.float(), kp.float(), vp.float(), tables, [100, 700])
    torch.testing.assert_close(out.float(), ref.reshape(2, -1), rtol=0, atol=ATOL_LOWP)
    assert ops.device_status(clear=True) == 0
    assert lib.as_debug_starve_next_launch(0) == N.AS_OK  # clears the pending prefill bit
    num_cached, num_new = [0, 32], [17, 130]
    tables, kp, vp, q, cu, lens = prefill_case(num_cached, num_new, 32, 8, 64, torch.bfloat16, 6)
    out = run_prefill(tables, kp, vp, q, cu, lens)
    ref = OA.prefill_attention_from_pool(q.float(), kp.float(), vp.float(), tables, cu, lens)
    torch.testing.assert_close(out.float(), ref, rtol=0, atol=ATOL_LOWP)
    assert ops.device_status(clear=True) == 0
