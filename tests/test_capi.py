"""The C-ABI library loads and exports every entry point include/agentserve_b200.h
declares; argument validation works without a GPU (no compute calls here)."""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

from agentserve_b200 import _native as N

REPO = Path(__file__).resolve().parent.parent
HEADER = REPO / "include" / "agentserve_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^AS_API\s+[\w\s\*]+?\b(as_\w+)\s*\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def lib():
    if not N.LIB_PATH.exists():
        from agentserve_b200.build import build
        build()
    return N.load()


def test_header_declares_entry_points():
    syms = declared_symbols()
    for name in ("as_pack_decode", "as_pack_prefill", "as_rope_reshape_and_cache",
                 "as_paged_decode_attention", "as_varlen_prefill_attention", "as_block_copy",
                 "as_paged_decode_workspace_size", "as_last_error", "as_device_status",
                 "as_varlen_prefill_attention_ws", "as_varlen_prefill_workspace_size"):
        assert name in syms


def test_library_exports_every_declared_symbol(lib):
    out = subprocess.run(["nm", "-D", "--defined-only", str(N.LIB_PATH)], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\bT (as_\w+)$", out, flags=re.M))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    # nothing else leaks out of the library with default visibility
    extra = sorted(exported - set(declared_symbols()))
    assert not extra, f"exported but not declared: {extra}"
    for s in declared_symbols():
        assert hasattr(lib, s)
        assert s in N.SIGNATURES, f"{s} has no ctypes signature"


def test_version(lib):
    assert lib.as_version() >= 100


def test_workspace_size_is_host_arithmetic(lib):
    # B=64, H=32, Kh=8, D=64, 272 blocks max, 32 blocks per split -> 9 splits
    n = lib.as_paged_decode_workspace_size(64, 32, 8, 64, 272, 32)
    counters = 64 * 32 * 4
    partial = 64 * 32 * 9
    expect = counters + 2 * partial * 4 + partial * 64 * 4
    assert n >= expect and n - expect < 4 * 256
    assert lib.as_paged_decode_workspace_size(0, 32, 8, 64, 272, 32) == 0


def test_invalid_arguments_rejected_before_any_cuda_call(lib):
    rc = lib.as_paged_decode_attention(None, None, 0, None, None, None, 0, None, 4, 32, 8, 64,
                                       8, 100, 10, 0.125, 16, None, 0, 0, N.AS_DTYPE_BF16, None)
    assert rc == N.AS_ERR_UNSUPPORTED
    assert "block_size must be 16" in N.last_error()
    rc = lib.as_paged_decode_attention(None, None, 0, None, None, None, 0, None, 4, 30, 8, 64,
                                       16, 100, 10, 0.125, 16, None, 0, 0, N.AS_DTYPE_BF16, None)
    assert rc == N.AS_ERR_INVALID_ARG  # H not a multiple of Kh
    rc = lib.as_rope_reshape_and_cache(None, 0, None, 0, None, 0, None, None, None, 0, None,
                                       None, 0, None, 4, 32, 8, 64, 7, None)
    assert rc == N.AS_ERR_INVALID_ARG and "dtype" in N.last_error()
    rc = lib.as_block_copy(None, None, None, None, 3, 100, 1, 0, 0, 1, 1, None)
    assert rc == N.AS_ERR_INVALID_ARG
    rc = lib.as_pack_decode(None, 4, None, None, 2, 8, 16, None, None, None, None, None, None)
    assert rc == N.AS_ERR_INVALID_ARG  # stride < max_blocks
    with pytest.raises(ValueError):
        N.check(N.AS_ERR_INVALID_ARG, "x")
    with pytest.raises(N.KernelError):
        N.check(N.AS_ERR_CUDA, "x")


def test_zero_sized_calls_are_no_ops(lib):
    assert lib.as_pack_decode(None, 8, None, None, 0, 8, 16, None, None, None, None, None,
                              None) == N.AS_OK
    assert lib.as_block_copy(None, None, None, None, 0, 16, 1, 0, 0, 1, 1, None) == N.AS_OK
    assert lib.as_varlen_prefill_attention(None, None, 2048, None, None, None, 8, None, None, 0,
                                           0, 0, 32, 8, 64, 16, 10, 8, 0.125, N.AS_DTYPE_BF16,
                                           None) == N.AS_OK


def test_new_entry_points_host_checks(lib):
    """Workspace-size arithmetic and argument checks of the split-KV prefill, the
    small-batch projection and the greedy sampler, all answered on the host."""
    # split-KV prefill: 1 sequence, 16 new tokens, 32/8 heads, D=64 -> 1 pair per head;
    # 4 forced splits -> 8 heads * 4 * 256 rows of (m, l) + D fp32 values
    rows = 8 * 4 * 256
    n = lib.as_varlen_prefill_workspace_size(1, 16, 32, 8, 64, 1900, 4, N.AS_DTYPE_BF16)
    assert n == -(-rows * 8 // 256) * 256 + -(-rows * 64 * 4 // 256) * 256
    assert lib.as_varlen_prefill_workspace_size(1, 16, 32, 8, 64, 1900, 1, N.AS_DTYPE_BF16) == 0
    assert lib.as_varlen_prefill_workspace_size(1, 16, 32, 8, 64, 1900, 4, N.AS_DTYPE_F32) == 0
    assert lib.as_varlen_prefill_workspace_size(1, 16, 32, 8, 96, 1900, 4, N.AS_DTYPE_BF16) == 0
    rc = lib.as_linear_small_m(None, 16, None, 16, None, 4, 16, 16, N.AS_DTYPE_F32, None)
    assert rc == N.AS_ERR_UNSUPPORTED
    rc = lib.as_linear_small_m(None, 16, None, 16, None, 300, 16, 16, N.AS_DTYPE_BF16, None)
    assert rc == N.AS_ERR_UNSUPPORTED and "M > 256" in N.last_error()
    # greedy: keys [rows] u64 and counters [rows] i32, each rounded to 256 B
    assert lib.as_greedy_workspace_size(64) == 512 + 256
    rc = lib.as_greedy_argmax(None, None, 100, 4, 100, N.AS_DTYPE_BF16, None, 0, None)
    assert rc == N.AS_ERR_INVALID_ARG  # null pointers
    rc = lib.as_greedy_argmax(None, None, 50, 4, 100, N.AS_DTYPE_BF16, None, 0, None)
    assert rc == N.AS_ERR_INVALID_ARG  # row stride < vocab
    assert lib.as_greedy_argmax(None, None, 100, 0, 100, N.AS_DTYPE_BF16, None, 0, None) == N.AS_OK


def test_noalloc_reports_bad_arguments_as_such(lib):
    """The allocation-free decode entry point checks its arguments before it looks at
    its static scratch, so a bad call gets the real cause (no GPU work is done)."""
    for H, Kh, D in ((30, 8, 64), (32, 8, 0)):
        rc = lib.as_paged_decode_attention_noalloc(None, None, 0, None, None, None, 64, None,
                                                   4, H, Kh, D, 16, 100, 64, 0.125, 0,
                                                   N.AS_LAYOUT_HEAD_MAJOR, N.AS_DTYPE_BF16,
                                                   None)
        assert rc == N.AS_ERR_INVALID_ARG
        assert "bad sizes" in N.last_error()
    rc = lib.as_paged_decode_attention_noalloc(None, None, 0, None, None, None, 64, None, 4, 32,
                                               8, 64, 8, 100, 64, 0.125, 0,
                                               N.AS_LAYOUT_HEAD_MAJOR, N.AS_DTYPE_BF16, None)
    assert rc == N.AS_ERR_UNSUPPORTED
    rc = lib.as_paged_decode_attention_noalloc(None, None, 0, None, None, None, 64, None, 4, 32,
                                               8, 64, 16, 100, 64, 0.125, 0, 7, N.AS_DTYPE_BF16,
                                               None)
    assert rc == N.AS_ERR_INVALID_ARG and "out_layout" in N.last_error()
    rc = lib.as_paged_decode_attention_noalloc(None, None, 2048, None, None, None, 64, None, 4,
                                               32, 8, 64, 16, 100, 64, 0.125, 0,
                                               N.AS_LAYOUT_HEAD_MAJOR, N.AS_DTYPE_BF16, None)
    assert rc == N.AS_ERR_INVALID_ARG and "null pointer" in N.last_error()


def test_wait_limit_and_starve_hook_are_host_settings(lib):
    prev = lib.as_set_wait_limit_ns(1_000_000)
    assert prev == 2_000_000_000
    assert lib.as_set_wait_limit_ns(0) == 1_000_000  # 0 restores the default
    assert lib.as_set_wait_limit_ns(0) == 2_000_000_000
    assert lib.as_debug_starve_next_launch(8) == N.AS_ERR_INVALID_ARG
