"""torch-facing wrappers of the C-ABI kernels.

Each wrapper checks shapes/devices, passes raw device pointers and the current CUDA
stream to the library, and raises on a non-zero status.  Tensors must live on a
CUDA device: there is no CPU path.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch

from . import _native as N

BLOCK_SIZE = 16

_DTYPES = {torch.float32: N.AS_DTYPE_F32, torch.float16: N.AS_DTYPE_F16,
           torch.bfloat16: N.AS_DTYPE_BF16}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPES[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; use float32, float16 or bfloat16") from None


def _cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("agentserve_b200 ops need CUDA tensors (no CPU fallback)")


def _require(ok: bool, what: str) -> None:
    """Argument checks raise ValueError (kept under python -O, unlike assert)."""
    if not ok:
        raise ValueError(what)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def device_status(clear: bool = True, device=None) -> int:
    """Read (and clear) the device status word: 1 bad block id, 2 bad slot, 4 wait
    timeout, 8 position outside the RoPE table, 16 sequence longer than its table row."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else device
    bits = ctypes.c_int(0)
    with torch.cuda.device(dev):
        N.check(N.load().as_device_status(int(clear), ctypes.byref(bits), _stream(dev)),
                "as_device_status")
    return bits.value


# ---------------------------------------------------------------------------
# (1) packing
# ---------------------------------------------------------------------------
@dataclass
class DecodePack:
    positions: torch.Tensor     # [B] int64
    slot_mapping: torch.Tensor  # [B] int64
    seq_lens_k: torch.Tensor    # [B] int32
    cu_seqlens_q: torch.Tensor  # [B+1] int32
    block_tables: torch.Tensor  # [B, max_blocks] int32


@dataclass
class PrefillPack:
    cu_seqlens_q: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    seq_lens_k: torch.Tensor
    block_tables: torch.Tensor


def pack_decode(block_tables: torch.Tensor, seq_lens: torch.Tensor,
                row_ids: Optional[torch.Tensor] = None, max_blocks: Optional[int] = None,
                out: Optional[DecodePack] = None) -> DecodePack:
    """block_tables [rows, stride] int32 (device-resident allocator table),
    seq_lens [B] int32 = cached tokens (position of the new token), row_ids [B] int32."""
    _cuda(block_tables, seq_lens, row_ids)
    B = seq_lens.shape[0]
    mb = max_blocks if max_blocks is not None else block_tables.shape[1]
    dev = seq_lens.device
    if out is None:
        out = DecodePack(torch.empty(B, dtype=torch.int64, device=dev),
                         torch.empty(B, dtype=torch.int64, device=dev),
                         torch.empty(B, dtype=torch.int32, device=dev),
                         torch.empty(B + 1, dtype=torch.int32, device=dev),
                         torch.empty(B, mb, dtype=torch.int32, device=dev))
    _require(block_tables.dtype == torch.int32 and seq_lens.dtype == torch.int32,
             "pack_decode: block_tables and seq_lens must be int32")
    _require(block_tables.stride(1) == 1, "pack_decode: block_tables rows must be contiguous")
    N.check(N.load().as_pack_decode(
        _ptr(block_tables), block_tables.stride(0), _ptr(row_ids), _ptr(seq_lens), B, mb,
        BLOCK_SIZE, _ptr(out.positions), _ptr(out.slot_mapping), _ptr(out.seq_lens_k),
        _ptr(out.cu_seqlens_q), _ptr(out.block_tables), _stream(dev)), "as_pack_decode")
    return out


def pack_prefill(block_tables: torch.Tensor, num_cached: torch.Tensor, num_new: torch.Tensor,
                 total_new: int, row_ids: Optional[torch.Tensor] = None,
                 max_blocks: Optional[int] = None) -> PrefillPack:
    _cuda(block_tables, num_cached, num_new, row_ids)
    R = num_new.shape[0]
    mb = max_blocks if max_blocks is not None else block_tables.shape[1]
    dev = num_new.device
    out = PrefillPack(torch.empty(R + 1, dtype=torch.int32, device=dev),
                      torch.empty(total_new, dtype=torch.int64, device=dev),
                      torch.empty(total_new, dtype=torch.int64, device=dev),
                      torch.empty(R, dtype=torch.int32, device=dev),
                      torch.empty(R, mb, dtype=torch.int32, device=dev))
    N.check(N.load().as_pack_prefill(
        _ptr(block_tables), block_tables.stride(0), _ptr(row_ids), _ptr(num_cached),
        _ptr(num_new), R, total_new, mb, BLOCK_SIZE, _ptr(out.cu_seqlens_q),
        _ptr(out.positions), _ptr(out.slot_mapping), _ptr(out.seq_lens_k),
        _ptr(out.block_tables), _stream(dev)), "as_pack_prefill")
    return out


# ---------------------------------------------------------------------------
# (2) fused RoPE + reshape_and_cache
# ---------------------------------------------------------------------------
def _row_view_ok(x: torch.Tensor) -> bool:
    return x.dim() == 3 and x.stride(2) == 1 and x.stride(1) == x.shape[2]


def rope_reshape_and_cache(q: Optional[torch.Tensor], k: torch.Tensor, v: torch.Tensor,
                           positions: Optional[torch.Tensor], slot_mapping: torch.Tensor,
                           cos_sin: Optional[torch.Tensor], k_cache: torch.Tensor,
                           v_cache: torch.Tensor, k_out: Optional[torch.Tensor] = None) -> None:
    """q [T, H, D] (rotated in place), k/v [T, Kh, D]; each may be a row-strided view
    (e.g. column slices of a fused QKV output).  k_cache/v_cache [NB, 16, Kh, D].
    cos_sin None: no rotation (plain write of k and v)."""
    _cuda(q, k, v, positions, slot_mapping, cos_sin, k_cache, v_cache, k_out)
    T, Kh, D = k.shape
    H = q.shape[1] if q is not None else 1
    for name, t in (("q", q), ("k", k), ("v", v)):
        if t is not None and not _row_view_ok(t):
            raise ValueError(f"{name} must be [T, heads, D] with contiguous rows")
    if cos_sin is not None:
        _require(cos_sin.dtype == torch.float32 and cos_sin.is_contiguous(),
                 "cos_sin must be a contiguous float32 table")
    _require(k_cache.is_contiguous() and v_cache.is_contiguous(), "KV planes must be contiguous")
    _require(k_cache.shape[1:] == (BLOCK_SIZE, Kh, D) and v_cache.shape == k_cache.shape,
             "k_cache / v_cache must be [NB, 16, Kh, D]")
    num_slots = k_cache.shape[0] * BLOCK_SIZE
    N.check(N.load().as_rope_reshape_and_cache(
        _ptr(q), q.stride(0) if q is not None else H * D, _ptr(k), k.stride(0), _ptr(v),
        v.stride(0), _ptr(positions), _ptr(slot_mapping), _ptr(cos_sin),
        cos_sin.shape[0] if cos_sin is not None else 0, _ptr(k_cache), _ptr(v_cache), num_slots,
        _ptr(k_out), T, H, Kh, D, dtype_code(k.dtype), _stream(k.device)),
        "as_rope_reshape_and_cache")


# ---------------------------------------------------------------------------
# (3) paged decode attention
# ---------------------------------------------------------------------------
def decode_workspace_bytes(num_seqs: int, num_heads: int, num_kv_heads: int, head_dim: int,
                           max_blocks: int, blocks_per_split: int) -> int:
    return int(N.load().as_paged_decode_workspace_size(num_seqs, num_heads, num_kv_heads,
                                                        head_dim, max_blocks, blocks_per_split))


def new_decode_workspace(num_seqs, num_heads, num_kv_heads, head_dim, max_blocks,
                         blocks_per_split, device) -> torch.Tensor:
    """Zero-filled workspace (the kernel keeps its counters at zero between calls)."""
    n = decode_workspace_bytes(num_seqs, num_heads, num_kv_heads, head_dim, max_blocks,
                               blocks_per_split)
    return torch.zeros(max(n, 256), dtype=torch.uint8, device=device)


class DecodeWorkspace:
    """Grow-only split-K workspace shared by calls with different batch sizes.

    The library keeps per-(sequence, head) arrival counters at the front of the
    workspace ([B*H] int32, rounded up to 256 bytes) and split partials after them,
    and leaves every counter it used at zero.  A call with a larger B than earlier
    calls extends the counter region over bytes that held partials, so that region
    is zeroed first; otherwise no memset is issued (fixed-B CUDA graphs issue none).
    """

    def __init__(self, num_heads: int, num_kv_heads: int, head_dim: int, device):
        self.H, self.Kh, self.D = num_heads, num_kv_heads, head_dim
        self.device = device
        self.buf: Optional[torch.Tensor] = None
        self._clean_upto = 0  # bytes [0, _clean_upto) are known to be zero

    def get(self, num_seqs: int, max_blocks: int, blocks_per_split: int) -> torch.Tensor:
        need = decode_workspace_bytes(num_seqs, self.H, self.Kh, self.D, max_blocks,
                                      blocks_per_split)
        counters = (num_seqs * self.H * 4 + 255) // 256 * 256
        if self.buf is None or self.buf.numel() < need:
            size = max(need, 1 << 20)
            if self.buf is not None:
                size = max(size, 2 * self.buf.numel())
            self.buf = torch.zeros(size, dtype=torch.uint8, device=self.device)
            self._clean_upto = counters
        elif counters > self._clean_upto:
            self.buf[:counters].zero_()
            self._clean_upto = counters
        else:
            self._clean_upto = counters  # partials of this call start right here
        return self.buf


def paged_decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                           block_tables: torch.Tensor, seq_lens_k: torch.Tensor, scale: float,
                           blocks_per_split: int, workspace: Optional[torch.Tensor],
                           out: Optional[torch.Tensor] = None,
                           out_layout: int = N.AS_LAYOUT_HEAD_MAJOR,
                           num_heads: Optional[int] = None) -> torch.Tensor:
    """q [B, H, D] (row-strided view allowed), k_cache/v_cache [NB, 16, Kh, D],
    block_tables [B, >=max_blocks] int32, seq_lens_k [B] int32 (keys incl. the new
    token).  Returns out [B, H*D] in out_layout."""
    _cuda(q, k_cache, v_cache, block_tables, seq_lens_k, workspace, out)
    B, H, D = q.shape
    NB, bs, Kh, D2 = k_cache.shape
    _require(bs == BLOCK_SIZE and D2 == D and v_cache.shape == k_cache.shape,
             "k_cache / v_cache must be [NB, 16, Kh, D] with q's head_dim")
    _require(_row_view_ok(q), "q must be [B, H, D] with contiguous rows")
    _require(block_tables.dtype == torch.int32 and block_tables.stride(1) == 1,
             "block_tables must be int32 with contiguous rows")
    max_blocks = block_tables.shape[1]
    if out is None:
        out = torch.empty(B, H * D, dtype=q.dtype, device=q.device)
    ws_ptr = _ptr(workspace)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    N.check(N.load().as_paged_decode_attention(
        _ptr(out), _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache), _ptr(block_tables),
        block_tables.stride(0), _ptr(seq_lens_k), B, H, Kh, D, BLOCK_SIZE, NB, max_blocks,
        float(scale), int(blocks_per_split), ws_ptr, ws_bytes, int(out_layout),
        dtype_code(q.dtype), _stream(q.device)), "as_paged_decode_attention")
    return out


def rope_decode_fusable(q: torch.Tensor, k_cache: torch.Tensor) -> bool:
    """True when rope_paged_decode_attention's one-launch path applies (bf16 / fp16,
    head_dim 64 or 128, at most 8 query heads per KV head)."""
    _, H, D = q.shape
    Kh = k_cache.shape[2]
    return (q.dtype in (torch.bfloat16, torch.float16) and D in (64, 128) and H % Kh == 0
            and H // Kh <= 8)


def rope_paged_decode_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                positions: torch.Tensor, slot_mapping: torch.Tensor,
                                cos_sin: torch.Tensor, k_cache: torch.Tensor,
                                v_cache: torch.Tensor, block_tables: torch.Tensor,
                                seq_lens_k: torch.Tensor, scale: float, blocks_per_split: int,
                                workspace: Optional[torch.Tensor],
                                out: Optional[torch.Tensor] = None,
                                out_layout: int = N.AS_LAYOUT_HEAD_MAJOR) -> torch.Tensor:
    """The decode step's RoPE + cache write of the new token and its attention in one
    launch (as_rope_paged_decode_attention): q [B, H, D], k / v [B, Kh, D] unrotated
    (row-strided views allowed, left unmodified), positions / slot_mapping [B] int64,
    cos_sin the fp32 table.  Same results as rope_reshape_and_cache followed by
    paged_decode_attention; fast path only (rope_decode_fusable)."""
    _cuda(q, k, v, positions, slot_mapping, cos_sin, k_cache, v_cache, block_tables,
          seq_lens_k, workspace, out)
    B, H, D = q.shape
    NB, bs, Kh, D2 = k_cache.shape
    _require(bs == BLOCK_SIZE and D2 == D and v_cache.shape == k_cache.shape,
             "k_cache / v_cache must be [NB, 16, Kh, D] with q's head_dim")
    _require(k_cache.is_contiguous() and v_cache.is_contiguous(), "KV planes must be contiguous")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require(_row_view_ok(t), f"{name} must be [B, heads, D] with contiguous rows")
    _require(k.shape == (B, Kh, D) and v.shape == (B, Kh, D), "k / v must be [B, Kh, D]")
    _require(cos_sin.dtype == torch.float32 and cos_sin.is_contiguous(),
             "cos_sin must be a contiguous float32 table")
    _require(block_tables.dtype == torch.int32 and block_tables.stride(1) == 1,
             "block_tables must be int32 with contiguous rows")
    if out is None:
        out = torch.empty(B, H * D, dtype=q.dtype, device=q.device)
    ws_bytes = workspace.numel() * workspace.element_size() if workspace is not None else 0
    N.check(N.load().as_rope_paged_decode_attention(
        _ptr(out), _ptr(q), q.stride(0), _ptr(k), k.stride(0), _ptr(v), v.stride(0),
        _ptr(positions), _ptr(slot_mapping), _ptr(cos_sin), cos_sin.shape[0], _ptr(k_cache),
        _ptr(v_cache), _ptr(block_tables), block_tables.stride(0), _ptr(seq_lens_k), B, H, Kh, D,
        BLOCK_SIZE, NB, block_tables.shape[1], float(scale), int(blocks_per_split),
        _ptr(workspace), ws_bytes, int(out_layout), dtype_code(q.dtype), _stream(q.device)),
        "as_rope_paged_decode_attention")
    return out


# ---------------------------------------------------------------------------
# (4) varlen prefill attention
# ---------------------------------------------------------------------------
def prefill_workspace_bytes(num_seqs: int, max_seqlen_q: int, num_heads: int, num_kv_heads: int,
                            head_dim: int, max_blocks: int, num_splits: int = 0,
                            dtype: torch.dtype = torch.bfloat16) -> int:
    """Split-KV workspace of varlen_prefill_attention (0 when no split applies)."""
    return int(N.load().as_varlen_prefill_workspace_size(
        num_seqs, max_seqlen_q, num_heads, num_kv_heads, head_dim, max_blocks, num_splits,
        dtype_code(dtype)))


def varlen_prefill_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                             block_tables: torch.Tensor, cu_seqlens_q: torch.Tensor,
                             seq_lens_k: torch.Tensor, max_seqlen_q: int, scale: float,
                             out: Optional[torch.Tensor] = None, num_splits: int = 0,
                             workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [total_q, H, D] (row-strided view allowed); returns out [total_q, H*D]
    (head-major, as prefill flattens it: llama.py:184).  num_splits: split-KV over
    CTAs (0 = chosen by the library, 1 = off); its fp32 partials go to `workspace`
    (uint8, prefill_workspace_bytes() long), allocated per call when not given."""
    _cuda(q, k_cache, v_cache, block_tables, cu_seqlens_q, seq_lens_k, out, workspace)
    Tq, H, D = q.shape
    NB, bs, Kh, D2 = k_cache.shape
    _require(bs == BLOCK_SIZE and D2 == D and v_cache.shape == k_cache.shape,
             "k_cache / v_cache must be [NB, 16, Kh, D] with q's head_dim")
    _require(_row_view_ok(q), "q must be [T, H, D] with contiguous rows")
    _require(block_tables.dtype == torch.int32 and block_tables.stride(1) == 1,
             "block_tables must be int32 with contiguous rows")
    R = seq_lens_k.shape[0]
    mb = block_tables.shape[1]
    if out is None:
        out = torch.empty(Tq, H * D, dtype=q.dtype, device=q.device)
    if workspace is None and num_splits != 1:
        need = prefill_workspace_bytes(R, int(max_seqlen_q), H, Kh, D, mb, num_splits, q.dtype)
        if need:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_ptr = _ptr(workspace) if workspace is not None else None
    ws_bytes = workspace.numel() if workspace is not None else 0
    N.check(N.load().as_varlen_prefill_attention_ws(
        _ptr(out), _ptr(q), q.stride(0), _ptr(k_cache), _ptr(v_cache), _ptr(block_tables),
        block_tables.stride(0), _ptr(cu_seqlens_q), _ptr(seq_lens_k), R, int(max_seqlen_q), Tq,
        H, Kh, D, BLOCK_SIZE, NB, mb, float(scale), dtype_code(q.dtype), int(num_splits),
        ws_ptr, ws_bytes, _stream(q.device)), "as_varlen_prefill_attention")
    return out


# ---------------------------------------------------------------------------
# (6) decode-step projections at small batch
# ---------------------------------------------------------------------------
LINEAR_MAX_M = 256


def linear_small_m(x: torch.Tensor, w: torch.Tensor,
                   out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [M, K] (row-strided view allowed, M <= 256) @ w[N, K]^T -> [M, N]: nn.Linear
    without bias on the tensor cores, K split over the CTAs of a cluster and reduced
    on chip."""
    _cuda(x, w, out)
    M, K = x.shape
    Nn = w.shape[0]
    _require(w.shape[1] == K and w.is_contiguous() and x.stride(1) == 1 and x.dtype == w.dtype,
             "linear_small_m: w must be a contiguous [N, K] of x's dtype, x rows contiguous")
    if out is None:
        out = torch.empty(M, Nn, dtype=x.dtype, device=x.device)
    _require(out.shape == (M, Nn) and out.stride(1) == 1 and out.dtype == x.dtype,
             "linear_small_m: out must be [M, N] of x's dtype with contiguous rows")
    N.check(N.load().as_linear_small_m(
        _ptr(out), out.stride(0), _ptr(x), x.stride(0), _ptr(w), M, Nn, K, dtype_code(x.dtype),
        _stream(x.device)), "as_linear_small_m")
    return out


def linear_small_m_swiglu(x: torch.Tensor, gate_up: torch.Tensor,
                          out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x [M, K] (M <= 256) -> silu(x W_gate^T) * (x W_up^T) [M, inter] in one launch from
    the fused [gate; up] weight [2*inter, K] (inter a multiple of 64): the same bits as
    silu_mul(linear_small_m(x, gate_up)) (llama.py:207-211)."""
    _cuda(x, gate_up, out)
    M, K = x.shape
    two_i = gate_up.shape[0]
    _require(gate_up.shape[1] == K and gate_up.is_contiguous() and x.stride(1) == 1 and
             x.dtype == gate_up.dtype and two_i % 128 == 0,
             "linear_small_m_swiglu: gate_up must be a contiguous [2*inter, K] of x's dtype, "
             "inter a multiple of 64")
    if out is None:
        out = torch.empty(M, two_i // 2, dtype=x.dtype, device=x.device)
    _require(out.shape == (M, two_i // 2) and out.stride(1) == 1 and out.dtype == x.dtype,
             "linear_small_m_swiglu: out must be [M, inter] of x's dtype with contiguous rows")
    N.check(N.load().as_linear_small_m_swiglu(
        _ptr(out), out.stride(0), _ptr(x), x.stride(0), _ptr(gate_up), M, two_i // 2, K,
        dtype_code(x.dtype), _stream(x.device)), "as_linear_small_m_swiglu")
    return out


# ---------------------------------------------------------------------------
# (7) greedy sampling
# ---------------------------------------------------------------------------
GREEDY_WS_ROWS = 4096
_greedy_ws: dict = {}


def greedy_argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[B, V] logits -> [B] int64 token ids: the reference's greedy sampling (fp32,
    nan_to_num(0, 1e4, -1e4), first argmax) in one kernel.  Its small workspace is one
    fixed buffer per device (so CUDA graphs keep its address), for up to 4096 rows."""
    _cuda(logits, out)
    B, V = logits.shape
    _require(logits.stride(1) == 1, "greedy_argmax: logits rows must be contiguous")
    _require(out is None or (out.shape == (B,) and out.dtype == torch.int64 and out.is_contiguous()),
             "greedy_argmax: out must be a contiguous int64 [B]")
    if out is None:
        out = torch.empty(B, dtype=torch.int64, device=logits.device)
    if B > GREEDY_WS_ROWS:
        ws = torch.zeros(int(N.load().as_greedy_workspace_size(B)), dtype=torch.uint8,
                         device=logits.device)
    else:
        ws = _greedy_ws.get(logits.device)
        if ws is None:
            ws = _greedy_ws[logits.device] = torch.zeros(
                int(N.load().as_greedy_workspace_size(GREEDY_WS_ROWS)), dtype=torch.uint8,
                device=logits.device)
    N.check(N.load().as_greedy_argmax(
        _ptr(out), _ptr(logits), logits.stride(0), B, V, dtype_code(logits.dtype), _ptr(ws),
        ws.numel(), _stream(logits.device)), "as_greedy_argmax")
    return out


# ---------------------------------------------------------------------------
# (5) block gather / copy
# ---------------------------------------------------------------------------
def block_copy(dst: torch.Tensor, src: torch.Tensor, src_ids: torch.Tensor,
               dst_ids: Optional[torch.Tensor], bytes_per_block: int, num_planes: int,
               src_plane_stride: int, dst_plane_stride: int, src_num_blocks: int,
               dst_num_blocks: int) -> None:
    """Byte-level block copy; strides in bytes.  See as_block_copy."""
    _cuda(dst, src, src_ids, dst_ids)
    n = src_ids.shape[0]
    N.check(N.load().as_block_copy(
        _ptr(dst), _ptr(src), _ptr(src_ids), _ptr(dst_ids), n, int(bytes_per_block),
        int(num_planes), int(src_plane_stride), int(dst_plane_stride), int(src_num_blocks),
        int(dst_num_blocks), _stream(dst.device)), "as_block_copy")


# ---------------------------------------------------------------------------
# fused elementwise stages of the decode step
# ---------------------------------------------------------------------------
def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """RMSNorm of the rows of x [rows, dim] (llama.py:39-56)."""
    _cuda(x, weight, out)
    _require(x.is_contiguous() and weight.is_contiguous(), "rmsnorm: x and weight must be contiguous")
    if out is None:
        out = torch.empty_like(x)
    _require(out.shape == x.shape and out.dtype == x.dtype and out.is_contiguous(),
             "rmsnorm: out must be a contiguous tensor like x")
    dim = x.shape[-1]
    N.check(N.load().as_rmsnorm(_ptr(out), _ptr(x), _ptr(weight), x.numel() // dim, dim,
                                float(eps), dtype_code(x.dtype), _stream(x.device)), "as_rmsnorm")
    return out


def add_rmsnorm(x: torch.Tensor, delta: torch.Tensor, weight: torch.Tensor, eps: float,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """x += delta in place (rounded to x.dtype), returns rmsnorm(x)."""
    _cuda(x, delta, weight, out)
    _require(x.is_contiguous() and delta.is_contiguous() and delta.shape == x.shape and
             weight.is_contiguous(), "add_rmsnorm: x, delta (same shape) and weight must be contiguous")
    if out is None:
        out = torch.empty_like(x)
    _require(out.shape == x.shape and out.dtype == x.dtype and out.is_contiguous(),
             "add_rmsnorm: out must be a contiguous tensor like x")
    dim = x.shape[-1]
    N.check(N.load().as_add_rmsnorm(_ptr(out), _ptr(x), _ptr(delta), _ptr(weight),
                                    x.numel() // dim, dim, float(eps), dtype_code(x.dtype),
                                    _stream(x.device)), "as_add_rmsnorm")
    return out


def silu_mul(gate_up: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """gate_up [rows, 2*I] -> silu(gate) * up [rows, I] (llama.py:207-211)."""
    _cuda(gate_up, out)
    _require(gate_up.is_contiguous() and gate_up.shape[1] % 2 == 0,
             "silu_mul: gate_up must be a contiguous [rows, 2*I]")
    rows, two_i = gate_up.shape
    inter = two_i // 2
    if out is None:
        out = torch.empty(rows, inter, dtype=gate_up.dtype, device=gate_up.device)
    _require(out.shape == (rows, inter) and out.dtype == gate_up.dtype and out.is_contiguous(),
             "silu_mul: out must be a contiguous [rows, I] of gate_up's dtype")
    N.check(N.load().as_silu_mul(_ptr(out), _ptr(gate_up), rows, inter,
                                 dtype_code(gate_up.dtype), _stream(gate_up.device)),
            "as_silu_mul")
    return out
