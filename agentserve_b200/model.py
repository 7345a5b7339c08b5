"""Llama decoder whose attention step runs on the sm_100a C-ABI kernels.

Drop-in for the object AgentServe's Engine calls (agentserve/model/llama.py):
same parameter names and shapes as LlamaModel (llama.py:245-262), and the three
methods Engine uses:

  forward(token_ids, kv_cache, position_offset)        llama.py:478-520, engine.py:304-308
  forward_decode_batch(last_token_ids, kv_caches, pos)  llama.py:265-376, engine.py:370-374
  forward_decode_paged(last, seq_lens, pos, allocator, request_ids)
                                                        llama.py:379-475, engine.py:360-366

Attention, RoPE, KV writes, packing, block gathers, RMSNorm (+ residual add),
SwiGLU and greedy argmax are the library's kernels; so are the projections and
lm_head of batches up to `small_batch_max_rows` (64) tokens — the decode step — on the
small-batch tensor-core kernel with SwiGLU fused into gate/up (`small_batch_linear`),
while larger batches (prefill) use cuBLAS GEMMs through torch.  With
reference_compat=True (default) two
behaviours of the reference's decode paths are reproduced so results match it:
the decode attention output is flattened dim-major before o_proj (llama.py:362,
470), and forward_decode_batch returns, for every sequence shorter than the
batch's longest, a zero K/V row in place of its new token (llama.py:327, 372).
reference_compat=False gives the head-major flatten of prefill (llama.py:184) and
keeps the new token's K/V.
"""

from __future__ import annotations

import math
from collections import OrderedDict
from typing import List, Optional, Sequence

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _native as N
from . import ops
from .cache import DeviceBlockAllocator

BS = ops.BLOCK_SIZE


def precompute_rope_freqs(head_dim: int, max_seq_len: int, theta: float) -> torch.Tensor:
    """fp32 cos||sin table [max_seq_len, head_dim] (llama.py:63-77), built on the CPU
    so every device gets the same bits."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    f = torch.outer(torch.arange(max_seq_len, dtype=torch.float32), inv)
    return torch.cat([f.cos(), f.sin()], dim=-1)


class RMSNorm(nn.Module):
    """llama.py:39-56."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim))

    def forward(self, x):
        xf = x.float()
        r = torch.rsqrt(xf.pow(2).mean(dim=-1, keepdim=True) + self.eps)
        return (xf * r).to(x.dtype) * self.weight


class _Attn(nn.Module):
    def __init__(self, c, tp_size: int = 1, split_o: bool = False):
        super().__init__()
        H, Kh, D = c.n_heads // tp_size, c.n_kv_heads // tp_size, c.head_dim
        self.q_proj = nn.Linear(c.hidden_dim, H * D, bias=False)
        self.k_proj = nn.Linear(c.hidden_dim, Kh * D, bias=False)
        self.v_proj = nn.Linear(c.hidden_dim, Kh * D, bias=False)
        self.o_proj = nn.Linear(H * D, c.hidden_dim, bias=False)
        # KV-head TP with the reference's two flattens: prefill feeds o_proj head-major
        # (llama.py:184), decode dim-major (llama.py:362, 470), so a rank's heads meet
        # two different column sets of the full o_proj; o_proj holds the decode set and
        # o_proj_prefill the prefill one
        self.o_proj_prefill = nn.Linear(H * D, c.hidden_dim, bias=False) if split_o else None


class _MLP(nn.Module):
    def __init__(self, c):
        super().__init__()
        self.gate_proj = nn.Linear(c.hidden_dim, c.intermediate_size, bias=False)
        self.up_proj = nn.Linear(c.hidden_dim, c.intermediate_size, bias=False)
        self.down_proj = nn.Linear(c.intermediate_size, c.hidden_dim, bias=False)


class _Layer(nn.Module):
    def __init__(self, c, tp_size: int = 1, split_o: bool = False):
        super().__init__()
        self.attn_norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.attn = _Attn(c, tp_size, split_o)
        self.ffn_norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.ffn = _MLP(c)


def shard_state_dict(full: dict, config, tp_size: int, tp_rank: int,
                     reference_compat: bool = True) -> dict:
    """KV-head tensor parallelism: the state dict of rank tp_rank out of tp_size.

    Rank r keeps query heads [r*H/N, (r+1)*H/N) and KV heads [r*Kh/N, (r+1)*Kh/N) (a
    GQA group never straddles ranks), i.e. row slices of q/k/v_proj, and the o_proj
    columns its heads feed.  Those columns are contiguous for the head-major flatten
    (h*D + d), and strided for the reference decode's dim-major flatten (d*H + h):
    the rank's local attention output is d*H_l + h_l, so its o_proj shard is
    W[:, d*H + r*H_l + h_l] in that order.  With reference_compat the prefill still
    flattens head-major, so the rank also gets the contiguous shard as
    attn.o_proj_prefill.weight.  Everything else is replicated."""
    H, Kh, D = config.n_heads, config.n_kv_heads, config.head_dim
    if H % tp_size or Kh % tp_size:
        raise ValueError(f"{tp_size} ranks cannot split {H} query / {Kh} KV heads")
    Hl, Khl = H // tp_size, Kh // tp_size
    out = {}
    if reference_compat:
        d = torch.arange(D).view(D, 1)
        h = torch.arange(Hl).view(1, Hl) + tp_rank * Hl
        ocols = (d * H + h).reshape(-1)
    else:
        ocols = torch.arange(tp_rank * Hl * D, (tp_rank + 1) * Hl * D)
    for name, w in full.items():
        if name.endswith("attn.q_proj.weight"):
            out[name] = w[tp_rank * Hl * D:(tp_rank + 1) * Hl * D]
        elif name.endswith("attn.k_proj.weight") or name.endswith("attn.v_proj.weight"):
            out[name] = w[tp_rank * Khl * D:(tp_rank + 1) * Khl * D]
        elif name.endswith("attn.o_proj.weight"):
            out[name] = w[:, ocols.to(w.device)]
            if reference_compat:
                out[name.replace("o_proj.weight", "o_proj_prefill.weight")] = \
                    w[:, tp_rank * Hl * D:(tp_rank + 1) * Hl * D]
        elif name.endswith("attn.o_proj_prefill.weight"):
            continue
        else:
            out[name] = w
    return {k: v.contiguous() for k, v in out.items()}


class B200LlamaModel(nn.Module):
    """tp_size > 1: KV-head tensor parallelism over tp_group (one process per GPU):
    this rank holds H/N query and Kh/N KV heads of every sequence (its allocator holds
    Kh/N heads too), o_proj is row-parallel and its output is summed over the group
    with one all-reduce per layer; the MLP, embedding and lm_head are replicated.
    Build the weights with shard_state_dict()."""

    def __init__(self, config, dtype: torch.dtype = torch.bfloat16,
                 device: str | torch.device = "cuda", fused_projections: bool = True,
                 reference_compat: bool = True, tp_size: int = 1, tp_rank: int = 0,
                 tp_group=None):
        super().__init__()
        c = self.config = config
        if c.n_heads % tp_size or c.n_kv_heads % tp_size:
            raise ValueError(f"{tp_size} ranks cannot split {c.n_heads}/{c.n_kv_heads} heads")
        self.tp_size, self.tp_rank, self.tp_group = tp_size, tp_rank, tp_group
        self.H, self.Kh, self.D = c.n_heads // tp_size, c.n_kv_heads // tp_size, c.head_dim
        self.embed = nn.Embedding(c.vocab_size, c.hidden_dim)
        split_o = tp_size > 1 and reference_compat
        self.layers = nn.ModuleList([_Layer(c, tp_size, split_o) for _ in range(c.n_layers)])
        self.norm = RMSNorm(c.hidden_dim, c.rms_norm_eps)
        self.lm_head = nn.Linear(c.hidden_dim, c.vocab_size, bias=False)
        self.to(device=device, dtype=dtype)
        # fp32 table whatever the model dtype (the reference's table is fp32 unless the
        # whole module is cast, llama.py:261-262)
        self.rope_table = precompute_rope_freqs(self.D, c.max_seq_len, c.rope_theta).to(device)
        self.scale = 1.0 / math.sqrt(self.D)  # SDPA's default scale (llama.py:183)
        self.fused_projections = fused_projections
        self.reference_compat = reference_compat
        self.decode_layout = N.AS_LAYOUT_DIM_MAJOR if reference_compat else N.AS_LAYOUT_HEAD_MAJOR
        self._fused = False
        self._workspaces = {}
        # forward_decode_batch's block buffers, kept while the caller feeds back the
        # caches it returned; free tokens each sequence gets when they are (re)packed
        self._batch_pool: Optional[dict] = None
        self.decode_batch_headroom: int = 64
        # decode attention split-K chunk in blocks: 0 = chosen by the library from the
        # batch's block count and the SM count (default); > 0 = fixed chunk
        self.decode_blocks_per_split: int = 0
        # forward_decode_paged replays a CUDA graph per (allocator, batch size, block
        # bucket) instead of launching ~5 kernels per layer from Python every step
        self.decode_graphs: bool = True
        # True (default): projections of at most small_batch_max_rows tokens (the decode
        # step) on the library's small-batch tensor-core kernel (as_linear_small_m, with
        # SwiGLU fused into gate/up) instead of cuBLAS; larger batches stay on cuBLAS.
        # Graphed 1B decode step on B200: 1.758 vs 1.761 ms at 64 sequences, 1.349 vs
        # 1.413 ms at 32; at 128 and 256 rows cuBLAS is faster.
        self.small_batch_linear: bool = True
        self.small_batch_max_rows: int = 64
        # True: the paged decode step does the new token's RoPE + cache write inside the
        # attention launch (as_rope_paged_decode_attention, bf16/fp16, head_dim 64/128);
        # False: separate RoPE + cache-write launch first (same results, bit for bit)
        self.fused_rope_decode: bool = True
        self.max_decode_graphs: int = 16
        self._graphs: "OrderedDict[tuple, _PagedStepGraph]" = OrderedDict()
        self._graph_pool = None

    @property
    def device(self) -> torch.device:
        return self.embed.weight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.weight.dtype

    # ------------------------------------------------------------------ weights
    @torch.no_grad()
    def fuse_projections_(self) -> None:
        """Store q/k/v and gate/up weights in one tensor each and point the Linear
        weights at views of it (state dict names unchanged), so one GEMM serves q, k, v
        and one serves gate, up."""
        if self._fused or not self.fused_projections:
            return
        for layer in self.layers:
            a, f = layer.attn, layer.ffn
            qkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous()
            nq, nk = a.q_proj.weight.shape[0], a.k_proj.weight.shape[0]
            a.q_proj.weight = nn.Parameter(qkv[:nq], requires_grad=False)
            a.k_proj.weight = nn.Parameter(qkv[nq:nq + nk], requires_grad=False)
            a.v_proj.weight = nn.Parameter(qkv[nq + nk:], requires_grad=False)
            a._qkv_w = qkv
            gu = torch.cat([f.gate_proj.weight, f.up_proj.weight], 0).contiguous()
            ni = f.gate_proj.weight.shape[0]
            f.gate_proj.weight = nn.Parameter(gu[:ni], requires_grad=False)
            f.up_proj.weight = nn.Parameter(gu[ni:], requires_grad=False)
            f._gu_w = gu
        self._fused = True

    def _linear(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        if self._small_batch(x):
            return ops.linear_small_m(x, w)
        return F.linear(x, w)

    def _qkv(self, layer: _Layer, h: torch.Tensor):
        n = h.shape[0]
        H, Kh, D = self.H, self.Kh, self.D
        a = layer.attn
        if self.fused_projections:
            qkv = self._linear(h, a._qkv_w)
            return (qkv[:, :H * D].view(n, H, D), qkv[:, H * D:(H + Kh) * D].view(n, Kh, D),
                    qkv[:, (H + Kh) * D:].view(n, Kh, D))
        return (a.q_proj(h).view(n, H, D), a.k_proj(h).view(n, Kh, D), a.v_proj(h).view(n, Kh, D))

    def _small_batch(self, x: torch.Tensor) -> bool:
        return (self.small_batch_linear and x.shape[0] <= min(self.small_batch_max_rows,
                                                              ops.LINEAR_MAX_M) and x.is_cuda
                and x.dtype in (torch.bfloat16, torch.float16))

    def _mlp(self, layer: _Layer, h: torch.Tensor) -> torch.Tensor:
        """SwiGLU on the already-normalised h (llama.py:207-211)."""
        f = layer.ffn
        if self.fused_projections:
            if self._small_batch(h) and f._gu_w.shape[0] % 128 == 0:
                # gate/up projection and SwiGLU in one launch
                return self._linear(ops.linear_small_m_swiglu(h, f._gu_w), f.down_proj.weight)
            return self._linear(ops.silu_mul(self._linear(h, f._gu_w)), f.down_proj.weight)
        return f.down_proj(F.silu(f.gate_proj(h)) * f.up_proj(h))

    def _run_layers(self, x: torch.Tensor, attention, prefill: bool = False) -> torch.Tensor:
        """The decoder stack (llama.py:218-238) with the residual adds fused into the
        next pre-norm: x is the embedding output (updated in place as the residual
        stream); attention(li, layer, h) returns the attention output fed to o_proj
        (head-major for prefill=True).  Returns the final-norm output."""
        L = len(self.layers)
        h = ops.rmsnorm(x, self.layers[0].attn_norm.weight, self.layers[0].attn_norm.eps)
        for li, layer in enumerate(self.layers):
            wo = layer.attn.o_proj.weight
            if prefill and layer.attn.o_proj_prefill is not None:
                wo = layer.attn.o_proj_prefill.weight
            a = self._linear(attention(li, layer, h), wo)
            if self.tp_size > 1:  # row-parallel o_proj: sum the ranks' partial outputs
                torch.distributed.all_reduce(a, group=self.tp_group)
            h = ops.add_rmsnorm(x, a, layer.ffn_norm.weight, layer.ffn_norm.eps)
            nxt = self.layers[li + 1].attn_norm if li + 1 < L else self.norm
            h = ops.add_rmsnorm(x, self._mlp(layer, h), nxt.weight, nxt.eps)
        return h

    def _logits(self, h: torch.Tensor) -> torch.Tensor:
        return self._linear(h, self.lm_head.weight)

    def _workspace(self, B: int, max_blocks: int, bps: int) -> torch.Tensor:
        ws = self._workspaces.get(self.device)
        if ws is None:
            ws = self._workspaces[self.device] = ops.DecodeWorkspace(self.H, self.Kh, self.D,
                                                                     self.device)
        return ws.get(B, max_blocks, bps)

    # ------------------------------------------------------------------ prefill
    @torch.inference_mode()
    def forward(self, token_ids, kv_cache=None, position_offset: int = 0):
        """Prefill T tokens after an optional cached prefix (llama.py:478-520).

        kv_cache: per-layer (k, v) [P, Kh, D] (the reference's list format) or None.
        Returns (logits [T, V], per-layer (k, v) [P+T, Kh, D]).  Each layer's K/V sit
        in a contiguous 16-token-block buffer that the prefill kernel reads as a pool
        with an identity block table; the returned tensors are views of it."""
        self.fuse_projections_()
        dev = self.device
        if not isinstance(token_ids, torch.Tensor):
            token_ids = torch.tensor(token_ids, dtype=torch.long)
        token_ids = token_ids.to(dev, non_blocking=True)
        T = int(token_ids.shape[0])
        # Attention covers the given prefix K/V plus the new tokens; position_offset only
        # drives RoPE (llama.py:506-507), exactly as in the reference, where a call with
        # kv_cache=None and an offset attends over the new tokens alone.
        P = int(kv_cache[0][0].shape[0]) if kv_cache is not None else 0
        total = P + T
        nblk = (total + BS - 1) // BS
        x = self.embed(token_ids)
        pos = torch.arange(position_offset, position_offset + T, device=dev, dtype=torch.int64)
        slots = torch.arange(P, total, device=dev, dtype=torch.int64)
        bt = torch.arange(nblk, dtype=torch.int32, device=dev).view(1, nblk)
        cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
        lk = torch.tensor([total], dtype=torch.int32, device=dev)
        new_cache = []

        def attention(li, layer, h):
            kbuf = torch.zeros(nblk, BS, self.Kh, self.D, dtype=self.dtype, device=dev)
            vbuf = torch.zeros_like(kbuf)
            kf, vf = kbuf.view(-1, self.Kh, self.D), vbuf.view(-1, self.Kh, self.D)
            if P:
                kf[:P].copy_(kv_cache[li][0])
                vf[:P].copy_(kv_cache[li][1])
            q, k, v = self._qkv(layer, h)
            ops.rope_reshape_and_cache(q, k, v, pos, slots, self.rope_table, kbuf, vbuf)
            new_cache.append((kf[:total], vf[:total]))
            return ops.varlen_prefill_attention(q, kbuf, vbuf, bt, cu, lk, T, self.scale)

        h = self._run_layers(x, attention, prefill=True)
        return self._logits(h), new_cache

    # ------------------------------------------------------------------ prefill (paged)
    @torch.inference_mode()
    def forward_prefill_paged(self, token_ids: Sequence[Sequence[int]],
                              num_cached: Sequence[int], allocator, request_ids: Sequence[str]):
        """Batched varlen prefill straight into the allocator's pool: request r's first
        num_cached[r] tokens are already in its blocks (a prefix-cache hit seeded with
        DeviceBlockAllocator.seed_blocks, engine.py:274-281) and the rest are computed
        here in one forward for all requests (the reference runs one request per forward,
        engine.py:228-229, then write_kv_prefill per layer, engine.py:311-315).  As in
        engine.py:299-302, a fully cached prompt re-feeds its last token at position
        len(prompt).  Returns the logits of each request's last token [R, V]."""
        if not isinstance(allocator, DeviceBlockAllocator):
            raise TypeError("forward_prefill_paged needs an agentserve_b200.DeviceBlockAllocator")
        self.fuse_projections_()
        R = len(token_ids)
        if R == 0:
            return torch.zeros(0, self.config.vocab_size)
        dev = self.device
        new_tok, nc, nn_ = [], [], []
        for toks, c in zip(token_ids, num_cached):
            c = int(c)
            rest = list(toks[c:])
            if not rest:  # engine.py:300-302: feed the last token again
                rest = list(toks[-1:])
            new_tok.extend(rest)
            nc.append(c)
            nn_.append(len(rest))
        total = len(new_tok)
        rows = allocator.rows_for(request_ids)
        meta = torch.tensor([nc, nn_, rows], dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        tokens = torch.tensor(new_tok, dtype=torch.long).pin_memory().to(dev, non_blocking=True)
        max_blocks = max(len(allocator._request_blocks[r]) for r in request_ids)
        pk = ops.pack_prefill(allocator.block_tables, meta[0].contiguous(), meta[1].contiguous(),
                              total, meta[2].contiguous(), max_blocks)
        max_new = max(nn_)

        def attention(li, layer, h):
            q, k, v = self._qkv(layer, h)
            kp, vp = allocator.k_plane(li), allocator.v_plane(li)
            ops.rope_reshape_and_cache(q, k, v, pk.positions, pk.slot_mapping, self.rope_table,
                                       kp, vp)
            return ops.varlen_prefill_attention(q, kp, vp, pk.block_tables, pk.cu_seqlens_q,
                                                pk.seq_lens_k, max_new, self.scale)

        h = self._run_layers(self.embed(tokens), attention, prefill=True)
        last = pk.cu_seqlens_q[1:].long() - 1
        return self._logits(h.index_select(0, last))

    @torch.inference_mode()
    def prefill_paged_greedy(self, token_ids: Sequence[Sequence[int]],
                             num_cached: Sequence[int], allocator,
                             request_ids: Sequence[str]) -> List[int]:
        """forward_prefill_paged followed by greedy sampling of each request's last
        position (engine.py:321), returning the first output tokens with one copy."""
        if len(token_ids) == 0:
            return []
        return greedy(self.forward_prefill_paged(token_ids, num_cached, allocator,
                                                 request_ids)).tolist()

    # ------------------------------------------------------------------ decode (lists)
    @torch.inference_mode()
    def forward_decode_batch(self, last_token_ids: List[int], kv_caches: list,
                             position_offsets: List[int]):
        """llama.py:265-376 with the per-request KV lists kept in one block buffer per
        layer (each sequence its own run of 16-token blocks with some free blocks after
        it), the new token written by the fused RoPE kernel and attention done by the
        paged decode kernel.

        The returned caches are views of those buffers.  When the next call passes them
        back unchanged (same requests in the same order, each cache exactly the view
        returned for it) and every sequence still has room, the histories are used in
        place and only the new token is written; otherwise (a new batch, a request
        whose run is full, caches from elsewhere) the histories are packed into new
        buffers first, each sequence getting `decode_batch_headroom` free tokens."""
        self.fuse_projections_()
        B = len(last_token_ids)
        c = self.config
        if B == 0:
            return torch.zeros(0, c.vocab_size), []
        dev = self.device
        L_layers = len(self.layers)
        lens = [int(kv_caches[b][0][0].shape[0]) for b in range(B)]
        max_len = max(lens)
        pool = self._batch_pool
        if not (pool is not None and pool["B"] == B and self._batch_pool_matches(pool, kv_caches, lens)):
            pool = self._batch_pool = self._pack_batch(kv_caches, lens)
        starts = pool["starts"]
        slots_host = [starts[b] * BS + lens[b] for b in range(B)]
        short = [b for b in range(B) if lens[b] < max_len]
        st = pool.get("static")
        if st is not None and st["bps"] != self.decode_blocks_per_split:
            st = None  # the workspace and any captured step follow the split size
            pool.pop("graph", None)
        if st is None:  # the step's inputs, staged with one copy per call
            n = 4 * B + len(short)
            host = torch.zeros(n, dtype=torch.int64).pin_memory()
            buf = torch.zeros(n, dtype=torch.int64, device=dev)
            st = pool["static"] = {
                "host": host, "np": host.numpy(), "buf": buf, "copied": torch.cuda.Event(),
                "tokens": buf[:B], "pos": buf[B:2 * B], "slots": buf[2 * B:3 * B],
                "lk": buf[3 * B:4 * B], "idx": buf[4 * B:], "n_short": len(short),
                "bps": self.decode_blocks_per_split,
                "ws": ops.new_decode_workspace(B, self.H, self.Kh, self.D, pool["mb"],
                                               self.decode_blocks_per_split, dev)}
        assert st["n_short"] == len(short)
        st["copied"].synchronize()  # the previous call's copy has left the pinned buffer
        h_np = st["np"]
        h_np[:B] = last_token_ids
        h_np[B:2 * B] = position_offsets
        h_np[2 * B:3 * B] = slots_host
        h_np[3 * B:4 * B] = [L + 1 for L in lens]
        h_np[4 * B:] = [slots_host[b] for b in short]
        st["buf"].copy_(st["host"], non_blocking=True)
        st["copied"].record()

        graphed = self.decode_graphs and dev.type == "cuda"
        if graphed and pool.get("graph") is None and pool.get("calls", 0) >= 2:
            # the first calls on these buffers ran eagerly (lazy initialisation, and a
            # batch that changes again at once is not worth a capture); capture, in a
            # memory pool of the graph's own (the graph goes when the buffers do)
            pool["mempool"] = torch.cuda.graph_pool_handle()
            s_ = torch.cuda.Stream(device=dev)
            s_.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, pool=pool["mempool"], stream=s_,
                                  capture_error_mode="relaxed"):
                pool["logits"] = self._decode_batch_body(pool)
            torch.cuda.current_stream().wait_stream(s_)
            pool["graph"] = graph
        if graphed and pool.get("graph") is not None:
            pool["graph"].replay()
            logits = pool["logits"].clone()
        else:
            logits = self._decode_batch_body(pool)
        pool["calls"] = pool.get("calls", 0) + 1

        # every sequence's [history + new token] view, one split per buffer
        sizes = []  # run b: its L_b + 1 tokens, then the rest of its blocks
        for b in range(B):
            sizes += [lens[b] + 1, pool["cap"][b] * BS - lens[b] - 1]
        views_k = [kb.view(-1, self.Kh, self.D).split(sizes)[0::2] for kb in pool["k"]]
        views_v = [vb.view(-1, self.Kh, self.D).split(sizes)[0::2] for vb in pool["v"]]
        new = [[(views_k[li][b], views_v[li][b]) for li in range(L_layers)] for b in range(B)]
        pool["lens"] = [L + 1 for L in lens]
        return logits, new

    def _decode_batch_body(self, pool) -> torch.Tensor:
        """forward_decode_batch's device work on the staged inputs of `pool` (no host
        reads: also the body of its captured graph)."""
        st = pool["static"]
        bps = self.decode_blocks_per_split
        lk = st["lk"].to(torch.int32)
        x = self.embed(st["tokens"])

        def attention(li, layer, h):
            kbuf, vbuf = pool["k"][li], pool["v"][li]
            q, k, v = self._qkv(layer, h)
            ops.rope_reshape_and_cache(q, k, v, st["pos"], st["slots"], self.rope_table, kbuf,
                                       vbuf)
            attn = ops.paged_decode_attention(q, kbuf, vbuf, pool["bt"], lk, self.scale, bps,
                                              st["ws"], out_layout=self.decode_layout)
            if self.reference_compat and st["n_short"]:
                # the reference returns a zero K/V row as the new token of every sequence
                # shorter than the batch's longest (llama.py:327, 372)
                kbuf.view(-1, self.Kh, self.D).index_fill_(0, st["idx"], 0)
                vbuf.view(-1, self.Kh, self.D).index_fill_(0, st["idx"], 0)
            return attn

        return self._logits(self._run_layers(x, attention))

    def _batch_pool_matches(self, pool, kv_caches, lens) -> bool:
        """The caches are exactly the views the last call returned (checked on every
        layer's K and V by address and length) and every sequence has room for one more
        token in its run."""
        if pool["lens"] != lens:
            return False
        kp, vp = pool["k_ptrs"], pool["v_ptrs"]
        for b, cache in enumerate(kv_caches):
            if lens[b] + 1 > pool["cap"][b] * BS:
                return False
            for li, (k, v) in enumerate(cache):
                if k.data_ptr() != kp[li][b] or v.data_ptr() != vp[li][b]:
                    return False
        return True

    def _pack_batch(self, kv_caches, lens) -> dict:
        """New per-layer block buffers holding every sequence's history (one
        multi-tensor copy per layer) with decode_batch_headroom free tokens after it."""
        dev = self.device
        B = len(lens)
        cap = [(L + 1 + self.decode_batch_headroom + BS - 1) // BS for L in lens]
        starts = [0]
        for n in cap[:-1]:
            starts.append(starts[-1] + n)
        total_blocks = starts[-1] + cap[-1]
        mb = max(cap)
        bt_host = torch.zeros(B, mb, dtype=torch.int32)
        for b in range(B):
            bt_host[b, :cap[b]] = torch.arange(starts[b], starts[b] + cap[b], dtype=torch.int32)
        kbufs, vbufs = [], []
        elt = torch.empty(0, dtype=self.dtype).element_size()
        row = self.Kh * self.D * elt
        for li in range(len(self.layers)):
            kbuf = torch.zeros(total_blocks, BS, self.Kh, self.D, dtype=self.dtype, device=dev)
            vbuf = torch.zeros_like(kbuf)
            kf, vf = kbuf.view(-1, self.Kh, self.D), vbuf.view(-1, self.Kh, self.D)
            dst = [kf[starts[b] * BS:starts[b] * BS + lens[b]] for b in range(B) if lens[b]]
            dst += [vf[starts[b] * BS:starts[b] * BS + lens[b]] for b in range(B) if lens[b]]
            src = [kv_caches[b][li][0] for b in range(B) if lens[b]]
            src += [kv_caches[b][li][1] for b in range(B) if lens[b]]
            if dst:
                torch._foreach_copy_(dst, [t.to(device=dev) for t in src])
            kbufs.append(kbuf)
            vbufs.append(vbuf)
        k_ptrs = [[kbufs[li].data_ptr() + starts[b] * BS * row for b in range(B)]
                  for li in range(len(self.layers))]
        v_ptrs = [[vbufs[li].data_ptr() + starts[b] * BS * row for b in range(B)]
                  for li in range(len(self.layers))]
        return {"B": B, "starts": starts, "cap": cap, "k": kbufs, "v": vbufs,
                "bt": bt_host.to(dev), "mb": mb, "lens": None, "k_ptrs": k_ptrs,
                "v_ptrs": v_ptrs}

    # ------------------------------------------------------------------ decode (paged)
    def _decode_core(self, tokens: torch.Tensor, seq_lens: torch.Tensor, row_ids: torch.Tensor,
                     allocator: DeviceBlockAllocator, max_blocks: int, bps: int,
                     positions: Optional[torch.Tensor] = None,
                     ws: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step entirely on the device (no host sync): pack -> per layer
        (norm, fused QKV GEMM, fused RoPE+cache write, paged attention, o_proj,
        MLP) -> norm -> lm_head.  Returns logits [B, V].  A CUDA graph passes its own
        split-K workspace `ws` (the shared one may be reallocated by later calls)."""
        B = tokens.shape[0]
        pk = ops.pack_decode(allocator.block_tables, seq_lens, row_ids, max_blocks)
        pos = pk.positions if positions is None else positions
        if ws is None:
            ws = self._workspace(B, max_blocks, bps)

        def attention(li, layer, h):
            q, k, v = self._qkv(layer, h)
            kp, vp = allocator.k_plane(li), allocator.v_plane(li)
            if self.fused_rope_decode and ops.rope_decode_fusable(q, kp):
                return ops.rope_paged_decode_attention(
                    q, k, v, pos, pk.slot_mapping, self.rope_table, kp, vp, pk.block_tables,
                    pk.seq_lens_k, self.scale, bps, ws, out_layout=self.decode_layout)
            ops.rope_reshape_and_cache(q, k, v, pos, pk.slot_mapping, self.rope_table, kp, vp)
            return ops.paged_decode_attention(q, kp, vp, pk.block_tables, pk.seq_lens_k,
                                              self.scale, bps, ws, out_layout=self.decode_layout)

        return self._logits(self._run_layers(self.embed(tokens), attention))

    @torch.inference_mode()
    def forward_decode_paged(self, last_token_ids: List[int], seq_lens: List[int],
                             position_offsets: List[int], allocator, request_ids: List[str]):
        """llama.py:379-475: K/V read in place from the allocator's device pool through
        its device block table; the new token's K/V is written by the fused RoPE kernel
        (write_kv_decode, llama.py:437-439).  Returns (logits [B, V], None)."""
        if not isinstance(allocator, DeviceBlockAllocator):
            raise TypeError("forward_decode_paged needs an agentserve_b200.DeviceBlockAllocator "
                            "(a device-resident pool and block table)")
        self.fuse_projections_()
        B = len(last_token_ids)
        if B == 0:
            return torch.zeros(0, self.config.vocab_size), None
        dev = self.device
        rows = allocator.rows_for(request_ids)
        max_blocks = max(len(allocator._request_blocks[r]) for r in request_ids)
        bps = self.decode_blocks_per_split
        if (self.decode_graphs and dev.type == "cuda" and
                (position_offsets is seq_lens or list(position_offsets) == list(seq_lens))):
            return self._graphed_decode(allocator, last_token_ids, seq_lens, rows, max_blocks,
                                        bps), None
        host = torch.tensor([list(last_token_ids), list(seq_lens), rows, list(position_offsets)],
                            dtype=torch.int64).pin_memory()
        d = host.to(dev, non_blocking=True)
        tokens = d[0]
        sl = d[1].to(torch.int32)
        rid = d[2].to(torch.int32)
        pos = None if list(position_offsets) == list(seq_lens) else d[3].contiguous()
        logits = self._decode_core(tokens, sl, rid, allocator, max_blocks, bps, positions=pos)
        return logits, None


    def _graphed_decode(self, allocator, tokens, seq_lens, rows, max_blocks: int,
                        bps: int, sample: bool = False) -> torch.Tensor:
        """forward_decode_paged through a cached CUDA graph.  Graphs are keyed by the
        allocator, the batch size and max_blocks rounded up to a power of two (capped by
        the allocator's table width); the split-K decomposition follows that bucket.
        sample=True captures greedy sampling too and returns next tokens instead of
        logits.  Least recently used graphs beyond max_decode_graphs are released."""
        g = self._step_graph(allocator, len(tokens), max_blocks, bps, sample)
        return g.run(tokens, seq_lens, rows)

    def _step_graph(self, allocator, B: int, max_blocks: int, bps: int,
                    sample: bool) -> "_PagedStepGraph":
        cap = allocator.block_tables.shape[1]
        mb = min(cap, 1 << max(0, (max_blocks - 1).bit_length()))
        key = (id(allocator), B, mb, bps, sample)
        g = self._graphs.get(key)
        if g is None or g.allocator is not allocator:
            if self._graph_pool is None:
                self._graph_pool = torch.cuda.graph_pool_handle()
            g = _PagedStepGraph(self, allocator, B, mb, bps, self._graph_pool, sample)
            self._graphs[key] = g
            while len(self._graphs) > self.max_decode_graphs:
                self._graphs.popitem(last=False)
        self._graphs.move_to_end(key)
        return g

    @torch.inference_mode()
    def decode_paged_greedy(self, last_token_ids: List[int], seq_lens: List[int], allocator,
                            request_ids: List[str]) -> List[int]:
        """One greedy decode step of the batch (forward_decode_paged with position =
        seq_len, then sampling.py:46-58's greedy branch) returning the next token ids
        with one device-to-host copy.  The step replays a CUDA graph captured for the
        batch size rounded up to a bucket (1, 2, 4, 8, then multiples of 8 up to 64 and
        of 32 above); the padding rows decode a dummy token in the allocator's scratch
        row and are dropped, so a batch that shrinks or grows by a few requests reuses
        the same graph."""
        return self.decode_paged_greedy_launch(last_token_ids, seq_lens, allocator,
                                               request_ids).result()

    @torch.inference_mode()
    def decode_paged_greedy_launch(self, last_token_ids: Optional[List[int]],
                                   seq_lens: List[int], allocator, request_ids: List[str],
                                   feed_from: Optional["DecodeHandle"] = None) -> "DecodeHandle":
        """decode_paged_greedy without waiting: the step is queued on the current stream
        and its tokens are copied to pinned host memory behind it; DecodeHandle.result()
        waits for them.  With feed_from (the handle of the previous step of the SAME
        batch, in the same order) the input tokens are that step's outputs, read on the
        device, so this step can be queued before the previous one's tokens reach the
        host; last_token_ids is then ignored."""
        if not isinstance(allocator, DeviceBlockAllocator):
            raise TypeError("decode_paged_greedy needs an agentserve_b200.DeviceBlockAllocator")
        self.fuse_projections_()
        B = len(seq_lens)
        if B == 0:
            return DecodeHandle(None, None, 0, [])
        rows = allocator.rows_for(request_ids)
        max_blocks = max(len(allocator._request_blocks[r]) for r in request_ids)
        Bp = _batch_bucket(B)
        if last_token_ids is None:
            last_token_ids = [0] * B
        if Bp > B:
            pad = allocator.scratch_row()
            last_token_ids = list(last_token_ids) + [0] * (Bp - B)
            seq_lens = list(seq_lens) + [0] * (Bp - B)
            rows = rows + [pad] * (Bp - B)
        if not (self.decode_graphs and self.device.type == "cuda"):
            host = torch.tensor([list(last_token_ids), list(seq_lens), rows], dtype=torch.int64)
            d = host.to(self.device)
            tok = d[0] if feed_from is None else feed_from.tokens.to(torch.int64)
            logits = self._decode_core(tok, d[1].to(torch.int32), d[2].to(torch.int32),
                                       allocator, max_blocks, self.decode_blocks_per_split)
            out = greedy(logits)
            return DecodeHandle(out, None, B, out[:B].tolist())
        g = self._step_graph(allocator, Bp, max_blocks, self.decode_blocks_per_split, True)
        return g.launch(last_token_ids, seq_lens, rows, B,
                        None if feed_from is None else feed_from.tokens)

    def release_decode_graphs(self) -> None:
        """Drop every cached decode graph now (e.g. before destroying a process group
        whose all-reduce the graphs captured: a live graph holding NCCL work keeps the
        group's teardown waiting)."""
        torch.cuda.synchronize()
        for g in self._graphs.values():
            g.release()
        self._graphs.clear()
        self._graph_pool = None
        if self._batch_pool is not None and self._batch_pool.get("graph") is not None:
            self._batch_pool.pop("graph").reset()  # forward_decode_batch's captured step


def _batch_bucket(B: int) -> int:
    """Decode batch sizes that share a captured graph: 1, 2, 4, 8, multiples of 8 up to
    64, multiples of 32 above."""
    if B <= 8:
        return 1 << max(0, (B - 1).bit_length())
    if B <= 64:
        return (B + 7) // 8 * 8
    return (B + 31) // 32 * 32


class _PagedStepGraph:
    """One captured forward_decode_paged step (logits only) for a fixed batch size and
    block bucket.  Inputs travel in one pinned int32 [3, B] buffer (tokens, seq_lens,
    table rows) with one host-to-device copy per call."""

    def __init__(self, model: "B200LlamaModel", allocator: DeviceBlockAllocator, B: int,
                 max_blocks: int, bps: int, pool, sample: bool = False):
        self.allocator = allocator
        self.sample = sample
        dev = model.device
        self.host = torch.zeros(3, B, dtype=torch.int32).pin_memory()
        self._host_np = self.host.numpy()
        self.inputs = torch.zeros(3, B, dtype=torch.int32, device=dev)
        self.copied = torch.cuda.Event()
        self.ws = ops.new_decode_workspace(B, model.H, model.Kh, model.D, max_blocks, bps, dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.model, self.max_blocks, self.bps = model, max_blocks, bps
        self._pool = pool
        self.logits: Optional[torch.Tensor] = None
        if sample:  # two pinned landing buffers for the tokens of consecutive launches
            self.out_host = [torch.zeros(B, dtype=torch.int64).pin_memory() for _ in range(2)]
            self.out_ready = [torch.cuda.Event(), torch.cuda.Event()]
            self._flip = 0

    def _body(self) -> torch.Tensor:
        logits = self.model._decode_core(self.inputs[0], self.inputs[1], self.inputs[2],
                                         self.allocator, self.max_blocks, self.bps, ws=self.ws)
        return greedy(logits) if self.sample else logits

    def release(self) -> None:
        if self.graph is not None:
            self.graph.reset()
            self.graph = None
        self.logits = None

    def _stage(self, tokens, seq_lens, rows) -> None:
        self.copied.synchronize()  # the previous call's copy has left the pinned buffer
        h = self._host_np
        h[0], h[1], h[2] = tokens, seq_lens, rows
        self.inputs.copy_(self.host, non_blocking=True)
        self.copied.record()

    def run(self, tokens, seq_lens, rows) -> torch.Tensor:
        """Called from forward_decode_paged (inference mode)."""
        self._stage(tokens, seq_lens, rows)
        self._replay()
        return self.logits.clone()

    def launch(self, tokens, seq_lens, rows, n: int,
               feed: Optional[torch.Tensor] = None) -> "DecodeHandle":
        """Queue one greedy step (sample=True graphs); feed: device tokens to use instead
        of `tokens` (the previous step's output of the same batch)."""
        self._stage(tokens, seq_lens, rows)
        if feed is not None:
            self.inputs[0].copy_(feed)
        self._replay()
        k = self._flip
        self._flip ^= 1
        self.out_host[k].copy_(self.logits, non_blocking=True)
        self.out_ready[k].record()
        return DecodeHandle(self.logits, self.out_ready[k], n, host=self.out_host[k])

    def _replay(self) -> None:
        if self.graph is None:
            # warm-up on a side stream (kernel attributes, cuBLAS workspaces), then
            # capture; the warm-up writes the same pool slots the replay rewrites
            s = torch.cuda.Stream(device=self.inputs.device)
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._body()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            self.graph = torch.cuda.CUDAGraph()
            # relaxed: a library kernel first used inside the capture (lazy module
            # loading, e.g. a cuBLAS algorithm the warm-up did not pick) must not
            # invalidate it
            with torch.cuda.graph(self.graph, pool=self._pool, stream=s,
                                  capture_error_mode="relaxed"):
                self.logits = self._body()
        self.graph.replay()


class DecodeHandle:
    """The greedy tokens of one queued decode step.  `tokens` is the step's device
    output (valid until the same graph is replayed again, which the stream orders after
    any reader queued before it); result() waits for the host copy."""

    def __init__(self, tokens: Optional[torch.Tensor], event, n: int,
                 values: Optional[List[int]] = None, host: Optional[torch.Tensor] = None):
        self.tokens, self.event, self.n = tokens, event, n
        self._values, self._host = values, host

    def result(self) -> List[int]:
        if self._values is None:
            self.event.synchronize()
            self._values = self._host[:self.n].tolist()
        return self._values


def greedy(logits: torch.Tensor) -> torch.Tensor:
    """sampling.py:46-58 with temperature <= 1e-6 (fp32, nan_to_num(0, 1e4, -1e4),
    first argmax) for [B, V] logits, in one kernel (as_greedy_argmax)."""
    return ops.greedy_argmax(logits)


class DecodeGraph:
    """One greedy decode step for a fixed batch, captured in a CUDA graph.

    Static device inputs: tokens [B] int64, seq_lens [B] int32 (cached tokens = position
    of the new token), row_ids [B] int32 (allocator table rows).  Output: next_tokens
    [B] int64.  With advance=True the graph also feeds next_tokens back into tokens and
    increments seq_lens, so replays run consecutive decode steps with no host work.
    """

    def __init__(self, model: B200LlamaModel, allocator: DeviceBlockAllocator, batch_size: int,
                 max_blocks: int, blocks_per_split: int, advance: bool = False):
        self.model = model
        self.allocator = allocator
        self.B = batch_size
        self.max_blocks = max_blocks
        self.bps = blocks_per_split
        self.advance = advance
        dev = model.device
        self.tokens = torch.zeros(batch_size, dtype=torch.int64, device=dev)
        self.seq_lens = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.row_ids = torch.zeros(batch_size, dtype=torch.int32, device=dev)
        self.next_tokens = torch.zeros(batch_size, dtype=torch.int64, device=dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None

    def _body(self):
        m = self.model
        logits = m._decode_core(self.tokens, self.seq_lens, self.row_ids, self.allocator,
                                self.max_blocks, self.bps)
        self.next_tokens.copy_(greedy(logits))
        if self.advance:
            self.tokens.copy_(self.next_tokens)
            self.seq_lens.add_(1)

    @torch.inference_mode()
    def capture(self, tokens, seq_lens, row_ids) -> None:
        """Warm up on a side stream (sets kernel attributes, cuBLAS handles) then
        capture.  The warm-up writes one token per sequence into the pool at
        seq_lens; the caller's next step overwrites the same slots."""
        self.model.fuse_projections_()
        self.load(tokens, seq_lens, row_ids)
        s = torch.cuda.Stream(device=self.model.device)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            saved = (self.tokens.clone(), self.seq_lens.clone())
            self._body()
            self.tokens.copy_(saved[0])
            self.seq_lens.copy_(saved[1])
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s, capture_error_mode="relaxed"):
            self._body()
        torch.cuda.synchronize()

    def load(self, tokens, seq_lens, row_ids) -> None:
        self.tokens.copy_(torch.as_tensor(tokens, dtype=torch.int64), non_blocking=True)
        self.seq_lens.copy_(torch.as_tensor(seq_lens, dtype=torch.int32), non_blocking=True)
        self.row_ids.copy_(torch.as_tensor(row_ids, dtype=torch.int32), non_blocking=True)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.next_tokens

    def release(self) -> None:
        """Free the captured graph now (before destroying a process group whose
        all-reduce it captured)."""
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None
