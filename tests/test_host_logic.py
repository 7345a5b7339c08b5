"""Host-side logic of the boundary, CPU only: the device allocator's bookkeeping keeps
the reference BlockAllocator semantics (agentserve/engine/cache.py:33-119, pinned by
the reference's tests/test_cache.py), its block-table rows mirror the host lists, and
the split-K helpers behave."""

import pytest
import torch

from agentserve_b200 import ops
from agentserve_b200.cache import DeviceBlockAllocator
from oracle import paged


@pytest.fixture
def alloc():
    return DeviceBlockAllocator(num_blocks=32, block_size=16, allocate_tensor=False,
                                device="cpu", max_seqs=64)


def test_allocation_counts(alloc):
    assert alloc.num_free_blocks() == 32 and alloc.num_used_blocks() == 0
    ids = alloc.allocate("r1", 4)
    assert len(ids) == 4 and alloc.num_free_blocks() == 28
    ids2 = alloc.allocate("r2", 4)
    assert set(ids).isdisjoint(ids2)
    alloc.free("r1")
    alloc.free("nonexistent")
    assert alloc.num_free_blocks() == 28
    assert alloc.memory_usage() == pytest.approx(4 / 32)


def test_exhaustion_and_recovery(alloc):
    with pytest.raises(MemoryError):
        alloc.allocate("r", 33)
    assert len(alloc.allocate("r", 32)) == 32
    alloc.free("r")
    assert len(alloc.allocate("r2", 32)) == 32


def test_churn_and_interleaving(alloc):
    for i in range(20):
        alloc.allocate(f"q{i}", 2)
        alloc.free(f"q{i}")
    assert alloc.num_free_blocks() == 32
    for i in range(16):
        alloc.allocate(f"x{i}", 1)
    for i in range(8):
        alloc.free(f"x{i}")
    assert alloc.num_free_blocks() == 24
    alloc.allocate("new", 8)
    assert alloc.num_free_blocks() == 16


def test_blocks_needed_and_blocks_for(alloc):
    assert [alloc.blocks_needed(n) for n in (0, 1, 16, 17, 31, 32)] == [0, 1, 1, 2, 2, 2]
    ids = alloc.allocate("a", 3)
    assert alloc.blocks_for("a") == ids
    alloc.free("a")
    assert alloc.blocks_for("a") == []


def test_same_free_order_as_reference_allocator():
    """The FIFO free list hands out the same ids as the reference for the same calls."""
    ours = DeviceBlockAllocator(32, allocate_tensor=False, device="cpu")
    ref = paged.OracleBlockAllocator(32)
    script = [("a", "A", 3), ("a", "B", 2), ("f", "A", 0), ("a", "C", 4), ("a", "B", 1),
              ("f", "B", 0), ("a", "D", 7)]
    for op, rid, n in script:
        if op == "a":
            assert ours.allocate(rid, n) == ref.allocate(rid, n)
        else:
            ours.free(rid)
            ref.free(rid)
    assert list(ours._free) == list(ref._free)


def test_device_table_rows_mirror_host_lists(alloc):
    alloc.allocate("a", 3)
    alloc.allocate("b", 2)
    alloc.allocate("a", 2)  # a request can grow
    ra, rb = alloc.row_of("a"), alloc.row_of("b")
    assert ra != rb
    assert alloc.block_tables[ra, :5].tolist() == alloc.blocks_for("a")
    assert alloc.block_tables[rb, :2].tolist() == alloc.blocks_for("b")
    alloc.free("a")
    alloc.allocate("c", 1)
    assert alloc.row_of("c") != rb  # rows are recycled without clobbering live ones
    assert alloc.block_tables[rb, :2].tolist() == alloc.blocks_for("b")


def test_row_capacity_limits():
    a = DeviceBlockAllocator(64, allocate_tensor=False, device="cpu", max_seqs=2,
                             max_blocks_per_seq=4)
    a.allocate("x", 4)
    with pytest.raises(MemoryError):
        a.allocate("x", 1)
    a.allocate("y", 1)
    with pytest.raises(MemoryError):
        a.allocate("z", 1)


def test_block_size_must_be_16():
    with pytest.raises(ValueError):
        DeviceBlockAllocator(8, block_size=4, allocate_tensor=False, device="cpu")


def test_decode_workspace_zeroes_counters_only_when_they_grow():
    ws = ops.DecodeWorkspace(32, 8, 64, "cpu")
    b = ws.get(8, 64, 16)
    b[1024:].fill_(7)  # partials of a B=8 call sit right after its 1 KB of counters
    b2 = ws.get(64, 64, 16)  # counters now cover 8 KB: must be zeroed again
    assert b2.data_ptr() == b.data_ptr() or b2.numel() > b.numel()
    assert int(b2[:64 * 32 * 4].sum()) == 0
    b2[64 * 32 * 4:].fill_(3)
    b3 = ws.get(8, 64, 16)  # smaller counter region: already zero, no memset needed
    assert int(b3[:8 * 32 * 4].sum()) == 0


def test_zero_copy_prefix_sharing_ref_counts(alloc):
    """A prefix-cache entry retains a finished request's full prefix blocks; a later
    request shares them (ref counts, no copy) and allocates the rest; blocks go back to
    the free list only when the last holder lets go."""
    a = alloc.allocate("A", 5)
    prefix = a[:3]
    alloc.retain_blocks(prefix)           # cache entry
    alloc.free("A")
    assert alloc.num_used_blocks() == 3 and all(alloc.ref_count(b) == 1 for b in prefix)
    alloc.share_blocks("B", prefix)
    own = alloc.allocate("B", 2)
    assert alloc.blocks_for("B") == prefix + own
    assert alloc.block_tables[alloc.row_of("B"), :5].tolist() == prefix + own
    assert all(alloc.ref_count(b) == 2 for b in prefix)
    alloc.share_blocks("C", prefix[:2])
    alloc.free("B")
    assert all(alloc.ref_count(b) == (2 if b in prefix[:2] else 1) for b in prefix)
    alloc.release_blocks(prefix)          # cache entry evicted
    assert alloc.ref_count(prefix[2]) == 0 and prefix[2] in alloc._free
    alloc.free("C")
    assert alloc.num_used_blocks() == 0 and alloc.num_free_blocks() == 32
    with pytest.raises(ValueError):
        alloc.share_blocks("D", [prefix[0]])  # no longer allocated
    alloc.allocate("E", 1)
    with pytest.raises(ValueError):
        alloc.share_blocks("E", alloc.blocks_for("E"))  # must share before allocating


def test_decode_batch_buffers_layout_and_reuse_rules():
    """forward_decode_batch's host bookkeeping (no kernel runs): each sequence's
    history is copied into its own run of blocks with the headroom after it, the
    returned-view addresses are recorded per layer, and a later call may reuse the
    buffers only with exactly those views, the same lengths and room left."""
    from agentserve_b200 import B200LlamaModel
    from agentserve_b200.config import ModelConfig
    cfg = ModelConfig(hidden_dim=64, n_heads=4, n_kv_heads=2, n_layers=2, vocab_size=100,
                      max_seq_len=512, intermediate_size=128)
    m = B200LlamaModel(cfg, dtype=torch.float32, device="cpu")
    m.decode_batch_headroom = 20
    lens = [0, 5, 16, 40]
    g = torch.Generator().manual_seed(0)
    caches = [[(torch.randn(L, 2, 16, generator=g), torch.randn(L, 2, 16, generator=g))
               for _ in range(2)] for L in lens]
    pool = m._pack_batch(caches, lens)
    assert pool["cap"] == [(L + 1 + 20 + 15) // 16 for L in lens]
    assert pool["starts"] == [0, 2, 4, 7]
    row = 2 * 16 * 4  # Kh * D * 4 bytes
    for li in range(2):
        kf = pool["k"][li].view(-1, 2, 16)
        for b, L in enumerate(lens):
            s0 = pool["starts"][b] * 16
            assert torch.equal(kf[s0:s0 + L], caches[b][li][0])
            assert pool["k_ptrs"][li][b] == pool["k"][li].data_ptr() + s0 * row
            assert int(pool["bt"][b, 0]) == pool["starts"][b]
    # the views the call would return (history + new token) match; anything else not
    pool["lens"] = [L + 1 for L in lens]
    views = [[(pool["k"][li].view(-1, 2, 16)[pool["starts"][b] * 16:][:L + 1],
               pool["v"][li].view(-1, 2, 16)[pool["starts"][b] * 16:][:L + 1])
              for li in range(2)] for b, L in enumerate(lens)]
    assert m._batch_pool_matches(pool, views, pool["lens"])
    assert not m._batch_pool_matches(pool, views, lens)                      # other lengths
    assert not m._batch_pool_matches(pool, views[::-1], pool["lens"][::-1])  # other order
    moved = [list(c) for c in views]
    moved[2][1] = (moved[2][1][0].clone(), moved[2][1][1])                   # one copied view
    assert not m._batch_pool_matches(pool, moved, pool["lens"])
    full = dict(pool, lens=[pool["cap"][0] * 16] + pool["lens"][1:])        # a full run
    assert not m._batch_pool_matches(full, views, full["lens"])
