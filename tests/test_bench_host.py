"""Host-side helpers of bench.py (no GPU): the per-step launch count it reports and the
pinning of each rank to its share of the host cores close to its GPU."""

import types

import pytest

import bench


def _model(small=True, max_rows=64, fused_rope=True):
    return types.SimpleNamespace(small_batch_linear=small, small_batch_max_rows=max_rows,
                                 fused_rope_decode=fused_rope)


def test_launches_per_step_counts_the_library_kernels_of_a_step():
    cfg = types.SimpleNamespace(n_layers=16)
    # pack + first RMSNorm + greedy + lm_head, and per layer: attention (RoPE fused),
    # 2 x add+RMSNorm, QKV, o_proj, gate/up+SwiGLU, down
    assert bench.launches_per_step(_model(), cfg, 64) == 4 + 7 * 16
    # batches above the small-batch limit keep cuBLAS projections (SwiGLU is ours)
    assert bench.launches_per_step(_model(), cfg, 128) == 3 + 4 * 16
    assert bench.launches_per_step(_model(small=False), cfg, 64) == 3 + 4 * 16
    # the separate RoPE + cache-write launch
    assert bench.launches_per_step(_model(fused_rope=False), cfg, 64) == 4 + 8 * 16


class _FakeAffinity:
    """os.sched_getaffinity / sched_setaffinity and torch.set_num_threads, recorded."""

    def __init__(self, allowed):
        self.allowed = set(allowed)
        self.set_to = None
        self.threads = None

    def install(self, monkeypatch, local_cores):
        monkeypatch.setattr(bench.os, "sched_getaffinity", lambda pid: set(self.allowed))
        monkeypatch.setattr(bench.os, "sched_setaffinity",
                            lambda pid, cores: setattr(self, "set_to", sorted(cores)))
        monkeypatch.setattr(bench.torch, "set_num_threads",
                            lambda n: setattr(self, "threads", n))
        monkeypatch.setattr(bench, "_gpu_local_cores", lambda i: set(local_cores[i]))
        fake_nvml = types.SimpleNamespace(nvmlInit=lambda: None)
        monkeypatch.setitem(__import__("sys").modules, "pynvml", fake_nvml)


def test_pinning_splits_the_cores_close_to_the_gpus_evenly(monkeypatch):
    # GPUs 0-1 close to cores 0-23, GPUs 2-3 close to 24-47; 48 cores allowed
    local = {0: range(24), 1: range(24), 2: range(24, 48), 3: range(24, 48)}
    for rank, want in ((0, list(range(12))), (1, list(range(12, 24))),
                       (2, list(range(24, 36))), (3, list(range(36, 48)))):
        fa = _FakeAffinity(range(48))
        fa.install(monkeypatch, local)
        bench.pin_rank_cores(rank, 4)
        assert fa.set_to == want and fa.threads == 12


def test_pinning_when_the_container_allows_only_some_close_cores(monkeypatch):
    # only cores 0-15 are allowed: GPUs 2-3 have no close core left, so all four
    # ranks share the allowed set
    local = {0: range(24), 1: range(24), 2: range(24, 48), 3: range(24, 48)}
    got = []
    for rank in range(4):
        fa = _FakeAffinity(range(16))
        fa.install(monkeypatch, local)
        bench.pin_rank_cores(rank, 4)
        got.append(fa.set_to)
    assert got == [list(range(4 * r, 4 * r + 4)) for r in range(4)]


@pytest.mark.parametrize("local_world", [1])
def test_no_pinning_for_a_single_rank(monkeypatch, local_world):
    fa = _FakeAffinity(range(8))
    fa.install(monkeypatch, {0: range(8)})
    bench.pin_rank_cores(0, local_world)
    assert fa.set_to is None


def test_no_pinning_when_a_share_would_be_a_single_core(monkeypatch):
    fa = _FakeAffinity(range(2))
    fa.install(monkeypatch, {i: range(2) for i in range(2)})
    bench.pin_rank_cores(1, 2)
    assert fa.set_to is None
