"""Pin the oracle (CPU restatement) to golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""

import hashlib

import numpy as np
import torch

from oracle import attention, paged, rope
from oracle.model import OracleLlama
from oracle.weights import init_weights_
from tests.golden import scenarios as S


def sha(t):
    return hashlib.sha256(t.detach().contiguous().cpu().numpy().tobytes()).hexdigest()


class Cfg:
    def __init__(self, **kw):
        self.__dict__.update(kw)
        self.head_dim = self.hidden_dim // self.n_heads


def test_rope_table_bit_exact(golden):
    t = rope.precompute_rope_freqs(64, 2048, 500000.0)
    assert sha(t) == str(golden["rope_table_sha"])
    assert sha(rope.precompute_rope_freqs(16, 512, 10000.0)) == str(golden["rope_tiny_sha"])


def test_apply_rope_bit_exact(golden):
    pos, x32, xbf = S.rope_inputs()
    cs = rope.precompute_rope_freqs(64, 2048, 500000.0)[pos]
    np.testing.assert_array_equal(rope.apply_rope(x32, cs).numpy(), golden["rope_out_f32"])
    np.testing.assert_array_equal(rope.apply_rope(xbf, cs).view(torch.int16).numpy(),
                                  golden["rope_out_bf16"])


def test_allocator_and_slots_bit_exact(golden):
    a = paged.OracleBlockAllocator(32, 16, num_layers=2, num_kv_heads=2, head_dim=16,
                                   allocate_tensor=True)
    a.allocate("A", 3)
    a.allocate("B", 2)
    a.free("A")
    a.allocate("C", 4)
    a.allocate("B", 1)
    kC, vC, kd, vd = S.cache_inputs()
    for layer in range(2):
        a.write_kv_prefill("C", layer, kC[layer], vC[layer])
        a.write_kv_decode("C", 37, layer, kd[layer], vd[layer])
    np.testing.assert_array_equal(np.array(a.blocks_for("B")), golden["cache_bt_B"])
    np.testing.assert_array_equal(np.array(a.blocks_for("C")), golden["cache_bt_C"])
    np.testing.assert_array_equal(np.array(list(a._free)), golden["cache_free_after"])
    np.testing.assert_array_equal(a.kv_pool.numpy(), golden["cache_pool"])
    k, v = a.gather_kv("C", 38, 1)
    np.testing.assert_array_equal(k.numpy(), golden["cache_gather_k"])
    np.testing.assert_array_equal(v.numpy(), golden["cache_gather_v"])
    np.testing.assert_array_equal(
        np.array([a.blocks_needed(n) for n in (0, 1, 15, 16, 17, 33)]),
        golden["cache_blocks_needed"])


def test_pack_decode_matches_allocator_slots(golden):
    bt_C = golden["cache_bt_C"].tolist()
    pos, slots, lk, cu = paged.pack_decode([bt_C, bt_C], [37, 16])
    assert pos.tolist() == [37, 16]
    assert slots.tolist() == [bt_C[2] * 16 + 5, bt_C[1] * 16]
    assert lk.tolist() == [38, 17] and cu.tolist() == [0, 1, 2]


def test_decode_attention_config1(golden):
    inp = S.decode_cfg1_inputs()
    assert sha(torch.cat([inp["q"].flatten(), inp["kpool"].flatten(), inp["vpool"].flatten(),
                          inp["kn"].flatten(), inp["vn"].flatten()])) == str(golden["cfg1_input_sha"])
    kp, vp = inp["kpool"].clone(), inp["vpool"].clone()
    for b, L in enumerate(inp["lens"]):
        paged.write_kv(kp, vp, inp["tables"][b], L, inp["kn"][b:b + 1], inp["vn"][b:b + 1])
    lk = [L + 1 for L in inp["lens"]]
    out = attention.decode_attention_from_pool(inp["q"], kp, vp, inp["tables"], lk)
    ref = torch.from_numpy(golden["cfg1_out"])
    torch.testing.assert_close(out, ref, rtol=0, atol=1e-6)
    assert sha(torch.stack([kp, vp])[:, None]) == str(golden["cfg1_pool_after_sha"])


def _model(tag):
    cfg = Cfg(**S.MODEL_CONFIGS[tag])
    m = OracleLlama(cfg)
    init_weights_(m, seed=0)
    return cfg, m.eval()


def test_oracle_model_matches_reference(golden):
    for tag in S.MODEL_CONFIGS:
        cfg, m = _model(tag)
        sc = S.model_scenario(tag, cfg)
        lg, kv = m.forward(sc["prompt"])
        np.testing.assert_allclose(lg.numpy(), golden[f"{tag}_prefill_logits"], rtol=0, atol=1e-5)
        pre = [(k[:32].clone(), v[:32].clone()) for k, v in kv]
        lg2, _ = m.forward(sc["prompt"][32:], kv_cache=pre, position_offset=32)
        np.testing.assert_allclose(lg2.numpy(), golden[f"{tag}_prefix_logits"], rtol=0, atol=1e-5)
        # padded-list decode
        caches, last, pos = [], [], []
        for p in sc["batch_prompts"]:
            l0, kvp = m.forward(p)
            caches.append(kvp)
            last.append(int(l0[-1].argmax()))
            pos.append(len(p))
        for step in range(S.DECODE_STEPS):
            lg, caches = m.forward_decode_batch(last, caches, pos)
            np.testing.assert_allclose(lg.numpy(), golden[f"{tag}_batch_logits"][step],
                                       rtol=0, atol=1e-5)
            last = [int(t) for t in lg.argmax(-1)]
            assert last == golden[f"{tag}_batch_tokens"][step].tolist()
            pos = [x + 1 for x in pos]
        # paged decode with the oracle allocator
        a = paged.OracleBlockAllocator(64, 16, cfg.n_layers, cfg.n_kv_heads, cfg.head_dim,
                                       allocate_tensor=True)
        rids, last, lens = [], [], []
        for i, p in enumerate(sc["batch_prompts"]):
            rid = f"r{i}"
            a.allocate(rid, a.blocks_needed(len(p) + S.DECODE_STEPS + 1))
            l0, kvp = m.forward(p)
            for li, (k, v) in enumerate(kvp):
                a.write_kv_prefill(rid, li, k, v)
            rids.append(rid)
            last.append(int(l0[-1].argmax()))
            lens.append(len(p))
        for step in range(S.DECODE_STEPS):
            lg, _ = m.forward_decode_paged(last, lens, lens, a, rids)
            np.testing.assert_allclose(lg.numpy(), golden[f"{tag}_paged_logits"][step],
                                       rtol=0, atol=1e-5)
            last = [int(t) for t in lg.argmax(-1)]
            assert last == golden[f"{tag}_paged_tokens"][step].tolist()
            lens = [x + 1 for x in lens]


def test_oracle_greedy_matches_reference_sampler(golden):
    """The oracle's greedy branch equals the reference's sample(temperature=0) on
    logits with NaN, +-inf, ties and values above the +inf replacement."""
    from oracle.model import greedy
    x32, xbf = S.greedy_logits()
    assert greedy(x32).numpy().tolist() == golden["greedy_tokens_f32"].tolist()
    assert greedy(xbf).numpy().tolist() == golden["greedy_tokens_bf16"].tolist()
