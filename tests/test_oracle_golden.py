"""The CPU oracle against the golden fixtures made by the reference's own code
(tests/golden/make_golden.py). CPU only."""
import numpy as np
import torch

from conftest import golden
from oracle import align, cache, gptq, layer, router


def test_pack_unpack_round_trip_4bit():
    # tests/test_gptq_unpack.py:41-46 of the reference
    rows = (np.arange(16 * 8).reshape(16, 8) % 16).astype(np.int32)
    cols = (np.arange(2 * 16).reshape(2, 16) % 16).astype(np.int32)
    assert np.array_equal(gptq.unpack_rows(gptq.pack_rows(rows)), rows)
    assert np.array_equal(gptq.unpack_cols(gptq.pack_cols(cols)), cols)


def test_dequant_matches_reference_bit_exact():
    g = golden("gptq_dequant.pt")
    for case in ("small", "seeded"):
        c = g[case]
        w = gptq.dequantize(c["qweight"].numpy(), c["qzeros"].numpy(), c["scales"].numpy(), c["g_idx"].numpy())
        assert w.dtype == np.float32
        assert np.array_equal(w, c["expected"].numpy()), case
    s = g["seeded"]
    assert np.array_equal(gptq.unpack_rows(s["qweight"].numpy()), s["unpacked_rows"].numpy())
    assert np.array_equal(gptq.unpack_cols(s["qzeros"].numpy()), s["unpacked_cols"].numpy())


def test_router_matches_reference_fallback():
    for c in golden("router.pt"):
        lg = c["logits"].numpy()
        assert not router.has_exact_ties(lg)
        w, ids, tei = router.topk_softmax(lg, c["k"], c["renormalize"])
        assert np.array_equal(ids, c["topk_ids"].numpy())
        np.testing.assert_allclose(w, c["topk_weights"].numpy(), rtol=2e-6, atol=1e-8)
        assert np.array_equal(tei, c["tei"].numpy())


def test_router_mtp_form_matches_reference():
    for name in ("moe_small.pt", "config0.pt"):
        g = golden(name)
        if "logits" in g:
            w, ids = router.router_topk_mtp_form(g["logits"].numpy(), g["topk_ids"].shape[1])
            assert np.array_equal(ids, g["topk_ids"].numpy())
            np.testing.assert_allclose(w, g["topk_weights"].numpy(), rtol=2e-6)


def test_moe_small_layer_matches_reference():
    g = golden("moe_small.pt")
    o = layer.MoeLayerOracle(g["experts"], g["shared"], group_size=g["group_size"])
    out = o.moe_tokens(g["x"].float(), g["topk_ids"], g["topk_weights"])
    torch.testing.assert_close(out, g["expected"], rtol=1e-5, atol=1e-4)


def _sha(t: torch.Tensor) -> str:
    import hashlib
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def test_config0_generator_pinned_and_layer_matches_reference():
    from mtp_b200.synthetic import CONFIG0, make_inputs, make_layer
    g = golden("config0.pt")
    experts, _ = make_layer(CONFIG0, seed=g["seed_layer"])
    x, logits = make_inputs(CONFIG0, 4, seed=g["seed_inputs"])
    for k, v in experts.items():
        assert _sha(v) == g["hashes"][k], k
    assert _sha(x) == g["hashes"]["x"] and _sha(logits) == g["hashes"]["logits"]
    w, ids = router.router_topk_mtp_form(logits.numpy(), CONFIG0.top_k)
    assert np.array_equal(ids, g["topk_ids"].numpy())
    o = layer.MoeLayerOracle(experts, None, group_size=CONFIG0.group_size)
    out = o.moe_tokens(x.float(), g["topk_ids"], g["topk_weights"])
    torch.testing.assert_close(out, g["expected"], rtol=1e-5, atol=2e-4)


def test_cache_managers_match_reference():
    for c in golden("cache.pt"):
        lru = cache.LruExpertCache(12)
        rt = cache.ReadyTimeExpertCache(**c["ready_params"])
        r1, r2 = [], []
        for kind, l, e, t in c["ops"]:
            if kind == "issue":
                r1.append(lru.issue_prefetch(l, e))
                r2.append(rt.issue_prefetch(l, e, arrival_us=t))
            else:
                r1.append(lru.demand(l, e))
                r2.append(rt.demand(l, e, arrival_us=t))
        rt.finish()
        assert r1 == c["lru_results"]
        assert r2 == c["ready_results"]
        assert lru.snapshot().as_dict() == c["lru_snapshot"]
        snap = rt.snapshot_ready()
        ref = c["ready_snapshot"]
        for key in ("capacity", "resident_count", "issued_fetch_count", "used_fetch_count",
                    "unused_fetch_count", "demand_count", "demand_hit_count", "demand_miss_count",
                    "evicted_before_use_count", "ready_late_miss_count", "late_completion_unused_count",
                    "queue_batch_count"):
            assert snap[key] == ref[key], key


def test_align_docstring_example():
    # vLLM moe_align_block_size docstring: ids 1..4, block 4 -> per-expert runs of
    # ascending flat indices padded with the sentinel 12.
    ids = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=np.int32)
    s, e, n, seg = align.moe_align_block_size(ids, 4, 5)
    assert n[0] == 16
    assert s[:16].tolist() == [3, 6, 9, 12, 0, 4, 10, 12, 1, 7, 11, 12, 2, 5, 8, 12]
    assert e[:4].tolist() == [1, 2, 3, 4]
    assert seg.tolist() == [[1, 0, 1], [2, 1, 1], [3, 2, 1], [4, 3, 1]]
