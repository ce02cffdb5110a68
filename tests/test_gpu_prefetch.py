"""Prefetch session on the GPU: the side-stream copies land the right bytes in
the right slots and publish the slot tables; evictions unpublish; a layer
computed through the session's slot table (resident slots from HBM, the rest
read from the pinned host store) equals the all-resident layer bit for bit."""
import pytest
import torch

pytestmark = pytest.mark.gpu

KEYS = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")


@pytest.fixture(scope="module")
def small_layers(cuda_device):
    from mtp_b200 import W4A16Experts
    from mtp_b200.synthetic import LayerConfig, make_layer
    cfg = LayerConfig(num_experts=16, hidden=256, inter=128, top_k=4, shared=False)
    layers = []
    for l in range(2):
        ex, _ = make_layer(cfg, seed=40 + l, device=cuda_device)
        layers.append(W4A16Experts.from_gptq(*(ex[k] for k in KEYS)))
    host = torch.empty((2, 16, layers[0].expert_bytes), dtype=torch.uint8).pin_memory()
    for l in range(2):
        host[l].copy_(layers[l].blobs.reshape(16, -1).cpu())
    return cfg, layers, host


def _slot_bytes(sess, l, slot):
    eb = sess.expert_bytes
    s0 = (l * sess.slots + slot) * eb
    return sess.cache[s0:s0 + eb].cpu()


def test_issue_copies_and_publishes(cuda_device, small_layers):
    from mtp_b200 import PrefetchSession
    cfg, layers, host = small_layers
    sess = PrefetchSession(2, 16, 4, layers[0].expert_bytes, host, device=cuda_device)
    assert (sess.slot_tables.cpu() == -1).all()
    assert sess.issue(1, [3, 5, 9]) == 3
    assert sess.issue(1, [3]) == 0              # resident or in flight: not issued again
    sess.sync()
    table = sess.slot_tables.cpu()
    assert (table[0] == -1).all()
    for e in (3, 5, 9):
        slot = int(table[1, e])
        assert 0 <= slot < 4
        assert torch.equal(_slot_bytes(sess, 1, slot), host[1, e])
    st = sess.poll()
    assert st["issued_fetch_count"] == 3 and st["resident_count"] == 3 and st["inflight_count"] == 0
    # demand: 3 hits, 7 misses and is inserted (4th slot); then a new issue evicts the LRU (5)
    assert sess.demand(1, [3, 7]) == 1
    sess.demand(1, [9])
    assert sess.issue(1, [11]) == 1
    sess.sync()
    table = sess.slot_tables.cpu()
    assert int(table[1, 5]) == -1
    for e in (3, 7, 9, 11):
        assert torch.equal(_slot_bytes(sess, 1, int(table[1, e])), host[1, e])
    st = sess.poll()
    assert st["demand_count"] == 3 and st["demand_hit_count"] == 2 and st["demand_miss_count"] == 1
    assert st["evicted_before_use_count"] == 1 and st["used_fetch_count"] == 2
    sess.close()


def test_layer_through_session_equals_all_resident(cuda_device, small_layers):
    import mtp_b200
    from mtp_b200 import PrefetchSession
    from mtp_b200.synthetic import make_inputs
    cfg, layers, host = small_layers
    sess = PrefetchSession(2, 16, 4, layers[0].expert_bytes, host, device=cuda_device)
    x, logits = make_inputs(cfg, 6, seed=77, device=cuda_device)
    ref = mtp_b200.moe_layer_w4a16(x, logits, layers[0], cfg.top_k)
    sess.issue(0, [0, 2, 4, 6])
    sess.sync()
    cache, table, hoststore = sess.layer_views(0)
    status = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    out = mtp_b200.moe_layer_w4a16(x, logits, layers[0], cfg.top_k, slot_table=table, slot_cache=cache,
                                   host_store=hoststore, status=status)
    sess.layer_used(0)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert int(status[1]) == 0            # no expert without a source
    resident = {0, 2, 4, 6}
    demanded = set(torch.topk(logits, cfg.top_k, dim=1).indices.flatten().tolist())
    assert int(status[0]) == len(demanded - resident)   # served from the host store
    sess.close()
