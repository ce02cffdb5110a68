"""Prefetch admission tiers (mtp_b200.admission) against the reference's own
build_priority_masks / build_premap_descriptors outputs
(tests/golden/premap.pt, made by tests/golden/make_golden.py), plus the budget
and the issue order on a simulated prefetch session. CPU only."""
import torch

from conftest import golden
from mtp_b200 import admission as adm


def test_priority_masks_match_reference():
    g = golden("premap.pt")
    masks = adm.priority_masks(g["transition"], g["mtp"])
    assert list(masks) == list(g["masks"])
    for name, m in masks.items():
        assert torch.equal(m, g["masks"][name]), name


def test_descriptors_match_reference_for_max_and_mean():
    g = golden("premap.pt")
    for red in ("max", "mean"):
        got = adm.premap_descriptors(g["transition"], g["mtp"], g["samples"], reduce=red)
        want = g[f"descriptors_{red}"]
        assert len(got) == len(want)
        for d, w in zip(got, want):
            assert (d.sample, d.layer, d.expert, d.priority, d.source) == tuple(w[:5])
            assert abs(d.score - w[5]) <= 1e-6 * max(1.0, abs(w[5]))


def test_budget_keeps_priority_order_and_issue_groups_by_layer():
    import mtp_b200
    g = golden("premap.pt")
    d = adm.premap_descriptors(g["transition"], g["mtp"], g["samples"])
    kept = adm.apply_budget(d, per_layer=5, max_priority=4)
    per = {}
    for x in kept:
        assert x.priority <= 4
        per[(x.sample, x.layer)] = per.get((x.sample, x.layer), 0) + 1
    assert max(per.values()) <= 5
    # within a (sample, layer) the budget takes the best first
    firsts = [x for x in d if x.priority <= 4]
    for key in per:
        assert [x for x in kept if (x.sample, x.layer) == key] == [x for x in firsts if (x.sample, x.layer) == key][:5]
    sess = mtp_b200.PrefetchSession(3, 64, 8, 1024, simulate=True)
    issued = adm.issue_descriptors(sess, [x for x in kept if x.sample == 0])
    st = sess.poll()
    assert issued == st["issued_fetch_count"] > 0
    sess.close()
