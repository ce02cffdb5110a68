"""Router, align, dequant and repack kernels against the CPU oracle (bit-exact
for ids, tables and dequantised values; fp32 router weights within 2e-6)."""
import numpy as np
import pytest
import torch

from conftest import golden
from oracle import align as oalign
from oracle import gptq as ogptq
from oracle import layout as olayout
from oracle import router as orouter

pytestmark = pytest.mark.gpu


def test_router_matches_reference_golden(cuda_device):
    import mtp_b200
    for c in golden("router.pt"):
        w, ids, tei = mtp_b200.topk_softmax(c["logits"].to(cuda_device), c["k"], c["renormalize"])
        assert torch.equal(ids.cpu(), c["topk_ids"])
        torch.testing.assert_close(w.cpu(), c["topk_weights"], rtol=2e-6, atol=1e-8)
        assert torch.equal(tei.cpu(), c["tei"])


@pytest.mark.parametrize("m,e,k", [(1, 256, 8), (3, 256, 8), (17, 128, 8), (256, 256, 8), (300, 512, 4),
                                   (5, 8, 2), (64, 1024, 8), (9, 33, 1), (4, 100, 32)])
@pytest.mark.parametrize("renorm", [True, False])
def test_router_matches_oracle(cuda_device, m, e, k, renorm):
    import mtp_b200
    g = torch.Generator().manual_seed(m * 1000 + e + k)
    logits = torch.randn(m, e, generator=g)
    assert not orouter.has_exact_ties(logits.numpy())
    w, ids, _ = mtp_b200.topk_softmax(logits.to(cuda_device), k, renorm)
    ow, oids, _ = orouter.topk_softmax(logits.numpy(), k, renorm)
    assert np.array_equal(ids.cpu().numpy(), oids)
    np.testing.assert_allclose(w.cpu().numpy(), ow, rtol=2e-6, atol=1e-9)


def test_router_tie_breaks_toward_lower_id(cuda_device):
    import mtp_b200
    logits = torch.zeros(2, 64)
    logits[0, [5, 9, 40]] = 3.0
    logits[1, :] = 1.0
    _, ids, _ = mtp_b200.topk_softmax(logits.to(cuda_device), 4)
    assert ids[0].tolist() == [5, 9, 40, 0]
    assert ids[1].tolist() == [0, 1, 2, 3]
    _, oids, _ = orouter.topk_softmax(logits.numpy(), 4)
    assert np.array_equal(ids.cpu().numpy(), oids)


def _align_case(ids, bm, e, emap=None, ignore=False, pad=False, dev=None):
    import mtp_b200
    t = torch.from_numpy(ids).to(dev)
    em = torch.from_numpy(emap).to(dev) if emap is not None else None
    s, ex, n, seg, nseg = mtp_b200.moe_align_block_size(t, bm, e, em, pad, ignore, return_segments=True)
    os_, oe, on, oseg = oalign.moe_align_block_size(ids, bm, e, emap, pad, ignore)
    assert int(n.item()) == int(on[0])
    assert np.array_equal(s.cpu().numpy(), os_)
    assert np.array_equal(ex.cpu().numpy(), oe)
    ns = int(nseg.item())
    assert ns == oseg.shape[0]
    assert np.array_equal(seg.cpu().numpy()[:ns], oseg)


def test_align_docstring_example(cuda_device):
    ids = np.array([[2, 3, 4], [1, 2, 4], [1, 3, 4], [1, 2, 3]], dtype=np.int32)
    _align_case(ids, 4, 5, dev=cuda_device)


@pytest.mark.parametrize("m,k,e,bm", [(1, 8, 256, 8), (1, 8, 256, 16), (3, 8, 256, 16), (17, 8, 128, 8),
                                      (256, 8, 256, 8), (256, 8, 256, 64), (1000, 4, 64, 16),
                                      (8192, 8, 256, 64), (5, 2, 8, 1), (33, 8, 1024, 32)])
def test_align_matches_oracle(cuda_device, m, k, e, bm):
    rng = np.random.default_rng(m * 7 + e)
    ids = np.stack([rng.choice(e, size=k, replace=False) for _ in range(m)]).astype(np.int32)
    _align_case(ids, bm, e, dev=cuda_device)
    _align_case(ids, bm, e, pad=True, dev=cuda_device)


def test_align_skewed_and_invalid_ids(cuda_device):
    rng = np.random.default_rng(3)
    ids = rng.integers(0, 4, size=(500, 8)).astype(np.int32)      # heavy collisions on 4 experts
    _align_case(ids, 16, 64, dev=cuda_device)
    ids2 = ids.copy()
    ids2[::7, 3] = -1                                               # invalid entries are dropped
    ids2[::11, 5] = 70
    _align_case(ids2, 16, 64, dev=cuda_device)


def test_align_expert_map(cuda_device):
    rng = np.random.default_rng(5)
    e = 64
    ids = np.stack([rng.choice(e, size=8, replace=False) for _ in range(40)]).astype(np.int32)
    emap = np.full(e, -1, dtype=np.int32)
    emap[16:32] = np.arange(16, dtype=np.int32)                     # this rank owns experts 16..31
    _align_case(ids, 8, e, emap=emap, ignore=True, dev=cuda_device)
    _align_case(ids, 8, e, emap=emap, ignore=False, dev=cuda_device)


def test_align_empty(cuda_device):
    import mtp_b200
    s, ex, n = mtp_b200.moe_align_block_size(torch.empty(0, 8, dtype=torch.int32, device=cuda_device), 16, 256)
    assert int(n.item()) == 0
    assert s.numel() == 0


def test_dequant_bit_exact_against_reference_golden(cuda_device):
    import mtp_b200
    g = golden("gptq_dequant.pt")
    for case in ("small", "seeded"):
        c = g[case]
        gs = 8 if case == "small" else 128
        w = mtp_b200.dequantize_gptq_projection(c["qweight"].to(cuda_device), c["qzeros"].to(cuda_device),
                                                c["scales"].to(cuda_device), c["g_idx"].to(cuda_device),
                                                group_size=gs)
        assert torch.equal(w.cpu(), c["expected"]), case


@pytest.mark.parametrize("k,n,gs,mode", [(2048, 1024, 128, "raw"), (512, 2048, 128, "sym8"), (256, 64, 64, "raw")])
def test_dequant_bit_exact_against_oracle(cuda_device, k, n, gs, mode):
    import mtp_b200
    g = torch.Generator().manual_seed(k + n)
    q = (torch.randint(0, 2 ** 32, (k // 8, n), generator=g, dtype=torch.int64) - 2 ** 31).to(torch.int32)
    z = (torch.randint(0, 2 ** 32, (k // gs, n // 8), generator=g, dtype=torch.int64) - 2 ** 31).to(torch.int32)
    s = (torch.randn(k // gs, n, generator=g).abs() * 0.02 + 1e-3).half()
    w = mtp_b200.dequantize_gptq_projection(q.to(cuda_device), z.to(cuda_device), s.to(cuda_device),
                                            group_size=gs, zero_mode=mode)
    ref = ogptq.dequantize(q.numpy(), z.numpy(), s.numpy(), group_size=gs, zero_mode=mode)
    assert np.array_equal(w.cpu().numpy(), ref)


@pytest.mark.parametrize("h,i,gs", [(256, 128, 128), (2048, 512, 128), (512, 256, 64)])
def test_repack_bit_exact_against_layout_oracle(cuda_device, h, i, gs):
    from mtp_b200 import W4A16Experts
    from mtp_b200.synthetic import gptq_experts
    g = torch.Generator().manual_seed(h + i)
    ex = gptq_experts(g, 3, h, i, gs, "cpu", random_zeros=True)
    w = W4A16Experts.from_gptq(*(ex[k].to(cuda_device) for k in
                                 ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")),
                               group_size=gs)
    blobs = w.blobs.cpu().numpy()
    for e in range(3):
        ref = olayout.repack_expert(ex, e, h, i, gs)
        assert np.array_equal(blobs[e][:ref.size], ref), e
