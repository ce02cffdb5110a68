"""The prefill path of the W4A16 MoE layer (mtp_w4a16_moe_prefill: 128-pair
bf16 tensor-core tiles) against the fp32 CPU oracle and against the decode
kernel. Same tolerance as the decode layer tests (rel-L2 <= 1e-2 and
normalised max-abs <= 2e-2, on the output's own scale); the prefill path
rounds dequantised weights to bf16 (as the reference's bf16 GEMM does) and the
W2 output per pair to bf16 (vLLM's intermediate_cache3) before the fp32
top-k sum."""
import numpy as np
import pytest
import torch

from oracle import layer as olayer
from oracle import router as orouter
from test_gpu_layer import KEYS, build, check

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("e,h,i,k,gs,m,shared", [
    (8, 256, 128, 2, 128, 300, True),     # ~75 pairs per expert: partial blocks (N < 128)
    (4, 512, 256, 2, 64, 700, True),      # ~350 pairs per expert: three blocks per expert, group 64
    (16, 1024, 384, 4, 128, 513, False),  # I = 384 (three W2 stages), no shared expert
    (32, 2048, 512, 8, 128, 257, True),   # config-1 H and I
])
def test_prefill_matches_oracle(cuda_device, e, h, i, k, gs, m, shared):
    import mtp_b200
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    cfg = LayerConfig(num_experts=e, hidden=h, inter=i, top_k=k, group_size=gs, shared=shared, tokens=(m,))
    experts, sh = make_layer(cfg, seed=e + h + i + m, random_zeros=True)
    w, s = build(experts, sh, cuda_device, gs=gs)
    x, logits = make_inputs(cfg, m, seed=21)
    tw = torch.empty(m, k, device=cuda_device)
    ti = torch.empty(m, k, dtype=torch.int32, device=cuda_device)
    status = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    out32 = torch.empty((m, h), dtype=torch.float32, device=cuda_device)
    out = mtp_b200.moe_layer_w4a16(x.to(cuda_device), logits.to(cuda_device), w, k, shared=s, topk_out=(tw, ti),
                                   status=status, out_f32=out32, path="prefill")
    ow, oids, _ = orouter.topk_softmax(logits.numpy(), k, True)
    assert np.array_equal(ti.cpu().numpy(), oids)
    assert status.cpu().tolist() == [0, 0, 0, 0]
    o = olayer.MoeLayerOracle(experts, sh, group_size=gs)
    ref = o.moe_tokens(x.float(), torch.as_tensor(oids), torch.as_tensor(ow))
    check(out, ref)
    check(out32, ref)
    # the decode kernel on the same call agrees within the same bound
    dec = mtp_b200.moe_layer_w4a16(x.to(cuda_device), logits.to(cuda_device), w, k, shared=s, path="decode")
    check(out, dec.float().cpu())


def test_prefill_given_ids_with_skipped_pairs_and_sym8(cuda_device):
    """Caller-given ids with -1 entries (the expert-parallel convention: pairs
    owned by another rank), some tokens with no routed pair at all, and the
    symmetric zero mode."""
    import mtp_b200
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    cfg = LayerConfig(num_experts=8, hidden=512, inter=256, top_k=4, shared=True, tokens=(400,))
    experts, sh = make_layer(cfg, seed=41)
    w, s = build(experts, sh, cuda_device)
    x, logits = make_inputs(cfg, 400, seed=43)
    ow, oids, _ = orouter.topk_softmax(logits.numpy(), 4, True)
    rng = np.random.default_rng(0)
    drop = rng.random(oids.shape) < 0.4
    drop[:20] = True                        # tokens 0-19: shared expert only
    ids = np.where(drop, -1, oids).astype(np.int32)
    wts = np.where(drop, 0.0, ow).astype(np.float32)
    out = mtp_b200.moe_layer_w4a16(x.to(cuda_device), None, w, 4, shared=s,
                                   topk_weights=torch.from_numpy(wts).to(cuda_device),
                                   topk_ids=torch.from_numpy(ids).to(cuda_device), zero_mode="sym8", path="prefill")
    o = olayer.MoeLayerOracle(experts, sh, zero_mode="sym8")
    ref = o.moe_tokens(x.float(), torch.as_tensor(np.where(drop, 0, oids)), torch.as_tensor(wts))
    check(out, ref)


def test_prefill_config4_shape_matches_decode_kernel(cuda_device):
    """Config-4 layer shape (E = 256, H = 2048, I = 512, top-8, shared expert)
    at M = 2048 through the router: the prefill path against the decode kernel
    (itself checked against the oracle), plus oracle rows; repeated calls are
    bit-identical."""
    import mtp_b200
    from mtp_b200.synthetic import CONFIG1, make_inputs, make_layer
    experts, sh = make_layer(CONFIG1, seed=0, device=cuda_device)
    w, s = build(experts, sh, cuda_device)
    x, logits = make_inputs(CONFIG1, 2048, seed=5, device=cuda_device)
    a = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="prefill")
    b = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="prefill")
    assert torch.equal(a, b)
    dec = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="decode")
    check(a, dec.float().cpu())
    ow, oids, _ = orouter.topk_softmax(logits.cpu().numpy(), 8, True)
    rows = [0, 1, 777, 2047]
    need = sorted({int(v) for r in rows for v in oids[r]})
    cpu_ex = {kk: {ee: experts[kk][ee].cpu() for ee in need} for kk in KEYS}
    o = olayer.MoeLayerOracle(cpu_ex, {kk: v.cpu() for kk, v in sh.items()})
    ref = o.moe_tokens(x[rows].float().cpu(), torch.as_tensor(oids[rows]), torch.as_tensor(ow[rows]))
    check(a[rows], ref)


def test_auto_path_choice(cuda_device):
    import mtp_b200
    assert mtp_b200.layer_path(16, 256, 8) == "decode"
    assert mtp_b200.layer_path(8192, 256, 8) == "prefill"
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    cfg = LayerConfig(num_experts=8, hidden=256, inter=128, top_k=2, shared=True, tokens=(256,))
    experts, sh = make_layer(cfg, seed=3)
    w, s = build(experts, sh, cuda_device)
    x, logits = make_inputs(cfg, 256, seed=4)
    x, logits = x.to(cuda_device), logits.to(cuda_device)
    auto = mtp_b200.moe_layer_w4a16(x, logits, w, 2, shared=s)
    pre = mtp_b200.moe_layer_w4a16(x, logits, w, 2, shared=s, path="prefill")
    assert torch.equal(auto, pre)
    with pytest.raises(ValueError):
        mtp_b200.moe_layer_w4a16(x, logits, w, 2, shared=s, path="prefill",
                                 slot_table=torch.arange(8, dtype=torch.int32, device=cuda_device),
                                 slot_cache=w.blobs)


def test_expert_parallel_layer_on_one_rank_is_the_layer_call(cuda_device):
    """Without a process group ExpertParallelMoE runs the whole layer as one
    call (router, experts, shared expert): the same bits as moe_layer_w4a16."""
    import mtp_b200
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    cfg = LayerConfig(num_experts=8, hidden=512, inter=256, top_k=2, shared=True, tokens=(300,))
    experts, sh = make_layer(cfg, seed=8)
    w, s = build(experts, sh, cuda_device)
    layer = mtp_b200.ExpertParallelMoE.for_gpu(w, 8, 2, shared=s)
    for m in (5, 300):
        x, logits = make_inputs(cfg, m, seed=m)
        x, logits = x.to(cuda_device), logits.to(cuda_device)
        assert torch.equal(layer(x, logits), mtp_b200.moe_layer_w4a16(x, logits, w, 2, shared=s))


def test_prefill_shared_expert_only_call(cuda_device):
    """The expert-parallel home rank's shared-expert call: every routed id -1,
    so the only pairs are the shared expert's."""
    import mtp_b200
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    cfg = LayerConfig(num_experts=8, hidden=512, inter=256, top_k=2, shared=True, tokens=(300,))
    experts, sh = make_layer(cfg, seed=12)
    w, s = build(experts, sh, cuda_device)
    x, _ = make_inputs(cfg, 300, seed=13)
    ids = torch.full((300, 2), -1, dtype=torch.int32, device=cuda_device)
    wts = torch.zeros((300, 2), dtype=torch.float32, device=cuda_device)
    out = mtp_b200.moe_layer_w4a16(x.to(cuda_device), None, w, 2, shared=s, topk_weights=wts, topk_ids=ids,
                                   path="prefill")
    o = olayer.MoeLayerOracle(experts, sh)
    ref = o.moe_tokens(x.float(), torch.zeros((300, 2), dtype=torch.long), torch.zeros((300, 2)))
    check(out, ref)
