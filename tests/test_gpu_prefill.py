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


def test_prefill_config4_matches_oracle_and_decode_kernel(cuda_device):
    """BASELINE config 4's layer (E = 256, H = 2048, I = 512, top-8, shared
    expert) at its own size, M = 8192, through the router: 64 strided rows
    against the fp32 oracle, every row against the decode kernel (itself
    checked against the oracle), and repeated calls bit-identical."""
    import mtp_b200
    from mtp_b200.synthetic import CONFIG1, make_inputs, make_layer
    m = 8192
    experts, sh = make_layer(CONFIG1, seed=0, device=cuda_device)
    w, s = build(experts, sh, cuda_device)
    x, logits = make_inputs(CONFIG1, m, seed=5, device=cuda_device)
    a = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="prefill")
    b = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="prefill")
    assert torch.equal(a, b)
    dec = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s, path="decode")
    check(a, dec.float().cpu())
    ow, oids, _ = orouter.topk_softmax(logits.cpu().numpy(), 8, True)
    rows = np.linspace(0, m - 1, num=64).astype(int).tolist()
    need = sorted({int(v) for r in rows for v in oids[r]})
    cpu_ex = {kk: {ee: experts[kk][ee].cpu() for ee in need} for kk in KEYS}
    o = olayer.MoeLayerOracle(cpu_ex, {kk: v.cpu() for kk, v in sh.items()})
    ref = o.moe_tokens(x[rows].float().cpu(), torch.as_tensor(oids[rows]), torch.as_tensor(ow[rows]))
    check(a[rows], ref)
    check(dec[rows], ref)


@pytest.mark.parametrize("e,h,i,k,m,shared", [
    (8, 256, 128, 2, 300, True),        # partial blocks, the shared expert as expert E
    (256, 2048, 512, 8, 8192, True),    # config 4
    (16, 512, 256, 4, 700, False),      # no shared expert
])
def test_prefill_align_tables_match_oracle(cuda_device, e, h, i, k, m, shared):
    """The prefill path's own align (histogram, offsets, stable scatter in
    three launches) against the moe_align_block_size restatement, bit for
    bit: the pairs extended by the shared expert (expert E), then sorted pair
    indices (valid region), expert of every used block and
    num_tokens_post_padded, at block size 128 with pad_sorted_ids."""
    import mtp_b200
    from mtp_b200 import _lib
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    from oracle import align as oalign
    cfg = LayerConfig(num_experts=e, hidden=h, inter=i, top_k=k, shared=shared, tokens=(m,))
    experts, sh = make_layer(cfg, seed=e + m, device=cuda_device)
    w, s = build(experts, sh, cuda_device)
    x, logits = make_inputs(cfg, m, seed=31, device=cuda_device)
    ws = mtp_b200.prefill_workspace(m, w, k, cuda_device)
    mtp_b200.moe_layer_w4a16(x, logits, w, k, shared=s, workspace=ws, path="prefill")
    torch.cuda.synchronize()
    t = _lib.prefill_tables(m, e, k, h, i, shared)
    kx = k + (1 if shared else 0)
    assert t.pairs_per_token == kx and t.block_size == 128

    def view(off, n):
        return ws[off:off + 4 * n].view(torch.int32).cpu().numpy()

    _, oids, _ = orouter.topk_softmax(logits.cpu().numpy(), k, True)
    ids_x = np.concatenate([oids, np.full((m, 1), e, np.int32)], axis=1) if shared else oids
    assert np.array_equal(view(t.pair_expert_ids, m * kx).reshape(m, kx), ids_x)
    ref_sorted, ref_eids, ref_ntpp, _ = oalign.moe_align_block_size(ids_x, 128, e + (1 if shared else 0),
                                                                     pad_sorted_ids=True)
    ntpp = int(view(t.num_tokens_post_padded, 1)[0])
    assert ntpp == int(ref_ntpp[0])
    assert t.capacity >= ntpp and t.capacity == ref_sorted.size
    assert np.array_equal(view(t.sorted_token_ids, ntpp), ref_sorted[:ntpp])
    assert np.array_equal(view(t.expert_ids, ntpp // 128), ref_eids[:ntpp // 128])


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


@pytest.mark.parametrize("path", ["decode", "prefill"])
def test_expert_map_and_shared_rows(cuda_device, path):
    """The expert-parallel fields of the layer call: global ids through an
    expert_map (this shard = global experts 8-15 of 16) give the same bits as
    the ids masked by hand; the shared expert restricted to rows [b, e) adds
    exactly the shared-only call's output on those rows (within the bf16
    bound) and nothing elsewhere."""
    import mtp_b200
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    m = 300 if path == "prefill" else 40
    cfg = LayerConfig(num_experts=8, hidden=512, inter=256, top_k=4, shared=True, tokens=(m,))
    experts, sh = make_layer(cfg, seed=71)
    w, s = build(experts, sh, cuda_device)
    x, _ = make_inputs(cfg, m, seed=72)
    x = x.to(cuda_device)
    g = torch.Generator().manual_seed(73)
    gids = torch.stack([torch.randperm(16, generator=g)[:4] for _ in range(m)]).to(torch.int32)
    gw = torch.rand((m, 4), generator=g)
    emap = torch.full((16,), -1, dtype=torch.int32)
    emap[8:] = torch.arange(8, dtype=torch.int32)
    lids = torch.where(gids >= 8, gids - 8, torch.full_like(gids, -1))
    lw = torch.where(gids >= 8, gw, torch.zeros(()))
    gids, gw, lids, lw, emap = (t.to(cuda_device) for t in (gids, gw, lids, lw, emap))
    a = mtp_b200.moe_layer_w4a16(x, None, w, 4, topk_weights=gw, topk_ids=gids, expert_map=emap, path=path)
    b = mtp_b200.moe_layer_w4a16(x, None, w, 4, topk_weights=lw, topk_ids=lids, path=path)
    assert torch.equal(a, b)
    r0, r1 = m // 4, m // 2
    c = mtp_b200.moe_layer_w4a16(x, None, w, 4, shared=s, topk_weights=gw, topk_ids=gids, expert_map=emap,
                                 shared_rows=(r0, r1), path=path)
    assert torch.equal(c[:r0], b[:r0]) and torch.equal(c[r1:], b[r1:])
    none_ids = torch.full((m, 4), -1, dtype=torch.int32, device=cuda_device)
    only = mtp_b200.moe_layer_w4a16(x, None, w, 4, shared=s, topk_weights=torch.zeros((m, 4), device=cuda_device),
                                    topk_ids=none_ids, path=path)
    check(c[r0:r1], (b[r0:r1].float() + only[r0:r1].float()).cpu())
    with pytest.raises(ValueError):
        mtp_b200.moe_layer_w4a16(x, torch.zeros((m, 8), device=cuda_device), w, 4, expert_map=emap, path=path)
