"""Generate the golden fixtures of tests/golden/ by running the REFERENCE's own
Python code (HUSRCF/MTP, importable from its ``src/`` directory).

Run in a container where the reference checkout exists:

    python tests/golden/make_golden.py --reference-src <reference>/src

The fixtures are small ``.pt`` files (torch.save of dicts of CPU tensors and
plain values); the tests load them and never need the reference itself.

Fixtures:
  gptq_dequant.pt   reference ``unpack_rows`` / ``unpack_cols`` /
                    ``dequantize_gptq_projection`` (repack/gptq_unpack.py:54-131)
                    on the reference test's own inputs (tests/test_gptq_unpack.py:49-82)
                    and on a seeded K=256, N=64, g=128 projection with random zeros.
  moe_small.pt      reference ``MtpExtraRunner.moe_tokens`` (mtp/extra_tensors.py:544-598)
                    over ``SingleExpertMlp`` experts dequantised by the reference
                    (fp32), routed by the reference ``router_topk`` (:341-355), on a
                    tiny layer E=8, H=256, I=128, k=2, M=5 with random GPTQ zeros and
                    a sigmoid-gated shared expert. Inputs are stored in the fixture.
  config0.pt        BASELINE config 0 (E=128, H=2048, I=768, k=8, M=4, seed 0) built
                    by mtp_b200.synthetic on the CPU; stores sha256 of the generated
                    tensors (pins the generator), the reference router outputs and the
                    reference moe_tokens output [4, 2048] fp32.
  router.pt         reference CPU ``topk_softmax`` fallback
                    (tracing/vllm_router_trace.py:4201-4227) on seeded logits [64, 256]
                    and [7, 128], renormalised and not.
  cache.pt          reference ``ControlledExpertCacheManager`` and
                    ``ReadyTimeExpertCacheManager`` (runtime/cache_manager.py:208-578)
                    counters after seeded issue/demand sequences.
  predictor_hr.pt   reference ``HiddenResidualExpertPredictor`` (training/
                    hidden_residual.py:44-103; hidden 256, 64 experts, 6 layers,
                    future window 4, width 128, seed 7, every parameter rounded to
                    bf16 so the kernel's bf16 copies are exact) on bf16 hidden
                    states [9, 256] with layer ids: its state dict, inputs, fp32
                    logits [9, 4, 64] and torch.topk(logits, 8) ids (the ranking of
                    recall_at_m, training/predictor.py:105).
  premap.pt         reference ``build_priority_masks`` / ``build_premap_descriptors``
                    (runtime/premap.py:78-192) on seeded transition and MTP scores
                    [5 tokens, 2 deltas, 3 layers, 64 experts] of 2 samples, max and
                    mean reductions.
  repack_manifest.json  the reference ``repack_qwen3_moe_gptq``
                    (repack/qwen3_moe_gptq.py:201-265) on the seeded synthetic snapshot
                    of mtp_b200.synthetic.make_gptq_snapshot (2 layers, 4 experts,
                    H=256, I=128, g=128, 2 shards, seed 0): its manifest.jsonl records
                    (per-tensor shape, dtype, sha256, source fields) and summary.json
                    without the machine paths.
"""
from __future__ import annotations

import argparse
import hashlib
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent


def sha(t: torch.Tensor) -> str:
    return hashlib.sha256(t.contiguous().view(torch.uint8).numpy().tobytes()).hexdigest()


def gen_dequant(ref):
    from mtp_expert_prefetch.repack import GptqProjectionTensors, dequantize_gptq_projection
    sys.path.insert(0, str(ROOT))
    from oracle import gptq as og

    out = {}
    # the reference test's own inputs (tests/test_gptq_unpack.py:49-82)
    int_weight = torch.arange(16 * 8, dtype=torch.int32).reshape(16, 8) % 16
    zeros = torch.stack([torch.full((8,), 2, dtype=torch.int32), torch.full((8,), 5, dtype=torch.int32)])
    scales = torch.stack([torch.linspace(0.25, 1.0, 8), torch.linspace(1.0, 1.75, 8)]).to(torch.float16)
    g_idx = torch.tensor([0] * 8 + [1] * 8, dtype=torch.int32)
    qweight = torch.from_numpy(og.pack_rows(int_weight.numpy()))
    qzeros = torch.from_numpy(og.pack_cols(zeros.numpy()))
    w = dequantize_gptq_projection(GptqProjectionTensors(qweight, qzeros, scales, g_idx), dtype=torch.float32)
    out["small"] = dict(qweight=qweight, qzeros=qzeros, scales=scales, g_idx=g_idx, expected=w)
    # seeded projection with random zeros
    g = torch.Generator().manual_seed(11)
    k, n, gs = 256, 64, 128
    qweight = (torch.randint(0, 2 ** 32, (k // 8, n), generator=g, dtype=torch.int64) - 2 ** 31).to(torch.int32)
    qzeros = (torch.randint(0, 2 ** 32, (k // gs, n // 8), generator=g, dtype=torch.int64) - 2 ** 31).to(torch.int32)
    scales = (torch.randn(k // gs, n, generator=g).abs() * 0.02 + 1e-3).to(torch.float16)
    g_idx = torch.arange(k, dtype=torch.int32) // gs
    w = dequantize_gptq_projection(GptqProjectionTensors(qweight, qzeros, scales, g_idx), dtype=torch.float32)
    from mtp_expert_prefetch.repack.gptq_unpack import unpack_cols, unpack_rows
    out["seeded"] = dict(qweight=qweight, qzeros=qzeros, scales=scales, g_idx=g_idx, expected=w,
                         unpacked_rows=unpack_rows(qweight), unpacked_cols=unpack_cols(qzeros))
    torch.save(out, HERE / "gptq_dequant.pt")


def _reference_runner(experts_gptq: dict, shared_gptq: dict | None, expert_ids, group_size: int):
    """Build a reference MtpExtraRunner (fp32) holding the given experts, the way the
    reference test builds one (tests/test_mtp_extra_tensors.py:18-55)."""
    from mtp_expert_prefetch.mtp import MtpExtraRunner
    from mtp_expert_prefetch.repack import (GptqProjectionTensors, SingleExpertMlp, SingleExpertWeights,
                                            TopKExpertMlp, dequantize_gptq_projection)

    def proj(q, z, s):
        k = q.shape[0] * 8
        g_idx = torch.arange(k, dtype=torch.int32) // group_size
        return dequantize_gptq_projection(GptqProjectionTensors(q, z, s, g_idx), dtype=torch.float32)

    def expert(src, e):
        w13 = proj(src["w13_qweight"][e], src["w13_qzeros"][e], src["w13_scales"][e]) if e is not None else \
            proj(src["w13_qweight"], src["w13_qzeros"], src["w13_scales"])
        w2 = proj(src["w2_qweight"][e], src["w2_qzeros"][e], src["w2_scales"][e]) if e is not None else \
            proj(src["w2_qweight"], src["w2_qzeros"], src["w2_scales"])
        inter = w13.shape[0] // 2
        return SingleExpertMlp(SingleExpertWeights(gate_proj=w13[:inter].contiguous(),
                                                   up_proj=w13[inter:].contiguous(), down_proj=w2))

    runner = MtpExtraRunner.__new__(MtpExtraRunner)
    torch.nn.Module.__init__(runner)
    runner.target_dtype = torch.float32
    runner.target_device = torch.device("cpu")
    uniq = sorted({int(e) for e in expert_ids})
    runner.topk_mlp = TopKExpertMlp({e: expert(experts_gptq, e) for e in uniq})
    if shared_gptq is not None:
        runner.shared_expert = expert(shared_gptq, None)
        runner.register_buffer("shared_expert_gate_weight",
                               shared_gptq["gate_weight"].to(torch.float32).reshape(1, -1), persistent=False)
    return runner


def _router(logits: torch.Tensor, k: int, router_weight_dim: int):
    """Reference router_topk (extra_tensors.py:341-355) on given logits: an identity
    router weight makes F.linear return the logits unchanged."""
    from mtp_expert_prefetch.mtp import MtpExtraRunner
    runner = MtpExtraRunner.__new__(MtpExtraRunner)
    torch.nn.Module.__init__(runner)
    runner.target_dtype = torch.float32
    runner.target_device = torch.device("cpu")
    runner.register_buffer("router_weight", torch.eye(router_weight_dim), persistent=False)
    # hidden_size is read from fc_weight's first dimension (extra_tensors.py:311-312)
    runner.register_buffer("fc_weight", torch.zeros(router_weight_dim, 1), persistent=False)
    r = runner.router_topk(logits, top_k=k)
    return r.topk_ids.to(torch.int32), r.topk_weights.to(torch.float32)


def gen_moe_small():
    sys.path.insert(0, str(ROOT))
    from mtp_b200.synthetic import LayerConfig, make_layer
    cfg = LayerConfig(num_experts=8, hidden=256, inter=128, top_k=2, shared=True)
    experts, shared = make_layer(cfg, seed=5, random_zeros=True)
    g = torch.Generator().manual_seed(6)
    x = torch.randn(5, 256, generator=g).to(torch.bfloat16)
    logits = torch.randn(5, 8, generator=g)
    ids, wts = _router(logits, 2, 8)
    runner = _reference_runner(experts, shared, ids.reshape(-1).tolist(), 128)
    out = runner.moe_tokens(x.float()[None], ids[None].long(), wts[None])[0]
    torch.save(dict(experts=experts, shared=shared, x=x, logits=logits, topk_ids=ids, topk_weights=wts,
                    expected=out, group_size=128, top_k=2), HERE / "moe_small.pt")


def gen_config0():
    sys.path.insert(0, str(ROOT))
    from mtp_b200.synthetic import CONFIG0, make_inputs, make_layer
    experts, _ = make_layer(CONFIG0, seed=0)
    x, logits = make_inputs(CONFIG0, 4, seed=1)
    ids, wts = _router(logits, CONFIG0.top_k, CONFIG0.num_experts)
    runner = _reference_runner(experts, None, ids.reshape(-1).tolist(), CONFIG0.group_size)
    runner.shared_expert = None
    # moe_tokens requires a shared expert; the config-0 layer has none, so the
    # routed part is taken with a zero shared gate weight and a zero shared MLP.
    from mtp_expert_prefetch.repack import SingleExpertMlp, SingleExpertWeights
    h, i = CONFIG0.hidden, CONFIG0.inter
    runner.shared_expert = SingleExpertMlp(SingleExpertWeights(torch.zeros(i, h), torch.zeros(i, h), torch.zeros(h, i)))
    runner.register_buffer("shared_expert_gate_weight", torch.zeros(1, h), persistent=False)
    out = runner.moe_tokens(x.float()[None], ids[None].long(), wts[None])[0]
    hashes = {k: sha(v) for k, v in experts.items()}
    hashes["x"] = sha(x)
    hashes["logits"] = sha(logits)
    torch.save(dict(hashes=hashes, topk_ids=ids, topk_weights=wts, expected=out, seed_layer=0, seed_inputs=1),
               HERE / "config0.pt")


def gen_router():
    import importlib
    trace = importlib.import_module("mtp_expert_prefetch.tracing.vllm_router_trace")
    trace._patch_missing_vllm_activation_ops_for_trace()
    op = torch.ops._moe_C.topk_softmax
    cases = []
    for seed, (m, e, k) in ((21, (64, 256, 8)), (22, (7, 128, 8)), (23, (3, 16, 4))):
        g = torch.Generator().manual_seed(seed)
        logits = torch.randn(m, e, generator=g)
        for renorm in (True, False):
            w = torch.empty(m, k)
            ids = torch.empty(m, k, dtype=torch.int32)
            tei = torch.empty(m, k, dtype=torch.int32)
            op(w, ids, tei, logits, renorm)
            cases.append(dict(logits=logits, k=k, renormalize=renorm, topk_weights=w, topk_ids=ids, tei=tei))
    torch.save(cases, HERE / "router.pt")


def gen_cache():
    from mtp_expert_prefetch.runtime.cache_manager import (ControlledExpertCacheManager,
                                                           ReadyTimeExpertCacheManager)
    cases = []
    for seed in range(4):
        rnd = random.Random(seed)
        ops = []
        t = 0.0
        for _ in range(400):
            t += rnd.choice([0.0, 5.0, 20.0, 50.0])
            kind = rnd.choice(["issue", "demand", "demand"])
            ops.append((kind, rnd.randrange(3), min(int(rnd.expovariate(0.15)), 31), t))
        lru = ControlledExpertCacheManager(capacity=12)
        ready = ReadyTimeExpertCacheManager(capacity=12, service_us_per_issue=30.0, service_us_per_batch=5.0,
                                            queue_batch_size=1 + seed, queue_deadline_us=10.0 * seed)
        res_lru, res_ready = [], []
        for kind, layer, expert, tt in ops:
            if kind == "issue":
                res_lru.append(lru.issue_prefetch(layer, expert))
                res_ready.append(ready.issue_prefetch(layer, expert, arrival_us=tt))
            else:
                res_lru.append(lru.demand(layer, expert))
                res_ready.append(ready.demand(layer, expert, arrival_us=tt))
        ready.finish()
        cases.append(dict(seed=seed, ops=ops, lru_results=res_lru, ready_results=res_ready,
                          lru_snapshot=lru.snapshot().as_dict(), ready_snapshot=ready.snapshot().as_dict(),
                          ready_params=dict(capacity=12, service_us_per_issue=30.0, service_us_per_batch=5.0,
                                            queue_batch_size=1 + seed, queue_deadline_us=10.0 * seed)))
    torch.save(cases, HERE / "cache.pt")


def gen_predictor_hr():
    from mtp_expert_prefetch.training.hidden_residual import HiddenResidualExpertPredictor
    torch.manual_seed(7)
    mod = HiddenResidualExpertPredictor(hidden_size=256, num_experts=64, num_layers=6, future_window=4, width=128)
    mod.eval()
    with torch.no_grad():
        for prm in mod.parameters():
            prm.copy_(prm.to(torch.bfloat16).to(torch.float32))
        # a LayerNorm affine that is not the identity
        mod.encoder[2].weight.copy_((1.0 + 0.1 * torch.randn(128)).to(torch.bfloat16).to(torch.float32))
        mod.encoder[2].bias.copy_((0.1 * torch.randn(128)).to(torch.bfloat16).to(torch.float32))
        hidden = torch.randn(9, 256).to(torch.bfloat16)
        layer_ids = torch.tensor([0, 5, 2, 3, 3, 1, 4, 0, 5], dtype=torch.int32)
        logits = mod(hidden.to(torch.float32), layer_ids=layer_ids.long())
    ids = torch.topk(logits, 8, dim=-1).indices.to(torch.int32)
    torch.save(dict(state={k: v.clone() for k, v in mod.state_dict().items()}, hidden=hidden, layer_ids=layer_ids,
                    logits=logits, topk_ids=ids, config=dict(hidden_size=256, num_experts=64, num_layers=6,
                                                                 future_window=4, width=128, ln_eps=1e-5)),
               HERE / "predictor_hr.pt")


def gen_repack():
    import json
    import tempfile

    from mtp_expert_prefetch.repack.qwen3_moe_gptq import repack_qwen3_moe_gptq
    sys.path.insert(0, str(ROOT))
    from mtp_b200.synthetic import make_gptq_snapshot
    with tempfile.TemporaryDirectory() as tmp:
        snap, out = Path(tmp) / "snapshot", Path(tmp) / "repacked"
        make_gptq_snapshot(snap, layers=2, experts=4, hidden=256, inter=128, group_size=128, shards=2, seed=0)
        repack_qwen3_moe_gptq(snap, out, num_experts=4)
        records = [json.loads(line) for line in (out / "manifest.jsonl").read_text().splitlines() if line.strip()]
        summary = json.loads((out / "summary.json").read_text())
    for key in ("snapshot_path", "output_dir"):
        summary.pop(key, None)
    (HERE / "repack_manifest.json").write_text(json.dumps({"records": records, "summary": summary,
                                                           "snapshot": dict(layers=2, experts=4, hidden=256,
                                                                            inter=128, group_size=128, shards=2,
                                                                            seed=0)}, indent=1, sort_keys=True))


def gen_premap():
    from mtp_expert_prefetch.runtime.premap import build_premap_descriptors, build_priority_masks
    g = torch.Generator().manual_seed(13)
    trans = torch.rand(5, 2, 3, 64, generator=g)
    mtp = torch.randn(5, 2, 3, 64, generator=g)
    samples = torch.tensor([0, 0, 1, 1, 1])
    masks = build_priority_masks(trans, mtp)
    out = dict(transition=trans, mtp=mtp, samples=samples, masks={k: v.clone() for k, v in masks.items()})
    for red in ("max", "mean"):
        d = build_premap_descriptors(trans, mtp, samples, reduce=red)
        out[f"descriptors_{red}"] = [(x.sample_idx, x.layer_idx, x.expert_id, x.priority, x.source, x.score)
                                     for x in d]
    torch.save(out, HERE / "premap.pt")


GENERATORS = {"gptq_dequant": lambda: gen_dequant(None), "moe_small": lambda: gen_moe_small(),
              "config0": lambda: gen_config0(), "router": lambda: gen_router(), "cache": lambda: gen_cache(),
              "predictor_hr": lambda: gen_predictor_hr(), "repack": lambda: gen_repack(),
              "premap": lambda: gen_premap()}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference-src", required=True)
    ap.add_argument("--only", nargs="*", choices=sorted(GENERATORS), help="generate only these fixtures")
    args = ap.parse_args()
    sys.path.insert(0, args.reference_src)
    torch.manual_seed(0)
    for name, gen in GENERATORS.items():
        if not args.only or name in args.only:
            gen()
    for f in sorted(HERE.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
