"""Benchmark: W4A16 MoE layer tok/s and % HBM roofline over the decode sweep
(E=256, H=2048, I=512, top-8, sigmoid-gated shared expert,
GPTQ int4 g128, M in {1,2,4,...,256}) on synthetic seeded weights and inputs.

One step = one layer forward at every M of the sweep, each through L layers of
distinct weights in sequence (a CUDA graph per M). Every layer call has fresh
router logits, and the L layers (L x 418 MB) and the sweep's traffic exceed the
126 MB L2, so weights come from HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Prints one JSON line (rank 0). Multi-GPU: one process per GPU (torchrun),
independent replicas (the decode layer does not shard), weak scaling, time =
max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SWEEP = (1, 2, 4, 8, 16, 32, 64, 128, 256)
METRIC = "W4A16 MoE layer tok/s and % HBM roofline, M=1-256; prefetch hit rate"
UNIT = "tokens/s"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def warm(self):
        """One untimed pass over the sweep (first-touch costs), then a fresh record."""
        for m, x, ids, w in self.batches:
            self.o.moe_tokens(x, ids, w)
        self.times = {m: [] for m in self.tokens}
        self.pos = 0

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in getattr(self, "lines", []):
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------
# CPU reference path (the reference's torch form; the oracle port)
# ---------------------------------------------------------------------------
class CpuReference:
    """The reference CPU path: per-token routed SiLU-MLP + sigmoid-gated shared
    expert with weights dequantised once to bf16 (the reference's
    load_topk_expert_mlp + moe_tokens form), torch on all host threads, over
    the same M sweep as the GPU value. Samples cycle through the sweep; the
    value is the sweep's tokens over the sum of the per-M mean layer times,
    the GPU value's definition, so a partial pass does not bias it."""

    def __init__(self, tokens=SWEEP):
        import torch

        from mtp_b200.synthetic import CONFIG1, make_inputs, make_layer
        from oracle import layer as olayer
        from oracle import router as orouter

        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        experts, shared = make_layer(CONFIG1, seed=0)
        self.o = olayer.MoeLayerOracle(experts, shared, dtype=torch.bfloat16)
        self.tokens = tuple(tokens)
        self.batches = []
        t0 = time.perf_counter()
        for m in self.tokens:
            x, logits = make_inputs(CONFIG1, m, seed=100 + m)
            w, ids, _ = orouter.topk_softmax(logits.numpy(), CONFIG1.top_k, True)
            self.o.prepare(ids)
            self.batches.append((m, x, torch.from_numpy(ids), torch.from_numpy(w)))
        self.dequant_s = time.perf_counter() - t0
        self.times = {m: [] for m in self.tokens}
        self.pos = 0

    def run(self, seconds: float):
        """Layer calls in sweep order (resuming where the last run stopped)
        until `seconds` have passed; at least one call."""
        deadline = time.perf_counter() + seconds
        calls = 0
        while time.perf_counter() < deadline or calls == 0:
            m, x, ids, w = self.batches[self.pos]
            t0 = time.perf_counter()
            self.o.moe_tokens(x, ids, w)
            self.times[m].append(time.perf_counter() - t0)
            self.pos = (self.pos + 1) % len(self.batches)
            calls += 1

    def warm(self):
        """One untimed pass over the sweep (first-touch costs), then a fresh record."""
        for m, x, ids, w in self.batches:
            self.o.moe_tokens(x, ids, w)
        self.times = {m: [] for m in self.tokens}
        self.pos = 0

    def summary(self):
        done = [m for m in self.tokens if self.times[m]]
        mean = {m: sum(self.times[m]) / len(self.times[m]) for m in done}
        calls = sum(len(v) for v in self.times.values())
        el = sum(sum(v) for v in self.times.values())
        complete = len(done) == len(self.tokens)
        value = sum(done) / sum(mean.values()) if done else 0.0
        return {
            "value": value, "unit": UNIT, "cores": self.threads, "kind": "port",
            "sample": (f"config-1 layer, M sweep {list(self.tokens)}{'' if complete else ' (partial: ' + str(done) + ')'}, "
                       f"{calls} layer calls, {el:.1f} s; value = sum(M) / sum over M of the mean layer time; bf16 "
                       f"weights dequantised once ({self.dequant_s:.1f} s, excluded); CPU {cpu_model()}"),
            "per_m_tok_s": {str(m): round(m / mean[m], 1) for m in done},
        }


def cpu_reference(seconds: float = 12.0):
    ref = CpuReference()
    ref.warm()
    ref.run(seconds)
    return ref.summary()


# ---------------------------------------------------------------------------
# GPU path
# ---------------------------------------------------------------------------
def algorithmic_bytes(num_unique: int, m: int, cfg, expert_bytes: int) -> int:
    weights = (num_unique + (1 if cfg.shared else 0)) * expert_bytes
    acts = m * cfg.hidden * 2 + m * cfg.num_experts * 4 + m * cfg.hidden * 2
    return weights + acts


def run_gpu(args, rank: int, world: int):
    import numpy as np
    import torch

    import mtp_b200
    from mtp_b200.ops import SharedExpert, W4A16Experts, layer_workspace
    from mtp_b200.synthetic import CONFIG1, make_inputs, make_layer

    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", 0)))
    torch.cuda.set_device(dev)
    cfg = CONFIG1
    keys = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")
    layers = []
    for l in range(args.layers):
        ex, sh = make_layer(cfg, seed=1000 * rank + l, device=dev)
        w = W4A16Experts.from_gptq(*(ex[k] for k in keys), group_size=cfg.group_size)
        s = SharedExpert.from_gptq(*(sh[k] for k in keys), sh["gate_weight"], group_size=cfg.group_size)
        del ex, sh
        layers.append((w, s))
    torch.cuda.synchronize()
    expert_bytes = layers[0][0].expert_bytes

    sweep = [int(v) for v in args.sweep.split(",")]
    # per-M inputs for every layer; routing differs per layer and per M
    state = {}
    for m in sweep:
        xs, lgs, outs, wss, ids = [], [], [], [], []
        for l in range(args.layers):
            x, lg = make_inputs(cfg, m, seed=10_000 * rank + 100 * l + m, device=dev)
            xs.append(x)
            lgs.append(lg)
            outs.append(torch.empty((m, cfg.hidden), dtype=torch.bfloat16, device=dev))
            wss.append(layer_workspace(m, layers[l][0], cfg.top_k, dev))
            ids.append(torch.empty((m, cfg.top_k), dtype=torch.int32, device=dev))
        state[m] = dict(x=xs, logits=lgs, out=outs, ws=wss, ids=ids,
                        tw=[torch.empty((m, cfg.top_k), device=dev) for _ in range(args.layers)])

    def run_m(m):
        st = state[m]
        for l in range(args.layers):
            w, s = layers[l]
            mtp_b200.moe_layer_w4a16(st["x"][l], st["logits"][l], w, cfg.top_k, shared=s, out=st["out"][l],
                                     workspace=st["ws"][l], topk_out=(st["tw"][l], st["ids"][l]))

    # eager warm-up, then one CUDA graph per M (the L layers in sequence)
    for m in sweep:
        run_m(m)
    torch.cuda.synchronize()
    graphs = {}
    cap_stream = torch.cuda.Stream(dev)
    for m in sweep:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap_stream):
            run_m(m)
        graphs[m] = g
    torch.cuda.synchronize()

    # unique experts per (M, layer) for the algorithmic bytes
    uniq = {m: [int(torch.unique(state[m]["ids"][l]).numel()) for l in range(args.layers)] for m in sweep}
    bytes_per_m = {m: sum(algorithmic_bytes(u, m, cfg, expert_bytes) for u in uniq[m]) for m in sweep}

    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        for m in sweep:
            graphs[m].replay()
    torch.cuda.synchronize()

    ev = {m: [] for m in sweep}
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    with ClockSampler(dev.index) as clocks:
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for _ in range(args.steps):
            for m in sweep:
                a = torch.cuda.Event(enable_timing=True)
                b = torch.cuda.Event(enable_timing=True)
                a.record(stream)
                graphs[m].replay()
                b.record(stream)
                ev[m].append((a, b))
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    elapsed_ms = t_start.elapsed_time(t_end)
    per_m_ms = {m: sum(a.elapsed_time(b) for a, b in ev[m]) / args.steps for m in sweep}
    if world > 1:
        t = torch.tensor([elapsed_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        elapsed_ms = float(t.item())

    hbm_gbs, peak_kind = peaks()
    tokens_per_step = sum(m * args.layers for m in sweep)
    value = tokens_per_step * args.steps * world / (elapsed_ms / 1e3)
    rows = []
    for m in sweep:
        us_layer = per_m_ms[m] * 1e3 / args.layers
        gbs = bytes_per_m[m] / (per_m_ms[m] / 1e3) / 1e9
        rows.append({"M": m, "us_per_layer": round(us_layer, 3), "tok_s": round(m / (us_layer / 1e6), 1),
                     "unique_experts": round(sum(uniq[m]) / args.layers, 2),
                     "bytes_per_layer": bytes_per_m[m] // args.layers, "hbm_gbs": round(gbs, 1),
                     "hbm_frac": round(gbs / hbm_gbs, 4)})
    total_bytes = sum(bytes_per_m.values())
    total_ms = sum(per_m_ms.values())
    achieved = total_bytes / (total_ms / 1e3) / 1e9
    # DRAM traffic per launch: the ncu-measured traffic/algorithmic ratios of
    # the layer kernel (profiles/traffic.json, one capture per listed M),
    # each sweep point taking the capture nearest in log2(M), applied to this
    # run's algorithmic bytes and averaged over the launches
    traffic = None
    tp = ROOT / "profiles" / "traffic.json"
    n_launch = len(sweep) * args.layers
    if tp.exists():
        caps = [(c["M"], c["traffic_over_algorithmic"]) for c in json.loads(tp.read_text()).get("captures", [])]
        if caps:
            import math

            def ratio_for(m):
                return min(caps, key=lambda c: (abs(math.log2(c[0]) - math.log2(m)), -c[0]))[1]

            traffic = round(sum(ratio_for(m) * bytes_per_m[m] for m in sweep) / n_launch)

    # end to end through the public API with host buffers (pinned), copies timed
    e2e = run_e2e(args, layers, cfg, sweep, dev, state) if not args.no_e2e else None

    result = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(elapsed_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "config1 decode sweep: W4A16 MoE layer E=256 H=2048 I=512 top-8 + shared expert, "
                               "GPTQ int4 g128 (raw zeros read)",
                   "tokens": sweep, "layers_per_graph": args.layers, "parallelism": f"replicas x{world}",
                   "l2": "inputs larger than L2: L distinct layers (L x 418 MB) and fresh routing per call"},
        "sweep": rows,
        "roofline": {"bound": "hbm", "kernel": "moe_fused_kernel (route+W1+W2+combine, one launch per layer), "
                                               "bytes and time summed over the sweep",
                     "achieved": round(achieved, 1), "peak": hbm_gbs, "unit": "GB/s",
                     "frac": round(achieved / hbm_gbs, 4), "peak_source": peak_kind,
                     "traffic": traffic},
        "gpu_launches": args.steps * len(sweep) * args.layers,
        "clocks": clocks.summary(),
    }
    if e2e is not None:
        result["e2e"] = e2e
    if not args.no_predictor:
        result["predictor"] = run_predictor(dev, hbm_gbs)
    if not args.no_prefetch and rank == 0:
        result["prefetch"] = run_prefetch(dev, layers[0][0], layers[0][1], cfg, args.prefetch_layers,
                                          args.prefetch_steps)
    del graphs, layers, state
    torch.cuda.empty_cache()
    if not args.no_prefill:
        result["prefill_ep"] = run_prefill_ep(args, rank, world, dev)
    return result


def bf16_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get("bf16_tflops_sustained") or d.get("bf16_tflops")
        if v:
            return float(v), "measured (sustained)" if d.get("bf16_tflops_sustained") else "measured"
    return 1400.0, "fallback (sustained)"


def run_prefill_ep(args, rank: int, world: int, dev):
    """Config 4: expert-parallel prefill. M = 8192 tokens in total, split evenly
    over the ranks (strong scaling), uniform-random top-8 routing over 256
    experts sharded by rank, L stacked layers with a bf16 residual add; each
    layer all-gathers the token rows and routing lists, runs one layer call
    on them (other ranks' experts dropped through an expert_map, the gated
    shared expert on this rank's own rows) and reduce-scatters the bf16
    partial rows home. After timing,
    every rank checks layer 0 on its own tokens against the single-GPU decode
    kernel over all 256 experts (gathered from the ranks' shards)."""
    import torch

    from mtp_b200 import ExpertParallelMoE, layer_path
    from mtp_b200.ops import SharedExpert, W4A16Experts
    from mtp_b200.synthetic import CONFIG1, gptq_experts

    cfg = CONFIG1
    m_total = args.prefill_tokens
    if m_total % world:
        raise ValueError("prefill tokens must split evenly over the ranks")
    m = m_total // world
    epr = cfg.num_experts // world
    keys = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")
    layers = []
    g = torch.Generator(device=dev)
    for l in range(args.prefill_layers):
        # this rank's expert shard of layer l (the same experts on every N) and the shared expert
        g.manual_seed(50_000 + 1_000 * l + rank)
        ex = gptq_experts(g, epr, cfg.hidden, cfg.inter, cfg.group_size, dev)
        local = W4A16Experts.from_gptq(*(ex[k] for k in keys), group_size=cfg.group_size)
        del ex
        g.manual_seed(90_000 + l)
        sh = gptq_experts(g, 1, cfg.hidden, cfg.inter, cfg.group_size, dev)
        gw = (torch.randn(cfg.hidden, generator=g, device=dev) * 0.02).to(torch.bfloat16)
        shared = SharedExpert.from_gptq(*(sh[k][0] for k in keys), gw, group_size=cfg.group_size)
        layers.append(ExpertParallelMoE.for_gpu(local, cfg.num_experts, cfg.top_k, shared=shared, tokens_per_rank=m))
        if l == 0:
            local0, shared0 = local, shared
    g.manual_seed(7_000 + rank)
    x0 = torch.randn((m, cfg.hidden), generator=g, device=dev).to(torch.bfloat16)
    logits = [torch.randn((m, cfg.num_experts), generator=g, device=dev) for _ in range(args.prefill_layers)]

    def step():
        x = x0
        for l, layer in enumerate(layers):
            x = x + layer(x, logits[l])
        return x

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index) as clocks:
        a.record(stream)
        for _ in range(args.prefill_steps):
            step()
        b.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    ms = a.elapsed_time(b)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    layer_ms = ms / args.prefill_steps / args.prefill_layers
    parity = prefill_ep_parity(layers[0], local0, shared0, x0, logits[0], cfg, world, dev)
    flops = 2 * m_total * (cfg.top_k + 1) * (cfg.hidden * 2 * cfg.inter + cfg.inter * cfg.hidden)
    peak, peak_kind = bf16_peak()
    per_gpu_tflops = flops / (layer_ms / 1e3) / world / 1e12
    return {
        "config": f"config4: M={m_total} tokens ({m} per rank), E=256 sharded {epr} per rank, top-8 uniform "
                  f"random routing, {args.prefill_layers} stacked layers with bf16 residual, shared expert at home",
        "n_gpus": world, "scaling": "strong", "steps": args.prefill_steps,
        "layer_ms": round(layer_ms, 4), "tok_s": round(m_total / (layer_ms / 1e3), 1),
        "flops_per_layer": flops,
        "roofline": {"bound": "tensor", "achieved": round(per_gpu_tflops, 2), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(per_gpu_tflops / peak, 4), "peak_source": peak_kind,
                     "note": "useful FLOPs (routed + shared pairs); the kernels also multiply the padding "
                             "columns of each expert's last 128-pair block"},
        "kernel_path": {"prefill": "moe_prefill.cu: 128-pair bf16 tcgen05 tiles (router, align, gather, W1, W2, "
                                   "combine launches)",
                        "decode": "moe_fused.cu: persistent layer kernel, 8-pair int8 tiles"}[
                            layer_path(m, epr, cfg.top_k)],
        "exchange": ("NCCL all_gather of bf16 token rows and int32 global id / fp32 weight lists; one layer call "
                     "on every gathered row (expert_map drops other ranks' pairs in the kernels, shared expert on "
                     "this rank's rows only); NCCL reduce_scatter (sum) of the bf16 partial rows; no host "
                     "synchronisation") if world > 1 else "single rank (no exchange)",
        "parity": parity,
        "clocks": clocks.summary(),
    }


def prefill_ep_parity(layer, local, shared, x, logits, cfg, world: int, dev):
    """Layer 0 of the expert-parallel stack on this rank's tokens against the
    single-GPU decode kernel (exact dequantisation) over all experts, the
    ranks' shards all-gathered into one expert array; max over ranks."""
    import torch

    import mtp_b200
    from mtp_b200.ops import W4A16Experts

    if world > 1:
        blobs = torch.empty((cfg.num_experts, local.expert_bytes), dtype=torch.uint8, device=dev)
        torch.distributed.all_gather_into_tensor(blobs, local.blobs.contiguous())
    else:
        blobs = local.blobs
    full = W4A16Experts(blobs, cfg.num_experts, local.hidden, local.inter, local.group_size, local.layout)
    out = layer(x, logits)
    ref = mtp_b200.moe_layer_w4a16(x, logits, full, cfg.top_k, shared=shared, path="decode")
    o, r = out.double().cpu(), ref.double().cpu()
    err = (o - r).abs()
    rel_l2 = float((o - r).norm() / r.norm().clamp_min(1e-30))
    vals = torch.tensor([rel_l2, float(err.max()) / max(1.0, float(r.abs().max())), float(err.max()),
                         float(r.abs().max())], dtype=torch.float64, device=dev)
    if world > 1:
        torch.distributed.all_reduce(vals, op=torch.distributed.ReduceOp.MAX)
    del blobs, full
    v = vals.tolist()
    return {"rel_l2": round(v[0], 6), "norm_max_abs": round(v[1], 6), "max_abs": round(v[2], 4),
            "max_ref": round(v[3], 3), "rows": int(x.shape[0]) * world,
            "against": "single-GPU decode kernel over all experts (exact dequantisation), layer 0, every row; "
                       "max over ranks",
            "bound": "rel-L2 <= 1e-2 and normalised max-abs <= 2e-2",
            "ok": bool(v[0] <= 1e-2 and v[1] <= 2e-2)}


def config2_choices(layers: int, steps: int, experts: int = 256, k: int = 8, hot: int = 32,
                    stay: float = 0.6, zipf_s: float = 1.1, seed: int = 2, model_seed: int = 2):
    """Synthetic config-2 routing: per layer a Zipf(s) popularity over a
    permutation of the experts (the "model", seeded by `model_seed`); pick j
    of a token at layer l + 1 comes from the layer's 32 most popular experts
    with probability `stay` when pick j at layer l did, else from the whole
    Zipf distribution (distinct picks); the tokens are drawn with `seed`."""
    import numpy as np
    model = np.random.default_rng(model_seed)
    rng = np.random.default_rng(seed)
    ranks = np.arange(1, experts + 1, dtype=np.float64)
    p_all = ranks ** -zipf_s
    p_all /= p_all.sum()
    p_hot = p_all[:hot] / p_all[:hot].sum()
    perms = [model.permutation(experts) for _ in range(layers)]
    out = np.zeros((steps, layers, k), dtype=np.int32)
    for t in range(steps):
        was_hot = rng.random(k) < 0.5
        for l in range(layers):
            picks, hot_flags = [], []
            for j in range(k):
                is_hot = was_hot[j] and rng.random() < stay
                while True:
                    r = rng.choice(hot, p=p_hot) if is_hot else rng.choice(experts, p=p_all)
                    e = int(perms[l][r])
                    if e not in picks:
                        break
                picks.append(e)
                hot_flags.append(r < hot)
            out[t, l] = picks
            was_hot = np.array(hot_flags)
    return out


def transition_tables(train: "np.ndarray", num_experts: int, deltas: int = 4):
    """T[d - 1][l][i][o]: the fraction of the (token, layer l) rows holding
    expert i whose layer l + d row holds expert o, counted on a held-out
    trace (the current -> future expert transition of
    training/baselines.py:22 train_transition_matrix, along the layer axis)."""
    import numpy as np
    steps, layers, k = train.shape
    T = np.zeros((deltas, layers, num_experts, num_experts), dtype=np.float32)
    cnt = np.zeros((layers, num_experts), dtype=np.float32)
    for t in range(steps):
        for l in range(layers):
            cur = train[t, l]
            cnt[l, cur] += 1
            for d in range(1, deltas + 1):
                if l + d < layers:
                    T[d - 1, l][np.ix_(cur, train[t, l + d])] += 1
    return T / np.maximum(cnt, 1)[None, :, :, None]


def run_prefetch(dev, experts, shared, cfg, n_layers: int, steps: int):
    """slot-indirected decode, M = 1, 64 of 256 experts
    resident per layer, 40 layers x 512 decode steps of the synthetic Zipf /
    layer-Markov trace. Every layer call demands its experts (hit = resident
    and copied; a miss is copied in and the layer waits for that copy, so the
    bytes cross the host link once), then an issue policy prefetches:

    * demand: no issue (demand-insert LRU only);
    * layer_transition: expert transition tables layer l -> l + d (d = 1..4)
      learned on a held-out trace; after layer l the top-12 experts of layers
      l + 1 and l + 2 are issued (12: a CPU simulation of the session over
      widths 8-24 gave the best hit rate with most issued copies used);
    * mtp_predictor: the same tables as the weights of one MTP predictor per
      layer (2048 -> 2048 -> 4 x 256, closed form: the hidden state holds the
      layer's experts as a multi-hot, W1 passes it through SiLU, W2 holds the
      four transition tables), run by the predictor kernel after each layer;
      its top-12 ids of the next layers are copied to the host (asynchronously,
      read two layers later) and issued for the layers 3 and 4 ahead of the
      layer that predicted them.

    Hit rate = demand_hit / demand_count with the counter definitions of
    runtime/cache_manager.py:193-263; late-miss and used-per-issued likewise.
    The pinned host store holds 40 x 256 experts (16.7 GB) when the host has
    room, else one 256-expert block that every layer reads (stated)."""
    import numpy as np
    import torch

    import mtp_b200

    e_bytes = experts.expert_bytes
    E, k = experts.num_experts, cfg.top_k
    one = experts.blobs.reshape(E, e_bytes).cpu()
    avail = 0
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable"):
                avail = int(line.split()[1]) * 1024
    except OSError:
        pass
    shared_layers = avail < 2 * n_layers * E * e_bytes
    if shared_layers:
        host = torch.empty((E, e_bytes), dtype=torch.uint8, pin_memory=True)
        host.copy_(one)
    else:
        host = torch.empty((n_layers, E, e_bytes), dtype=torch.uint8, pin_memory=True)
        for l in range(n_layers):
            host[l].copy_(one)
    trace = config2_choices(n_layers, steps, seed=2)
    # held out: the same model (expert popularity per layer), other tokens
    T = transition_tables(config2_choices(n_layers, 512, seed=3, model_seed=2), E)
    x = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(5)).to(torch.bfloat16).to(dev)
    ws = mtp_b200.layer_workspace(1, experts, k, dev)
    out = torch.empty(1, cfg.hidden, dtype=torch.bfloat16, device=dev)
    logits_host = torch.zeros(steps, n_layers, E, dtype=torch.float32)
    for t in range(steps):
        for l in range(n_layers):
            logits_host[t, l, trace[t, l]] = 8.0 + torch.arange(k, dtype=torch.float32) * 0.01
    logits_dev = logits_host.to(dev)
    stream = torch.cuda.current_stream(dev)

    # one closed-form predictor per layer (see the docstring)
    w1 = torch.zeros(cfg.hidden, cfg.hidden, dtype=torch.bfloat16)
    w1[torch.arange(E), torch.arange(E)] = 1.0
    w1 = w1.to(dev)
    preds = []
    for l in range(n_layers):
        w2 = torch.zeros(4 * E, cfg.hidden, dtype=torch.float32)
        for d in range(4):
            w2[d * E:(d + 1) * E, :E] = torch.from_numpy(T[d, l].T)
        preds.append(mtp_b200.MtpPredictor(w1, None, w2.to(torch.bfloat16).to(dev), None, future=4, experts=E))
    hvec = torch.zeros(n_layers, steps, cfg.hidden, dtype=torch.bfloat16)
    for t in range(steps):
        for l in range(n_layers):
            hvec[l, t, torch.from_numpy(trace[t, l]).long()] = 4.0
    hvec = hvec.to(dev)
    pws = preds[0].workspace(1, dev)
    width = 12
    ring = 4
    pids = [torch.empty(1, 4, width, dtype=torch.int32, device=dev) for _ in range(ring)]
    pids_host = [torch.empty(1, 4, width, dtype=torch.int32, pin_memory=True) for _ in range(ring)]
    pev = [torch.cuda.Event() for _ in range(ring)]
    # layer_transition: the issue lists follow from the trace and the tables
    # alone, so they are formed before the timed loop (a C++ runtime forms
    # one in microseconds; numpy's per-layer call overhead would otherwise be
    # what the timing measures)
    trans_issue = {}
    for t in range(steps):
        for l in range(n_layers):
            for d in (1, 2):
                if l + d < n_layers:
                    score = T[d - 1, l][trace[t, l]].sum(axis=0)
                    trans_issue[t, l, d] = np.ascontiguousarray(np.argsort(-score, kind="stable")[:width], dtype=np.int32)

    def policy_run(policy: str):
        sess = mtp_b200.PrefetchSession(n_layers, E, 64, e_bytes, host, device=dev, shared_host_layers=shared_layers)
        views = [sess.layer_views(l) for l in range(n_layers)]
        status = torch.zeros(4, dtype=torch.int32, device=dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        warm = 8
        base = None
        # the host runs at most two layers ahead of the device (events after
        # each layer call), as a decode loop that waits on recent layers does:
        # the session classifies a demand of an in-flight copy as ready-late
        # from the host's view, so an unbounded run-ahead would count copies
        # that land before their layer starts on the device as late
        lev = [torch.cuda.Event() for _ in range(3)]
        g = 0
        for t in range(steps):
            if t == warm:
                torch.cuda.synchronize()
                base = sess.poll()
                status.zero_()
                e0.record(stream)
            for l in range(n_layers):
                ids = trace[t, l]
                if g >= 2:
                    lev[(g - 2) % 3].synchronize()
                sess.demand(l, ids)
                sess.wait(l, ids, stream)
                cache, table, hst = views[l]
                mtp_b200.moe_layer_w4a16(x, logits_dev[t, l].reshape(1, E), experts, k, shared=shared,
                                         slot_table=table, slot_cache=cache, host_store=hst, workspace=ws, out=out,
                                         status=status)
                sess.layer_used(l, stream)
                lev[g % 3].record(stream)
                g += 1
                if policy == "layer_transition":
                    for d in (1, 2):
                        if l + d < n_layers:
                            sess.issue(l + d, trans_issue[t, l, d])
                elif policy == "mtp_predictor":
                    b = l % ring
                    preds[l].predict_topk(hvec[l, t:t + 1], width, ids_out=pids[b], workspace=pws)
                    pids_host[b].copy_(pids[b], non_blocking=True)
                    pev[b].record(stream)
                    if l >= 2:
                        # the prediction made two layers back, read late so the
                        # host does not wait for the device: its deltas 3 and 4
                        # are layers l + 1 and l + 2
                        pb = (l - 2) % ring
                        pev[pb].synchronize()
                        for d in (3, 4):
                            if l - 2 + d < n_layers:
                                sess.issue(l - 2 + d, pids_host[pb][0, d - 1].numpy())
        e1.record(stream)
        torch.cuda.synchronize()
        sess.sync()
        st = sess.poll()
        ms = e0.elapsed_time(e1)
        d = {kk: st[kk] - base[kk] for kk in ("issued_fetch_count", "used_fetch_count", "demand_count",
                                               "demand_hit_count", "demand_miss_count", "ready_late_miss_count",
                                               "evicted_before_use_count", "bytes_copied")}
        timed = steps - warm
        host_served = int(status[0].item())
        sess.close()
        return {"hit_rate": round(d["demand_hit_count"] / max(1, d["demand_count"]), 4),
                "late_miss_rate": round(d["ready_late_miss_count"] / max(1, d["demand_count"]), 4),
                "used_per_issued": round(d["used_fetch_count"] / max(1, d["issued_fetch_count"]), 4),
                "issued_fetch_count": d["issued_fetch_count"],
                "host_served_experts": host_served,
                "tok_s": round(timed / (ms / 1e3), 1), "ms_per_token": round(ms / timed, 3),
                "h2d_GBps": round((d["bytes_copied"] + host_served * e_bytes) / (ms / 1e3) / 1e9, 2),
                "counters": d}

    policies = {p: policy_run(p) for p in ("demand", "layer_transition", "mtp_predictor")}
    best = max(policies, key=lambda p: policies[p]["hit_rate"])
    return {"config": f"config2 slot cache: {n_layers} layers x {steps} steps, 256 experts, 64 slots/layer, M=1, "
                      "Zipf(1.1) popularity + layer Markov (stay 0.6 in top-32); pinned host store "
                      + ("one 256-expert block shared by all layers (host RAM short of 2x the 16.7 GB store)"
                         if shared_layers else f"{n_layers} x 256 experts"),
            "steps_timed": steps - 8, "policies": policies, "hit_rate": policies[best]["hit_rate"],
            "hit_rate_policy": best,
            "reference_hit_rate": {"model_only": 0.478, "measured_copy": 0.406,
                                   "source": "PROGRESS.md:4614-4673: W7900 copy envelope, dolly trace, "
                                             "previous-token transition issue, simulated ready-time queue"},
            "transfer": "every miss is copied into the slot cache on the session's side stream and the layer "
                        "waits for the copy (host bytes cross once); h2d_GBps counts every host byte",
            "timing": "CUDA events on the compute stream around the timed steps; includes the host-side "
                      "session bookkeeping, eager launches and (mtp_predictor) one device-to-host read per layer, "
                      "read two layers late; layer_transition's issue lists are formed before the timed loop; the host "
                      "runs at most two layer calls ahead of the device in every policy"}


def run_predictor(dev, hbm_gbs):
    """the MTP predictor (2048 -> 2048 -> 4 x 256, top-8 per
    future layer) at M = 1, 8, 64. Twelve predictors of distinct weights
    (12 x 12.6 MB, more than L2) run back to back in one CUDA graph, so every
    call streams its weights from HBM; device time per call from CUDA events
    around the graph replays, and GB/s on the weight bytes."""
    import torch

    import mtp_b200
    from mtp_b200.synthetic import CONFIG3, make_predictor, make_predictor_inputs

    cfg = CONFIG3
    copies = 12
    preds = []
    for c in range(copies):
        w1, b1, w2, b2 = (t.to(dev) for t in make_predictor(cfg, seed=c))
        preds.append(mtp_b200.MtpPredictor(w1, b1, w2, b2, future=cfg.future, experts=cfg.experts))
    wbytes = 2 * (cfg.width * cfg.hidden + cfg.future * cfg.experts * cfg.width)
    rows = []
    for m in cfg.tokens:
        h = make_predictor_inputs(cfg, m, seed=m).to(dev)
        ws = preds[0].workspace(m, dev)
        ids = torch.empty(m, cfg.future, cfg.top_k, dtype=torch.int32, device=dev)

        def calls():
            for p in preds:
                p.predict_topk(h, cfg.top_k, ids_out=ids, workspace=ws)

        calls()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            calls()
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (reps * copies)
        gbs = (wbytes + 2 * m * cfg.hidden) / (us / 1e6) / 1e9
        rows.append({"M": m, "us": round(us, 2), "hbm_gbs": round(gbs, 1), "hbm_frac": round(gbs / hbm_gbs, 4),
                     "launches_per_call": 3})
        del g
    # the reference's own architecture at its default size (hidden 2048,
    # width 256, 40 layers, 4 deltas, 256 experts; random weights)
    gen = torch.Generator(device="cpu").manual_seed(11)
    rnd = lambda *shape, s=0.02: (torch.randn(*shape, generator=gen) * s).to(torch.bfloat16).to(dev)
    hr = [mtp_b200.HiddenResidualPredictor(rnd(256, 2048), rnd(256), 1.0 + rnd(256), rnd(256), rnd(40, 256, s=1.0),
                                           rnd(4, 256, s=1.0), rnd(256, 256), rnd(256)) for _ in range(copies)]
    hr_bytes = 2 * (256 * 2048 + 256 * 256 + 40 * 256 + 4 * 256 + 4 * 256)
    hr_rows = []
    for m in cfg.tokens:
        h = make_predictor_inputs(cfg, m, seed=m).to(dev)
        lids = torch.arange(m, dtype=torch.int32, device=dev) % 40
        ws = hr[0].workspace(m, dev)
        ids = torch.empty(m, 4, cfg.top_k, dtype=torch.int32, device=dev)

        def hcalls():
            for p in hr:
                p.predict_topk(h, lids, cfg.top_k, ids_out=ids, workspace=ws)

        hcalls()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            hcalls()
        for _ in range(3):
            g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(10):
            g.replay()
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / (10 * copies)
        hr_rows.append({"M": m, "us": round(us, 2), "launches_per_call": 4})
        del g
    return {"config": "config3 predictor 2048->2048->4x256 bf16, top-8 per future layer; 12 weight copies "
                      "(151 MB > L2) per CUDA graph", "weight_bytes": wbytes, "sweep": rows,
            "hidden_residual": {"config": "reference HiddenResidualExpertPredictor shape: hidden 2048 -> width 256 "
                                          "-> LayerNorm + layer/delta embeddings -> classifier 256 experts, 4 deltas, "
                                          "top-8; 12 weight copies per CUDA graph (weights fit L2: latency-bound)",
                                "weight_bytes": hr_bytes, "sweep": hr_rows}}


def run_e2e(args, layers, cfg, sweep, dev, state):
    """Same metric through the public call with pinned host inputs: every
    step copies all of its inputs (hidden states + router logits of every
    layer call, one H2D per M) from pinned host memory, runs the layer calls,
    and reads every output back (one D2H per M). Timed two ways: the step's
    copies and calls captured once in a CUDA graph and replayed (how a
    serving loop runs a decode step, the reference's vLLM included), and
    eager (every call launched from Python)."""
    import torch

    import mtp_b200

    steps = max(1, min(args.steps, args.e2e_steps))
    host = {}
    for m in sweep:
        # [L, m, ...] contiguous so that one copy moves every layer call's rows
        hx = torch.stack([t.cpu() for t in state[m]["x"]]).pin_memory()
        hl = torch.stack([t.cpu() for t in state[m]["logits"]]).pin_memory()
        ho = torch.empty((args.layers, m, cfg.hidden), dtype=torch.bfloat16).pin_memory()
        dx, dl = torch.empty_like(hx, device=dev), torch.empty_like(hl, device=dev)
        do = torch.empty_like(ho, device=dev)
        host[m] = (hx, hl, ho, dx, dl, do)

    # copies on their own stream: every M's inputs go in at the start of the
    # step (in sweep order), each M's outputs come back while the next M runs
    copy = torch.cuda.Stream(dev)
    ev_in = {m: torch.cuda.Event() for m in sweep}
    ev_out = {m: torch.cuda.Event() for m in sweep}

    def one_step():
        cur = torch.cuda.current_stream(dev)
        copy.wait_stream(cur)
        with torch.cuda.stream(copy):
            for m in sweep:
                hx, hl, ho, dx, dl, do = host[m]
                dx.copy_(hx, non_blocking=True)
                dl.copy_(hl, non_blocking=True)
                ev_in[m].record(copy)
        for m in sweep:
            hx, hl, ho, dx, dl, do = host[m]
            cur.wait_event(ev_in[m])
            for l in range(args.layers):
                w, s = layers[l]
                mtp_b200.moe_layer_w4a16(dx[l], dl[l], w, cfg.top_k, shared=s, out=do[l], workspace=state[m]["ws"][l])
            ev_out[m].record(cur)
            copy.wait_event(ev_out[m])
            with torch.cuda.stream(copy):
                ho.copy_(do, non_blocking=True)
        cur.wait_stream(copy)

    def timed(run):
        stream = torch.cuda.current_stream(dev)
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(stream)
        for _ in range(steps):
            run()
        b.record(stream)
        torch.cuda.synchronize()
        return a.elapsed_time(b)

    for _ in range(2):
        one_step()
    torch.cuda.synchronize()
    eager_ms = timed(one_step)
    side = torch.cuda.Stream(dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=side):
        one_step()
    torch.cuda.synchronize()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    graph_ms = timed(g.replay)
    del g
    tok = sum(m * args.layers for m in sweep) * steps
    h2d = sum(m * cfg.hidden * 2 + m * cfg.num_experts * 4 for m in sweep) * args.layers
    d2h = sum(m * cfg.hidden * 2 for m in sweep) * args.layers
    return {"value": round(tok / (graph_ms / 1e3), 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "steps": steps,
            "path": "mtp_b200.moe_layer_w4a16 per layer call (ctypes C-ABI); every step copies its inputs from "
                    "pinned host memory (one H2D per M for all layer calls) and reads every output back (one D2H "
                    "per M), the copies on a second stream overlapping the layer calls of other M; the step's copies "
                    "and calls captured in one CUDA graph and replayed every step",
            "eager_value": round(tok / (eager_ms / 1e3), 1),
            "eager_path": "the same calls launched eagerly from Python every step"}


def run_reference(args, rank: int):
    """``--impl reference``: the reference CPU path alone, rank 0 only, on the
    GPU arm's workload (the config-1 M sweep) and metric."""
    if rank != 0:
        return None
    ref = CpuReference()
    per_step = min(8.0, max(0.5, 120.0 / max(1, args.steps + args.warmup)))
    ref.warm()
    for _ in range(args.warmup):
        ref.run(per_step)
    ref.times = {m: [] for m in ref.tokens}
    for _ in range(args.steps):
        ref.run(per_step)
    res = ref.summary()
    value = res["value"]
    return {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic", "impl": "reference",
        "config": {"workload": "config1 decode sweep: W4A16 MoE layer E=256 H=2048 I=512 top-8 + shared expert, "
                               "GPTQ int4 g128 (reference CPU torch path, weights dequantised once)",
                   "tokens": list(ref.tokens)},
        "sweep": [{"M": int(m), "tok_s": v} for m, v in res["per_m_tok_s"].items()],
        "cpu_baseline": {"value": round(value, 2), "unit": UNIT, "cores": res["cores"], "kind": res["kind"],
                         "sample": res["sample"]},
        "e2e": {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mtp_b200", choices=["mtp_b200", "reference"])
    ap.add_argument("--layers", type=int, default=16)
    ap.add_argument("--sweep", default=",".join(str(m) for m in SWEEP))
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-predictor", action="store_true")
    ap.add_argument("--no-prefetch", action="store_true")
    ap.add_argument("--prefetch-layers", type=int, default=40)
    ap.add_argument("--prefetch-steps", type=int, default=512)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-prefill", action="store_true")
    ap.add_argument("--prefill-tokens", type=int, default=8192)
    ap.add_argument("--prefill-layers", type=int, default=40)
    ap.add_argument("--prefill-steps", type=int, default=3)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        res = run_reference(args, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    if world > 1:
        import datetime

        import torch
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", 0)))
        # NVLink SHARP off: the exchange here is all_to_all (no in-switch
        # reduction to gain), and a rank that dies while bound to an NVLink
        # multicast object can fault its peers' GPUs.
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # stdout carries only the JSON line
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    res = run_gpu(args, rank, world)
    if rank == 0 and world == 1 and not args.no_cpu:
        # on the host cores of a one-GPU run only (other ranks would compete
        # for the same cores)
        cb = cpu_reference(seconds=args.cpu_seconds)
        per_m = cb.pop("per_m_tok_s")
        res["cpu_baseline"] = cb
        for row in res.get("sweep", []):
            row["cpu_tok_s"] = per_m.get(str(row["M"]))
    if world > 1:
        import torch
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    if rank == 0:
        print(json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
