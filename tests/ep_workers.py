"""Rank bodies for the expert-parallel tests (spawned processes import them).

CPU ranks (gloo): the exchange of :class:`mtp_b200.ExpertParallelMoE` with the
oracle as the local expert compute, checked against the single-process oracle
layer on the same tokens. GPU ranks (NCCL): the same exchange around the CUDA
layer kernel, checked against the one-GPU layer over all experts.
"""
from __future__ import annotations

import datetime
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

KEYS = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")


def _init(backend: str, rank: int, world: int, port: int):
    import os

    import torch.distributed as dist
    # NVLink SHARP off: a rank that dies while its memory is bound to an NVLink
    # multicast object can fault the other ranks' GPUs, and the test harness
    # ends ranks that do not exit in time.
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))


def cpu_rank(rank: int, world: int, port: int, cfg: dict, queue):
    """Oracle experts on CPU; every rank checks its own tokens."""
    import numpy as np
    import torch
    import torch.distributed as dist
    import torch.nn.functional as F

    from mtp_b200.ep import ExpertParallelMoE
    from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
    from oracle import layer as olayer
    from oracle import router as orouter

    try:
        _init("gloo", rank, world, port)
        c = LayerConfig(num_experts=cfg["E"], hidden=cfg["H"], inter=cfg["I"], top_k=cfg["k"],
                        group_size=cfg["G"], shared=cfg["shared"])
        experts, shared = make_layer(c, seed=3, random_zeros=True)
        dq = {e: olayer.dequant_expert(*(experts[kk][e] for kk in KEYS), group_size=c.group_size)
              for e in range(c.num_experts)}
        epr = c.num_experts // world
        m = cfg["M"][rank]
        x, logits = make_inputs(c, max(m, 1), seed=100 + rank)
        x, logits = x[:m], logits[:m]
        if cfg.get("skip_rank") is not None:
            # no token of any rank picks the experts of this rank
            lo = cfg["skip_rank"] * epr
            logits[:, lo:lo + epr] = -1e4

        def local_fn(rows, ids, w, f32=False):
            out = torch.zeros(rows.shape, dtype=torch.float32)
            xf = rows.float()
            for r in range(rows.shape[0]):
                for j in range(ids.shape[1]):
                    e = int(ids[r, j])
                    if e >= 0:
                        out[r] += float(w[r, j]) * olayer.expert_mlp(xf[r:r + 1], *dq[rank * epr + e])[0]
            return out if f32 else out.to(torch.bfloat16)

        def router_fn(lg, k):
            w, ids, _ = orouter.topk_softmax(lg.numpy(), k, True)
            return torch.from_numpy(w), torch.from_numpy(ids.astype(np.int32))

        shared_fn = None
        if shared is not None:
            sdq = olayer.dequant_expert(*(shared[kk] for kk in KEYS), group_size=c.group_size)
            gw = shared["gate_weight"].float()

            def shared_fn(xx):
                xf = xx.float()
                return (torch.sigmoid(F.linear(xf, gw[None]))[:, :1] * olayer.expert_mlp(xf, *sdq)).to(torch.bfloat16)

        layer = ExpertParallelMoE(c.num_experts, c.top_k, c.hidden, local_fn, router_fn, shared_fn,
                                  tokens_per_rank=m if cfg.get("gather") else None)
        out = layer(x, logits)
        w, ids, _ = orouter.topk_softmax(logits.numpy(), c.top_k, True)
        if m:
            o = olayer.MoeLayerOracle(experts, shared, group_size=c.group_size)
            ref = o.moe_tokens(x.float(), torch.as_tensor(ids), torch.as_tensor(w))
            res = (olayer.relative_l2(out.float(), ref), olayer.normalized_max_abs(out.float(), ref))
        else:
            res = (0.0, 0.0) if out.shape == (0, c.hidden) else (1.0, 1.0)
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, res, None))
    except Exception as exc:  # reported to the test, which fails on it
        queue.put((rank, None, repr(exc)))


def gpu_rank(rank: int, world: int, port: int, cfg: dict, queue):
    """CUDA layer kernel on each rank's expert shard (one GPU per rank)."""
    import torch
    import torch.distributed as dist

    try:
        torch.cuda.set_device(rank)
        _init("nccl", rank, world, port)
        import mtp_b200
        from mtp_b200 import ExpertParallelMoE, SharedExpert, W4A16Experts
        from mtp_b200.synthetic import LayerConfig, make_inputs, make_layer
        from oracle import layer as olayer

        dev = torch.device("cuda", rank)
        c = LayerConfig(num_experts=cfg["E"], hidden=cfg["H"], inter=cfg["I"], top_k=cfg["k"],
                        group_size=cfg["G"], shared=True)
        experts, shared = make_layer(c, seed=5, device=dev)
        full = W4A16Experts.from_gptq(*(experts[kk] for kk in KEYS), group_size=c.group_size)
        sh = SharedExpert.from_gptq(*(shared[kk] for kk in KEYS), shared["gate_weight"], group_size=c.group_size)
        layer = ExpertParallelMoE.for_gpu(full.shard(rank, world), c.num_experts, c.top_k, shared=sh,
                                          tokens_per_rank=cfg["M"] if cfg.get("gather") else None)
        x, logits = make_inputs(c, cfg["M"], seed=200 + rank, device=dev)
        out = layer(x, logits)
        ref = mtp_b200.moe_layer_w4a16(x, logits, full, c.top_k, shared=sh)
        torch.cuda.synchronize()
        res = (olayer.relative_l2(out.float().cpu(), ref.float().cpu()),
               olayer.normalized_max_abs(out.float().cpu(), ref.float().cpu()))
        dist.barrier()
        dist.destroy_process_group()
        queue.put((rank, res, None))
    except Exception as exc:
        queue.put((rank, None, repr(exc)))
