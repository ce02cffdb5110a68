"""Expert-parallel W4A16 MoE layer for prefill: experts sharded across the
ranks of a process group, tokens dispatched to the ranks that own their
experts and the partial outputs combined back, one all-to-all each way.

Rank g owns the experts [g * E / G, (g + 1) * E / G). A token's pairs on
another rank reach it as local expert ids with every foreign pair marked -1,
which is the ``expert_map`` convention of the kernels this path replaces
(vLLM ``fused_moe`` with ``expert_map``; the reference consumes it at
tracing/vllm_wna16_group_plan.py:87-95, and reads the EP map at
tracing/vllm_router_trace.py:7661-7689). Each rank routes its own tokens, then

Two exchange forms:

* ``tokens_per_rank`` given (every rank holds the same number of tokens, as a
  prefill chunk does): no host synchronisation and fixed message sizes.
  1. all-gather the token rows and their global (id, weight) lists;
  2. one layer call on every gathered row (``gathered_fn``): on the GPU the
     kernels take the global ids through an ``expert_map`` (other ranks'
     experts -> -1) and add the gated shared expert to this rank's own rows
     only, writing bf16 partial rows;
  3. reduce-scatter (sum) of the partials back to the home ranks (bf16 on the
     GPU: each rank's partial is rounded once to bf16 before the sum, and the
     sum once more; fp32 partials where the backend has no bf16 reduction).
  The bytes moved equal those of an all-to-all padded to the per-rank
  capacity a fixed-size exchange needs (a token may use every rank).
* otherwise (ranks with different token counts): a deduplicated all-to-all.
  1. dispatch: every token row goes once to each rank that owns at least one
     of its experts, with its k local ids and weights (weight 0 and id -1 for
     pairs owned elsewhere); the split sizes are exchanged first (host syncs);
  2. local compute: the layer kernel on the received rows (no router, no
     shared expert), each row becoming the weighted sum over its local
     experts, rounded to bf16 for the return trip;
  3. combine: the partial rows go back to their home rank, which adds them in
     fp32 to its shared-expert output and rounds once to bf16 (one more bf16
     rounding per remote rank than the single-device layer).

The exchanges run on ``torch.distributed`` (NCCL over NVLink on the GPU, gloo
in the CPU tests). Row payloads travel as bf16 bits in int32 views (two values
per word; H is even), the id / weight lists as one int32 tensor. The decode
configs do not shard: they run one replica per GPU.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable

import torch
import torch.distributed as dist


@dataclass
class DispatchPlan:
    """Send side of one dispatch: rows ordered by destination rank, then token."""

    tokens: torch.Tensor        # [S] int64 source token of each sent row
    counts: list[int]           # rows per destination rank (sums to S)
    local_ids: torch.Tensor     # [S, k] int32 destination-local expert id, -1 if owned elsewhere
    local_weights: torch.Tensor  # [S, k] fp32 routing weight, 0 where the id is -1


def experts_per_rank(num_experts: int, world: int) -> int:
    if world < 1 or num_experts % world:
        raise ValueError(f"{num_experts} experts do not shard evenly over {world} ranks")
    return num_experts // world


def plan_dispatch(topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
                  world: int) -> DispatchPlan:
    """Rows to send per destination: token t goes to rank d once when any of
    its top-k experts lives on d. Ids outside [0, E) are never sent."""
    if topk_ids.shape != topk_weights.shape or topk_ids.dim() != 2:
        raise ValueError("topk_ids and topk_weights must both be [M, k]")
    epr = experts_per_rank(num_experts, world)
    m, k = topk_ids.shape
    ids = topk_ids.long()
    valid = (ids >= 0) & (ids < num_experts)
    dest = torch.where(valid, ids // epr, torch.full_like(ids, world))   # world = nowhere
    sends = torch.zeros((m, world + 1), dtype=torch.bool, device=ids.device)
    sends.scatter_(1, dest, True)
    sends = sends[:, :world]
    # (destination, token) pairs in destination-major, token-ascending order
    pairs = sends.t().nonzero()
    d_of_row, tokens = pairs[:, 0], pairs[:, 1]
    counts = torch.bincount(d_of_row, minlength=world).tolist()
    row_ids = ids[tokens]
    mine = (dest[tokens] == d_of_row[:, None])
    local_ids = torch.where(mine, row_ids - d_of_row[:, None] * epr, torch.full_like(row_ids, -1))
    local_w = torch.where(mine, topk_weights[tokens].float(), torch.zeros_like(topk_weights[tokens].float()))
    return DispatchPlan(tokens, counts, local_ids.to(torch.int32).contiguous(), local_w.contiguous())


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def _all_to_all(out: torch.Tensor, inp: torch.Tensor, out_splits: list[int], in_splits: list[int], group,
                world: int):
    if world == 1:
        out.copy_(inp)
    else:
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=group)


def _all_gather(out: torch.Tensor, inp: torch.Tensor, group, world: int):
    """Rank-ordered concatenation along dim 0 (NCCL all_gather_into_tensor;
    the list form on backends without it)."""
    if world == 1:
        out.copy_(inp)
    elif inp.device.type == "cuda":
        dist.all_gather_into_tensor(out, inp, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), inp, group=group)


def _all_gather_many(pairs, group, world: int, device):
    """Several rank-ordered all-gathers, one call each. (torch's coalescing
    manager would make them one NCCL launch, but it blocked the host for the
    whole exchange in a measurement on two B200s: 1.1 ms per layer against
    0.6 ms with plain calls.)"""
    for out, inp in pairs:
        _all_gather(out, inp, group, world)


def _reduce_scatter_sum(out: torch.Tensor, inp: torch.Tensor, group, world: int):
    """out = sum over ranks of this rank's dim-0 chunk of inp (NCCL
    reduce_scatter_tensor; all_reduce then slice on backends without it)."""
    if world == 1:
        out.copy_(inp)
    elif inp.device.type == "cuda":
        dist.reduce_scatter_tensor(out, inp, group=group)
    else:
        dist.all_reduce(inp, group=group)
        out.copy_(inp.chunk(world)[dist.get_rank(group)])


def _exchange_counts(counts: list[int], device, group, world: int) -> list[int]:
    if world == 1:
        return list(counts)
    send = torch.tensor(counts, dtype=torch.int64, device=device)
    recv = torch.empty_like(send)
    dist.all_to_all_single(recv, send, group=group)
    return recv.tolist()


class ExpertParallelMoE:
    """One expert-parallel MoE layer on this rank.

    ``local_fn(rows, ids, weights, f32=False)`` computes the received rows:
    bf16 [R, H], int32 [R, k] local ids (-1 = skip), fp32 [R, k] weights ->
    [R, H] (bf16, or fp32 with ``f32=True``).
    ``router_fn(logits, k)`` returns (weights fp32 [M, k], ids int32 [M, k]),
    ``shared_fn(x)`` the gated shared-expert output bf16 [M, H] (or None).
    :meth:`for_gpu` wires them to the CUDA kernels; the tests inject CPU
    versions to check the exchange on gloo ranks. Without an initialised
    process group (or in a group of one) the layer runs as a single rank that
    owns every expert; ``single_fn(x, logits)``, when given, then computes the
    whole layer in one call (no dispatch bookkeeping). With ``tokens_per_rank``
    every call must bring exactly that many tokens and the exchange is the
    all-gather / reduce-scatter form (no host synchronisation)."""

    def __init__(self, num_experts: int, top_k: int, hidden: int, local_fn: Callable,
                 router_fn: Callable, shared_fn: Callable | None = None, group=None,
                 single_fn: Callable | None = None, tokens_per_rank: int | None = None,
                 gathered_fn: Callable | None = None):
        self.world, self.rank = _world(group)
        self.num_experts = num_experts
        self.epr = experts_per_rank(num_experts, self.world)
        self.top_k = top_k
        self.hidden = hidden
        self.local_fn = local_fn
        self.router_fn = router_fn
        self.shared_fn = shared_fn
        self.group = group
        self.single_fn = single_fn
        self.tokens_per_rank = tokens_per_rank
        # gathered_fn(rows, global_ids, weights, home) -> partial rows [n*m, H]
        # (bf16 or fp32): this rank's experts on every gathered row, plus the
        # shared expert on rows [home[0], home[1]); by default from local_fn
        # and shared_fn with the foreign ids masked here
        self.gathered_fn = gathered_fn or self._gathered_from_local

    @classmethod
    def for_gpu(cls, local_experts, num_experts: int, top_k: int, shared=None, renormalize: bool = True,
                group=None, zero_mode: str = "raw", tokens_per_rank: int | None = None) -> "ExpertParallelMoE":
        """``local_experts``: this rank's shard (``W4A16Experts.shard``)."""
        from . import _lib
        from .ops import layer_path, layer_workspace, moe_layer_w4a16, prefill_workspace, topk_softmax

        cache = {}

        def workspace(m, dev, path):
            # one workspace per path, grown on demand: the decode one is
            # zero-filled once and every call leaves its counters zero, so
            # calls of any size up to its own can reuse it; the prefill one
            # keeps nothing between calls
            size = _lib.prefill_workspace_bytes if path == "prefill" else _lib.layer_workspace_bytes
            need = size(m, local_experts.num_experts, top_k, local_experts.hidden, local_experts.inter)
            ws = cache.get(path)
            if ws is None or ws.numel() < need or ws.device != dev:
                make = prefill_workspace if path == "prefill" else layer_workspace
                cache[path] = ws = make(m, local_experts, top_k, dev)
            return ws

        def local_fn(rows, ids, weights, f32=False):
            m = rows.shape[0]
            path = layer_path(m, local_experts.num_experts, top_k)
            out32 = torch.empty((m, rows.shape[1]), dtype=torch.float32, device=rows.device) if f32 else None
            out = moe_layer_w4a16(rows, None, local_experts, top_k, topk_weights=weights, topk_ids=ids,
                                  zero_mode=zero_mode, workspace=workspace(m, rows.device, path), path=path,
                                  out_f32=out32)
            return out32 if f32 else out

        def router_fn(logits, k):
            w, ids, _ = topk_softmax(logits, k, renormalize)
            return w, ids

        shared_fn = None
        if shared is not None:
            def shared_fn(x):
                m = x.shape[0]
                none_w = torch.zeros((m, top_k), dtype=torch.float32, device=x.device)
                none_ids = torch.full((m, top_k), -1, dtype=torch.int32, device=x.device)
                # the shared expert alone: m pairs on one expert
                path = layer_path(m, 1, 1)
                return moe_layer_w4a16(x, None, local_experts, top_k, shared=shared, topk_weights=none_w,
                                       topk_ids=none_ids, zero_mode=zero_mode,
                                       workspace=workspace(m, x.device, path), path=path)

        def single_fn(x, logits):
            m = x.shape[0]
            path = layer_path(m, local_experts.num_experts, top_k)
            return moe_layer_w4a16(x, logits, local_experts, top_k, renormalize, shared=shared, zero_mode=zero_mode,
                                   workspace=workspace(m, x.device, path), path=path)

        world, rank = _world(group)
        epr = experts_per_rank(num_experts, world)
        maps = {}

        def gathered_fn(rows, gids, gweights, home):
            # global ids straight into the kernels: expert_map drops other
            # ranks' pairs, shared_rows puts the shared expert on the home rows
            dev = rows.device
            emap = maps.get(dev)
            if emap is None:
                g = torch.arange(num_experts, dtype=torch.int32, device=dev)
                lo = rank * epr
                emap = maps[dev] = torch.where((g >= lo) & (g < lo + epr), g - lo, torch.full_like(g, -1))
            m = rows.shape[0]
            path = layer_path(m, local_experts.num_experts, top_k)
            return moe_layer_w4a16(rows, None, local_experts, top_k, shared=shared if home[1] > home[0] else None,
                                   topk_weights=gweights, topk_ids=gids, zero_mode=zero_mode,
                                   workspace=workspace(m, dev, path), path=path, expert_map=emap,
                                   shared_rows=home if shared is not None and home[1] > home[0] else None)

        return cls(num_experts, top_k, local_experts.hidden, local_fn, router_fn, shared_fn, group, single_fn,
                   tokens_per_rank, gathered_fn)

    def forward(self, x: torch.Tensor, router_logits: torch.Tensor) -> torch.Tensor:
        """x bf16 [M, H] and router_logits fp32 [M, E] of this rank's tokens -> bf16 [M, H]."""
        if x.dim() != 2 or x.shape[1] != self.hidden or x.dtype != torch.bfloat16:
            raise ValueError(f"x must be bf16 [M, {self.hidden}]")
        if router_logits.shape != (x.shape[0], self.num_experts) or router_logits.dtype != torch.float32:
            raise ValueError(f"router_logits must be fp32 [M, {self.num_experts}]")
        m, h, k = x.shape[0], self.hidden, self.top_k
        dev = x.device
        if self.world == 1 and self.single_fn is not None and m > 0:
            return self.single_fn(x, router_logits)
        weights, ids = self.router_fn(router_logits, k)
        if self.tokens_per_rank is not None:
            if m != self.tokens_per_rank:
                raise ValueError(f"this layer exchanges {self.tokens_per_rank} tokens per rank, got {m}")
            return self._forward_gathered(x, ids, weights)
        plan = plan_dispatch(ids, weights, self.num_experts, self.world)
        recv_counts = _exchange_counts(plan.counts, dev, self.group, self.world)
        r = sum(recv_counts)
        # dispatch: token rows (bf16 bits) and the id | weight lists
        send_rows = x[plan.tokens].view(torch.int32)
        recv_rows = torch.empty((r, h // 2), dtype=torch.int32, device=dev)
        _all_to_all(recv_rows, send_rows, recv_counts, plan.counts, self.group, self.world)
        send_meta = torch.cat([plan.local_ids, plan.local_weights.view(torch.int32)], dim=1)
        recv_meta = torch.empty((r, 2 * k), dtype=torch.int32, device=dev)
        _all_to_all(recv_meta, send_meta, recv_counts, plan.counts, self.group, self.world)
        # local experts on the received rows
        if r > 0:
            y = self.local_fn(recv_rows.view(torch.bfloat16), recv_meta[:, :k].contiguous(),
                              recv_meta[:, k:].contiguous().view(torch.float32))
        else:
            y = torch.empty((0, h), dtype=torch.bfloat16, device=dev)
        # combine: partial rows back to their home rank, summed in fp32
        back = torch.empty((len(plan.tokens), h // 2), dtype=torch.int32, device=dev)
        _all_to_all(back, y.contiguous().view(torch.int32), plan.counts, recv_counts, self.group, self.world)
        acc = torch.zeros((m, h), dtype=torch.float32, device=dev)
        if self.shared_fn is not None and m > 0:
            acc += self.shared_fn(x).float()
        acc.index_add_(0, plan.tokens, back.view(torch.bfloat16).float())
        return acc.to(torch.bfloat16)

    def _gathered_from_local(self, rows: torch.Tensor, gids: torch.Tensor, gweights: torch.Tensor,
                             home: tuple[int, int]) -> torch.Tensor:
        """The default gathered_fn: foreign ids masked to -1 here, local_fn in
        fp32 on every row, shared_fn on the home rows."""
        lo = self.rank * self.epr
        mine = (gids >= lo) & (gids < lo + self.epr)
        lids = torch.where(mine, gids - lo, torch.full_like(gids, -1)).contiguous()
        lw = torch.where(mine, gweights, torch.zeros((), device=gweights.device)).contiguous()
        part = self.local_fn(rows, lids, lw, f32=True).float().contiguous()
        if self.shared_fn is not None and home[1] > home[0]:
            part[home[0]:home[1]] += self.shared_fn(rows[home[0]:home[1]].contiguous()).float()
        return part

    def _forward_gathered(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        """All-gather rows and lists, this rank's experts on every row and
        the shared expert on the home rows (gathered_fn), reduce-scatter of
        the partial rows."""
        m, h, k, n = x.shape[0], self.hidden, self.top_k, self.world
        dev = x.device
        rows = torch.empty((n * m, h // 2), dtype=torch.int32, device=dev)
        gids = torch.empty((n * m, k), dtype=torch.int32, device=dev)
        gw = torch.empty((n * m, k), dtype=torch.float32, device=dev)
        _all_gather_many([(rows, x.contiguous().view(torch.int32)), (gids, ids.to(torch.int32).contiguous()),
                          (gw, weights.float().contiguous())], self.group, n, dev)
        home = (self.rank * m, self.rank * m + m)
        part = self.gathered_fn(rows.view(torch.bfloat16), gids, gw, home).contiguous()
        if part.dtype == torch.bfloat16 and dev.type != "cuda":
            part = part.float()  # CPU backends reduce fp32
        out = torch.empty((m, h), dtype=part.dtype, device=dev)
        _reduce_scatter_sum(out, part, self.group, n)
        return out if out.dtype == torch.bfloat16 else out.to(torch.bfloat16)

    __call__ = forward
