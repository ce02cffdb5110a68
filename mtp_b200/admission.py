"""Prefetch admission: priority tiers over predicted experts and the
descriptors that feed the prefetch session, in priority order under a budget.

Semantics of the reference's premap descriptor build
(runtime/premap.py:78-192, with select_topk_mask / novel_mtp_extra_mask of
admission.py:129-160); the tier names and the descriptor order are kept the
same so descriptor lists compare one to one:

  P2  transition top-16 (protected, highest predicted value)
  P3  transition top 17 .. transition_topk (protected)
  P4  the first four MTP candidates (of the MTP top-mtp_topk, in score
      order) outside the transition top-transition_topk ("novel extras")
  P5  the next novel extras, up to max_extra

Scores are [tokens, future, layers, experts] (one row per token and future
delta). A descriptor is one (sample, layer, expert) over all tokens and
deltas of the sample; an expert in several tiers keeps the highest (lowest
number); its score is the tier's max over the rows that selected it (or mean
/ sum); descriptors sort by (sample, layer, priority, -score, expert). The
operations are torch tensor operations, so the masks build on the device the
scores live on (the predictor's logits stay on the GPU until the descriptor
list is taken).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class PrefetchDescriptor:
    sample: int
    layer: int
    expert: int
    priority: int
    source: str
    score: float


def select_topk_mask(scores: torch.Tensor, k: int) -> torch.Tensor:
    """True at the top-k entries along the last (expert) axis."""
    k = min(max(0, int(k)), scores.shape[-1])
    mask = torch.zeros(scores.shape, dtype=torch.bool, device=scores.device)
    if k:
        mask.scatter_(-1, torch.topk(scores.float(), k, dim=-1).indices, True)
    return mask


def novel_extra_mask(base: torch.Tensor, mtp_scores: torch.Tensor, mtp_topk: int, max_extra: int) -> torch.Tensor:
    """Up to max_extra of the MTP top-mtp_topk (in score order) outside base."""
    max_extra = max(0, int(max_extra))
    mtp_topk = min(max(0, int(mtp_topk)), mtp_scores.shape[-1])
    out = torch.zeros_like(base)
    if not max_extra or not mtp_topk:
        return out
    s = mtp_scores.float()
    s = s.masked_fill(~torch.isfinite(s), -float("inf"))
    ranked = torch.topk(s, mtp_topk, dim=-1).indices
    novel = ~base.gather(-1, ranked)
    keep = novel & (novel.to(torch.int32).cumsum(-1) <= max_extra)
    out.scatter_(-1, ranked, keep)
    return out & ~base


def priority_masks(transition: torch.Tensor, mtp: torch.Tensor, *, transition_topk: int = 32, mtp_topk: int = 64,
                   max_extra: int = 8) -> dict[str, torch.Tensor]:
    head = select_topk_mask(transition, min(16, int(transition_topk)))
    full = select_topk_mask(transition, transition_topk)
    x_head = novel_extra_mask(full, mtp, mtp_topk, min(4, int(max_extra)))
    x_all = novel_extra_mask(full, mtp, mtp_topk, max_extra)
    return {
        "P2_transition_top16": head,
        f"P3_transition_top17_to_{int(transition_topk)}": full & ~head,
        "P4_mtp_extra1_to_4": x_head,
        f"P5_mtp_extra5_to_{max(int(max_extra), 4)}": x_all & ~x_head,
    }


def _reduce(scores: torch.Tensor, mask: torch.Tensor, how: str) -> torch.Tensor:
    if how == "max":
        return scores.float().masked_fill(~mask, -float("inf")).amax(dim=(0, 1)).clamp_min(0.0)
    masked = scores.float().masked_fill(~mask, 0.0).sum(dim=(0, 1))
    if how == "sum":
        return masked
    if how == "mean":
        return masked / mask.float().sum(dim=(0, 1)).clamp_min(1.0)
    raise ValueError(f"unknown score reduction {how!r}")


def premap_descriptors(transition: torch.Tensor, mtp: torch.Tensor, sample_of_token: torch.Tensor, *,
                       transition_topk: int = 32, mtp_topk: int = 64, max_extra: int = 8,
                       reduce: str = "max") -> list[PrefetchDescriptor]:
    """Deduplicated, priority-ordered descriptors (see the module docstring)."""
    if transition.shape != mtp.shape or transition.dim() != 4:
        raise ValueError("transition and mtp scores must both be [tokens, future, layers, experts]")
    if sample_of_token.numel() != transition.shape[0]:
        raise ValueError("one sample index per token")
    masks = priority_masks(transition, mtp, transition_topk=transition_topk, mtp_topk=mtp_topk, max_extra=max_extra)
    tiers = [(name, int(name[1]), src, sc) for name, src, sc in zip(
        masks, ("transition_head", "transition_tail", "mtp_token_extra_head", "mtp_token_extra_tail"),
        (transition, transition, mtp, mtp))]
    out: list[PrefetchDescriptor] = []
    samples = sample_of_token.to(torch.long).cpu()
    for s in torch.unique(samples).tolist():
        rows = (samples == s).to(transition.device)
        claimed = torch.zeros(transition.shape[2:], dtype=torch.bool, device=transition.device)
        for name, prio, src, sc in tiers:
            m = masks[name][rows]
            le = m.any(dim=(0, 1)) & ~claimed
            if not bool(le.any()):
                continue
            red = _reduce(sc[rows], m, reduce)
            layers, experts = torch.nonzero(le, as_tuple=True)
            vals = red[layers, experts].tolist()
            out += [PrefetchDescriptor(int(s), int(l), int(e), prio, src, float(v))
                    for l, e, v in zip(layers.tolist(), experts.tolist(), vals)]
            claimed |= le
    out.sort(key=lambda d: (d.sample, d.layer, d.priority, -d.score, d.expert))
    return out


def apply_budget(descriptors: list[PrefetchDescriptor], *, per_layer: int | None = None,
                 total: int | None = None, max_priority: int = 5) -> list[PrefetchDescriptor]:
    """The descriptors the issue path admits: tiers up to max_priority, at most
    per_layer per (sample, layer) and total overall, best first (the input
    order is already priority, then score)."""
    kept, per = [], {}
    for d in descriptors:
        if d.priority > max_priority:
            continue
        key = (d.sample, d.layer)
        if per_layer is not None and per.get(key, 0) >= per_layer:
            continue
        if total is not None and len(kept) >= total:
            break
        per[key] = per.get(key, 0) + 1
        kept.append(d)
    return kept


def issue_descriptors(session, descriptors: list[PrefetchDescriptor]) -> int:
    """Issue admitted descriptors to a PrefetchSession in order (one issue
    call per layer run); returns the number of copies started."""
    issued, i = 0, 0
    while i < len(descriptors):
        j = i
        while j < len(descriptors) and descriptors[j].layer == descriptors[i].layer:
            j += 1
        issued += session.issue(descriptors[i].layer, [d.expert for d in descriptors[i:j]])
        i = j
    return issued
