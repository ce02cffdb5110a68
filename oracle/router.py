"""Router softmax / top-k / renormalise, restated in numpy fp32.

Test infrastructure (see ``oracle/__init__.py``).

Reference forms:
  * vLLM ``topk_softmax`` as the reference restates it for CPU use,
    src/mtp_expert_prefetch/tracing/vllm_router_trace.py:4201-4227:
    ``softmax(logits.float())`` -> ``topk`` (descending) -> optional
    ``v / v.sum().clamp_min(1e-20)``; ``token_expert_indices`` = arange(k).
  * ``MtpExtraRunner.router_topk``, src/mtp_expert_prefetch/mtp/extra_tensors.py:341-355:
    top-k on the fp32 logits, then softmax over the k selected values. Same ids;
    the weights equal the renormalised vLLM weights up to fp32 rounding.

Selection order: experts are ranked by logit (softmax is monotonic, so this is
the same ranking as by probability), descending, with exact ties broken toward
the lower expert id. The reference leaves tie order to ``torch.topk``; the
synthetic N(0,1) logits have no exact ties, which the fixtures assert.
"""
from __future__ import annotations

import numpy as np


def topk_order(logits: np.ndarray, k: int) -> np.ndarray:
    """[M, E] -> [M, k] int32 expert ids, descending logit, ties -> lower id."""
    lg = np.asarray(logits, dtype=np.float32)
    # lexsort: last key is primary. Sort by (-logit, expert id).
    m, e = lg.shape
    ids = np.empty((m, k), dtype=np.int32)
    cols = np.arange(e)
    for r in range(m):
        order = np.lexsort((cols, -lg[r].astype(np.float64)))
        ids[r] = order[:k]
    return ids


def topk_softmax(logits: np.ndarray, k: int, renormalize: bool = True):
    """Returns (topk_weights fp32 [M,k], topk_ids int32 [M,k], token_expert_indices int32 [M,k])."""
    lg = np.asarray(logits, dtype=np.float32)
    mx = lg.max(axis=-1, keepdims=True)
    ex = np.exp((lg - mx).astype(np.float32)).astype(np.float32)
    probs = (ex / ex.sum(axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    ids = topk_order(lg, k)
    vals = np.take_along_axis(probs, ids.astype(np.int64), axis=-1).astype(np.float32)
    if renormalize:
        denom = np.maximum(vals.sum(axis=-1, keepdims=True, dtype=np.float32), np.float32(1e-20))
        vals = (vals / denom).astype(np.float32)
    tei = np.broadcast_to(np.arange(k, dtype=np.int32), ids.shape).copy()
    return vals, ids, tei


def router_topk_mtp_form(logits: np.ndarray, k: int):
    """extra_tensors.py:353-354: top-k on logits, softmax over the k values."""
    lg = np.asarray(logits, dtype=np.float32)
    ids = topk_order(lg, k)
    vals = np.take_along_axis(lg, ids.astype(np.int64), axis=-1)
    vals = vals - vals.max(axis=-1, keepdims=True)
    ex = np.exp(vals).astype(np.float32)
    return (ex / ex.sum(axis=-1, keepdims=True)).astype(np.float32), ids


def has_exact_ties(logits: np.ndarray) -> bool:
    lg = np.asarray(logits, dtype=np.float32)
    for row in lg:
        if np.unique(row).size != row.size:
            return True
    return False
