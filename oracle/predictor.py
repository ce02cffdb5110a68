"""MTP expert-demand predictor: BF16 MLP + per-future-layer top-k (torch fp32 on the CPU).

Test infrastructure (see ``oracle/__init__.py``).

Reference family: ``HiddenResidualExpertPredictor`` (src/mtp_expert_prefetch/
training/hidden_residual.py:44-134: Linear -> SiLU -> ... -> Linear classifier
over experts per future delta) and ``MtpRouterOnlyPredictor``
(training/predictor.py:193-241); ranking metric ``recall_at_m`` (predictor.py:105)
takes ``topk(logits.float())``. The BASELINE shape is
``logits = W2 . silu(W1 . h + b1) + b2`` with H -> H -> [F x E] and top-k per
future layer f.

The hidden activation is rounded to bf16 between the two linears, as the
CUDA kernel stores it (the second GEMV consumes a bf16 operand).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .router import topk_order


def predictor_logits(h, w1, b1, w2, b2, *, round_hidden_bf16: bool = True) -> torch.Tensor:
    h = h.to(torch.float32)
    a = F.linear(h, w1.to(torch.float32), None if b1 is None else b1.to(torch.float32))
    a = F.silu(a)
    if round_hidden_bf16:
        a = a.to(torch.bfloat16).to(torch.float32)
    return F.linear(a, w2.to(torch.float32), None if b2 is None else b2.to(torch.float32))


def predict_topk(h, w1, b1, w2, b2, *, future: int, experts: int, k: int):
    """Returns (logits [M, F, E] fp32, ids [M, F, k] int32)."""
    logits = predictor_logits(h, w1, b1, w2, b2)
    m = logits.shape[0]
    lg = logits.reshape(m, future, experts)
    ids = topk_order(lg.reshape(m * future, experts).numpy(), k).reshape(m, future, k)
    return lg, torch.from_numpy(ids)
