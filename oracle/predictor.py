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


def hidden_residual_logits(h, layer_ids, w1, b1, ln_w, ln_b, eps, layer_emb, delta_emb, wc, bc, *,
                           round_context_bf16: bool = True) -> torch.Tensor:
    """HiddenResidualExpertPredictor.forward (training/hidden_residual.py:86-103)
    in fp32: state = LayerNorm(silu(W1 h + b1)); logits[:, f] =
    Wc silu(state + layer_emb[layer_ids] + delta_emb[f]) + bc, [M, F, E].
    With ``round_context_bf16`` the classifier's input is rounded to bf16, as
    the CUDA kernel feeds its bf16 MMA."""
    f32 = lambda t: None if t is None else t.to(torch.float32)
    a = F.silu(F.linear(h.to(torch.float32), f32(w1), f32(b1)))
    state = F.layer_norm(a, (a.shape[-1],), f32(ln_w), f32(ln_b), eps)
    lids = torch.as_tensor(layer_ids).long().clamp(0, layer_emb.shape[0] - 1)
    ctx = state[:, None, :] + f32(layer_emb)[lids][:, None, :] + f32(delta_emb)[None, :, :]
    z = F.silu(ctx)
    if round_context_bf16:
        z = z.to(torch.bfloat16).to(torch.float32)
    return F.linear(z, f32(wc), f32(bc))
