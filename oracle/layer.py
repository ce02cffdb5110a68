"""The W4A16 MoE layer forward on the CPU: dequantise, then matmul (torch).

Test infrastructure (see ``oracle/__init__.py``); also the timed CPU path of
``bench.py --impl reference`` (the reference's own CPU torch form).

Reference:
  * expert MLP - ``SingleExpertMlp.forward``,
    src/mtp_expert_prefetch/repack/gptq_unpack.py:247-256:
    ``linear(silu(linear(x, gate)) * linear(x, up), down)``;
  * weights dequantised once per expert (``load_topk_expert_mlp``,
    gptq_unpack.py:350-371, via ``dequantize_gptq_projection`` :88-131);
  * routed sum + sigmoid-gated shared expert - ``MtpExtraRunner.moe_tokens``,
    src/mtp_expert_prefetch/mtp/extra_tensors.py:544-598: for each top-k slot,
    for each unique expert in that slot, ``out[mask] += w[mask] * expert(x[mask])``;
    then ``out += sigmoid(linear(x, w_g)) * shared(x)``;
  * w13 holds the gate rows first and the up rows next (vLLM ``w13``;
    ``silu_and_mul`` restated at vllm_router_trace.py:4175-4182).
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import gptq


def expert_mlp(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    """gptq_unpack.py:252-256."""
    return F.linear(F.silu(F.linear(x, gate)) * F.linear(x, up), down)


def dequant_expert(qw13, qz13, sc13, qw2, qz2, sc2, *, group_size=128, zero_mode="raw"):
    """One expert's (gate, up, down) fp32 torch tensors in Linear orientation."""
    to_np = lambda t: t.cpu().numpy() if isinstance(t, torch.Tensor) else np.asarray(t)
    w13 = gptq.dequantize(to_np(qw13), to_np(qz13), to_np(sc13), group_size=group_size, zero_mode=zero_mode)
    w2 = gptq.dequantize(to_np(qw2), to_np(qz2), to_np(sc2), group_size=group_size, zero_mode=zero_mode)
    inter = w13.shape[0] // 2
    return (torch.from_numpy(w13[:inter].copy()), torch.from_numpy(w13[inter:].copy()),
            torch.from_numpy(w2))


class MoeLayerOracle:
    """Holds the GPTQ tensors of one layer and dequantises experts on first use.

    ``experts`` maps the attribute names of the GPTQ checkpoint form
    (``w13_qweight [E, H/8, 2I]``, ``w13_qzeros [E, H/g, 2I/8]``,
    ``w13_scales [E, H/g, 2I]``, ``w2_*`` with H and I swapped) to tensors;
    ``shared`` (optional) holds the same keys without the leading E axis plus
    ``gate_weight [H]``.
    """

    def __init__(self, experts: dict, shared: dict | None = None, *, group_size: int = 128,
                 zero_mode: str = "raw", dtype: torch.dtype = torch.float32):
        self.experts = experts
        self.shared = shared
        self.group_size = group_size
        self.zero_mode = zero_mode
        self.dtype = dtype
        self._cache: dict[int, tuple] = {}
        self._shared_w = None

    def _expert(self, e: int):
        if e not in self._cache:
            ex = self.experts
            w = dequant_expert(ex["w13_qweight"][e], ex["w13_qzeros"][e], ex["w13_scales"][e],
                               ex["w2_qweight"][e], ex["w2_qzeros"][e], ex["w2_scales"][e],
                               group_size=self.group_size, zero_mode=self.zero_mode)
            self._cache[e] = tuple(t.to(self.dtype).contiguous() for t in w)
        return self._cache[e]

    def _shared(self):
        if self._shared_w is None and self.shared is not None:
            s = self.shared
            w = dequant_expert(s["w13_qweight"], s["w13_qzeros"], s["w13_scales"],
                               s["w2_qweight"], s["w2_qzeros"], s["w2_scales"],
                               group_size=self.group_size, zero_mode=self.zero_mode)
            gw = s["gate_weight"].reshape(1, -1).to(torch.float32)
            self._shared_w = tuple(t.to(self.dtype).contiguous() for t in w) + (gw.to(self.dtype),)
        return self._shared_w

    def prepare(self, expert_ids) -> None:
        """Dequantise the given experts (and the shared one) ahead of timing."""
        for e in sorted({int(v) for v in np.asarray(expert_ids).reshape(-1)}):
            self._expert(e)
        self._shared()

    def moe_tokens(self, x: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor) -> torch.Tensor:
        """extra_tensors.py:544-598 on [T, H] tokens; returns [T, H] in ``self.dtype``."""
        flat_x = x.reshape(-1, x.shape[-1]).to(self.dtype)
        ids = torch.as_tensor(topk_ids).to(torch.long).reshape(flat_x.shape[0], -1)
        wts = torch.as_tensor(topk_weights).to(self.dtype).reshape(flat_x.shape[0], -1)
        out = torch.zeros_like(flat_x)
        for slot in range(ids.shape[1]):
            slot_ids = ids[:, slot]
            slot_w = wts[:, slot]
            for e in torch.unique(slot_ids).tolist():
                mask = slot_ids == int(e)
                if not bool(mask.any()):
                    continue
                gate, up, down = self._expert(int(e))
                y = expert_mlp(flat_x[mask], gate, up, down)
                out[mask] = out[mask] + slot_w[mask, None] * y
        sw = self._shared()
        if sw is not None:
            gate, up, down, gw = sw
            out = out + torch.sigmoid(F.linear(flat_x, gw)) * expert_mlp(flat_x, gate, up, down)
        return out


def relative_l2(out: torch.Tensor, ref: torch.Tensor) -> float:
    out = out.double()
    ref = ref.double()
    return float((out - ref).norm() / ref.norm().clamp_min(1e-30))


def normalized_max_abs(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max|out - ref| / max(1, max|ref|): the max-abs bound on the output's own scale."""
    out = out.double()
    ref = ref.double()
    return float((out - ref).abs().max() / max(1.0, float(ref.abs().max())))
