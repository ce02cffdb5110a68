"""Route vLLM's fused-MoE expert computation for GPTQ int4 (W4A16) models to
this library, at run time, without changing vLLM.

``install()`` replaces ``fused_experts_impl`` in
``vllm.model_executor.layers.fused_moe.fused_moe`` (the function vLLM's
``fused_experts`` custom ops call; the reference's trace harness replaces the
same symbol, tracing/vllm_router_trace.py:19286-19842, to time it). Calls
that this library covers go to :func:`mtp_b200.fused_experts` (the layer
kernels: W1 + SiLU * up + W2 + routed-weight sum in one call); every other
call goes to the original function unchanged. ``uninstall()`` puts it back.

Covered: ``use_int4_w4a16`` without any other quantisation flag, SiLU,
bf16 activations, no routed weight on the input, no zero points (symmetric
GPTQ), no biases or activation scales, group 64 or 128, H a multiple of 256
up to 2048, I a multiple of 128 up to 1024, at most 1024 experts and top-32,
``expert_map`` allowed (its -1 entries skip the pair). The weights stay in
vLLM's moe_wna16 layout; they are repacked into the kernel layout once per
weight tensor (see :func:`mtp_b200.experts_from_vllm_wna16`).
"""
from __future__ import annotations

import importlib
from dataclasses import dataclass, field
from types import SimpleNamespace

import torch

MODULE = "vllm.model_executor.layers.fused_moe.fused_moe"


@dataclass
class ShimStats:
    routed_calls: int = 0
    fallback_calls: int = 0
    fallback_reasons: dict = field(default_factory=dict)


stats = ShimStats()
_original = None


def unsupported_reason(hidden_states, w1, w2, topk_ids, activation, apply_router_weight_on_input, use_fp8_w8a8,
                       use_int8_w8a8, use_int8_w8a16, use_int4_w4a16, ocp_mx_scheme, per_channel_quant, w1_scale,
                       w2_scale, w1_zp, w2_zp, a1_scale, a2_scale, block_shape, w1_bias, w2_bias) -> str | None:
    """None when the call is one the library computes, else why not."""
    if not use_int4_w4a16 or use_fp8_w8a8 or use_int8_w8a8 or use_int8_w8a16 or ocp_mx_scheme is not None:
        return "not int4_w4a16"
    name = str(getattr(activation, "value", activation)).lower()
    if name != "silu":
        return f"activation {name}"
    if apply_router_weight_on_input or per_channel_quant:
        return "router weight on input / per-channel"
    if w1_zp is not None or w2_zp is not None:
        return "zero points"
    if a1_scale is not None or a2_scale is not None or w1_bias is not None or w2_bias is not None:
        return "activation scales or biases"
    if w1_scale is None or w2_scale is None:
        return "no weight scales"
    if not (isinstance(hidden_states, torch.Tensor) and hidden_states.is_cuda and hidden_states.dtype == torch.bfloat16
            and hidden_states.dim() == 2):
        return "hidden states not 2-D bf16 on a GPU"
    if w1.dtype != torch.uint8 or w2.dtype != torch.uint8 or w1.dim() != 3 or w2.dim() != 3:
        return "weights not in the moe_wna16 uint8 layout"
    e, two_i, h_half = w1.shape
    h, i = 2 * h_half, two_i // 2
    if h % 256 or h > 2048 or i % 128 or i > 1024 or e > 1024 or topk_ids.shape[1] > 32:
        return f"shape E={e} H={h} I={i} k={topk_ids.shape[1]}"
    g = h // w1_scale.shape[2]
    if g not in (64, 128) or (block_shape is not None and list(block_shape)[-1] != g):
        return f"group size {g}"
    return None


def _route(original):
    def fused_experts_impl(hidden_states, w1, w2, topk_weights, topk_ids, inplace, activation="silu",
                           apply_router_weight_on_input=False, use_fp8_w8a8=False, use_int8_w8a8=False,
                           use_int8_w8a16=False, use_int4_w4a16=False, ocp_mx_scheme=None, per_channel_quant=False,
                           global_num_experts=-1, expert_map=None, w1_scale=None, w2_scale=None, w1_zp=None,
                           w2_zp=None, a1_scale=None, a2_scale=None, block_shape=None, w1_bias=None, w2_bias=None):
        why = unsupported_reason(hidden_states, w1, w2, topk_ids, activation, apply_router_weight_on_input,
                                 use_fp8_w8a8, use_int8_w8a8, use_int8_w8a16, use_int4_w4a16, ocp_mx_scheme,
                                 per_channel_quant, w1_scale, w2_scale, w1_zp, w2_zp, a1_scale, a2_scale, block_shape,
                                 w1_bias, w2_bias)
        if why is not None:
            stats.fallback_calls += 1
            stats.fallback_reasons[why] = stats.fallback_reasons.get(why, 0) + 1
            return original(hidden_states, w1, w2, topk_weights, topk_ids, inplace, activation,
                            apply_router_weight_on_input, use_fp8_w8a8, use_int8_w8a8, use_int8_w8a16,
                            use_int4_w4a16, ocp_mx_scheme, per_channel_quant, global_num_experts, expert_map,
                            w1_scale, w2_scale, w1_zp, w2_zp, a1_scale, a2_scale, block_shape, w1_bias, w2_bias)
        from .ops import fused_experts
        stats.routed_calls += 1
        qc = SimpleNamespace(w1_scale=w1_scale, w2_scale=w2_scale, w1_zp=None, w2_zp=None, block_shape=block_shape)
        return fused_experts(hidden_states, w1, w2, topk_weights, topk_ids, inplace=inplace, activation="silu",
                             global_num_experts=global_num_experts, expert_map=expert_map, quant_config=qc)

    fused_experts_impl.mtp_b200_original = original
    return fused_experts_impl


def install() -> None:
    """Replace vLLM's fused_experts_impl (idempotent)."""
    global _original
    mod = importlib.import_module(MODULE)
    if getattr(mod.fused_experts_impl, "mtp_b200_original", None) is not None:
        return
    _original = mod.fused_experts_impl
    mod.fused_experts_impl = _route(_original)


def uninstall() -> None:
    """Restore vLLM's own fused_experts_impl."""
    global _original
    mod = importlib.import_module(MODULE)
    orig = getattr(mod.fused_experts_impl, "mtp_b200_original", None)
    if orig is not None:
        mod.fused_experts_impl = orig
    _original = None


def installed() -> bool:
    mod = importlib.import_module(MODULE)
    return getattr(mod.fused_experts_impl, "mtp_b200_original", None) is not None
