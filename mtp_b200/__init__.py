"""mtp_b200: B200-native (sm_100a) GPTQ-int4 W4A16 mixture-of-experts layer
forward and its MTP-driven expert-prefetch path.

The compute runs in ``lib/libmtp_b200.so`` (hand-written CUDA behind a C ABI,
``include/mtp_b200.h``); this package is the host-side mirror of the reference
interfaces. There is no CPU fallback.
"""
from ._lib import MtpError, load as load_library  # noqa: F401
from .ep import ExpertParallelMoE, plan_dispatch  # noqa: F401
from .ops import (  # noqa: F401
    HiddenResidualPredictor,
    MtpPredictor,
    PrefetchSession,
    SharedExpert,
    W4A16Experts,
    dequantize_gptq_projection,
    experts_from_vllm_wna16,
    fused_experts,
    layer_path,
    layer_workspace,
    moe_align_block_size,
    moe_layer_w4a16,
    prefill_workspace,
    topk_softmax,
    vllm_wna16_to_gptq,
)

__all__ = [
    "ExpertParallelMoE",
    "HiddenResidualPredictor",
    "MtpError",
    "MtpPredictor",
    "PrefetchSession",
    "load_library",
    "SharedExpert",
    "W4A16Experts",
    "dequantize_gptq_projection",
    "experts_from_vllm_wna16",
    "fused_experts",
    "layer_path",
    "layer_workspace",
    "moe_align_block_size",
    "moe_layer_w4a16",
    "plan_dispatch",
    "prefill_workspace",
    "topk_softmax",
    "vllm_wna16_to_gptq",
]
