"""The vLLM integration shim (mtp_b200.vllm_shim) on the CPU: install and
uninstall swap vLLM's fused_experts_impl and back, calls outside what the
library covers reach vLLM's original function with every argument unchanged,
and the coverage rules reject what the kernels do not compute. The routed
path itself runs on the GPU (tests/test_gpu_layer.py)."""
import pytest
import torch

vllm_fm = pytest.importorskip("vllm.model_executor.layers.fused_moe.fused_moe")


def test_install_uninstall_and_fallback(monkeypatch):
    from mtp_b200 import vllm_shim
    seen = {}

    def fake_original(*args):
        seen["args"] = args
        return "vllm"

    monkeypatch.setattr(vllm_fm, "fused_experts_impl", fake_original)
    vllm_shim.install()
    vllm_shim.install()  # idempotent
    assert vllm_shim.installed() and vllm_fm.fused_experts_impl is not fake_original
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    w1 = torch.zeros(4, 256, 128, dtype=torch.uint8)
    w2 = torch.zeros(4, 256, 64, dtype=torch.uint8)
    ids = torch.zeros(2, 2, dtype=torch.int32)
    before = vllm_shim.stats.fallback_calls
    # bf16 weights (not int4_w4a16): vLLM's own path, arguments passed through
    out = vllm_fm.fused_experts_impl(x, w1, w2, torch.ones(2, 2), ids, False, "silu")
    assert out == "vllm" and seen["args"][0] is x and seen["args"][5] is False
    assert vllm_shim.stats.fallback_calls == before + 1
    vllm_shim.uninstall()
    assert vllm_fm.fused_experts_impl is fake_original and not vllm_shim.installed()


def test_coverage_rules():
    from mtp_b200.vllm_shim import unsupported_reason
    x = torch.zeros(2, 256, dtype=torch.bfloat16)
    w1 = torch.zeros(4, 256, 128, dtype=torch.uint8)
    w2 = torch.zeros(4, 256, 64, dtype=torch.uint8)
    s1, s2 = torch.zeros(4, 256, 2), torch.zeros(4, 256, 1)
    ids = torch.zeros(2, 2, dtype=torch.int32)
    base = dict(hidden_states=x, w1=w1, w2=w2, topk_ids=ids, activation="silu", apply_router_weight_on_input=False,
                use_fp8_w8a8=False, use_int8_w8a8=False, use_int8_w8a16=False, use_int4_w4a16=True,
                ocp_mx_scheme=None, per_channel_quant=False, w1_scale=s1, w2_scale=s2, w1_zp=None, w2_zp=None,
                a1_scale=None, a2_scale=None, block_shape=[0, 128], w1_bias=None, w2_bias=None)
    # on the CPU the hidden states are rejected (the kernels run on the GPU)
    assert unsupported_reason(**base) == "hidden states not 2-D bf16 on a GPU"
    assert unsupported_reason(**{**base, "use_int4_w4a16": False}) == "not int4_w4a16"
    assert unsupported_reason(**{**base, "activation": "gelu"}) == "activation gelu"
    assert unsupported_reason(**{**base, "w1_zp": torch.zeros(1)}) == "zero points"
    assert unsupported_reason(**{**base, "apply_router_weight_on_input": True}).startswith("router weight")
