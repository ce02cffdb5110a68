"""vLLM's moe_wna16 GPTQ weight layout back to the checkpoint form (CPU).

vLLM's loader keeps, per expert, ``qweight.T.contiguous().view(uint8)`` and
``scales.T`` (vllm/model_executor/layers/quantization/moe_wna16.py,
moe_wna16_weight_loader, GPTQ branch); the test restates that transform,
applies mtp_b200.vllm_wna16_to_gptq and expects the checkpoint tensors back
bit for bit (zero points: the symmetric 8 in every nibble)."""
import torch

from mtp_b200.synthetic import LayerConfig, make_layer


def vllm_layout(gptq: dict):
    """The moe_wna16 GPTQ branch of vLLM's weight loader, per stacked expert."""
    w = lambda q: torch.stack([q[e].T.contiguous().view(torch.uint8) for e in range(q.shape[0])])
    s = lambda sc: torch.stack([sc[e].T for e in range(sc.shape[0])]).to(torch.bfloat16)
    return w(gptq["w13_qweight"]), w(gptq["w2_qweight"]), s(gptq["w13_scales"]), s(gptq["w2_scales"])


def test_vllm_layout_round_trips_to_gptq():
    from mtp_b200 import vllm_wna16_to_gptq
    cfg = LayerConfig(num_experts=4, hidden=512, inter=256, group_size=128)
    experts, _ = make_layer(cfg, seed=1)
    w1, w2, s1, s2 = vllm_layout(experts)
    assert w1.shape == (4, 2 * 256, 512 // 2) and w2.shape == (4, 512, 256 // 2)
    back = vllm_wna16_to_gptq(w1, w2, s1, s2)
    for key in ("w13_qweight", "w2_qweight", "w13_qzeros", "w2_qzeros"):
        assert torch.equal(back[key], experts[key]), key
    # scales went through bf16 in vLLM's parameters: equal to the fp16 values
    # rounded to bf16
    for key in ("w13_scales", "w2_scales"):
        assert torch.equal(back[key], experts[key].to(torch.bfloat16).to(torch.float16)), key
