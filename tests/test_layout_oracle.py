"""The kernel weight layout, decoded on the CPU, reproduces the reference
dequantisation exactly (fp32, including non-8 zero points). CPU only."""
import numpy as np
import torch

from conftest import golden
from oracle import gptq, layout


def test_layout_decode_equals_gptq_dequant():
    g = golden("moe_small.pt")
    ex = g["experts"]
    h, i, gs = 256, 128, 128
    L = layout.expert_layout(h, i, gs)
    for e in (0, 3, 7):
        blob = layout.repack_expert(ex, e, h, i, gs)
        w13 = layout.decode_projection(blob, L["w13_qweight"], L["w13_scales"], L["w13_zeros"], 2 * i, h, gs,
                                       gated=True)
        w2 = layout.decode_projection(blob, L["w2_qweight"], L["w2_scales"], L["w2_zeros"], h, i, gs)
        ref13 = gptq.dequantize(ex["w13_qweight"][e].numpy(), ex["w13_qzeros"][e].numpy(), ex["w13_scales"][e].numpy())
        ref2 = gptq.dequantize(ex["w2_qweight"][e].numpy(), ex["w2_qzeros"][e].numpy(), ex["w2_scales"][e].numpy())
        assert np.array_equal(w13, ref13)
        assert np.array_equal(w2, ref2)


def test_layout_sym8_mode_ignores_stored_zeros():
    g = golden("moe_small.pt")
    ex = g["experts"]
    h, i, gs = 256, 128, 128
    L = layout.expert_layout(h, i, gs)
    blob = layout.repack_expert(ex, 1, h, i, gs)
    w2 = layout.decode_projection(blob, L["w2_qweight"], L["w2_scales"], L["w2_zeros"], h, i, gs, zero_mode="sym8")
    ref = gptq.dequantize(ex["w2_qweight"][1].numpy(), ex["w2_qzeros"][1].numpy(), ex["w2_scales"][1].numpy(),
                          zero_mode="sym8")
    assert np.array_equal(w2, ref)


def test_layout_sizes_equal_gptq_sizes():
    g = golden("moe_small.pt")
    ex = g["experts"]
    blob = layout.repack_expert(ex, 0, 256, 128, 128)
    sections = [ex[k][0].numel() * ex[k][0].element_size() for k in
                ("w13_qweight", "w13_scales", "w13_qzeros", "w2_qweight", "w2_scales", "w2_qzeros")]
    # same bytes as the GPTQ tensors, each section padded to a 256-byte boundary
    assert blob.size == sum((b + 255) // 256 * 256 for b in sections)
