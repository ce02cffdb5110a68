"""The C-ABI library loads, exports every symbol include/mtp_b200.h declares,
and answers size queries and argument errors without touching a GPU. CPU only."""
import ctypes as C
import re

import numpy as np
import pytest

from conftest import ROOT
from oracle import align as oalign
from oracle import layout as olayout


def header_symbols():
    text = (ROOT / "include" / "mtp_b200.h").read_text()
    return sorted(set(re.findall(r"MTP_API\s+[\w\s\*]*?\b(mtp_\w+)\s*\(", text)))


def test_library_exports_every_header_symbol(built_lib):
    from mtp_b200 import _lib
    lib = _lib.load()
    syms = header_symbols()
    assert syms, "no declarations found in the header"
    for name in syms:
        assert hasattr(lib, name), name
    assert sorted(_lib.EXPORTS) == syms
    assert lib.mtp_abi_version() >= 1


def test_status_strings(built_lib):
    from mtp_b200 import _lib
    lib = _lib.load()
    for code in range(10):
        assert lib.mtp_status_string(code)
    assert lib.mtp_status_string(0) == b"ok"


@pytest.mark.parametrize("numel,e,bm,pad", [(8, 256, 8, 0), (8, 256, 16, 1), (2048, 256, 8, 0),
                                            (65536, 256, 64, 1), (12, 5, 4, 0), (0, 4, 16, 0)])
def test_align_sizes_match_vllm_wrapper(built_lib, numel, e, bm, pad):
    from mtp_b200 import _lib
    cap, blocks, segs = _lib.align_sizes(numel, e, bm, bool(pad))
    ocap, oblocks = oalign.buffer_sizes(numel, e, bm, bool(pad))
    assert (cap, blocks, segs) == (ocap, oblocks, min(numel, e))


@pytest.mark.parametrize("h,i,g", [(2048, 512, 128), (2048, 768, 128), (256, 128, 128), (512, 256, 64)])
def test_expert_layout_offsets(built_lib, h, i, g):
    from mtp_b200 import _lib
    lay = _lib.expert_layout(h, i, g)
    ref = olayout.expert_layout(h, i, g)
    for f in ("w13_qweight", "w13_scales", "w13_zeros", "w2_qweight", "w2_scales", "w2_zeros", "bytes"):
        assert getattr(lay, f) == ref[f], f
    if (h, i, g) == (2048, 512, 128):
        assert lay.bytes == 1_634_304  # BASELINE's bytes per expert incl. qzeros


def test_argument_errors_need_no_gpu(built_lib):
    from mtp_b200 import _lib
    lib = _lib.load()
    w = (C.c_float * 8)()
    ids = (C.c_int32 * 8)()
    assert lib.mtp_router_topk(None, 1, 256, 8, 1, w, ids, None, None) == 1          # NULL logits
    assert lib.mtp_router_topk(w, 1, 2048, 8, 1, w, ids, None, None) == 2            # E too large
    assert lib.mtp_router_topk(w, 1, 256, 33, 1, w, ids, None, None) == 2            # k too large
    assert lib.mtp_gptq_dequant(ids, ids, ids, None, 256, 64, 128, 7, w, None) == 9  # bad zero mode
    assert lib.mtp_w4a16_moe_layer(None, None) == 1
    args = _lib.MtpMoeLayerArgs()
    args.num_tokens, args.hidden, args.inter, args.num_experts = 1, 2048, 512, 256
    args.top_k, args.group_size = 8, 128
    assert lib.mtp_w4a16_moe_layer(C.byref(args), None) == 1                         # NULL buffers
    args.hidden = 3000
    assert lib.mtp_w4a16_moe_layer(C.byref(args), None) == 2                         # bad hidden
    ws = C.c_int64()
    assert lib.mtp_w4a16_moe_layer_workspace_size(1, 256, 8, 2048, 512, C.byref(ws)) == 0
    assert ws.value > 0


def test_prefill_argument_errors_need_no_gpu(built_lib):
    from mtp_b200 import _lib
    lib = _lib.load()
    assert lib.mtp_w4a16_moe_prefill(None, None) == 1
    args = _lib.MtpMoeLayerArgs()
    args.num_tokens, args.hidden, args.inter, args.num_experts = 8192, 2048, 512, 256
    args.top_k, args.group_size = 8, 128
    assert lib.mtp_w4a16_moe_prefill(C.byref(args), None) == 1                       # NULL buffers
    table = (C.c_int32 * 256)()
    args.slot_table = C.cast(table, C.c_void_p)
    assert lib.mtp_w4a16_moe_prefill(C.byref(args), None) == 9                       # slot table: decode only
    args.slot_table = None
    args.inter = 200
    assert lib.mtp_w4a16_moe_prefill(C.byref(args), None) == 2                       # I not a multiple of 128
    args.inter, args.num_experts = 512, 1024
    buf = (C.c_uint8 * 16)()
    args.shared_blob = C.cast(buf, C.c_void_p)
    assert lib.mtp_w4a16_moe_prefill(C.byref(args), None) == 2                       # E + shared > 1024
    # workspace: sorted capacity for 128-pair blocks of E + 1 experts, then the
    # x / h / y rows of every position
    ws = C.c_int64()
    assert lib.mtp_w4a16_moe_prefill_workspace_size(8192, 256, 8, 2048, 512, C.byref(ws)) == 0
    cap = -(-(8192 * 9 + 257 * 127) // 128) * 128
    assert ws.value >= cap * (2048 + 512 + 2048) * 2
    assert ws.value < cap * (2048 + 512 + 2048) * 2 + 64 * cap


def test_python_api_rejects_cpu_tensors(built_lib):
    import torch
    import mtp_b200
    with pytest.raises(ValueError):
        mtp_b200.topk_softmax(torch.zeros(2, 8), 2)
    with pytest.raises(ValueError):
        mtp_b200.moe_align_block_size(torch.zeros(2, 2, dtype=torch.int32), 8, 8)
    # the product entry points have no CPU path: host tensors are refused
    # before anything runs
    from mtp_b200.ops import MtpPredictor, W4A16Experts, dequantize_gptq_projection, moe_layer_w4a16
    i32 = dict(dtype=torch.int32)
    with pytest.raises(ValueError, match="CUDA"):
        dequantize_gptq_projection(torch.zeros(16, 8, **i32), torch.zeros(1, 1, **i32),
                                   torch.zeros(1, 8, dtype=torch.float16))
    with pytest.raises(ValueError, match="CUDA"):
        W4A16Experts.from_gptq(torch.zeros(2, 32, 256, **i32), torch.zeros(2, 2, 32, **i32),
                               torch.zeros(2, 2, 256, dtype=torch.float16), torch.zeros(2, 16, 256, **i32),
                               torch.zeros(2, 1, 32, **i32), torch.zeros(2, 1, 256, dtype=torch.float16))
    experts = W4A16Experts(None, 2, 256, 128, 128, None)
    with pytest.raises(ValueError, match="CUDA"):
        moe_layer_w4a16(torch.zeros(4, 256, dtype=torch.bfloat16), torch.zeros(4, 2), experts, 1)
    with pytest.raises(ValueError, match="CUDA"):
        mtp_b200.fused_experts(torch.zeros(4, 256, dtype=torch.bfloat16), experts,
                               topk_weights=torch.ones(4, 1), topk_ids=torch.zeros(4, 1, **i32))
    with pytest.raises(ValueError, match="CUDA"):
        MtpPredictor(torch.zeros(64, 256, dtype=torch.bfloat16), None, torch.zeros(8, 64, dtype=torch.bfloat16),
                     None, future=1, experts=8)
