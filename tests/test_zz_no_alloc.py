"""mtp_w4a16_moe_layer_noalloc: the layer forward for callers that cannot
allocate device memory (an FFI host that only passes pointers it was given, a
serving loop whose device memory belongs to another allocator). It must give
the same results as the allocating entry point, on consecutive calls that
share its built-in scratch, and refuse requests larger than that scratch.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one; it also passes on its own in a fresh
process.
"""
import ctypes as C

import pytest
import torch

from oracle import layer as olayer

pytestmark = pytest.mark.gpu

KEYS = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")


def _args(x, logits, experts, shared, out, k=8):
    from mtp_b200 import _lib
    a = _lib.MtpMoeLayerArgs()
    m, h = x.shape
    a.num_tokens, a.hidden, a.inter, a.num_experts = m, h, experts.inter, experts.num_experts
    a.top_k, a.group_size, a.renormalize, a.zero_mode = k, experts.group_size, 1, _lib.MTP_ZERO_RAW
    a.hidden_states = x.data_ptr()
    a.router_logits = logits.data_ptr()
    a.expert_blobs = experts.blobs.data_ptr()
    a.expert_bytes = experts.expert_bytes
    a.shared_blob = shared.blob.data_ptr()
    a.shared_gate_weight = shared.gate_weight.data_ptr()
    a.out = out.data_ptr()
    a.workspace = None          # ignored by the no-alloc entry point
    a.workspace_bytes = 0
    return a


@pytest.fixture(scope="module")
def layer(cuda_device):
    from mtp_b200 import SharedExpert, W4A16Experts
    from mtp_b200.synthetic import CONFIG1, make_layer
    ex, sh = make_layer(CONFIG1, seed=21, device=cuda_device)
    w = W4A16Experts.from_gptq(*(ex[k] for k in KEYS))
    s = SharedExpert.from_gptq(*(sh[k] for k in KEYS), sh["gate_weight"])
    return w, s


@pytest.mark.parametrize("m", [1, 16, 48])
def test_noalloc_matches_allocating_entry_point_twice(cuda_device, layer, m):
    import mtp_b200
    from mtp_b200 import _lib
    from mtp_b200.synthetic import CONFIG1, make_inputs
    lib = _lib.load()
    w, s = layer
    stream = C.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    for call in range(2):
        x, logits = make_inputs(CONFIG1, m, seed=500 + 10 * m + call, device=cuda_device)
        ref = mtp_b200.moe_layer_w4a16(x, logits, w, 8, shared=s)
        out = torch.full((m, CONFIG1.hidden), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        args = _args(x, logits, w, s, out)
        status = lib.mtp_w4a16_moe_layer_noalloc(C.byref(args), stream)
        assert status == 0, lib.mtp_status_string(status)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        # the layer is deterministic: the same call on other scratch memory
        # gives the same bits
        assert torch.equal(out, ref), (
            f"rel-L2 {olayer.relative_l2(out.float().cpu(), ref.float().cpu()):.3e}, "
            f"normalised max-abs {olayer.normalized_max_abs(out.float().cpu(), ref.float().cpu()):.3e}")


def test_noalloc_rejects_requests_beyond_its_scratch(cuda_device, layer):
    from mtp_b200 import _lib
    from mtp_b200.synthetic import CONFIG1, make_inputs
    lib = _lib.load()
    w, s = layer
    m = 256  # needs ~21 MB of scratch, far above the 6 MiB array
    x, logits = make_inputs(CONFIG1, m, seed=9, device=cuda_device)
    out = torch.zeros((m, CONFIG1.hidden), dtype=torch.bfloat16, device=cuda_device)
    args = _args(x, logits, w, s, out)
    stream = C.c_void_p(torch.cuda.current_stream(cuda_device).cuda_stream)
    assert lib.mtp_w4a16_moe_layer_noalloc(C.byref(args), stream) == 4  # MTP_ERR_WORKSPACE
    torch.cuda.synchronize()
    assert int(out.abs().max().item()) == 0  # nothing was launched
