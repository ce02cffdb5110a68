"""MTP expert-demand predictor on the GPU against the fp32
CPU oracle (oracle/predictor.py): logits within tolerance and the top-k ids
per future layer equal, except where two candidates are closer than the
logits' own tolerance (the bf16 rounding of the hidden activation can flip
them)."""
import numpy as np
import pytest
import torch

from oracle import predictor as opred

pytestmark = pytest.mark.gpu

LOGIT_TOL = 1e-2       # max |gpu - oracle| / max |oracle|
EXACT_ROW_FRACTION = 0.95


def _check(cfg, m, seed, bias, dev):
    import mtp_b200
    from mtp_b200.synthetic import make_predictor, make_predictor_inputs
    w1, b1, w2, b2 = make_predictor(cfg, seed=seed, bias=bias)
    h = make_predictor_inputs(cfg, m, seed=seed)
    ref_logits, ref_ids = opred.predict_topk(h, w1, b1, w2, b2, future=cfg.future, experts=cfg.experts, k=cfg.top_k)
    pred = mtp_b200.MtpPredictor(w1.to(dev), None if b1 is None else b1.to(dev), w2.to(dev),
                                 None if b2 is None else b2.to(dev), future=cfg.future, experts=cfg.experts)
    logits = torch.empty(m, cfg.future * cfg.experts, dtype=torch.float32, device=dev)
    ids = pred.predict_topk(h.to(dev), cfg.top_k, logits_out=logits)
    torch.cuda.synchronize()
    lg = logits.cpu().reshape(m, cfg.future, cfg.experts)
    scale = ref_logits.abs().max().item()
    assert (lg - ref_logits).abs().max().item() <= LOGIT_TOL * scale
    got = ids.cpu().numpy()
    exp = ref_ids.numpy()
    ref = ref_logits.numpy()
    exact = 0
    for i in range(m):
        for f in range(cfg.future):
            g_row, e_row = got[i, f], exp[i, f]
            assert len(set(g_row.tolist())) == cfg.top_k and g_row.min() >= 0 and g_row.max() < cfg.experts
            if np.array_equal(g_row, e_row):
                exact += 1
                continue
            # every pick is within tolerance of the oracle's k-th best logit
            kth = np.sort(ref[i, f])[::-1][cfg.top_k - 1]
            assert (ref[i, f][g_row] >= kth - LOGIT_TOL * scale).all()
    assert exact >= EXACT_ROW_FRACTION * m * cfg.future


@pytest.mark.parametrize("m", [1, 8, 64])
def test_predictor_config3_matches_oracle(cuda_device, m):
    from mtp_b200.synthetic import CONFIG3
    _check(CONFIG3, m, seed=3 + m, bias=True, dev=cuda_device)


def test_predictor_without_bias_and_odd_m(cuda_device):
    from mtp_b200.synthetic import PredictorConfig
    cfg = PredictorConfig(hidden=512, width=256, future=2, experts=128, top_k=4)
    _check(cfg, 37, seed=11, bias=False, dev=cuda_device)


def test_predictor_rejects_bad_shapes(cuda_device):
    import ctypes as C
    from mtp_b200 import _lib
    lib = _lib.load()
    buf = torch.zeros(1 << 20, dtype=torch.uint8, device=cuda_device)
    p = C.c_void_p(buf.data_ptr())
    # hidden not a multiple of 128
    assert lib.mtp_predict_topk(p, 1, 100, p, None, 256, p, None, 4, 256, 8, None, p, p, buf.numel(), None) == 2
    # top_k > 32
    assert lib.mtp_predict_topk(p, 1, 256, p, None, 256, p, None, 4, 256, 33, None, p, p, buf.numel(), None) == 2
    # workspace too small
    assert lib.mtp_predict_topk(p, 64, 256, p, None, 256, p, None, 4, 256, 8, None, p, p, 16, None) == 4


def test_hidden_residual_predictor_matches_reference_golden(cuda_device):
    """The reference predictor architecture (HiddenResidualExpertPredictor:
    encoder Linear -> SiLU -> LayerNorm, layer and delta embeddings, shared
    classifier) run by the kernel on the reference module's own weights and
    inputs (tests/golden/predictor_hr.pt): logits within LOGIT_TOL of the
    reference's fp32 logits and of the bf16-context oracle, top-8 ids equal to
    the reference's on at least EXACT_ROW_FRACTION of the (token, delta)
    rows, every other pick within tolerance of the k-th best."""
    import mtp_b200
    from conftest import golden
    g = golden("predictor_hr.pt")
    st, c = g["state"], g["config"]
    bf = lambda t: t.to(torch.bfloat16).to(cuda_device).contiguous()
    pred = mtp_b200.HiddenResidualPredictor(bf(st["encoder.0.weight"]), bf(st["encoder.0.bias"]),
                                            bf(st["encoder.2.weight"]), bf(st["encoder.2.bias"]),
                                            bf(st["layer_embedding.weight"]), bf(st["delta_embedding.weight"]),
                                            bf(st["classifier.weight"]), bf(st["classifier.bias"]), ln_eps=c["ln_eps"])
    m, f, e = g["logits"].shape
    logits = torch.empty(m, f, e, dtype=torch.float32, device=cuda_device)
    ids = pred.predict_topk(g["hidden"].to(cuda_device), g["layer_ids"].to(cuda_device), 8, logits_out=logits)
    torch.cuda.synchronize()
    got = logits.cpu()
    ref = g["logits"]
    scale = ref.abs().max().item()
    orc = opred.hidden_residual_logits(g["hidden"], g["layer_ids"], st["encoder.0.weight"], st["encoder.0.bias"],
                                       st["encoder.2.weight"], st["encoder.2.bias"], c["ln_eps"],
                                       st["layer_embedding.weight"], st["delta_embedding.weight"],
                                       st["classifier.weight"], st["classifier.bias"])
    assert (got - orc).abs().max().item() <= LOGIT_TOL * scale
    assert (got - ref).abs().max().item() <= LOGIT_TOL * scale
    gi, ri = ids.cpu().numpy(), g["topk_ids"].numpy()
    exact = 0
    for i in range(m):
        for j in range(f):
            if np.array_equal(gi[i, j], ri[i, j]):
                exact += 1
                continue
            kth = np.sort(ref[i, j].numpy())[::-1][7]
            assert (ref[i, j].numpy()[gi[i, j]] >= kth - LOGIT_TOL * scale).all()
    assert exact >= EXACT_ROW_FRACTION * m * f
