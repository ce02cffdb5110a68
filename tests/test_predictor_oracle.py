"""The predictor oracle on the CPU: shapes, descending order with ties to the
lower expert id, and agreement with a direct torch restatement of the
BASELINE config-3 MLP. CPU only."""
import torch

from oracle import predictor as opred


def test_oracle_topk_descending_and_consistent():
    from mtp_b200.synthetic import PredictorConfig, make_predictor, make_predictor_inputs
    cfg = PredictorConfig(hidden=256, width=256, future=2, experts=64, top_k=8)
    w1, b1, w2, b2 = make_predictor(cfg, seed=1)
    h = make_predictor_inputs(cfg, 5, seed=1)
    logits, ids = opred.predict_topk(h, w1, b1, w2, b2, future=cfg.future, experts=cfg.experts, k=cfg.top_k)
    assert logits.shape == (5, 2, 64) and ids.shape == (5, 2, 8)
    for i in range(5):
        for f in range(2):
            vals = logits[i, f][ids[i, f].long()]
            assert torch.all(vals[:-1] >= vals[1:])
            kth = torch.sort(logits[i, f], descending=True).values[cfg.top_k - 1]
            assert vals.min() >= kth
    # direct restatement: silu MLP with the hidden rounded to bf16
    a = torch.nn.functional.silu(h.float() @ w1.float().T + b1.float()).to(torch.bfloat16).float()
    direct = (a @ w2.float().T + b2.float()).reshape(5, 2, 64)
    assert torch.allclose(direct, logits, rtol=0, atol=1e-5)


def test_oracle_ties_go_to_lower_id():
    from oracle.router import topk_order
    import numpy as np
    row = np.zeros((1, 16), dtype=np.float32)
    row[0, [3, 7, 9]] = 1.0
    assert topk_order(row, 2).tolist() == [[3, 7]]


def test_hidden_residual_oracle_matches_reference_golden():
    """oracle.predictor.hidden_residual_logits (fp32, no bf16 rounding) equals
    the reference HiddenResidualExpertPredictor's own logits (fixture made by
    tests/golden/make_golden.py) and ranks the same top-8."""
    import torch

    from conftest import golden
    from oracle import predictor as opred
    g = golden("predictor_hr.pt")
    st, c = g["state"], g["config"]
    lg = opred.hidden_residual_logits(g["hidden"], g["layer_ids"], st["encoder.0.weight"], st["encoder.0.bias"],
                                      st["encoder.2.weight"], st["encoder.2.bias"], c["ln_eps"],
                                      st["layer_embedding.weight"], st["delta_embedding.weight"],
                                      st["classifier.weight"], st["classifier.bias"], round_context_bf16=False)
    torch.testing.assert_close(lg, g["logits"], rtol=1e-5, atol=1e-5)
    assert torch.equal(torch.topk(lg, 8, dim=-1).indices.to(torch.int32), g["topk_ids"])
