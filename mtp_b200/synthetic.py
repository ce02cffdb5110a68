"""Seeded synthetic inputs for the BASELINE configurations (no checkpoint or
dataset exists on this machine; these stand in with the shapes and value
distributions the BASELINE fixes).

GPTQ int4 symmetric, group 128: qweight int32 with uniform random nibbles,
qzeros packed with the value 8, scales fp16 ``|N(0,1)| * 0.02 + 1e-3``;
activations bf16 N(0,1), router logits fp32 N(0,1); the shared expert's gate
weight bf16 ``N(0,1) * 0.02``.

Draw order per layer (fixed so fixtures are reproducible from the seed):
w13_qweight, w13_scales, w2_qweight, w2_scales, [w13_qzeros, w2_qzeros when
random zeros], then the shared expert in the same order and its gate weight.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

SYM_ZERO_WORD = -2004318072  # 0x88888888 as int32: eight nibbles of value 8


@dataclass(frozen=True)
class LayerConfig:
    num_experts: int
    hidden: int
    inter: int
    top_k: int = 8
    group_size: int = 128
    shared: bool = True
    tokens: tuple[int, ...] = field(default_factory=tuple)


# BASELINE.json configs (0-based).
CONFIG0 = LayerConfig(num_experts=128, hidden=2048, inter=768, shared=False, tokens=(4,))
CONFIG1 = LayerConfig(num_experts=256, hidden=2048, inter=512, shared=True,
                      tokens=(1, 2, 4, 8, 16, 32, 64, 128, 256))


def _qweight(g: torch.Generator, shape, device) -> torch.Tensor:
    x = torch.randint(0, 2 ** 32, shape, generator=g, dtype=torch.int64, device=device)
    return (x - 2 ** 31).to(torch.int32)


def _scales(g: torch.Generator, shape, device) -> torch.Tensor:
    return (torch.randn(shape, generator=g, device=device).abs() * 0.02 + 1e-3).to(torch.float16)


def _zeros(g: torch.Generator | None, shape, device, random_zeros: bool) -> torch.Tensor:
    if not random_zeros:
        return torch.full(shape, SYM_ZERO_WORD, dtype=torch.int32, device=device)
    return _qweight(g, shape, device)


def gptq_experts(g: torch.Generator, e: int, hidden: int, inter: int, group: int, device,
                 random_zeros: bool = False) -> dict[str, torch.Tensor]:
    """GPTQ checkpoint form with a leading expert axis (w13 = gate rows, then up rows)."""
    t = {
        "w13_qweight": _qweight(g, (e, hidden // 8, 2 * inter), device),
        "w13_scales": _scales(g, (e, hidden // group, 2 * inter), device),
        "w2_qweight": _qweight(g, (e, inter // 8, hidden), device),
        "w2_scales": _scales(g, (e, inter // group, hidden), device),
    }
    t["w13_qzeros"] = _zeros(g, (e, hidden // group, 2 * inter // 8), device, random_zeros)
    t["w2_qzeros"] = _zeros(g, (e, inter // group, hidden // 8), device, random_zeros)
    return t


def make_layer(cfg: LayerConfig, seed: int = 0, device="cpu", random_zeros: bool = False):
    """Returns (experts dict, shared dict or None) in GPTQ checkpoint form."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    experts = gptq_experts(g, cfg.num_experts, cfg.hidden, cfg.inter, cfg.group_size, device, random_zeros)
    shared = None
    if cfg.shared:
        s = gptq_experts(g, 1, cfg.hidden, cfg.inter, cfg.group_size, device, random_zeros)
        shared = {k: v[0] for k, v in s.items()}
        shared["gate_weight"] = (torch.randn(cfg.hidden, generator=g, device=device) * 0.02).to(torch.bfloat16)
    return experts, shared


def make_inputs(cfg: LayerConfig, m: int, seed: int = 1, device="cpu"):
    """(hidden_states bf16 [M, H], router_logits fp32 [M, E])."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    x = torch.randn((m, cfg.hidden), generator=g, device=device).to(torch.bfloat16)
    logits = torch.randn((m, cfg.num_experts), generator=g, device=device, dtype=torch.float32)
    return x, logits


# the MTP predictor, hidden 2048 -> 2048 -> 4 future layers x 256 experts.
@dataclass(frozen=True)
class PredictorConfig:
    hidden: int = 2048
    width: int = 2048
    future: int = 4
    experts: int = 256
    top_k: int = 8
    tokens: tuple[int, ...] = (1, 8, 64)


CONFIG3 = PredictorConfig()


def make_predictor(cfg: PredictorConfig, seed: int = 0, device="cpu", bias: bool = True):
    """W1 [width, hidden], W2 [future*experts, width] bf16 N(0,1)*0.02, biases bf16 N(0,1)*0.02 (or None)."""
    g = torch.Generator(device="cpu").manual_seed(seed)
    w1 = (torch.randn(cfg.width, cfg.hidden, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(cfg.future * cfg.experts, cfg.width, generator=g) * 0.02).to(torch.bfloat16)
    b1 = (torch.randn(cfg.width, generator=g) * 0.02).to(torch.bfloat16) if bias else None
    b2 = (torch.randn(cfg.future * cfg.experts, generator=g) * 0.02).to(torch.bfloat16) if bias else None
    mv = lambda t: None if t is None else t.to(device)  # noqa: E731
    return mv(w1), mv(b1), mv(w2), mv(b2)


def make_predictor_inputs(cfg: PredictorConfig, m: int, seed: int = 0, device="cpu") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(10_000 + seed)
    return torch.randn(m, cfg.hidden, generator=g).to(torch.bfloat16).to(device)


def make_gptq_snapshot(path, *, layers: int = 2, experts: int = 4, hidden: int = 256, inter: int = 128,
                       group_size: int = 128, shards: int = 2, seed: int = 0) -> dict:
    """A small Hugging Face style GPTQ checkpoint snapshot on disk (sharded
    safetensors + model.safetensors.index.json) with the Qwen3 MoE expert key
    names (model.language_model.layers.{l}.mlp.experts.{e}.{gate,up,down}_proj.
    {qweight,qzeros,scales,g_idx}), seeded: GPTQ int4 weights and zeros of 8,
    fp16 scales |N(0,1)| * 0.02 + 1e-3, g_idx = k // group_size. Experts are
    spread over `shards` files. Returns the tensors by key."""
    import json
    from pathlib import Path

    from safetensors.torch import save_file

    path = Path(path)
    path.mkdir(parents=True, exist_ok=True)
    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for l in range(layers):
        for e in range(experts):
            for proj, (k, n) in (("gate_proj", (hidden, inter)), ("up_proj", (hidden, inter)),
                                 ("down_proj", (inter, hidden))):
                key = f"model.language_model.layers.{l}.mlp.experts.{e}.{proj}"
                tensors[f"{key}.qweight"] = _qweight(g, (k // 8, n), "cpu")
                tensors[f"{key}.qzeros"] = _zeros(None, (k // group_size, n // 8), "cpu", False)
                tensors[f"{key}.scales"] = _scales(g, (k // group_size, n), "cpu")
                tensors[f"{key}.g_idx"] = torch.arange(k, dtype=torch.int32) // group_size
    names = sorted(tensors)
    weight_map = {}
    for s in range(shards):
        part = {n: tensors[n] for i, n in enumerate(names) if i % shards == s}
        fname = f"model-{s + 1:05d}-of-{shards:05d}.safetensors"
        save_file(part, str(path / fname))
        weight_map.update({n: fname for n in part})
    (path / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    return tensors
