"""GPTQ checkpoint repack and loading for the W4A16 MoE layer.

A Hugging Face snapshot keeps one tensor per (layer, expert, projection, kind)
(``model.language_model.layers.{l}.mlp.experts.{e}.{gate,up,down}_proj.
{qweight,qzeros,scales,g_idx}``, sharded safetensors with an index). The
reference repacks them into one file per layer with the experts stacked
(``layer_{l:02d}.safetensors``, keys ``experts.{projection}.{kind}``) plus a
``manifest.jsonl`` (per tensor: shape, dtype, sha256, source shape / dtype /
count / key template) and a ``summary.json``
(repack/qwen3_moe_gptq.py:142-265, read back by repack/store.py:39-245).
This module writes and reads that same layout (the format is kept alike so a
store made by either tool serves both) and turns a layer into the kernel's
expert blobs: w13 = gate rows then up rows (the vLLM w13 order), w2 = down.

Only the trivial group order is supported (g_idx = k // group_size: no
act-order permutation); a layer with another g_idx is rejected.
"""
from __future__ import annotations

import hashlib
import json
import re
from pathlib import Path

import torch

PROJECTIONS = ("down_proj", "gate_proj", "up_proj")
KINDS = ("g_idx", "qweight", "qzeros", "scales")
EXPERT_KEY = re.compile(r"^model\.language_model\.layers\.(\d+)\.mlp\.experts\.(\d+)\."
                        r"(down_proj|gate_proj|up_proj)\.(g_idx|qweight|qzeros|scales)$")


def tensor_sha256(t: torch.Tensor) -> str:
    """sha256 of the tensor's bytes (bf16 viewed as int16), as the reference
    manifest records it (repack/qwen3_moe_gptq.py:116-122)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


class SnapshotReader:
    """Reads single tensors of a sharded safetensors snapshot through its index."""

    def __init__(self, snapshot: str | Path):
        self.path = Path(snapshot)
        index = self.path / "model.safetensors.index.json"
        if not index.exists():
            raise FileNotFoundError(f"missing safetensors index: {index}")
        self.weight_map: dict[str, str] = json.loads(index.read_text())["weight_map"]
        self._files = {}

    def get(self, key: str) -> torch.Tensor:
        from safetensors import safe_open
        name = self.weight_map[key]
        f = self._files.get(name)
        if f is None:
            shard = self.path / name
            if not shard.exists():
                raise FileNotFoundError(f"missing shard for {key}: {shard}")
            f = self._files[name] = safe_open(str(shard), framework="pt", device="cpu")
        return f.get_tensor(key)

    def expert_keys(self) -> dict[int, dict[tuple[str, str], dict[int, str]]]:
        out: dict[int, dict[tuple[str, str], dict[int, str]]] = {}
        for key in self.weight_map:
            m = EXPERT_KEY.match(key)
            if m:
                l, e, proj, kind = int(m.group(1)), int(m.group(2)), m.group(3), m.group(4)
                out.setdefault(l, {}).setdefault((proj, kind), {})[e] = key
        return out


def repack_snapshot(snapshot: str | Path, out_dir: str | Path, *, layers: list[int] | None = None,
                    num_experts: int = 256, overwrite: bool = False) -> Path:
    """Stack every expert of each layer into ``layer_{l:02d}.safetensors`` and
    write ``manifest.jsonl`` (one record per layer) and ``summary.json``.
    Returns the manifest path. A layer missing an expert's tensor raises."""
    from safetensors.torch import save_file
    snapshot, out_dir = Path(snapshot).resolve(), Path(out_dir).resolve()
    out_dir.mkdir(parents=True, exist_ok=True)
    manifest = out_dir / "manifest.jsonl"
    if manifest.exists() and not overwrite:
        raise FileExistsError(f"refusing to overwrite {manifest} (pass overwrite=True)")
    reader = SnapshotReader(snapshot)
    keys = reader.expert_keys()
    chosen = sorted(keys) if layers is None else sorted(layers)
    missing_layers = [l for l in chosen if l not in keys]
    if missing_layers or not chosen:
        raise ValueError(f"layers not in the snapshot: {missing_layers or chosen}")
    n_src = n_out = 0
    with manifest.open("w", encoding="utf-8") as mf:
        for l in chosen:
            tensors, meta = {}, {}
            for proj in PROJECTIONS:
                for kind in KINDS:
                    by_expert = keys[l].get((proj, kind), {})
                    missing = [e for e in range(num_experts) if e not in by_expert]
                    if missing:
                        raise RuntimeError(f"layer {l} {proj}.{kind} is missing {len(missing)} experts: {missing[:16]}")
                    pieces = [reader.get(by_expert[e]) for e in range(num_experts)]
                    stacked = torch.stack(pieces).contiguous()
                    name = f"experts.{proj}.{kind}"
                    tensors[name] = stacked
                    meta[name] = {
                        "shape": list(stacked.shape), "dtype": str(stacked.dtype).replace("torch.", ""),
                        "sha256": tensor_sha256(stacked), "source_count": num_experts,
                        "source_shape": list(pieces[0].shape),
                        "source_dtype": str(pieces[0].dtype).replace("torch.", ""),
                        "source_key_template": f"model.language_model.layers.{l}.mlp.experts.{{expert}}.{proj}.{kind}",
                    }
            fname = f"layer_{l:02d}.safetensors"
            save_file(tensors, str(out_dir / fname))
            rec = {"layer": l, "path": fname, "num_experts": num_experts,
                   "num_source_tensors": len(PROJECTIONS) * len(KINDS) * num_experts,
                   "num_output_tensors": len(tensors), "tensors": meta}
            n_src += rec["num_source_tensors"]
            n_out += rec["num_output_tensors"]
            mf.write(json.dumps(rec, sort_keys=True) + "\n")
    summary = {"snapshot_path": str(snapshot), "output_dir": str(out_dir), "manifest_path": manifest.name,
               "layers": chosen, "num_layers": len(chosen), "num_experts": num_experts,
               "projections": list(PROJECTIONS), "kinds": list(KINDS), "total_source_tensors": n_src,
               "total_output_tensors": n_out, "reduction_factor": n_src / n_out if n_out else None,
               "verify": False}
    (out_dir / "summary.json").write_text(json.dumps(summary, indent=2, sort_keys=True) + "\n", encoding="utf-8")
    return manifest


class RepackedStore:
    """A repacked layer store (the reference's layout): manifest checks,
    sha256 verification, and the layer in the GPTQ form the kernel repack
    takes (w13 = gate | up along N, w2 = down)."""

    def __init__(self, path: str | Path):
        self.path = Path(path)
        summary = self.path / "summary.json"
        manifest = self.path / "manifest.jsonl"
        if not summary.exists():
            raise FileNotFoundError(f"missing repack summary: {summary}")
        if not manifest.exists():
            raise FileNotFoundError(f"missing repack manifest: {manifest}")
        self.summary = json.loads(summary.read_text())
        self.manifest: dict[int, dict] = {}
        for i, line in enumerate(manifest.read_text().splitlines(), start=1):
            if line.strip():
                rec = json.loads(line)
                if int(rec["layer"]) in self.manifest:
                    raise RuntimeError(f"duplicate layer {rec['layer']} in {manifest}:{i}")
                self.manifest[int(rec["layer"])] = rec
        if not self.manifest:
            raise RuntimeError(f"empty repack manifest: {manifest}")
        self.layers = tuple(sorted(self.manifest))
        self.num_experts = int(self.summary.get("num_experts", self.manifest[self.layers[0]]["num_experts"]))

    def tensors(self, layer: int, *, verify: bool = True) -> dict[str, torch.Tensor]:
        """The layer's stacked tensors; shape, dtype and (``verify``) sha256
        checked against the manifest (a mismatch raises ValueError)."""
        from safetensors import safe_open
        rec = self.manifest.get(layer)
        if rec is None:
            raise KeyError(f"layer {layer} is not in the store")
        out = {}
        with safe_open(str(self.path / rec["path"]), framework="pt", device="cpu") as f:
            for name, info in rec["tensors"].items():
                t = f.get_tensor(name)
                if list(t.shape) != info["shape"] or str(t.dtype).replace("torch.", "") != info["dtype"]:
                    raise ValueError(f"layer {layer} {name}: {list(t.shape)} {t.dtype} does not match the manifest "
                                     f"{info['shape']} {info['dtype']}")
                if verify and info.get("sha256") and tensor_sha256(t) != info["sha256"]:
                    raise ValueError(f"layer {layer} {name}: sha256 does not match the manifest")
                out[name] = t
        return out

    def gptq_layer(self, layer: int, *, verify: bool = True) -> tuple[dict[str, torch.Tensor], int]:
        """(GPTQ tensors with a leading expert axis in the keys of
        W4A16Experts.from_gptq, group size)."""
        t = self.tensors(layer, verify=verify)
        g_gate, g_down = t["experts.gate_proj.g_idx"], t["experts.down_proj.g_idx"]
        hidden, inter = g_gate.shape[1], g_down.shape[1]
        group = hidden // t["experts.gate_proj.scales"].shape[1]
        for name, gi, k in (("gate_proj", g_gate, hidden), ("up_proj", t["experts.up_proj.g_idx"], hidden),
                            ("down_proj", g_down, inter)):
            want = (torch.arange(k, dtype=gi.dtype) // group).expand_as(gi)
            if not torch.equal(gi, want):
                raise ValueError(f"layer {layer} {name}: g_idx is not k // {group} (act-order is not supported)")
        cat = lambda kind: torch.cat([t[f"experts.gate_proj.{kind}"], t[f"experts.up_proj.{kind}"]], dim=2).contiguous()
        return ({"w13_qweight": cat("qweight"), "w13_qzeros": cat("qzeros"), "w13_scales": cat("scales"),
                 "w2_qweight": t["experts.down_proj.qweight"].contiguous(),
                 "w2_qzeros": t["experts.down_proj.qzeros"].contiguous(),
                 "w2_scales": t["experts.down_proj.scales"].contiguous()}, group)

    def load_layer(self, layer: int, device, *, verify: bool = True):
        """The layer's experts in the kernel layout on ``device`` (a GPU)."""
        from .ops import W4A16Experts
        g, group = self.gptq_layer(layer, verify=verify)
        keys = ("w13_qweight", "w13_qzeros", "w13_scales", "w2_qweight", "w2_qzeros", "w2_scales")
        return W4A16Experts.from_gptq(*(g[k].to(device) for k in keys), group_size=group)
