"""GPTQ checkpoint repack and store (mtp_b200.checkpoint), CPU only.

The repack of a seeded synthetic snapshot must reproduce, record for record,
the manifest the reference's own repack_qwen3_moe_gptq wrote for the same
snapshot (tests/golden/repack_manifest.json, made by
tests/golden/make_golden.py): same stacked tensors (sha256), shapes, dtypes
and source fields. The store then verifies hashes, rejects corruption and
act-order g_idx, and returns the layer in the GPTQ form the kernel repack
takes (w13 = gate | up along N)."""
import json

import pytest
import torch

from conftest import GOLDEN
from mtp_b200 import checkpoint as ck
from mtp_b200.synthetic import make_gptq_snapshot


@pytest.fixture(scope="module")
def golden_manifest():
    return json.loads((GOLDEN / "repack_manifest.json").read_text())


@pytest.fixture()
def repacked(tmp_path, golden_manifest):
    p = golden_manifest["snapshot"]
    src = make_gptq_snapshot(tmp_path / "snap", layers=p["layers"], experts=p["experts"], hidden=p["hidden"],
                             inter=p["inter"], group_size=p["group_size"], shards=p["shards"], seed=p["seed"])
    ck.repack_snapshot(tmp_path / "snap", tmp_path / "out", num_experts=p["experts"])
    return tmp_path / "out", src


def test_repack_matches_reference_manifest(repacked, golden_manifest):
    out, _ = repacked
    records = [json.loads(line) for line in (out / "manifest.jsonl").read_text().splitlines() if line.strip()]
    assert records == golden_manifest["records"]
    summary = json.loads((out / "summary.json").read_text())
    for key in ("snapshot_path", "output_dir"):
        summary.pop(key)
    assert summary == golden_manifest["summary"]


def test_store_returns_gptq_layer(repacked):
    out, src = repacked
    store = ck.RepackedStore(out)
    assert store.layers == (0, 1) and store.num_experts == 4
    g, group = store.gptq_layer(1)
    assert group == 128
    key = lambda e, p, k: f"model.language_model.layers.1.mlp.experts.{e}.{p}.{k}"
    for e in range(4):
        for kind, name in (("qweight", "qweight"), ("qzeros", "qzeros"), ("scales", "scales")):
            w13 = torch.cat([src[key(e, "gate_proj", kind)], src[key(e, "up_proj", kind)]], dim=1)
            assert torch.equal(g[f"w13_{name}"][e], w13)
            assert torch.equal(g[f"w2_{name}"][e], src[key(e, "down_proj", kind)])
    assert g["w13_qweight"].shape == (4, 256 // 8, 2 * 128) and g["w2_qweight"].shape == (4, 128 // 8, 256)


def test_store_rejects_corruption_and_act_order(repacked):
    from safetensors.torch import load_file, save_file
    out, _ = repacked
    path = out / "layer_00.safetensors"
    t = load_file(str(path))
    t["experts.up_proj.scales"][0, 0, 0] += 1.0
    save_file(t, str(path))
    store = ck.RepackedStore(out)
    with pytest.raises(ValueError, match="sha256"):
        store.tensors(0)
    store.tensors(0, verify=False)  # shapes and dtypes still match
    t = load_file(str(out / "layer_01.safetensors"))
    t["experts.gate_proj.g_idx"] = t["experts.gate_proj.g_idx"].flip(1).contiguous()
    save_file(t, str(out / "layer_01.safetensors"))
    with pytest.raises(ValueError, match="act-order"):
        ck.RepackedStore(out).gptq_layer(1, verify=False)


def test_repack_refuses_missing_experts_and_overwrite(tmp_path):
    make_gptq_snapshot(tmp_path / "snap", layers=1, experts=2, shards=1, seed=1)
    with pytest.raises(RuntimeError, match="missing"):
        ck.repack_snapshot(tmp_path / "snap", tmp_path / "out", num_experts=3)
    ck.repack_snapshot(tmp_path / "snap", tmp_path / "out2", num_experts=2)
    with pytest.raises(FileExistsError):
        ck.repack_snapshot(tmp_path / "snap", tmp_path / "out2", num_experts=2)
