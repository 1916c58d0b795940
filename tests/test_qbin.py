"""The QWENBIN1 writer (qwen2.5-jetson-inference_b200/qbin.py) reproduces the
reference exporter's archives: every tensor's dtype, shape, offset, size and
SHA-256 (golden from tools/export_model.py, tests/golden/qbin_kat.json)."""
import importlib
import json
import os

import pytest

from conftest import REPO


@pytest.fixture(scope="module")
def qbin(b200):
    return importlib.import_module("qwen25_b200.qbin")


@pytest.mark.parametrize("precision", ["fp32", "w16a16", "w8a16"])
def test_archive_matches_reference_exporter(qbin, tmp_path, precision):
    kat = json.load(open(os.path.join(REPO, "tests", "golden", "qbin_kat.json")))
    tensors = qbin.synthetic_qwen2(kat["config"], seed=3)
    tensors["model.layers.1.mlp.down_proj.weight"][:, :64] = 0.0
    path = str(tmp_path / "m.qbin")
    qbin.write_archive(path, tensors, precision)
    meta = qbin.read_records(path)
    meta.pop("source")
    assert meta == kat["archives"][precision]


def test_synthetic_model_shapes(qbin):
    t = qbin.synthetic_qwen2(dict(qbin.QWEN25_05B, num_hidden_layers=1, vocab_size=64))
    assert t["model.layers.0.self_attn.k_proj.weight"].shape == (128, 896)
    assert t["model.layers.0.mlp.down_proj.weight"].shape == (896, 4864)
    assert "lm_head.weight" not in t  # tied
