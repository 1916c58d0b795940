"""Generates the CPU golden fixtures in this directory from the REFERENCE itself.

Run in a container that has the reference checkout (--reference, default
$QWEN_REFERENCE_DIR or BASELINE.json's reference_path) and the reference CPU Linear built into
oracle/_ref (``make -C oracle ref``):

    python tests/golden/make_golden.py

Outputs (committed, small):
  exporter_kat.npz   reference tools/export_model.py float32_to_bfloat16 and
                     quantize_groupwise on seeded inputs (group 64, a K=70
                     tail, an all-zero group), i.e. the W8A16 qbin format;
  qbin_kat.json      archive metadata (dtype/shape/offset/size/SHA-256 of every
                     tensor) the reference exporter writes for a seeded tiny
                     Qwen2 in fp32 / w16a16 / w8a16 (weights from
                     qbin.synthetic_qwen2(TINY_QWEN2, seed=3) with zero groups);
  cpu_linear.npz     reference src/cpu_ops.cpp linear_fp32 / linear_fp32_batch
                     (OpenBLAS FP32) on the deterministic BF16 patterns of the
                     reference's tests/test_cuda.cpp:621-703 (check_bf16_linear_case).
The tests compare the oracle (oracle/linear_oracle.c) against these.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)


def bf16_linear_patterns(tokens, out_features, in_features):
    """Input patterns of reference tests/test_cuda.cpp:621-637."""
    idx_w = np.arange(out_features * in_features)
    weight = ((idx_w % 17) - 8).astype(np.float32) * 0.015625
    idx_x = np.arange(tokens * in_features)
    x = ((idx_x % 13) - 6).astype(np.float32) * 0.03125
    bias = ((np.arange(out_features) % 5) - 2).astype(np.float32) * 0.0625
    return (weight.reshape(out_features, in_features),
            x.reshape(tokens, in_features), bias)


BF16_CASES = [(3, 11, 14, True), (2, 5, 7, True), (3, 23, 14, False),
              (32, 64, 64, True), (31, 37, 33, True), (65, 70, 67, False)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=None)
    args = ap.parse_args()
    if args.reference is None:
        args.reference = os.environ.get("QWEN_REFERENCE_DIR")
    if args.reference is None:
        with open(os.path.join(REPO, "BASELINE.json")) as f:
            args.reference = json.load(f)["reference_path"]
    sys.path.insert(0, os.path.join(args.reference, "tools"))
    import export_model as E  # the reference exporter
    from oracle import oracle as O

    rng = np.random.default_rng(20240611)
    # --- BF16 conversion known answers (exporter self-test values + random).
    special = np.array([0.0, -0.0, 1.0, -2.5, np.inf, -np.inf, np.nan,
                        1.0 + 1.0 / 256.0,
                        np.nextafter(np.float32(1.0 + 1.0 / 256.0), np.float32(np.inf)),
                        3.0e38, -1.0e-40, 65504.0, 1.0 / 3.0], dtype=np.float32)
    randv = (rng.standard_normal(4096) * np.exp(rng.uniform(-20, 20, 4096))).astype(np.float32)
    f32 = np.concatenate([special, randv])
    bf16_bits = E.float32_to_bfloat16(f32)

    # --- Quantiser: seeded N(0, 0.02) weights, group 64, tails and a zero group.
    quant = {}
    for name, (rows, cols) in {"q_24x200": (24, 200), "q_8x70": (8, 70),
                               "q_16x896": (16, 896), "q_5x65": (5, 65)}.items():
        w = rng.normal(0.0, 0.02, (rows, cols)).astype(np.float32)
        w[rows - 1, :min(64, cols)] = 0.0      # an all-zero group -> scale 1.0
        w[0, 0] = 0.04                          # a row whose max is a round value
        q, s, _, _ = E.quantize_groupwise(w, 64)
        quant[name + "_w"] = w
        quant[name + "_q"] = q
        quant[name + "_s"] = E.float32_to_bfloat16(s).reshape(s.shape)
    np.savez_compressed(os.path.join(HERE, "exporter_kat.npz"),
                        f32=f32, bf16_bits=bf16_bits, **quant)

    # --- Reference CPU FP32 Linear on the reference test patterns.
    if O.ref_cpu() is None:
        raise SystemExit("oracle/_ref/libref_cpu_linear.so missing: make -C oracle ref")
    out = {}
    for (m, n, k, with_bias) in BF16_CASES:
        w, x, b = bf16_linear_patterns(m, n, k)
        wb, xb, bb = (O.bf16_to_f32(E.float32_to_bfloat16(a)).reshape(a.shape)
                      for a in (w, x, b))
        y = O.ref_cpu_linear(wb, bb if with_bias else None, xb)
        y1 = O.ref_cpu_linear(wb, bb if with_bias else None, xb[0])
        tag = f"{m}x{n}x{k}"
        out[tag + "_batch"] = y
        out[tag + "_gemv"] = y1
    np.savez_compressed(os.path.join(HERE, "cpu_linear.npz"), **out)
    make_qbin_kat(args.reference)
    print("wrote exporter_kat.npz, cpu_linear.npz, qbin_kat.json")



TINY_QWEN2 = dict(hidden_size=64, intermediate_size=160, num_hidden_layers=2,
                  num_attention_heads=4, num_key_value_heads=2, vocab_size=300,
                  max_position_embeddings=512, rms_norm_eps=1e-6, rope_theta=1000000.0,
                  tie_word_embeddings=True, bos_token_id=1, eos_token_id=2,
                  model_type="qwen2")


def make_qbin_kat(reference: str):
    """Archive metadata the reference exporter writes for a seeded tiny Qwen2
    (every tensor's dtype, shape, offset, size and SHA-256): the writer in
    qwen2.5-jetson-inference_b200/qbin.py must reproduce it exactly."""
    import importlib.util
    import struct
    import tempfile
    sys.path.insert(0, os.path.join(reference, "tools"))
    import export_model as E
    spec = importlib.util.spec_from_file_location(
        "qbin", os.path.join(REPO, "qwen2.5-jetson-inference_b200", "qbin.py"))
    Q = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(Q)
    tensors = Q.synthetic_qwen2(TINY_QWEN2, seed=3)
    tensors["model.layers.1.mlp.down_proj.weight"][:, :64] = 0.0  # zero groups
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        src = os.path.join(tmp, "src")
        os.makedirs(src)
        header, payload, off = {}, [], 0
        for name in sorted(tensors):
            a = np.ascontiguousarray(tensors[name], dtype="<f4")
            header[name] = {"dtype": "F32", "shape": list(a.shape),
                            "data_offsets": [off, off + a.nbytes]}
            payload.append(a)
            off += a.nbytes
        enc = json.dumps(header).encode()
        with open(os.path.join(src, "model.safetensors"), "wb") as f:
            f.write(struct.pack("<Q", len(enc)))
            f.write(enc)
            for a in payload:
                a.tofile(f)
        from pathlib import Path
        for prec in ("fp32", "w16a16", "w8a16"):
            dst = os.path.join(tmp, f"model.{prec}.qbin")
            E.export(Path(src), Path(dst), prec, 64)
            meta = Q.read_records(dst)
            meta.pop("source")
            out[prec] = meta
    with open(os.path.join(HERE, "qbin_kat.json"), "w") as f:
        json.dump({"config": TINY_QWEN2, "archives": out}, f, indent=0)


if __name__ == "__main__":
    main()
