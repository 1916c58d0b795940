"""QWENBIN1 weight archives (the engine's on-disk weight layouts).

Writes the three archives the reference engine loads --- ``model.fp32.qbin``,
``model.w16a16.qbin`` and ``model.w8a16.qbin`` (group-64 INT8 Linear weights +
BF16 scales) --- plus ``config.json``, from FP32 arrays.  The format is the
one the reference exporter writes and its archive reader checks
(reference tools/export_model.py:25-30, 99-107, 202-223, 273-345;
src/archive.cpp:49-102):

* header ``<8sIIQQ``: magic ``QWENBIN1``, version 1, JSON size, data offset
  (1 MiB), 0; the JSON metadata follows the header;
* tensors sorted by name, each at a 256-byte aligned offset relative to the
  data offset, with name / shape / dtype / offset / nbytes / sha256;
* ``w8a16``: 2-D tensors other than the embedding / LM head become int8 with
  a BF16 ``<name>.scale`` tensor written right after them (symmetric,
  group 64 along K, scale = max|w|/127, 0 -> 1.0, round-half-even, clip
  +-127); every other tensor is BF16 (round-to-nearest-even);
* ``w16a16``: every tensor BF16; ``fp32``: every tensor FP32.

Also makes the seeded synthetic Qwen2.5-0.5B weights of BASELINE configs[0]
(N(0, 0.02) matrices, zero biases, unit norm gains, tied embeddings), which
stand in for the real checkpoint (not available offline).
"""
from __future__ import annotations

import hashlib
import json
import os
import struct

import numpy as np

MAGIC = b"QWENBIN1"
VERSION = 1
DATA_OFFSET = 1024 * 1024
ALIGNMENT = 256
HEADER = struct.Struct("<8sIIQQ")
ARCHIVE_NAMES = {"fp32": "model.fp32.qbin", "w16a16": "model.w16a16.qbin",
                 "w8a16": "model.w8a16.qbin"}

QWEN25_05B = dict(hidden_size=896, intermediate_size=4864, num_hidden_layers=24,
                  num_attention_heads=14, num_key_value_heads=2, vocab_size=151936,
                  max_position_embeddings=32768, rms_norm_eps=1e-6,
                  rope_theta=1000000.0, tie_word_embeddings=True, bos_token_id=151643,
                  eos_token_id=151645, model_type="qwen2")


def bf16_bits(a: np.ndarray) -> np.ndarray:
    """FP32 -> BF16 bits, round-to-nearest-even, NaN kept quiet."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32)
    out = ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype("<u2")
    nan = np.isnan(a)
    if nan.any():
        out[nan] = ((u[nan] >> 16) | np.uint32(0x40)).astype("<u2")
    return out


def quantize_groupwise(w: np.ndarray, group: int = 64):
    """(int8 q, FP32 scale [rows, groups]) by the exporter's rule."""
    rows, cols = w.shape
    groups = (cols + group - 1) // group
    pad = groups * group - cols
    wp = np.pad(w, ((0, 0), (0, pad))) if pad else w
    blocks = wp.reshape(rows, groups, group)
    scale = (np.abs(blocks).max(axis=2) / np.float32(127.0)).astype(np.float32)
    scale = np.where(scale == 0.0, np.float32(1.0), scale).astype(np.float32)
    q = np.clip(np.rint(blocks / scale[:, :, None]), -127, 127).astype(np.int8)
    return np.ascontiguousarray(q.reshape(rows, groups * group)[:, :cols]), scale


def _quantized(name: str, a: np.ndarray) -> bool:
    return a.ndim == 2 and name not in ("model.embed_tokens.weight", "lm_head.weight")


def write_archive(path: str, tensors: dict, precision: str, group_size: int = 64,
                  source: str = "synthetic") -> None:
    """Writes one QWENBIN1 archive from {name: FP32 array}."""
    records = []
    with open(path, "w+b") as f:
        f.truncate(DATA_OFFSET)
        f.seek(DATA_OFFSET)

        def put(name, arr, dtype, quant=None):
            rel = f.tell() - DATA_OFFSET
            pad = (-rel) % ALIGNMENT
            if pad:
                f.write(b"\0" * pad)
            offset = f.tell() - DATA_OFFSET
            arr = np.ascontiguousarray(arr)
            f.write(memoryview(arr).cast("B"))
            rec = {"name": name, "shape": list(arr.shape), "dtype": dtype, "offset": offset,
                   "nbytes": arr.nbytes,
                   "sha256": hashlib.sha256(memoryview(arr).cast("B")).hexdigest()}
            if quant is not None:
                rec["quant"] = quant
            records.append(rec)

        for name in sorted(tensors):
            a = np.asarray(tensors[name], dtype=np.float32)
            if precision == "w8a16" and _quantized(name, a):
                q, scale = quantize_groupwise(a, group_size)
                sname = name + ".scale"
                put(name, q, "int8", {"scheme": "symmetric_group_w8a16",
                                      "group_size": group_size, "axis": 1,
                                      "scale_tensor": sname, "scale_dtype": "bfloat16"})
                put(sname, bf16_bits(scale).reshape(scale.shape), "bfloat16")
            elif precision in ("w16a16", "w8a16"):
                put(name, bf16_bits(a).reshape(a.shape), "bfloat16")
            else:
                put(name, a, "float32")
        meta = {"format": "QWENBIN1", "version": VERSION, "source": source,
                "precision": precision,
                "group_size": group_size if precision == "w8a16" else None,
                "tensors": records}
        enc = json.dumps(meta, ensure_ascii=False, separators=(",", ":")).encode("utf-8")
        if HEADER.size + len(enc) > DATA_OFFSET:
            raise RuntimeError("archive JSON exceeds the reserved header region")
        f.seek(0)
        f.write(HEADER.pack(MAGIC, VERSION, len(enc), DATA_OFFSET, 0))
        f.write(enc)


def read_records(path: str) -> dict:
    """Metadata JSON of an archive (for checks)."""
    with open(path, "rb") as f:
        magic, version, json_size, data_offset, _ = HEADER.unpack(f.read(HEADER.size))
        if magic != MAGIC or version != VERSION:
            raise ValueError("not a QWENBIN1 archive")
        return json.loads(f.read(json_size))


def synthetic_qwen2(config: dict, seed: int = 0) -> dict:
    """Seeded synthetic weights: N(0, 0.02) matrices, zero biases, unit gains."""
    rng = np.random.default_rng(seed)
    h, ffn = config["hidden_size"], config["intermediate_size"]
    nh, nkv = config["num_attention_heads"], config["num_key_value_heads"]
    hd = h // nh
    t = {}

    def mat(rows, cols):
        return (rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(0.02))

    t["model.embed_tokens.weight"] = mat(config["vocab_size"], h)
    for i in range(config["num_hidden_layers"]):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = np.ones(h, np.float32)
        t[p + "post_attention_layernorm.weight"] = np.ones(h, np.float32)
        t[p + "self_attn.q_proj.weight"] = mat(nh * hd, h)
        t[p + "self_attn.k_proj.weight"] = mat(nkv * hd, h)
        t[p + "self_attn.v_proj.weight"] = mat(nkv * hd, h)
        t[p + "self_attn.q_proj.bias"] = np.zeros(nh * hd, np.float32)
        t[p + "self_attn.k_proj.bias"] = np.zeros(nkv * hd, np.float32)
        t[p + "self_attn.v_proj.bias"] = np.zeros(nkv * hd, np.float32)
        t[p + "self_attn.o_proj.weight"] = mat(h, nh * hd)
        t[p + "mlp.gate_proj.weight"] = mat(ffn, h)
        t[p + "mlp.up_proj.weight"] = mat(ffn, h)
        t[p + "mlp.down_proj.weight"] = mat(h, ffn)
    t["model.norm.weight"] = np.ones(h, np.float32)
    if not config.get("tie_word_embeddings", True):
        t["lm_head.weight"] = mat(config["vocab_size"], h)
    return t


def write_model(directory: str, config: dict, seed: int = 0,
                precisions=("fp32", "w16a16", "w8a16")) -> None:
    """config.json + the requested archives of the synthetic model."""
    os.makedirs(directory, exist_ok=True)
    with open(os.path.join(directory, "config.json"), "w") as f:
        json.dump(config, f, indent=1)
    tensors = synthetic_qwen2(config, seed)
    for p in precisions:
        write_archive(os.path.join(directory, ARCHIVE_NAMES[p]), tensors, p)


def load_archive(path: str) -> dict:
    """{name: numpy array} of an archive (BF16 as uint16 bit patterns), as
    views of a read-only memory map."""
    meta = read_records(path)
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    dt = {"float32": np.float32, "bfloat16": np.uint16, "int8": np.int8}
    out = {}
    for rec in meta["tensors"]:
        raw = mm[DATA_OFFSET + rec["offset"]:DATA_OFFSET + rec["offset"] + rec["nbytes"]]
        out[rec["name"]] = raw.view(dt[rec["dtype"]]).reshape(rec["shape"])
    return out
