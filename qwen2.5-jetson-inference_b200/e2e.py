"""End-to-end runs of the reference engine with the b200 Linear kernels.

The engine (reference src/qwen2.cpp, unchanged) is built by adapter/Makefile
twice: ``e2e_b200`` (Linear layers from libb200linear.so through the C++
adapter) and ``e2e_reference`` (the reference's own Linear kernels), both
driving adapter/e2e_driver.cpp.  This module writes the seeded synthetic
model (qbin.py), runs either binary and parses its JSON line.
"""
from __future__ import annotations

import json
import os
import subprocess

import numpy as np

from . import qbin

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "adapter", "_build")


def binary(kind: str) -> str:
    """Path of the e2e driver linked with 'b200' or 'reference' Linear kernels."""
    path = os.path.join(BUILD, f"e2e_{kind}")
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (make -C adapter, needs the "
                                "reference sources)")
    return path


def ensure_model(directory: str, config: dict, seed: int = 0,
                 precisions=("fp32", "w16a16", "w8a16")) -> str:
    """Writes the synthetic model once (a marker file records the config)."""
    marker = os.path.join(directory, "synthetic.json")
    want = {"config": config, "seed": seed, "precisions": list(precisions)}
    if os.path.exists(marker):
        with open(marker) as f:
            if json.load(f) == want:
                return directory
    qbin.write_model(directory, config, seed, precisions)
    with open(marker, "w") as f:
        json.dump(want, f)
    return directory


def prompt_ids(n: int = 32, vocab: int = 151936, seed: int = 0) -> list[int]:
    """Seeded prompt of token ids uniform in [0, vocab)."""
    return np.random.default_rng(seed).integers(0, vocab, n).tolist()


def run(kind: str, model_dir: str, prompt: list[int], backend: str = "cuda",
        precision: str = "w16a16", linear_kernel: str = "custom", new_tokens: int = 128,
        warmup: int = 5, repeat: int = 20, max_seq_len: int = 256,
        logits_out: str | None = None, force_tokens: list[int] | None = None,
        timeout: int = 1800, summation_order: str | None = None) -> dict:
    """Runs one binary; summation_order ("reference" / "fast") sets the b200
    library's decode summation order (B200_SUMMATION_ORDER) for that run."""
    cmd = [binary(kind), "--model", model_dir, "--backend", backend, "--precision",
           precision, "--linear-kernel", linear_kernel, "--token-ids",
           ",".join(map(str, prompt)), "--new-tokens", str(new_tokens), "--warmup",
           str(warmup), "--repeat", str(repeat), "--max-seq-len", str(max_seq_len)]
    if logits_out:
        cmd += ["--logits-out", logits_out]
    if force_tokens:
        cmd += ["--force-tokens", ",".join(map(str, force_tokens))]
    env = dict(os.environ)
    if summation_order is not None:
        env["B200_SUMMATION_ORDER"] = summation_order
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    if proc.returncode != 0:
        raise RuntimeError(f"{' '.join(cmd[:2])} failed: {proc.stderr[-2000:]}")
    return json.loads(proc.stdout.strip().splitlines()[-1])


def forced_agreement(ours: dict, reference_tokens: list[int]) -> dict:
    """Teacher-forced comparison: our argmax at every step when fed the
    reference engine's tokens.  Disagreements are classified by the gap
    between our two largest logits, in BF16 ulps of the top logit (the LM head
    argmax runs on BF16-rounded logits)."""
    am, gaps = ours["forced_argmax"], ours["forced_gap"]
    n = min(len(am), len(reference_tokens))
    dis = [j for j in range(n) if am[j] != reference_tokens[j]]
    return {"steps": n, "agree": n - len(dis),
            "disagree_steps": dis,
            "disagree_gaps": [round(gaps[j], 5) for j in dis]}
