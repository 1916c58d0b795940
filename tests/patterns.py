"""Deterministic inputs of the reference's CUDA tests (integer patterns, no
RNG) and the seeded synthetic inputs of the benchmark configs."""
import functools

import numpy as np


def w8a16_case(tokens, out_features, in_features):
    """reference tests/test_cuda.cpp:519-547 (check_w8a16_linear_case)."""
    g = 64
    groups = (in_features + g - 1) // g
    idx = np.arange(out_features * in_features, dtype=np.int64)
    q = ((idx * 17 % 31) - 15).astype(np.int8)
    if q.size >= 2:
        q[0], q[1] = -127, 127
    q = q.reshape(out_features, in_features)
    s = ((1 + np.arange(out_features * groups) % 7) / 1024.0).astype(np.float32)
    s = s.reshape(out_features, groups)
    x = (((np.arange(tokens * in_features, dtype=np.int64) * 13 % 29) - 14) / 64.0)
    x = x.astype(np.float32).reshape(tokens, in_features)
    bias = (((np.arange(out_features) % 9) - 4) / 32.0).astype(np.float32)
    if in_features > g:
        q[out_features - 1, :g] = 0
        s[out_features - 1, 0] = 1.0
    return q, s, x, bias


def gemv_bf16_case(out_features, in_features, seed=5):
    """reference tests/test_cuda.cpp:706-752 (make_gemv_weight + inputs)."""
    idx = np.arange(out_features * in_features, dtype=np.int64)
    w = ((((idx + seed) % 19) - 9) * 0.0078125).astype(np.float32)
    x = (((np.arange(in_features) % 11) - 5) * 0.015625).astype(np.float32)
    bias = (((np.arange(out_features) % 7) - 3) * 0.03125).astype(np.float32)
    return w.reshape(out_features, in_features), x, bias


def lm_head_tie_case(vocab, hidden, tie_a, tie_b):
    """reference tests/test_cuda.cpp:790-808 (check_lm_head_fused_case)."""
    w, _, _ = gemv_bf16_case(vocab, hidden, seed=11)
    w[tie_a, :] = 2.0
    w[tie_b, :] = 2.0
    x = np.empty(hidden, np.float32)
    x[0] = 100.0
    x[1:] = ((np.arange(1, hidden) % 13) - 6) * 0.0234375
    return w, x


# Decode GEMV sweep and prefill GEMM sweep: K -> N.
QWEN_SHAPES = [(896, 896), (896, 128), (896, 4864), (4864, 896), (896, 151936)]
PREFILL_M = [32, 128, 512, 2048, 8192]


@functools.lru_cache(maxsize=8)
def seeded_linear(n, k, seed, bias=False):
    """Seeded synthetic Linear: W ~ N(0, 0.02) FP32 (cached; do not mutate)."""
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    b = rng.normal(0.0, 0.02, n).astype(np.float32) if bias else None
    return w, b
