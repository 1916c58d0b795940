"""The oracle (CPU restatement) pinned against the reference itself.

Golden fixtures come from the reference's own exporter and its CPU FP32
Linear (tests/golden/make_golden.py); the known answers below are the
reference exporter's self-test values (tools/export_model.py:414-428)."""
import os

import numpy as np
import pytest

from conftest import golden
from golden.make_golden import BF16_CASES, bf16_linear_patterns


def test_bf16_known_answers(oracle):
    # tools/export_model.py:414-428: exact values, tie-to-even, NaN stays NaN.
    exact = np.array([0.0, -0.0, 1.0, -2.5, np.inf, -np.inf], dtype=np.float32)
    assert np.array_equal(oracle.bf16_to_f32(oracle.f32_to_bf16(exact)), exact)
    tie = np.array([1.0 + 1.0 / 256.0], dtype=np.float32)
    assert int(oracle.f32_to_bf16(tie)[0]) == 0x3F80
    above = np.nextafter(tie, np.float32(np.inf))
    assert int(oracle.f32_to_bf16(above)[0]) == 0x3F81
    assert np.isnan(oracle.bf16_to_f32(oracle.f32_to_bf16(np.array([np.nan], np.float32)))[0])


def test_bf16_matches_reference_exporter(oracle):
    g = golden("exporter_kat.npz")
    assert np.array_equal(oracle.f32_to_bf16(g["f32"]), g["bf16_bits"])


@pytest.mark.parametrize("name", ["q_24x200", "q_8x70", "q_16x896", "q_5x65"])
def test_quantizer_matches_reference_exporter(oracle, name):
    g = golden("exporter_kat.npz")
    q, s = oracle.quantize_groupwise(g[name + "_w"], 64)
    assert np.array_equal(q, g[name + "_q"])
    assert np.array_equal(s, g[name + "_s"])


@pytest.mark.parametrize("case", BF16_CASES)
def test_linear_bf16_matches_reference_cpu(oracle, case):
    m, n, k, with_bias = case
    g = golden("cpu_linear.npz")
    w, x, b = bf16_linear_patterns(m, n, k)
    wb, xb, bb = oracle.f32_to_bf16(w), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    y = oracle.linear_bf16(wb, bb if with_bias else None, xb)
    ref = g[f"{m}x{n}x{k}_batch"]
    # Same products, different summation order (OpenBLAS): FP32 rounding only.
    np.testing.assert_allclose(y, ref, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(y[0], g[f"{m}x{n}x{k}_gemv"], rtol=1e-5, atol=1e-5)


def test_w8a16_gemv_and_gemm_dequant_forms(oracle):
    # Reference test pattern (tests/test_cuda.cpp:524-547) at K=70 (tail group).
    n, k, m = 5, 70, 3
    idx = np.arange(n * k)
    q = ((idx * 17 % 31) - 15).astype(np.int8).reshape(n, k)
    q.flat[0], q.flat[1] = -127, 127
    groups = (k + 63) // 64
    s = ((1 + np.arange(n * groups) % 7) / 1024.0).astype(np.float32).reshape(n, groups)
    q[n - 1, :64] = 0
    s[n - 1, 0] = 1.0
    x = (((np.arange(m * k) * 13 % 29) - 14) / 64.0).astype(np.float32).reshape(m, k)
    sb, xb = oracle.f32_to_bf16(s), oracle.f32_to_bf16(x)
    y0 = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, None, xb, gemm=False))
    y1 = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, None, xb, gemm=True))
    # Plain float64 evaluation of the same dequantised product.
    deq = q.astype(np.float64) * oracle.bf16_to_f32(sb).astype(np.float64).repeat(64, 1)[:, :k]
    exact = oracle.bf16_to_f32(xb).astype(np.float64) @ deq.T
    tol = np.maximum(1.0 / 64, np.abs(exact) * 0.01)
    assert np.all(np.abs(y0 - exact) <= tol)
    assert np.all(np.abs(y1 - exact) <= tol)


def test_argmax_ties_and_degenerate(oracle):
    v = oracle.f32_to_bf16(np.array([1.0, 3.0, 2.0, 3.0], np.float32))
    assert oracle.argmax_bf16(v) == 1
    v = oracle.f32_to_bf16(np.array([-np.inf, np.nan, -np.inf], np.float32))
    assert oracle.argmax_bf16(v) == 0
    assert oracle.argmax_bf16(np.zeros(0, np.uint16)) == 0


def test_reference_order_matches_reference_cuda_kernels(oracle):
    """The CPU restatement of the reference decode kernels' FP32 operation
    order (oracle_gemv_reference_order) against outputs of the reference's
    own CUDA kernels, bit for bit (fixture made on a B200 by
    tests/golden/make_ref_kernel_golden.py)."""
    from golden.make_ref_kernel_golden import REF_ORDER_CASES, ref_order_inputs
    path = os.path.join(os.path.dirname(__file__), "golden", "ref_kernels_order.npz")
    if not os.path.exists(path):
        pytest.skip("ref_kernels_order.npz not generated yet")
    g = np.load(path)
    for i, (name, kind, n, k) in enumerate(REF_ORDER_CASES):
        w, s, b, x = ref_order_inputs(kind, n, k, 100 + i)
        got = oracle.gemv_reference_order(w, b, x, scales=s, lm_head=(kind == "lm"))
        assert np.array_equal(got, g[name]), name
