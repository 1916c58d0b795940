"""Decode GEMV (BF16 and W8A16) on the GPU against the oracle, the
reference's own CUDA kernels (built for sm_100a) and the reference test
tolerances (tests/test_cuda.cpp:611-619, 596-598)."""
import numpy as np
import pytest

from conftest import from_bits, to_bits
from patterns import QWEN_SHAPES, gemv_bf16_case, seeded_linear, w8a16_case

pytestmark = pytest.mark.gpu


def bf16_tol(expected):
    return np.maximum(0.004, np.abs(expected) * 0.008)


def w8_tol(expected):
    return np.maximum(1.0 / 64, np.abs(expected) * 0.01)


def north_star_ok(actual, expected):
    return np.all(np.abs(actual - expected) <= 2e-2 + 1e-2 * np.abs(expected))


# reference tests/test_cuda.cpp:775-786
BF16_GEMV_CASES = [(896, 896, True), (128, 896, True), (4864, 896, False),
                   (896, 4864, False), (1024, 1024, True), (897, 896, False),
                   (3, 1024, False), (512, 70, True)]


@pytest.mark.parametrize("n,k,with_bias", BF16_GEMV_CASES)
def test_gemv_bf16_reference_shapes(b200, oracle, cuda, n, k, with_bias):
    import torch
    w, x, b = gemv_bf16_case(n, k)
    wb, xb, bb = oracle.f32_to_bf16(w), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    dw, dx = from_bits(wb, cuda), from_bits(xb, cuda)
    db = from_bits(bb, cuda) if with_bias else None
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    b200.gemv_bf16(dw, db, dx, y, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.linear_bf16(wb, bb if with_bias else None, xb)[0]
    assert np.all(np.abs(got - exp) <= bf16_tol(exp))


@pytest.mark.parametrize("tokens,n,k,with_bias",
                         [(1, 5, 70, True), (1, 7, 65, False), (1, 896, 896, True),
                          (1, 128, 896, True), (1, 4864, 896, False),
                          (1, 896, 4864, False), (1, 896, 1024, True),
                          (1, 896, 1216, False), (1, 24, 896, True), (1, 96, 912, False)])
def test_gemv_w8a16_reference_shapes(b200, oracle, cuda, tokens, n, k, with_bias):
    import torch
    q, s, x, b = w8a16_case(tokens, n, k)
    sb, xb, bb = oracle.f32_to_bf16(s), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    b200.gemv_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64,
                    from_bits(bb, cuda) if with_bias else None,
                    from_bits(xb[0], cuda), y, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb if with_bias else None,
                                                 xb[0], gemm=False))[0]
    assert np.all(np.abs(got - exp) <= w8_tol(exp))


@pytest.mark.parametrize("k,n", QWEN_SHAPES)
@pytest.mark.parametrize("w8", [True, False])
def test_gemv_baseline_shapes_seeded(b200, oracle, cuda, k, n, w8):
    """N(0,0.02) weights (exporter quantiser), x ~ N(0,1)."""
    import torch
    w, bias = seeded_linear(n, k, seed=1000 + k + n, bias=(n <= 896 and k == 896))
    x = np.random.default_rng(k * 7 + n).standard_normal(k).astype(np.float32)
    xb = oracle.f32_to_bf16(x)
    bb = oracle.f32_to_bf16(bias) if bias is not None else None
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    db = from_bits(bb, cuda) if bb is not None else None
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        b200.gemv_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64, db,
                        from_bits(xb, cuda), y, n, k)
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb, xb, gemm=False))[0]
    else:
        wb = oracle.f32_to_bf16(w)
        b200.gemv_bf16(from_bits(wb, cuda), db, from_bits(xb, cuda), y, n, k)
        exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, bb, xb)[0]))
    got = oracle.bf16_to_f32(to_bits(y))
    assert north_star_ok(got, exp)
    # Differences are FP32 summation order only: at most 1 BF16 ulp.
    ulp = np.abs(exp) * 2.0 ** -7 + 1e-30
    assert np.all(np.abs(got - exp) <= ulp * 1.01 + 1e-4)


def test_gemv_matches_reference_cuda_kernels(b200, oracle, cuda):
    """Same device buffers through the reference's own kernels (sm_100a)."""
    import ctypes
    import torch
    ref = oracle.ref_cuda()
    if ref is None:
        pytest.skip("oracle/_ref/libref_kernels.so not built")
    for (k, n) in QWEN_SHAPES[:4]:
        w, _ = seeded_linear(n, k, seed=k + 3 * n)
        q, sb = oracle.quantize_groupwise(w)
        x = oracle.f32_to_bf16(np.random.default_rng(n).standard_normal(k).astype(np.float32))
        dq, ds, dx = torch.from_numpy(q).to(cuda), from_bits(sb, cuda), from_bits(x, cuda)
        ours = torch.empty(n, dtype=torch.bfloat16, device=cuda)
        theirs = torch.empty_like(ours)
        b200.gemv_w8a16(dq, ds, 64, None, dx, ours, n, k)
        s = torch.cuda.current_stream().cuda_stream
        assert ref.ref_gemv_w8a16(dq.data_ptr(), ds.data_ptr(), 64, None, dx.data_ptr(),
                                  theirs.data_ptr(), n, k, s) == 0
        a, r = oracle.bf16_to_f32(to_bits(ours)), oracle.bf16_to_f32(to_bits(theirs))
        assert north_star_ok(a, r)
        assert np.all(np.abs(a - r) <= w8_tol(r))
        wb = oracle.f32_to_bf16(w)
        dw = from_bits(wb, cuda)
        b200.gemv_bf16(dw, None, dx, ours, n, k)
        assert ref.ref_gemv_bf16(dw.data_ptr(), None, dx.data_ptr(), theirs.data_ptr(),
                                 n, k, s) == 0
        a, r = oracle.bf16_to_f32(to_bits(ours)), oracle.bf16_to_f32(to_bits(theirs))
        assert np.all(np.abs(a - r) <= bf16_tol(r))


def test_gemv_unaligned_and_k_zero(b200, oracle, cuda):
    import torch
    n, k = 37, 40
    w, x, b = gemv_bf16_case(n, k)
    wb, xb, bb = oracle.f32_to_bf16(w), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    # Offset every buffer by one element: 2-byte aligned only.
    dw = from_bits(np.concatenate([[0], wb.ravel()]).astype(np.uint16), cuda)[1:]
    dx = from_bits(np.concatenate([[0], xb]).astype(np.uint16), cuda)[1:]
    y = torch.empty(n + 1, dtype=torch.bfloat16, device=cuda)[1:]
    b200.gemv_bf16(dw, from_bits(bb, cuda), dx, y, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.linear_bf16(wb, bb, xb)[0]
    assert np.all(np.abs(got - exp) <= bf16_tol(exp))
    # K = 0: output is the bias (empty dot product).
    b200.gemv_bf16(dw, from_bits(bb, cuda), dx, y, n, 0)
    assert np.array_equal(to_bits(y), bb)
    assert b200.device_status() == 0


@pytest.mark.parametrize("n,k", [(8, 64), (16, 128), (24, 896), (40, 4864), (1000, 896),
                                 (2056, 1024), (4096, 2048), (512, 8192), (64, 12288),
                                 (8, 30000)])
@pytest.mark.parametrize("w8", [True, False])
def test_gemv_tile_geometries(b200, oracle, cuda, n, k, w8):
    """Partial tiles, split rows and the large-K fallbacks of the TMA path."""
    import torch
    w, _ = seeded_linear(n, k, seed=n * 31 + k)
    x = oracle.f32_to_bf16(np.random.default_rng(n + k).standard_normal(k).astype(np.float32))
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        b200.gemv_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64, None,
                        from_bits(x, cuda), y, n, k)
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, None, x, gemm=False))[0]
    else:
        wb = oracle.f32_to_bf16(w)
        b200.gemv_bf16(from_bits(wb, cuda), None, from_bits(x, cuda), y, n, k)
        exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, None, x)[0]))
    got = oracle.bf16_to_f32(to_bits(y))
    assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)
    assert b200.device_status() == 0
