"""W8A16 decode GEMV on the integer tensor cores (gemv_i8tc.cu, the default
W8A16 GEMV kernel selected by B200_GEMV_I8TC=1) against the oracle
(oracle_linear_w8a16: reference tests/test_cuda.cpp:494-517 arithmetic).  Matrices of fewer rows
take the CUDA-core kernels; they stay in the parametrisation as a check of
the default W8A16 GEMV at the Qwen2.5 shapes.

The kernel sums each 64-wide group exactly in INT32 (x split into integer
limbs per group) and rounds only when combining groups, so every output must
be within one BF16 ulp of the oracle's sequential FP32 sum; edge cases: all
zero x, an exponent spread of more than 2^13 inside one group, ragged row
counts, one group (K = 64), long K, and the fused LM-head argmax with ties."""
import numpy as np
import pytest

from conftest import from_bits, to_bits

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def i8tc_on():
    import os
    os.environ["B200_GEMV_I8TC"] = "1"
    yield
    del os.environ["B200_GEMV_I8TC"]


def one_ulp_ok(got, exp):
    """|got - exp| <= one BF16 ulp of exp (plus the FP32 noise floor)."""
    e = np.abs(exp).astype(np.float32)
    ulp = np.where(e > 0, 2.0 ** (np.floor(np.log2(np.maximum(e, 1e-30))) - 7), 2.0 ** -133)
    return np.abs(got - exp) <= ulp * 1.0001 + 1e-6


def run(b200, oracle, cuda, n, k, x_f32, seed=0, bias=True):
    import torch
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    q, sb = oracle.quantize_groupwise(w)
    xb = oracle.f32_to_bf16(x_f32)
    bb = oracle.f32_to_bf16(rng.normal(0, 0.02, n).astype(np.float32)) if bias else None
    y = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    b200.gemv_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64,
                    from_bits(bb, cuda) if bias else None, from_bits(xb, cuda), y, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb, xb))[0]
    assert b200.device_status() == 0
    return got, exp


@pytest.mark.parametrize("n,k", [(896, 896), (4864, 896), (896, 4864), (151936, 896),
                                 (80000, 64), (76000, 1088), (75800, 2048)])
def test_i8tc_gemv_within_one_ulp(b200, oracle, cuda, n, k):
    x = np.random.default_rng(n + k).standard_normal(k).astype(np.float32)
    got, exp = run(b200, oracle, cuda, n, k, x)
    assert one_ulp_ok(got, exp).all()
    assert np.mean(got == exp) > 0.95


def test_i8tc_gemv_edge_inputs(b200, oracle, cuda):
    k, n = 896, 75904
    # all-zero x: y == bias exactly
    got, exp = run(b200, oracle, cuda, n, k, np.zeros(k, np.float32))
    assert np.array_equal(got, exp)
    # exponent spread of > 2^13 inside groups (dropped bits below 2^-20 of
    # the group's largest element)
    x = np.random.default_rng(3).standard_normal(k).astype(np.float32) * 1e-4
    x[::64] = 300.0
    x[5::64] = -7e-6
    got, exp = run(b200, oracle, cuda, n, k, x, seed=4)
    assert np.all(np.abs(got - exp) <= 2e-2 + 1e-2 * np.abs(exp))
    assert one_ulp_ok(got, exp).mean() > 0.99
    # subnormal-free tiny values and signed zeros
    x = np.random.default_rng(5).standard_normal(k).astype(np.float32)
    x[1::7] = -0.0
    got, exp = run(b200, oracle, cuda, n, k, x, seed=6, bias=False)
    assert one_ulp_ok(got, exp).all()


def test_i8tc_lm_head_argmax_and_ties(b200, oracle, cuda):
    import torch
    v, k = 151936, 896
    rng = np.random.default_rng(9)
    w = rng.normal(0, 0.02, (v, k)).astype(np.float32)
    q, sb = oracle.quantize_groupwise(w)
    for tie in [(17, 9000), (128 * 7 - 1, 128 * 7), (v - 2, v - 1)]:
        q2 = q.copy()
        q2[tie[0]] = 100
        q2[tie[1]] = 100
        s2 = sb.copy()
        s2[tie[0]] = s2[tie[1]] = oracle.f32_to_bf16(np.full(k // 64, 0.01, np.float32))
        x = rng.standard_normal(k).astype(np.float32)
        x[:] = np.abs(x) + 0.1
        xb = oracle.f32_to_bf16(x)
        logits = torch.empty(v, dtype=torch.bfloat16, device=cuda)
        bv, bi = b200.lm_head_workspace(v, cuda)
        am = torch.empty(1, dtype=torch.int32, device=cuda)
        b200.lm_head_w8a16(torch.from_numpy(q2).to(cuda), from_bits(s2, cuda), 64, None,
                           from_bits(xb, cuda), logits, bv, bi, am, v, k)
        lg = to_bits(logits)
        assert int(am.item()) == oracle.argmax_bf16(lg) == tie[0]
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q2, s2, None, xb))[0]
        assert one_ulp_ok(oracle.bf16_to_f32(lg), exp).all()
