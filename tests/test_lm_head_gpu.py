"""Fused LM head (GEMV + argmax) on the GPU: the reference's tie cases
(tests/test_cuda.cpp:790-880) and the full 896 -> 151936 head."""
import numpy as np
import pytest

from conftest import from_bits, to_bits
from patterns import lm_head_tie_case, seeded_linear

pytestmark = pytest.mark.gpu


def run_lm_head(b200, cuda, w_dev, x_dev, vocab, k, scales=None):
    import torch
    logits = torch.empty(vocab, dtype=torch.bfloat16, device=cuda)
    bv, bi = b200.lm_head_workspace(vocab, cuda)
    am = torch.full((1,), -7, dtype=torch.int32, device=cuda)
    if scales is None:
        b200.lm_head_bf16(w_dev, None, x_dev, logits, bv, bi, am, vocab, k)
    else:
        b200.lm_head_w8a16(w_dev, scales, 64, None, x_dev, logits, bv, bi, am, vocab, k)
    return logits, int(am.item())


@pytest.mark.parametrize("vocab,hidden,tie_a,tie_b",
                         [(512, 64, 3, 4), (1002, 64, 7, 71), (200, 10, 5, 22),
                          (8, 4, 0, 3), (64, 896, 1, 31), (4096, 896, 70, 4000),
                          (65536, 896, 30001, 30002), (151936, 896, 151934, 151935)])
def test_lm_head_ties_resolve_to_lowest_index(b200, oracle, cuda, vocab, hidden,
                                              tie_a, tie_b):
    w, x = lm_head_tie_case(vocab, hidden, tie_a, tie_b)
    wb, xb = oracle.f32_to_bf16(w), oracle.f32_to_bf16(x)
    logits, am = run_lm_head(b200, cuda, from_bits(wb, cuda), from_bits(xb, cuda),
                             vocab, hidden)
    got = oracle.bf16_to_f32(to_bits(logits))
    exp_bits, exp_am = oracle.lm_head(wb, None, xb)
    exp = oracle.bf16_to_f32(exp_bits)
    assert np.all(np.abs(got - exp) <= np.maximum(0.008, np.abs(exp) * 0.01))
    assert am == oracle.argmax_bf16(to_bits(logits))
    assert am == tie_a == exp_am


@pytest.mark.parametrize("w8", [False, True])
def test_lm_head_full_vocab(b200, oracle, cuda, w8):
    import torch
    vocab, k = 151936, 896
    w, _ = seeded_linear(vocab, k, seed=4242)
    x = oracle.f32_to_bf16(np.random.default_rng(99).standard_normal(k).astype(np.float32))
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        logits, am = run_lm_head(b200, cuda, torch.from_numpy(q).to(cuda),
                                 from_bits(x, cuda), vocab, k, scales=from_bits(sb, cuda))
        exp_bits, exp_am = oracle.lm_head(q, None, x, scales=sb)
    else:
        wb = oracle.f32_to_bf16(w)
        logits, am = run_lm_head(b200, cuda, from_bits(wb, cuda), from_bits(x, cuda),
                                 vocab, k)
        exp_bits, exp_am = oracle.lm_head(wb, None, x)
    bits = to_bits(logits)
    got, exp = oracle.bf16_to_f32(bits), oracle.bf16_to_f32(exp_bits)
    assert np.all(np.abs(got - exp) <= np.maximum(0.008, np.abs(exp) * 0.01))
    assert np.mean(bits == exp_bits) > 0.95
    # The fused argmax is the argmax of its own BF16 logits (reference criterion)...
    assert am == oracle.argmax_bf16(bits)
    # ...and the oracle's whenever the oracle's top two differ by more than 1 ulp.
    top = np.sort(exp)[-2:]
    if top[1] - top[0] > abs(top[1]) * 2.0 ** -7:
        assert am == exp_am


def test_argmax_bf16(b200, oracle, cuda):
    import torch
    rng = np.random.default_rng(3)
    for n in (1, 7, 1000, 151936):
        v = oracle.f32_to_bf16(rng.standard_normal(n).astype(np.float32))
        v[n // 2] = v[n - 1] = oracle.f32_to_bf16(np.array([9.0], np.float32))[0]
        out = torch.empty(1, dtype=torch.int32, device=cuda)
        b200.argmax_bf16(from_bits(v, cuda), n, out)
        assert int(out.item()) == oracle.argmax_bf16(v)
