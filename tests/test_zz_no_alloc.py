"""The allocation-free LM head (b200_lm_head_bf16_noalloc).

Some callers cannot allocate device memory: a plugin host that passes a
kernel only its inputs and outputs, or code that is already recording a CUDA
graph (cudaMalloc is not allowed there).  This entry point keeps its argmax
scratch in a fixed array owned by the library.  The test calls it through the
C ABI twice in a row and checks each result against the workspace-taking
b200_lm_head_bf16 on the same inputs, with the LM-head tolerance used by the
other tests (max(0.008, 1%) on logits, identical argmax).  The file name
makes pytest collect it last."""
import numpy as np
import pytest

from conftest import from_bits, to_bits
from patterns import lm_head_tie_case, seeded_linear

pytestmark = pytest.mark.gpu


def _run_reference_entry(b200, cuda, w, x, vocab, k):
    import torch
    logits = torch.empty(vocab, dtype=torch.bfloat16, device=cuda)
    bv, bi = b200.lm_head_workspace(vocab, cuda)
    am = torch.empty(1, dtype=torch.int32, device=cuda)
    b200.lm_head_bf16(w, None, x, logits, bv, bi, am, vocab, k)
    return to_bits(logits), int(am.item())


def _run_noalloc(b200, cuda, w, x, vocab, k):
    import torch
    logits = torch.empty(vocab, dtype=torch.bfloat16, device=cuda)
    am = torch.full((1,), -5, dtype=torch.int32, device=cuda)
    stream = torch.cuda.current_stream().cuda_stream
    rc = b200.ABI.b200_lm_head_bf16_noalloc(w.data_ptr(), None, x.data_ptr(),
                                            logits.data_ptr(), am.data_ptr(),
                                            vocab, k, stream)
    assert rc == 0, b200.ABI.b200_status_string(rc)
    return to_bits(logits), int(am.item())


@pytest.mark.parametrize("vocab,k,tie", [(151936, 896, (70001, 70002)),
                                         (1000, 64, (3, 900)), (64, 896, (1, 31)),
                                         (262144, 64, (5, 262143)),  # the stated limit
                                         (1003, 70, (2, 1002))])     # generic path
def test_noalloc_matches_workspace_entry_point_twice(b200, oracle, cuda, vocab, k, tie):
    w, x = lm_head_tie_case(vocab, k, *tie) if vocab <= 1000 else (None, None)
    if w is None:
        w, _ = seeded_linear(vocab, k, seed=11)
        w = w.copy()
        w[tie[0], :] = w[tie[1], :] = 2.0
        x = np.random.default_rng(5).standard_normal(k).astype(np.float32)
        x[0] = 100.0  # the two tied rows dominate every other logit
    dw = from_bits(oracle.f32_to_bf16(w), cuda)
    dx = from_bits(oracle.f32_to_bf16(x), cuda)
    ref_bits, ref_am = _run_reference_entry(b200, cuda, dw, dx, vocab, k)
    ref = oracle.bf16_to_f32(ref_bits)
    for _ in range(2):
        bits, am = _run_noalloc(b200, cuda, dw, dx, vocab, k)
        got = oracle.bf16_to_f32(bits)
        assert np.all(np.abs(got - ref) <= np.maximum(0.008, np.abs(ref) * 0.01))
        assert am == ref_am == tie[0]


def test_noalloc_rejects_vocab_beyond_limit(b200, cuda):
    limit = int(b200.ABI.b200_lm_head_noalloc_max_vocab())
    assert limit == 262144
    rc = b200.ABI.b200_lm_head_bf16_noalloc(None, None, None, None, None,
                                            limit + 8, 896, None)
    assert rc == -1  # NULL argmax is checked first
    import torch
    am = torch.empty(1, dtype=torch.int32, device=cuda)
    rc = b200.ABI.b200_lm_head_bf16_noalloc(None, None, None, None, am.data_ptr(),
                                            limit + 8, 896, None)
    assert rc == -4
