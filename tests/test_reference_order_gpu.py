"""Reference summation order (b200_set_summation_order(B200_ORDER_REFERENCE)):
the decode GEMVs and the fused LM head must be BIT-IDENTICAL to the
reference's own CUDA kernels (src/cuda/kernels.cu, built unchanged for
sm_100a) and to the CPU restatement of their operation order
(oracle_gemv_reference_order), at the configs[1] shapes.  The prefill GEMMs
need no mode: their tensor-core K order gives the reference WMMA kernels'
results exactly, checked here at configs[2] token counts."""
import numpy as np
import pytest

from conftest import from_bits, to_bits
from patterns import QWEN_SHAPES, seeded_linear

pytestmark = pytest.mark.gpu


@pytest.fixture
def reference_order(b200):
    b200.set_summation_order("reference")
    assert b200.summation_order() == b200.ORDER_REFERENCE
    yield b200
    b200.set_summation_order("fast")


@pytest.fixture(scope="module")
def ref(oracle):
    r = oracle.ref_cuda()
    if r is None:
        pytest.skip("oracle/_ref/libref_kernels.so not built")
    return r


def _case(oracle, n, k, seed):
    w, b = seeded_linear(n, k, seed, bias=True)
    rng = np.random.default_rng(seed + 1)
    x = oracle.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    return w, oracle.f32_to_bf16(b), x


@pytest.mark.parametrize("k,n", QWEN_SHAPES)
@pytest.mark.parametrize("w8", [True, False], ids=["w8a16", "bf16"])
def test_gemv_bit_identical_to_reference_kernels(reference_order, oracle, ref, cuda,
                                                 k, n, w8):
    import torch
    b200 = reference_order
    w, bb, xb = _case(oracle, n, k, seed=n + k)
    st = torch.cuda.current_stream().cuda_stream
    db, dx = from_bits(bb, cuda), from_bits(xb, cuda)
    ours = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    theirs = torch.empty_like(ours)
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        dq, ds = torch.from_numpy(q).to(cuda), from_bits(sb, cuda)
        b200.gemv_w8a16(dq, ds, 64, db, dx, ours, n, k)
        assert ref.ref_gemv_w8a16(dq.data_ptr(), ds.data_ptr(), 64, db.data_ptr(),
                                  dx.data_ptr(), theirs.data_ptr(), n, k, st) == 0
        exp = oracle.gemv_reference_order(q, bb, xb, scales=sb)
    else:
        wb = oracle.f32_to_bf16(w)
        dw = from_bits(wb, cuda)
        b200.gemv_bf16(dw, db, dx, ours, n, k)
        assert ref.ref_gemv_bf16(dw.data_ptr(), db.data_ptr(), dx.data_ptr(),
                                 theirs.data_ptr(), n, k, st) == 0
        exp = oracle.gemv_reference_order(wb, bb, xb)
    a, r = to_bits(ours), to_bits(theirs)
    assert np.array_equal(r, exp), "oracle vs reference kernels"
    assert np.array_equal(a, r), f"{int((a != r).sum())} of {n} outputs differ"
    assert b200.device_status() == 0


def test_lm_head_bit_identical_to_reference_kernel(reference_order, oracle, ref, cuda):
    """Full 151936 vocabulary: logits and argmax equal to the reference's
    lm_head_bf16; the workspace and the no-allocation entry points alike."""
    import torch
    b200 = reference_order
    v, k = 151936, 896
    st = torch.cuda.current_stream().cuda_stream
    for seed in (3, 4):
        w, _, xb = _case(oracle, v, k, seed=seed)
        wb = oracle.f32_to_bf16(w)
        dw, dx = from_bits(wb, cuda), from_bits(xb, cuda)
        ours = torch.empty(v, dtype=torch.bfloat16, device=cuda)
        theirs = torch.empty_like(ours)
        nl = torch.empty_like(ours)
        bv, bi = b200.lm_head_workspace(v, cuda)
        am = torch.empty(1, dtype=torch.int32, device=cuda)
        am_ref = torch.empty_like(am)
        am_na = torch.empty_like(am)
        b200.lm_head_bf16(dw, None, dx, ours, bv, bi, am, v, k)
        rbv = torch.empty((v + 7) // 8, dtype=torch.float32, device=cuda)
        rbi = torch.empty((v + 7) // 8, dtype=torch.int32, device=cuda)
        assert ref.ref_lm_head_bf16(dw.data_ptr(), None, dx.data_ptr(), theirs.data_ptr(),
                                    rbv.data_ptr(), rbi.data_ptr(), am_ref.data_ptr(),
                                    v, k, st) == 0
        b200.ABI.b200_lm_head_bf16_noalloc(dw.data_ptr(), None, dx.data_ptr(), nl.data_ptr(),
                                           am_na.data_ptr(), v, k, st)
        torch.cuda.synchronize()
        a, r = to_bits(ours), to_bits(theirs)
        assert np.array_equal(a, r), f"{int((a != r).sum())} logits differ"
        assert np.array_equal(to_bits(nl), r)
        assert int(am.item()) == int(am_ref.item()) == int(am_na.item())
        exp = oracle.gemv_reference_order(wb, None, xb, lm_head=True)
        assert np.array_equal(r, exp), "oracle vs reference kernel"


@pytest.mark.parametrize("m", [32, 128, 2048])
@pytest.mark.parametrize("k,n", QWEN_SHAPES)
def test_prefill_gemm_bit_identical_to_reference_wmma(reference_order, oracle, ref, cuda, m,
                                                       k, n):
    """The tcgen05 GEMMs (both precisions; W8A16 one-pass and dequantise-once
    routes) against the reference WMMA kernels on the same buffers (in the
    reference order: the fast order splits K for short prompts)."""
    import torch
    b200 = reference_order
    if n == 151936 and m > 128:
        pytest.skip("reference WMMA kernel at this size takes long; covered at M<=128")
    w, bb, _ = _case(oracle, n, k, seed=7 * n + k)
    x = oracle.f32_to_bf16(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32))
    st = torch.cuda.current_stream().cuda_stream
    db, dx = from_bits(bb, cuda), from_bits(x, cuda)
    ours = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    theirs = torch.empty_like(ours)
    q, sb = oracle.quantize_groupwise(w)
    dq, ds = torch.from_numpy(q).to(cuda), from_bits(sb, cuda)
    b200.gemm_w8a16(dq, ds, 64, db, dx, ours, m, n, k)
    assert ref.ref_gemm_w8a16(dq.data_ptr(), ds.data_ptr(), 64, db.data_ptr(), dx.data_ptr(),
                              theirs.data_ptr(), m, n, k, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(ours, theirs), "w8a16"
    dw = from_bits(oracle.f32_to_bf16(w), cuda)
    b200.gemm_bf16(dw, db, dx, ours, m, n, k)
    assert ref.ref_gemm_bf16(dw.data_ptr(), db.data_ptr(), dx.data_ptr(), theirs.data_ptr(),
                             m, n, k, st) == 0
    torch.cuda.synchronize()
    assert torch.equal(ours, theirs), "bf16"
