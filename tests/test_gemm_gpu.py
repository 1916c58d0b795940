"""Prefill GEMM (tcgen05 tensor-core path and CUDA-core fallback) on the GPU
against the oracle: the reference test shapes (tests/test_cuda.cpp:694-703,
882-919) and the BASELINE prefill sweep on sampled rows."""
import numpy as np
import pytest

from conftest import from_bits, to_bits
from patterns import PREFILL_M, QWEN_SHAPES, seeded_linear, w8a16_case

pytestmark = pytest.mark.gpu


def bf16_tol(e):
    return np.maximum(0.004, np.abs(e) * 0.008)


def w8_tol(e):
    return np.maximum(1.0 / 64, np.abs(e) * 0.01)


def north_star_ok(a, e):
    return np.all(np.abs(a - e) <= 2e-2 + 1e-2 * np.abs(e))


def bf16_linear_patterns(tokens, n, k):
    from golden.make_golden import bf16_linear_patterns as p
    return p(tokens, n, k)


@pytest.mark.parametrize("m,n,k,with_bias",
                         [(3, 11, 14, True), (2, 5, 7, True), (3, 23, 14, False),
                          (32, 64, 64, True), (31, 37, 33, True), (65, 70, 67, False),
                          (130, 200, 136, True), (257, 384, 512, False)])
def test_gemm_bf16_reference_shapes(b200, oracle, cuda, m, n, k, with_bias):
    import torch
    w, x, b = bf16_linear_patterns(m, n, k)
    wb, xb, bb = oracle.f32_to_bf16(w), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    b200.gemm_bf16(from_bits(wb, cuda), from_bits(bb, cuda) if with_bias else None,
                   from_bits(xb, cuda), y, m, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.linear_bf16(wb, bb if with_bias else None, xb)
    assert np.all(np.abs(got - exp) <= bf16_tol(exp))


W8_CASES = ([(3, 5, 70, True), (2, 7, 65, False)] +
            [(2, n, k, bias) for (n, k, bias) in [(896, 896, True), (128, 896, True),
                                                   (4864, 896, False), (896, 4864, False)]] +
            [(t, n, k, bias) for t in (32, 128, 512)
             for (n, k, bias) in [(896, 896, True), (4864, 896, False), (896, 4864, False)]] +
            [(200, 96, 912, False), (129, 24, 1024, True)])


@pytest.mark.parametrize("m,n,k,with_bias", W8_CASES)
def test_gemm_w8a16_reference_shapes(b200, oracle, cuda, m, n, k, with_bias):
    """reference check_w8a16_linear_case: GEMM vs the dequantised reference
    and GEMV row 0 vs GEMM row 0."""
    import torch
    q, s, x, b = w8a16_case(m, n, k)
    sb, xb, bb = oracle.f32_to_bf16(s), oracle.f32_to_bf16(x), oracle.f32_to_bf16(b)
    dq, ds, dx = torch.from_numpy(q).to(cuda), from_bits(sb, cuda), from_bits(xb, cuda)
    db = from_bits(bb, cuda) if with_bias else None
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    b200.gemm_w8a16(dq, ds, 64, db, dx, y, m, n, k)
    got = oracle.bf16_to_f32(to_bits(y))
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb if with_bias else None, xb,
                                                 gemm=True))
    assert np.all(np.abs(got - exp) <= w8_tol(exp))
    gv = torch.empty(n, dtype=torch.bfloat16, device=cuda)
    b200.gemv_w8a16(dq, ds, 64, db, dx[0], gv, n, k)
    gvf = oracle.bf16_to_f32(to_bits(gv))
    assert np.all(np.abs(gvf - got[0]) <= w8_tol(got[0]))


@pytest.mark.parametrize("m", PREFILL_M)
@pytest.mark.parametrize("k,n", QWEN_SHAPES)
@pytest.mark.parametrize("w8", [True, False])
def test_gemm_prefill_sweep_sampled_rows(b200, oracle, cuda, m, k, n, w8):
    """configs[2] sizes; the oracle checks 24 sampled rows (all rows at M=32)."""
    import torch
    if m * n > 8192 * 4864 and not w8:
        m = 2048  # keep the BF16 896->151936 case at a size the oracle samples quickly
    w, bias = seeded_linear(n, k, seed=77 + k + n, bias=(n <= 896))
    rng = np.random.default_rng(m + k + n)
    x = oracle.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    bb = oracle.f32_to_bf16(bias) if bias is not None else None
    db = from_bits(bb, cuda) if bb is not None else None
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    rows = np.arange(m) if m <= 32 else np.unique(np.concatenate(
        [[0, m - 1], rng.choice(m, 22, replace=False)]))
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        b200.gemm_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64, db,
                        from_bits(x, cuda), y, m, n, k)
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb, x[rows], gemm=True))
    else:
        wb = oracle.f32_to_bf16(w)
        b200.gemm_bf16(from_bits(wb, cuda), db, from_bits(x, cuda), y, m, n, k)
        exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, bb, x[rows])))
    ybits = to_bits(y)
    got = oracle.bf16_to_f32(ybits[rows])
    assert north_star_ok(got, exp)
    assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)
    assert np.isfinite(oracle.bf16_to_f32(ybits)).all()


def test_gemm_matches_reference_cuda_kernels(b200, oracle, cuda):
    import torch
    ref = oracle.ref_cuda()
    if ref is None:
        pytest.skip("oracle/_ref/libref_kernels.so not built")
    s = torch.cuda.current_stream().cuda_stream
    for (m, k, n) in [(128, 896, 896), (512, 896, 4864), (128, 4864, 896)]:
        w, _ = seeded_linear(n, k, seed=m + n)
        q, sb = oracle.quantize_groupwise(w)
        x = oracle.f32_to_bf16(np.random.default_rng(m).standard_normal((m, k)).astype(np.float32))
        dq, ds, dx = torch.from_numpy(q).to(cuda), from_bits(sb, cuda), from_bits(x, cuda)
        ours = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        theirs = torch.empty_like(ours)
        b200.gemm_w8a16(dq, ds, 64, None, dx, ours, m, n, k)
        assert ref.ref_gemm_w8a16(dq.data_ptr(), ds.data_ptr(), 64, None, dx.data_ptr(),
                                  theirs.data_ptr(), m, n, k, s) == 0
        a, r = oracle.bf16_to_f32(to_bits(ours)), oracle.bf16_to_f32(to_bits(theirs))
        assert north_star_ok(a, r)
        assert np.all(np.abs(a - r) <= w8_tol(r))
        wb = oracle.f32_to_bf16(w)
        dw = from_bits(wb, cuda)
        b200.gemm_bf16(dw, None, dx, ours, m, n, k)
        assert ref.ref_gemm_bf16(dw.data_ptr(), None, dx.data_ptr(), theirs.data_ptr(),
                                 m, n, k, s) == 0
        a, r = oracle.bf16_to_f32(to_bits(ours)), oracle.bf16_to_f32(to_bits(theirs))
        assert np.all(np.abs(a - r) <= bf16_tol(r))


def test_gemm_output_guard_band_and_status(b200, oracle, cuda):
    """Nothing is written outside Y (guard bands), tails in M and N."""
    import torch
    m, n, k = 133, 200, 192
    w, _ = seeded_linear(n, k, seed=5)
    q, sb = oracle.quantize_groupwise(w)
    x = oracle.f32_to_bf16(np.random.default_rng(1).standard_normal((m, k)).astype(np.float32))
    guard = 4096
    buf = torch.full((m * n + 2 * guard,), 7.0, dtype=torch.bfloat16, device=cuda)
    y = buf[guard:guard + m * n].view(m, n)
    b200.gemm_w8a16(torch.from_numpy(q).to(cuda), from_bits(sb, cuda), 64, None,
                    from_bits(x, cuda), y, m, n, k)
    head, tail = to_bits(buf[:guard]), to_bits(buf[guard + m * n:])
    seven = oracle.f32_to_bf16(np.array([7.0], np.float32))[0]
    assert (head == seven).all() and (tail == seven).all()
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, None, x, gemm=True))
    got = oracle.bf16_to_f32(to_bits(y))
    assert np.all(np.abs(got - exp) <= w8_tol(exp))
    assert b200.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(8192, 896, 4864), (2048, 896, 151936), (4100, 1088, 8200)])
def test_w8a16_one_pass_and_two_pass_agree(b200, oracle, cuda, m, k, n):
    """Large-M W8A16 with a reserved buffer runs as dequantise-once + BF16
    tensor-core GEMM; the one-pass kernel that keeps the dequantised weights
    in tensor memory (B200_GEMM_ONE_PASS, and the default without a
    reservation) must give the same bits: both multiply bf16(q*s) and walk K
    16 at a time in ascending order."""
    import os
    import torch
    assert b200.ABI.b200_gemm_reserve_scratch(0) == 0
    g = torch.Generator(device=cuda)
    g.manual_seed(m + n)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    q, s = b200.quantize_groupwise(w)
    bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    two = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    one = torch.empty_like(two)
    b200.gemm_w8a16(q, s, 64, bias, x, two, m, n, k)
    os.environ["B200_GEMM_ONE_PASS"] = "1"
    try:
        b200.gemm_w8a16(q, s, 64, bias, x, one, m, n, k)
    finally:
        del os.environ["B200_GEMM_ONE_PASS"]
    torch.cuda.synchronize()
    a, r = two.float(), one.float()
    assert torch.equal(two, one), float((a - r).abs().max())
    assert b200.device_status() == 0
    rows = [0, m // 2, m - 1]
    qn, sn = q.cpu().numpy(), s.view(torch.int16).cpu().numpy().view(np.uint16)
    xb = x[rows].view(torch.int16).cpu().numpy().view(np.uint16)
    bb = bias.view(torch.int16).cpu().numpy().view(np.uint16)
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(qn, sn, bb, xb, gemm=True))
    got = a[rows].cpu().numpy()
    assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)


@pytest.mark.parametrize("m,k,n", [(32, 4864, 896), (128, 4864, 896), (7, 2112, 264),
                                   (96, 8192, 128)])
@pytest.mark.parametrize("w8", [True, False], ids=["w8a16", "bf16"])
def test_short_prompt_split_k(b200, oracle, cuda, m, k, n, w8):
    """Fast order, <= 128 tokens, K >= 2048, with a reservation: K splits
    across grid z with FP32 partials and a fixed-order reduce.  Every row
    against the oracle; the unsplit kernel (B200_GEMM_NO_SPLITK) on the same
    inputs within one BF16 ulp; two runs bit-identical."""
    import os
    import torch
    assert b200.ABI.b200_gemm_reserve_scratch(0) == 0
    rng = np.random.default_rng(m * 31 + k + n)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    bb = oracle.f32_to_bf16(rng.normal(0, 0.02, n).astype(np.float32))
    xb = oracle.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    dx, db = from_bits(xb, cuda), from_bits(bb, cuda)
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        dq, ds = torch.from_numpy(q).to(cuda), from_bits(sb, cuda)
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb, xb, gemm=True))

        def call(y):
            b200.gemm_w8a16(dq, ds, 64, db, dx, y, m, n, k)
    else:
        wb = oracle.f32_to_bf16(w)
        dw = from_bits(wb, cuda)
        exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, bb, xb)))

        def call(y):
            b200.gemm_bf16(dw, db, dx, y, m, n, k)
    ys = [torch.empty(m, n, dtype=torch.bfloat16, device=cuda) for _ in range(3)]
    # the cluster split (which takes these shapes first) off: this test
    # covers the reserved-buffer split
    os.environ["B200_GEMM_CSPLIT"] = "0"
    try:
        call(ys[0])
        call(ys[1])
        os.environ["B200_GEMM_NO_SPLITK"] = "1"
        call(ys[2])
    finally:
        os.environ.pop("B200_GEMM_NO_SPLITK", None)
        del os.environ["B200_GEMM_CSPLIT"]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1])
    got = oracle.bf16_to_f32(to_bits(ys[0]))
    ulp = np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4
    assert np.all(np.abs(got - exp) <= ulp)
    unsplit = oracle.bf16_to_f32(to_bits(ys[2]))
    assert np.all(np.abs(got - unsplit) <= np.abs(unsplit) * 2.0 ** -7 * 1.01 + 1e-4)
    assert b200.device_status() == 0


@pytest.mark.parametrize("m,k,n", [(32, 896, 151936), (128, 896, 4864), (7, 896, 896),
                                   (64, 4864, 896), (100, 1088, 264)])
def test_bf16_transposed_form_matches_default(b200, oracle, cuda, m, k, n):
    """BF16 GEMM for <= 128 tokens in the transposed form (weights the MMA's
    M side, B200_GEMM_W16T=1) against the CTA-tile kernel (=0) on the same inputs
    (bit-identical: same products, same K order) and the oracle."""
    import os
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(m * 7 + n)
    w = (torch.randn(n, k, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    ref = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    got = torch.empty_like(ref)
    try:
        os.environ["B200_GEMM_W16T"] = "0"
        b200.gemm_bf16(w, bias, x, ref, m, n, k)
        os.environ["B200_GEMM_W16T"] = "1"
        b200.gemm_bf16(w, bias, x, got, m, n, k)
    finally:
        del os.environ["B200_GEMM_W16T"]
    torch.cuda.synchronize()
    assert b200.device_status() == 0
    assert torch.equal(got, ref), float((got.float() - ref.float()).abs().max())
    rows = [0, m // 2, m - 1]
    wb = w.view(torch.int16).cpu().numpy().view(np.uint16)
    xb = x[rows].view(torch.int16).cpu().numpy().view(np.uint16)
    bb = bias.view(torch.int16).cpu().numpy().view(np.uint16)
    exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, bb, xb)))
    g32 = got[rows].float().cpu().numpy()
    assert np.all(np.abs(g32 - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)


@pytest.mark.parametrize("m,k,n", [(2048, 896, 4864), (1000, 1088, 1000), (200, 896, 300),
                                   (1200, 4864, 896)])
def test_w8a16_cta_pair_form_matches_one_sm_form(b200, oracle, cuda, m, k, n):
    """The CTA-pair W8A16 kernel (cta_group::2: A from each SM's TMEM, X split
    between the pair; B200_W8T_CFG=p192) gives the same bits as the one-SM
    kernel (192x2) on the same inputs, ragged sizes included, and matches the
    oracle on sampled rows."""
    import os
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(m + 3 * n)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    q, s = b200.quantize_groupwise(w)
    bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    ys = []
    try:
        for cfg in ("192x2", "p192", "p192"):
            os.environ["B200_W8T_CFG"] = cfg
            y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
            b200.gemm_w8a16(q, s, 64, bias, x, y, m, n, k)
            ys.append(y)
    finally:
        del os.environ["B200_W8T_CFG"]
    torch.cuda.synchronize()
    assert b200.device_status() == 0
    assert torch.equal(ys[0], ys[1]) and torch.equal(ys[1], ys[2])
    rows = [0, m // 2, m - 1]
    qn, sn = q.cpu().numpy(), s.view(torch.int16).cpu().numpy().view(np.uint16)
    xb = x[rows].view(torch.int16).cpu().numpy().view(np.uint16)
    bb = bias.view(torch.int16).cpu().numpy().view(np.uint16)
    exp = oracle.bf16_to_f32(oracle.linear_w8a16(qn, sn, bb, xb, gemm=True))
    got = ys[1][rows].float().cpu().numpy()
    assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)


@pytest.mark.parametrize("m,k,n", [(32, 896, 151936), (1, 896, 896), (100, 1088, 264),
                                   (128, 4864, 896), (2048, 896, 4864), (1500, 896, 1000)])
def test_w8a16_packed_weights_bit_identical(b200, oracle, cuda, m, k, n):
    """Weights pre-packed at upload (b200_pack_w8a16: tile-major 16 KB blocks
    in the kernels' shared-memory layout) give the same bits as the plain
    W8A16 GEMM, ragged sizes and the CTA-pair route included; the packed image
    itself is checked against a host restatement of the layout."""
    import torch
    g = torch.Generator(device=cuda)
    g.manual_seed(m * 5 + n)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    q, s = b200.quantize_groupwise(w)
    bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    packed = b200.pack_w8a16(q, n, k)
    y0 = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    y1 = torch.empty_like(y0)
    import os
    os.environ["B200_GEMM_NO_SPLITK"] = "1"  # same kernel as the packed call
    os.environ["B200_GEMM_CSPLIT"] = "0"
    try:
        b200.gemm_w8a16(q, s, 64, bias, x, y0, m, n, k)
    finally:
        del os.environ["B200_GEMM_NO_SPLITK"]
        del os.environ["B200_GEMM_CSPLIT"]
    b200.gemm_w8a16_packed(packed, s, 64, bias, x, y1, m, n, k)
    torch.cuda.synchronize()
    assert b200.device_status() == 0
    if m > 1:
        assert torch.equal(y0, y1)
    else:
        # one token: the plain entry takes the GEMV (FP32 q * x * s), the
        # packed one keeps the GEMM arithmetic (products of bf16(q * s)): the
        # packed result against the oracle's GEMM form
        qn_, sn_ = q.cpu().numpy(), s.view(torch.int16).cpu().numpy().view(np.uint16)
        exp1 = oracle.bf16_to_f32(oracle.linear_w8a16(
            qn_, sn_, bias.view(torch.int16).cpu().numpy().view(np.uint16),
            x.view(torch.int16).cpu().numpy().view(np.uint16), gemm=True))
        got1 = y1.float().cpu().numpy()
        assert np.all(np.abs(got1 - exp1) <= np.abs(exp1) * 2.0 ** -7 * 1.01 + 1e-4)
    # layout restatement on the first and the last tile row
    tk = (k + 127) // 128
    pk = packed.cpu().numpy()
    qn = q.cpu().numpy().view(np.uint8)
    for tn in (0, (n - 1) // 128):
        for kt in (0, tk - 1):
            blk = pk[(tn * tk + kt) * 16384:(tn * tk + kt + 1) * 16384].reshape(128, 8, 16)
            for r in (0, 5, 127):
                row = tn * 128 + r
                for c in range(8):
                    col = kt * 128 + c * 16
                    exp = qn[row, col:col + 16] if row < n and col < k else np.zeros(16, np.uint8)
                    assert np.array_equal(blk[r, c ^ (r & 7)], exp)


@pytest.mark.parametrize("m,k,n", [(32, 896, 896), (32, 4864, 896), (128, 4864, 896),
                                   (7, 2112, 264), (100, 2176, 1000), (17, 896, 128),
                                   (256, 4864, 896), (300, 4864, 264), (512, 4864, 896)])
@pytest.mark.parametrize("w8", [True, False], ids=["w8a16", "bf16"])
def test_cluster_split_k(b200, oracle, cuda, m, k, n, w8):
    """Short prompts on narrow matrices in the fast order: K split across a
    thread-block cluster, partials summed in rank order through distributed
    shared memory.  Every row against the oracle; two runs bit-identical; the
    unsplit kernels (B200_GEMM_CSPLIT=0, no reserved K split) within one BF16
    ulp on the same inputs."""
    import os
    import torch
    rng = np.random.default_rng(m * 13 + k + n)
    w = rng.normal(0, 0.02, (n, k)).astype(np.float32)
    bb = oracle.f32_to_bf16(rng.normal(0, 0.02, n).astype(np.float32))
    xb = oracle.f32_to_bf16(rng.standard_normal((m, k)).astype(np.float32))
    dx, db = from_bits(xb, cuda), from_bits(bb, cuda)
    if w8:
        q, sb = oracle.quantize_groupwise(w)
        dq, ds = torch.from_numpy(q).to(cuda), from_bits(sb, cuda)
        exp = oracle.bf16_to_f32(oracle.linear_w8a16(q, sb, bb, xb, gemm=True))

        def call(y):
            b200.gemm_w8a16(dq, ds, 64, db, dx, y, m, n, k)
    else:
        wb = oracle.f32_to_bf16(w)
        dw = from_bits(wb, cuda)
        exp = oracle.bf16_to_f32(oracle.f32_to_bf16(oracle.linear_bf16(wb, bb, xb)))

        def call(y):
            b200.gemm_bf16(dw, db, dx, y, m, n, k)
    ys = [torch.empty(m, n, dtype=torch.bfloat16, device=cuda) for _ in range(3)]
    call(ys[0])
    call(ys[1])
    os.environ["B200_GEMM_CSPLIT"] = "0"
    os.environ["B200_GEMM_NO_SPLITK"] = "1"
    try:
        call(ys[2])
    finally:
        del os.environ["B200_GEMM_CSPLIT"]
        del os.environ["B200_GEMM_NO_SPLITK"]
    torch.cuda.synchronize()
    assert b200.device_status() == 0
    assert torch.equal(ys[0], ys[1])
    got = oracle.bf16_to_f32(to_bits(ys[0]))
    assert np.all(np.abs(got - exp) <= np.abs(exp) * 2.0 ** -7 * 1.01 + 1e-4)
    unsplit = oracle.bf16_to_f32(to_bits(ys[2]))
    assert np.all(np.abs(got - unsplit) <= np.abs(unsplit) * 2.0 ** -7 * 1.01 + 1e-4)


@pytest.mark.parametrize("w8", [True, False], ids=["w8a16", "bf16"])
def test_full_size_prefill_every_output(b200, cuda, w8):
    """configs[2]'s largest case, 8192 x 896 -> 151936 (1.24 G outputs), every
    output against a torch FP32 product of X with the GEMM's weights (BF16 W,
    or bf16(q * s) for W8A16), TF32 off, computed in row blocks: each within
    one BF16 ulp of the FP32 value (plus 1e-4 absolute)."""
    import torch
    m, k, n = 8192, 896, 151936
    g = torch.Generator(device=cuda)
    g.manual_seed(8192)
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    if w8:
        q, s = b200.quantize_groupwise(w)
        b200.gemm_w8a16(q, s, 64, bias, x, y, m, n, k)
        wd = (q.float() * s.float().repeat_interleave(64, dim=1)).to(torch.bfloat16).float()
        del q, s
    else:
        wb = w.to(torch.bfloat16)
        b200.gemm_bf16(wb, bias, x, y, m, n, k)
        wd = wb.float()
        del wb
    del w
    torch.cuda.synchronize()
    assert b200.device_status() == 0
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        bad = 0
        for r0 in range(0, m, 1024):
            ref = x[r0:r0 + 1024].float() @ wd.t() + bias.float()
            got = y[r0:r0 + 1024].float()
            tol = ref.abs() * 2.0 ** -7 * 1.01 + 1e-4
            bad += int(((got - ref).abs() > tol).sum())
            del ref, got, tol
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    assert bad == 0, f"{bad} outputs off"
