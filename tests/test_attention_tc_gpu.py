"""Tensor-core causal GQA prefill attention (b200_attention_prefill_bf16,
csrc/attention_tc.cu) against an FP32 torch restatement of the reference's
attention_prefill_bf16_kernel (src/cuda/kernels.cu:221-283: FP32 scores
q.k / 8, softmax with the row maximum subtracted, FP32 weighted sum of V)
on the same BF16 inputs.  P is rounded to BF16 for the tensor cores, so the
check is the attention tolerance |a - b| <= 2e-2 + 1e-2 |b|, plus a tight
mean error."""
import ctypes

import pytest

pytestmark = pytest.mark.gpu


def reference_attention(q, kc, vc, tokens, pos0, heads, kv_heads):
    import torch
    hd = 64
    out = torch.empty(tokens, heads * hd, dtype=torch.float32, device=q.device)
    group = heads // kv_heads
    for h in range(heads):
        kvh = h // group
        qh = q[:, h * hd:(h + 1) * hd].float()                      # [T, 64]
        keys = kc[kvh, :pos0 + tokens].float()                       # [S, 64]
        vals = vc[kvh, :pos0 + tokens].float()
        s = (qh @ keys.t()) / 8.0                                    # [T, S]
        qpos = torch.arange(tokens, device=q.device)[:, None] + pos0
        kpos = torch.arange(pos0 + tokens, device=q.device)[None, :]
        s = s.masked_fill(kpos > qpos, float("-inf"))
        p = torch.softmax(s, dim=1)
        out[:, h * hd:(h + 1) * hd] = p @ vals
    return out


@pytest.mark.parametrize("tokens,pos0", [(1, 0), (32, 0), (127, 0), (128, 0), (300, 0),
                                         (1000, 0), (64, 17), (200, 300)])
def test_prefill_attention_tc_matches_fp32(b200, cuda, tokens, pos0):
    import torch
    heads, kv_heads, hd, max_seq = 14, 2, 64, 1536
    g = torch.Generator(device=cuda)
    g.manual_seed(tokens * 7 + pos0)
    qkv_dim = (heads + 2 * kv_heads) * hd
    q = torch.randn(tokens, qkv_dim, generator=g, device=cuda).to(torch.bfloat16)
    kc = torch.randn(kv_heads, max_seq, hd, generator=g, device=cuda).to(torch.bfloat16)
    vc = torch.randn(kv_heads, max_seq, hd, generator=g, device=cuda).to(torch.bfloat16)
    out = torch.full((tokens, heads * hd), float("nan"), dtype=torch.bfloat16, device=cuda)
    fn = b200.ABI.b200_attention_prefill_bf16
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p,
                   ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    fn.restype = ctypes.c_int
    rc = fn(q.data_ptr(), qkv_dim, kc.data_ptr(), vc.data_ptr(), out.data_ptr(), heads * hd,
            tokens, pos0, heads, kv_heads, max_seq, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    torch.cuda.synchronize()
    exp = reference_attention(q, kc, vc, tokens, pos0, heads, kv_heads)
    got = out.float()
    err = (got - exp).abs()
    assert bool((err <= 2e-2 + 1e-2 * exp.abs()).all()), float(err.max())
    assert float(err.mean()) < 2e-3
    assert b200.device_status() == 0


def test_prefill_attention_tc_rejects_bad_arguments(b200, cuda):
    fn = b200.ABI.b200_attention_prefill_bf16
    fn.restype = ctypes.c_int
    assert fn(None, 1152, None, None, None, 896, 4, 0, 14, 2, 64, None) == b200.B200_ERR_INVALID_ARGUMENT
