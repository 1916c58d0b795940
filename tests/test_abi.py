"""C-ABI surface checks that need no GPU: the library loads, exports every
symbol include/b200_linear.h declares, and rejects bad arguments before
touching the device (reference error behaviour, src/cuda/kernels.cu:1631,1661
and tests/test_cuda.cpp:887-890)."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO


def declared_functions():
    text = open(os.path.join(REPO, "include", "b200_linear.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported(b200):
    names = declared_functions()
    assert len(names) >= 10
    for name in names:
        assert hasattr(b200.ABI, name), name


def test_status_strings(b200):
    assert b200.ABI.b200_status_string(0) == b"ok"
    assert b"64" in b200.ABI.b200_status_string(-2)
    assert b200.version() >= 100


def test_group_size_other_than_64_is_rejected(b200):
    null = None
    assert b200.ABI.b200_gemv_w8a16(null, null, 32, null, null, null, 1, 1, null) == -2
    assert b200.ABI.b200_gemm_w8a16(null, null, 32, null, null, null, 1, 1, 1, null) == -2
    assert b200.ABI.b200_lm_head_w8a16(null, null, 128, null, null, null, null, null,
                                       null, 1, 1, null) == -2
    with pytest.raises(b200.Error):
        b200.gemv_w8a16(None, None, 32, None, None, None, 1, 1, stream=0)


def test_invalid_arguments_are_rejected(b200):
    A = b200.ABI
    assert A.b200_gemv_bf16(None, None, None, None, -1, 4, None) == -1
    assert A.b200_gemv_bf16(None, None, None, None, 4, 4, None) == -1
    assert A.b200_gemm_bf16(None, None, None, None, 2, 4, -4, None) == -1
    assert A.b200_lm_head_bf16(None, None, None, None, None, None, None, 8, 4, None) == -1
    assert A.b200_argmax_bf16(None, 4, None, None) == -1
    assert A.b200_gemm_w8a16_packed(None, None, 32, None, None, None, 1, 1, 1, None) == -2
    assert A.b200_gemm_w8a16_packed(None, None, 64, None, None, None, 2, 4, 16, None) == -1
    assert A.b200_pack_w8a16(None, 4, 16, None, None) == -1
    assert A.b200_pack_w8a16(None, 4, 24, None, None) == -1


def test_packed_size(b200):
    A = b200.ABI
    # [2 ceil(N/256)][ceil(K/128)] blocks of 16 KB
    assert A.b200_w8a16_packed_bytes(896, 896) == 8 * 7 * 16384
    assert A.b200_w8a16_packed_bytes(151936, 896) == 1188 * 7 * 16384
    assert A.b200_w8a16_packed_bytes(128, 4864) == 2 * 38 * 16384
    assert A.b200_w8a16_packed_bytes(0, 896) == 0


def test_empty_shapes_are_noops(b200):
    A = b200.ABI
    assert A.b200_gemv_bf16(None, None, None, None, 0, 896, None) == 0
    assert A.b200_gemm_bf16(None, None, None, None, 0, 896, 896, None) == 0
    assert A.b200_gemm_w8a16(None, None, 64, None, None, None, 4, 0, 896, None) == 0


def test_lm_head_workspace_is_reference_sized(b200):
    for v in (1, 8, 9, 151936):
        assert b200.lm_head_workspace_bytes(v, 896) == ((v + 7) // 8) * 8


def test_quantizer_matches_oracle_bit_exact(b200, oracle):
    import torch
    rng = np.random.default_rng(7)
    for rows, cols in [(33, 896), (7, 70), (4, 65), (3, 4864)]:
        w = rng.normal(0, 0.02, (rows, cols)).astype(np.float32)
        w[-1, :64] = 0.0
        q, s = b200.quantize_groupwise(torch.from_numpy(w))
        qo, so = oracle.quantize_groupwise(w)
        assert np.array_equal(q.numpy(), qo)
        assert np.array_equal(s.view(torch.int16).numpy().view(np.uint16), so)


def test_engine_header_symbols_are_exported(b200):
    text = open(os.path.join(REPO, "include", "b200_engine.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = sorted(set(re.findall(r"\b(b200_[a-z0-9_]+)\s*\(", text)))
    assert len(names) >= 10
    for name in names:
        assert hasattr(b200.ABI, name), name


def test_engine_and_window_reject_bad_arguments_before_the_device(b200):
    """Null handles and impossible sizes return B200_ERR_INVALID_ARGUMENT (-1)
    without any CUDA call (so this runs without a GPU)."""
    import importlib
    importlib.import_module("qwen25_b200.engine")   # sets the engine argtypes
    importlib.import_module("qwen25_b200.sharded")  # and the sharded ones
    A = b200.ABI
    assert A.b200_engine_decode(None, 1) == -1
    assert A.b200_engine_prefill(None, None, 4) == -1
    assert A.b200_engine_set_decode_mode(None, 0) == -1
    assert A.b200_engine_decode_mode(None) == -1
    assert A.b200_engine_force_token(None, 5) == -1
    assert A.b200_engine_test_stall(None, 3) == -1
    assert A.b200_engine_set_trace(None, 4) == -1
    assert A.b200_engine_read_trace(None, None) == -1
    assert A.b200_engine_destroy(None) == 0
    out = ctypes.c_void_p()
    assert A.b200_engine_create(ctypes.byref(out), None, None, None, None, None) == -1
    assert A.b200_window_create(None, 1024, None, ctypes.byref(out)) == -1
    assert A.b200_window_ptr(None) is None
    assert A.b200_window_destroy(None) == 0
    assert A.b200_sharded_gemm_w8a16_p2p(None, None, None, None, 64, None, None,
                                         4, 8, 16, None) == -1
    assert A.b200_sharded_gemm_w8a16_p2p(None, None, None, None, 32, None, None,
                                         4, 8, 16, None) == -2  # group size
