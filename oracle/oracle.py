"""Python face of the CPU parity checker (TEST INFRASTRUCTURE ONLY).

Wraps ``liboracle.so`` (oracle/linear_oracle.c, the CPU restatement of the
reference's Linear arithmetic) and, when present, the reference itself built
from its own sources into ``oracle/_ref``:

* ``_ref/libref_cpu_linear.so`` - reference src/cpu_ops.cpp (FP32 OpenBLAS);
* ``_ref/libref_kernels.so``    - reference src/cuda/kernels.cu for sm_100a.

Only tests/, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` may import this module.  No product code path uses it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF_CPU = None
_REF_CUDA = None

_p = ctypes.c_void_p
_i = ctypes.c_int


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def lib():
    """Load (building with gcc if needed) the oracle shared library."""
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        src = os.path.join(HERE, "linear_oracle.c")
        if not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(src):
            subprocess.run(["make", "-C", HERE, "liboracle.so"], check=True,
                           stdout=subprocess.DEVNULL)
        L = ctypes.CDLL(path)
        L.oracle_f32_to_bf16_array.argtypes = [_p, _p, ctypes.c_int64]
        L.oracle_bf16_to_f32_array.argtypes = [_p, _p, ctypes.c_int64]
        L.oracle_linear_bf16.argtypes = [_p, _p, _p, _p, _i, _i, _i]
        L.oracle_linear_w8a16.argtypes = [_p, _p, _i, _p, _p, _p, _i, _i, _i, _i]
        L.oracle_argmax_bf16.argtypes = [_p, _i]
        L.oracle_argmax_bf16.restype = _i
        L.oracle_lm_head.argtypes = [_p, _p, _i, _p, _p, _p, _i, _i, _i]
        L.oracle_lm_head.restype = _i
        L.oracle_quantize_groupwise.argtypes = [_p, _i, _i, _i, _p, _p]
        L.oracle_gemv_reference_order.argtypes = [_p, _i, _p, _p, _p, _p, _i, _i, _i]
        _LIB = L
    return _LIB


# ---------------------------------------------------------------- BF16 bits
def f32_to_bf16(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    out = np.empty(a.shape, dtype=np.uint16)
    lib().oracle_f32_to_bf16_array(_ptr(a), _ptr(out), a.size)
    return out


def bf16_to_f32(a) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.uint16)
    out = np.empty(a.shape, dtype=np.float32)
    lib().oracle_bf16_to_f32_array(_ptr(a), _ptr(out), a.size)
    return out


# ------------------------------------------------------------- arithmetic
def linear_bf16(weight, bias, x) -> np.ndarray:
    """FP32 result of the BF16 Linear (reference tests/test_cuda.cpp:474-490)."""
    weight = np.ascontiguousarray(weight, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    n, k = weight.shape
    m = x.size // k if k else (x.shape[0] if x.ndim == 2 else 1)
    out = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    lib().oracle_linear_bf16(_ptr(weight), _ptr(b), _ptr(x), _ptr(out), m, n, k)
    return out


def linear_w8a16(q, scales, bias, x, group_size=64, gemm=False) -> np.ndarray:
    """BF16 bits of the W8A16 Linear; gemm=True rounds q*s to BF16 first."""
    q = np.ascontiguousarray(q, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.uint16)
    x = np.ascontiguousarray(x, dtype=np.uint16)
    n, k = q.shape
    m = x.size // k if k else (x.shape[0] if x.ndim == 2 else 1)
    out = np.empty((m, n), dtype=np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    lib().oracle_linear_w8a16(_ptr(q), _ptr(scales), group_size, _ptr(b), _ptr(x),
                              _ptr(out), m, n, k, 1 if gemm else 0)
    return out


def argmax_bf16(values) -> int:
    v = np.ascontiguousarray(values, dtype=np.uint16)
    return int(lib().oracle_argmax_bf16(_ptr(v), v.size))


def lm_head(weight, bias, x, scales=None, group_size=64):
    """(logits BF16 bits, argmax) of the fused LM head; int8 weight => W8 form."""
    x = np.ascontiguousarray(x, dtype=np.uint16)
    is8 = weight.dtype == np.int8
    weight = np.ascontiguousarray(weight)
    v, k = weight.shape
    logits = np.empty(v, dtype=np.uint16)
    s = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    idx = lib().oracle_lm_head(_ptr(weight), _ptr(s), group_size, _ptr(b), _ptr(x),
                               _ptr(logits), v, k, 1 if is8 else 0)
    return logits, int(idx)


def gemv_reference_order(weight, bias, x, scales=None, lm_head=False) -> np.ndarray:
    """BF16 bits of the decode GEMV (int8 weight => W8A16) or the BF16 LM-head
    logits, computed in the reference CUDA kernels' own FP32 operation order
    (src/cuda/kernels.cu:359-384, 438-603, 953-1041)."""
    x = np.ascontiguousarray(x, dtype=np.uint16).reshape(-1)
    is8 = weight.dtype == np.int8
    weight = np.ascontiguousarray(weight)
    n, k = weight.shape
    out = np.empty(n, dtype=np.uint16)
    s = None if scales is None else np.ascontiguousarray(scales, dtype=np.uint16)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.uint16)
    lib().oracle_gemv_reference_order(_ptr(weight), 1 if is8 else 0, _ptr(s), _ptr(b),
                                      _ptr(x), _ptr(out), n, k, 1 if lm_head else 0)
    return out


def quantize_groupwise(weight, group_size=64):
    """(int8 q, BF16-bits scales) by the exporter's rule."""
    w = np.ascontiguousarray(weight, dtype=np.float32)
    rows, cols = w.shape
    groups = (cols + group_size - 1) // group_size
    q = np.empty((rows, cols), dtype=np.int8)
    s = np.empty((rows, groups), dtype=np.uint16)
    lib().oracle_quantize_groupwise(_ptr(w), rows, cols, group_size, _ptr(q), _ptr(s))
    return q, s


# --------------------------------------------------- reference (built here)
def ref_cpu():
    """Reference src/cpu_ops.cpp Linear (FP32, OpenBLAS) or None if not built."""
    global _REF_CPU
    if _REF_CPU is None:
        path = os.path.join(HERE, "_ref", "libref_cpu_linear.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_cpu_linear_fp32.argtypes = [_p, _p, _p, _p, _i, _i]
        L.ref_cpu_linear_fp32_batch.argtypes = [_p, _p, _p, _p, _i, _i, _i]
        L.ref_cpu_set_threads.argtypes = [_i]
        L.ref_cpu_get_threads.restype = _i
        _REF_CPU = L
    return _REF_CPU


def ref_cpu_linear(weight_f32, bias_f32, x_f32):
    """Reference CPU FP32 Linear; x is [K] (sgemv) or [M, K] (sgemm)."""
    L = ref_cpu()
    w = np.ascontiguousarray(weight_f32, dtype=np.float32)
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    b = None if bias_f32 is None else np.ascontiguousarray(bias_f32, dtype=np.float32)
    n, k = w.shape
    if x.ndim == 1:
        out = np.empty(n, dtype=np.float32)
        rc = L.ref_cpu_linear_fp32(_ptr(w), _ptr(b), _ptr(x), _ptr(out), n, k)
    else:
        out = np.empty((x.shape[0], n), dtype=np.float32)
        rc = L.ref_cpu_linear_fp32_batch(_ptr(w), _ptr(b), _ptr(x), _ptr(out),
                                         x.shape[0], n, k)
    assert rc == 0
    return out


def ref_cuda():
    """Reference src/cuda/kernels.cu built for sm_100a, or None if not built."""
    global _REF_CUDA
    if _REF_CUDA is None:
        path = os.path.join(HERE, "_ref", "libref_kernels.so")
        if not os.path.exists(path):
            return None
        L = ctypes.CDLL(path)
        L.ref_gemv_bf16.argtypes = [_p, _p, _p, _p, _i, _i, _p]
        L.ref_gemv_w8a16.argtypes = [_p, _p, _i, _p, _p, _p, _i, _i, _p]
        L.ref_gemm_bf16.argtypes = [_p, _p, _p, _p, _i, _i, _i, _p]
        L.ref_gemm_w8a16.argtypes = [_p, _p, _i, _p, _p, _p, _i, _i, _i, _p]
        L.ref_lm_head_bf16.argtypes = [_p, _p, _p, _p, _p, _p, _p, _i, _i, _p]
        L.ref_argmax_bf16.argtypes = [_p, _i, _p, _p]
        _REF_CUDA = L
    return _REF_CUDA
