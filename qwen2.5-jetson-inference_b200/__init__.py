"""B200 (sm_100a) Linear-layer kernels for the Qwen2.5 batch-1 engine.

Python face of ``libb200linear.so``.  The functions below mirror the
reference engine's C++ Linear interface, ``infer::cuda::*`` (reference
include/infer/cuda_ops.hpp:24-55,102-103): same names, same argument order
and meaning, and the same error behaviour (the reference throws
``infer::Error``; here :class:`Error` is raised).  Tensors are torch CUDA
tensors (BF16 as ``torch.bfloat16``, INT8 weights as ``torch.int8``); the
raw device pointers go through the C ABI declared in include/b200_linear.h.

There is no CPU fallback: if the library is missing, importing this package
raises ImportError.  Build it with ``python build.py`` in this directory (or
``__graft_entry__.build()`` at the repository root).
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libb200linear.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is not built; run build.py (no CPU fallback exists)")

_lib = ctypes.CDLL(LIB_PATH)
_p = ctypes.c_void_p
_i = ctypes.c_int

_SIGNATURES = {
    "b200_version": ([], _i),
    "b200_status_string": ([_i], ctypes.c_char_p),
    "b200_device_status": ([_i], _i),
    "b200_gemv_bf16": ([_p, _p, _p, _p, _i, _i, _p], _i),
    "b200_gemv_w8a16": ([_p, _p, _i, _p, _p, _p, _i, _i, _p], _i),
    "b200_gemm_bf16": ([_p, _p, _p, _p, _i, _i, _i, _p], _i),
    "b200_gemm_w8a16": ([_p, _p, _i, _p, _p, _p, _i, _i, _i, _p], _i),
    "b200_lm_head_workspace_bytes": ([_i, _i], ctypes.c_size_t),
    "b200_lm_head_bf16": ([_p, _p, _p, _p, _p, _p, _p, _i, _i, _p], _i),
    "b200_lm_head_w8a16": ([_p, _p, _i, _p, _p, _p, _p, _p, _p, _i, _i, _p], _i),
    "b200_argmax_bf16": ([_p, _i, _p, _p], _i),
    "b200_gemm_reserve_scratch": ([ctypes.c_size_t], _i),
    "b200_w8a16_packed_bytes": ([_i, _i], ctypes.c_size_t),
    "b200_pack_w8a16": ([_p, _i, _i, _p, _p], _i),
    "b200_gemm_w8a16_packed": ([_p, _p, _i, _p, _p, _p, _i, _i, _i, _p], _i),
    "b200_lm_head_noalloc_max_vocab": ([], ctypes.c_size_t),
    "b200_lm_head_bf16_noalloc": ([_p, _p, _p, _p, _p, _i, _i, _p], _i),
    "b200_set_summation_order": ([_i], _i),
    "b200_summation_order": ([], _i),
}
for _name, (_args, _res) in _SIGNATURES.items():
    _fn = getattr(_lib, _name)
    _fn.argtypes = _args
    _fn.restype = _res

ABI = _lib

B200_OK = 0
B200_ERR_INVALID_ARGUMENT = -1
B200_ERR_GROUP_SIZE = -2
B200_ERR_WORKSPACE = -3
B200_ERR_TOO_LARGE = -4
B200_ERR_NCCL = -5
ORDER_FAST = 0
ORDER_REFERENCE = 1


class Error(RuntimeError):
    """Raised for any non-zero status (reference: infer::Error)."""

    def __init__(self, status: int, what: str):
        self.status = status
        text = _lib.b200_status_string(status).decode()
        super().__init__(f"{what}: {text} (status {status})")


def _check(status: int, what: str) -> None:
    if status != 0:
        raise Error(status, what)


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    if not t.is_cuda:
        raise Error(B200_ERR_INVALID_ARGUMENT, "tensor must live on a CUDA device")
    return t.data_ptr()


def _stream(stream):
    if stream is None:
        return torch.cuda.current_stream().cuda_stream
    if isinstance(stream, int):
        return stream
    return stream.cuda_stream


def version() -> int:
    return _lib.b200_version()


def device_status(clear: bool = False) -> int:
    """Device-side error word (B200_DEVICE_*); synchronises the device."""
    return _lib.b200_device_status(1 if clear else 0)


def set_summation_order(order) -> None:
    """Decode GEMV / LM-head summation order: ORDER_FAST (default) or
    ORDER_REFERENCE (every FP32 operation in the reference kernels' order;
    bit-identical outputs on the reference's fast-path shapes).  Also accepts
    "fast" / "reference".  Process-wide."""
    if isinstance(order, str):
        order = {"fast": ORDER_FAST, "reference": ORDER_REFERENCE}[order]
    _check(_lib.b200_set_summation_order(int(order)), "set_summation_order")


def summation_order() -> int:
    return _lib.b200_summation_order()


# ---------------------------------------------------------------- Linear API
def gemv_bf16(weight, bias, input, output, out_features, in_features, stream=None):
    """y = bf16(W x + b); reference infer::cuda::gemv_bf16."""
    _check(_lib.b200_gemv_bf16(_ptr(weight), _ptr(bias), _ptr(input), _ptr(output),
                               out_features, in_features, _stream(stream)),
           "gemv_bf16")


def gemv_w8a16(weight, scales, group_size, bias, input, output, out_features,
               in_features, stream=None):
    """y = bf16(sum float(q) s x + b); reference infer::cuda::gemv_w8a16."""
    _check(_lib.b200_gemv_w8a16(_ptr(weight), _ptr(scales), group_size, _ptr(bias),
                                _ptr(input), _ptr(output), out_features, in_features,
                                _stream(stream)),
           "gemv_w8a16")


def gemm_bf16(weight, bias, input, output, tokens, out_features, in_features,
              stream=None):
    """Y = bf16(X W^T + b); reference infer::cuda::gemm_bf16."""
    _check(_lib.b200_gemm_bf16(_ptr(weight), _ptr(bias), _ptr(input), _ptr(output),
                               tokens, out_features, in_features, _stream(stream)),
           "gemm_bf16")


def gemm_w8a16(weight, scales, group_size, bias, input, output, tokens,
               out_features, in_features, stream=None):
    """Y = bf16(X bf16(q s)^T + b); reference infer::cuda::gemm_w8a16."""
    _check(_lib.b200_gemm_w8a16(_ptr(weight), _ptr(scales), group_size, _ptr(bias),
                                _ptr(input), _ptr(output), tokens, out_features,
                                in_features, _stream(stream)),
           "gemm_w8a16")


def pack_w8a16(weight, out_features, in_features, stream=None):
    """Pre-packs INT8 weights [N, K] once at upload into the prefill
    kernels' tile layout (b200_pack_w8a16); returns the packed uint8 tensor."""
    nbytes = int(_lib.b200_w8a16_packed_bytes(out_features, in_features))
    packed = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=weight.device)
    _check(_lib.b200_pack_w8a16(_ptr(weight), out_features, in_features, _ptr(packed),
                                _stream(stream)), "pack_w8a16")
    return packed


def gemm_w8a16_packed(packed, scales, group_size, bias, input, output, tokens,
                      out_features, in_features, stream=None):
    """gemm_w8a16 on weights pre-packed by pack_w8a16 (bit-identical)."""
    _check(_lib.b200_gemm_w8a16_packed(_ptr(packed), _ptr(scales), group_size, _ptr(bias),
                                       _ptr(input), _ptr(output), tokens, out_features,
                                       in_features, _stream(stream)),
           "gemm_w8a16_packed")


def lm_head_workspace_bytes(vocab: int, in_features: int) -> int:
    return int(_lib.b200_lm_head_workspace_bytes(vocab, in_features))


def lm_head_bf16(weight, bias, input, logits, block_max_value, block_max_index,
                 argmax, vocab, in_features, stream=None):
    """Fused logits + argmax; reference infer::cuda::lm_head_bf16."""
    _check(_lib.b200_lm_head_bf16(_ptr(weight), _ptr(bias), _ptr(input), _ptr(logits),
                                  _ptr(block_max_value), _ptr(block_max_index),
                                  _ptr(argmax), vocab, in_features, _stream(stream)),
           "lm_head_bf16")


def lm_head_w8a16(weight, scales, group_size, bias, input, logits, block_max_value,
                  block_max_index, argmax, vocab, in_features, stream=None):
    """INT8-weight form of the fused LM head (no reference counterpart)."""
    _check(_lib.b200_lm_head_w8a16(_ptr(weight), _ptr(scales), group_size, _ptr(bias),
                                   _ptr(input), _ptr(logits), _ptr(block_max_value),
                                   _ptr(block_max_index), _ptr(argmax), vocab,
                                   in_features, _stream(stream)),
           "lm_head_w8a16")


def argmax_bf16(values, n, output, stream=None):
    """Argmax, lowest index on ties; reference infer::cuda::argmax_bf16."""
    _check(_lib.b200_argmax_bf16(_ptr(values), n, _ptr(output), _stream(stream)),
           "argmax_bf16")


def lm_head_workspace(vocab: int, device=None):
    """(block_max_value float32[ceil(V/8)], block_max_index int32[ceil(V/8)])."""
    blocks = (vocab + 7) // 8
    dev = device or torch.device("cuda")
    return (torch.empty(blocks, dtype=torch.float32, device=dev),
            torch.empty(blocks, dtype=torch.int32, device=dev))


# ------------------------------------------------------ W8A16 weight format
def quantize_groupwise(weight: torch.Tensor, group_size: int = 64):
    """Symmetric group-wise INT8 quantisation, group along K, on the GPU.

    Restates the exporter's rule (reference tools/export_model.py:226-247,
    289-296): scale = max|w|/127 per (row, group) in FP32, 0 -> 1.0;
    q = clip(round_half_even(w / scale), -127, 127); the stored scale is the
    BF16 (round-to-nearest-even) of the FP32 scale.  Returns (int8 [N, K],
    bfloat16 [N, ceil(K / group_size)]).
    """
    w = weight.to(torch.float32)
    rows, cols = w.shape
    groups = (cols + group_size - 1) // group_size
    pad = groups * group_size - cols
    wp = torch.nn.functional.pad(w, (0, pad)) if pad else w
    blocks = wp.view(rows, groups, group_size)
    scale = blocks.abs().amax(dim=2) / 127.0
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    q = torch.clamp(torch.round(blocks / scale[:, :, None]), -127, 127).to(torch.int8)
    q = q.view(rows, groups * group_size)[:, :cols].contiguous()
    return q, scale.to(torch.bfloat16)
