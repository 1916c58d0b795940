"""Host side of the column-sharded Linear (one process per GPU).

Mirrors the C ABI of include/b200_linear.h (b200_comm_*, b200_sharded_*):
an NCCL communicator is created from a unique id that rank 0 makes and the
other ranks receive through ``torch.distributed`` (any backend, gloo
included), then the sharded W8A16 GEMM (+ NCCL all-gather, or fused with
the exchange through a symmetric window of NVLink-mapped buffers) and the
vocabulary-sharded LM head (+ cross-GPU argmax) run on each rank's stream.
The reference is single-GPU; these are the sharded forms of its gemm_w8a16
and lm_head_bf16 (src/cuda/kernels.cu:1566-1579, 1657-1684).
"""
from __future__ import annotations

import ctypes
import struct

import torch

from . import ABI, Error, _check, _ptr, _stream

_p = ctypes.c_void_p
_i = ctypes.c_int
for _name, (_args, _res) in {
    "b200_nccl_unique_id_bytes": ([], _i),
    "b200_nccl_get_unique_id": ([_p], _i),
    "b200_comm_init": ([ctypes.POINTER(_p), ctypes.c_char_p, _i, _i], _i),
    "b200_comm_wrap": ([ctypes.POINTER(_p), _p, _i, _i], _i),
    "b200_comm_destroy": ([_p], _i),
    "b200_sharded_gemm_workspace_bytes": ([_i, _i, _i], ctypes.c_size_t),
    "b200_sharded_gemm_w8a16_allgather": (
        [_p, _p, _p, _i, _p, _p, _p, _p, _i, _i, _i, _p], _i),
    "b200_sharded_lm_head_workspace_bytes": ([_i, _i], ctypes.c_size_t),
    "b200_window_create": ([_p, ctypes.c_size_t, _p, ctypes.POINTER(_p)], _i),
    "b200_window_ptr": ([_p], _p),
    "b200_window_destroy": ([_p], _i),
    "b200_sharded_gemm_w8a16_p2p": ([_p, _p, _p, _p, _i, _p, _p, _i, _i, _i, _p], _i),
    "b200_sharded_lm_head_bf16": ([_p, _p, _p, _p, _p, _p, _p, _i, _i, _p], _i),
}.items():
    _fn = getattr(ABI, _name)
    _fn.argtypes = _args
    _fn.restype = _res


def shard_range(total: int, nranks: int, rank: int) -> tuple[int, int]:
    """(first row, row count) of `rank`'s contiguous shard; total % nranks == 0."""
    if nranks < 1 or not 0 <= rank < nranks:
        raise ValueError(f"bad rank {rank} of {nranks}")
    if total % nranks:
        raise ValueError(f"{total} rows do not split evenly over {nranks} ranks")
    n = total // nranks
    return rank * n, n


def exchange_unique_id(rank: int, group=None, make_id=None) -> bytes:
    """Rank 0 makes an NCCL unique id; every rank returns it (broadcast over
    torch.distributed, which may be a CPU/gloo group)."""
    import torch.distributed as dist
    payload = [None]
    if rank == 0:
        payload[0] = make_id() if make_id else new_unique_id()
    dist.broadcast_object_list(payload, src=0, group=group)
    return payload[0]


def new_unique_id() -> bytes:
    n = ABI.b200_nccl_unique_id_bytes()
    buf = ctypes.create_string_buffer(n)
    _check(ABI.b200_nccl_get_unique_id(buf), "ncclGetUniqueId")
    return buf.raw


class Comm:
    """An NCCL communicator whose rank drives the current CUDA device."""

    def __init__(self, unique_id: bytes, nranks: int, rank: int):
        self.nranks, self.rank = nranks, rank
        self.handle = _p()
        _check(ABI.b200_comm_init(ctypes.byref(self.handle), unique_id, nranks, rank),
               "ncclCommInitRank")

    @classmethod
    def from_process_group(cls, group=None):
        import torch.distributed as dist
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        return cls(exchange_unique_id(rank, group), world, rank)

    def close(self):
        if self.handle:
            _check(ABI.b200_comm_destroy(self.handle), "ncclCommDestroy")
            self.handle = _p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_w8a16_allgather(comm: Comm, weight_shard, scales_shard, bias_shard, input,
                         output, workspace, tokens, out_features, in_features,
                         stream=None):
    """Full Y on every rank from this rank's rows of W (see the C ABI)."""
    _check(ABI.b200_sharded_gemm_w8a16_allgather(
        comm.handle, _ptr(weight_shard), _ptr(scales_shard), 64, _ptr(bias_shard),
        _ptr(input), _ptr(output), _ptr(workspace), tokens, out_features, in_features,
        _stream(stream)), "sharded_gemm_w8a16_allgather")


class Window:
    """A symmetric device buffer: `nbytes` on every rank, every rank's buffer
    mapped into every process (collective over `comm`)."""

    def __init__(self, comm: Comm, nbytes: int, stream=None):
        self.handle = _p()
        self.nbytes = nbytes
        _check(ABI.b200_window_create(comm.handle, nbytes, _stream(stream),
                                      ctypes.byref(self.handle)), "window_create")

    def ptr(self) -> int:
        return ABI.b200_window_ptr(self.handle)

    def tensor(self, shape, dtype=torch.bfloat16, device=None):
        """This rank's buffer viewed as a tensor (no copy; valid while open)."""
        n = 1
        for d in shape:
            n *= d
        itemsize = torch.empty((), dtype=dtype).element_size()
        if n * itemsize > self.nbytes:
            raise ValueError("shape exceeds the window")
        dev = device or torch.device("cuda", torch.cuda.current_device())

        class _Iface:  # __cuda_array_interface__ view of the raw pointer
            pass
        iface = _Iface()
        typestr = {torch.bfloat16: "<f2", torch.float16: "<f2", torch.float32: "<f4",
                   torch.int32: "<i4", torch.uint8: "|u1"}[dtype]
        iface.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr,
                                          "data": (self.ptr(), False), "version": 3}
        t = torch.as_tensor(iface, device=dev)
        return t.view(dtype) if dtype == torch.bfloat16 else t

    def close(self):
        if self.handle:
            _check(ABI.b200_window_destroy(self.handle), "window_destroy")
            self.handle = _p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def gemm_w8a16_p2p(comm: Comm, window: Window, weight_shard, scales_shard, bias_shard,
                   input, tokens, out_features, in_features, stream=None):
    """Fused sharded GEMM + all-gather: the full Y lands in every rank's window."""
    _check(ABI.b200_sharded_gemm_w8a16_p2p(
        comm.handle, window.handle, _ptr(weight_shard), _ptr(scales_shard), 64,
        _ptr(bias_shard), _ptr(input), tokens, out_features, in_features,
        _stream(stream)), "sharded_gemm_w8a16_p2p")


def gemm_workspace(tokens, out_features, nranks, device=None):
    n = ABI.b200_sharded_gemm_workspace_bytes(tokens, out_features, nranks)
    return torch.empty(n, dtype=torch.uint8, device=device or "cuda")


def lm_head_bf16(comm: Comm, weight_shard, bias_shard, input, logits_shard, workspace,
                 argmax, vocab, in_features, stream=None):
    """Vocabulary-sharded fused LM head; *argmax = global index on every rank."""
    _check(ABI.b200_sharded_lm_head_bf16(
        comm.handle, _ptr(weight_shard), _ptr(bias_shard), _ptr(input),
        _ptr(logits_shard), _ptr(workspace), _ptr(argmax), vocab, in_features,
        _stream(stream)), "sharded_lm_head_bf16")


def lm_head_workspace(vocab, nranks, device=None):
    n = ABI.b200_sharded_lm_head_workspace_bytes(vocab, nranks)
    return torch.empty((n + 7) // 8 * 8, dtype=torch.uint8, device=device or "cuda")


# ---- host mirror of the 64-bit argmax key (used by the CPU tests) --------
def order_key(value: float) -> int:
    """Orderable 32-bit key of an FP32 value (larger value -> larger key)."""
    u = struct.unpack("<I", struct.pack("<f", value))[0]
    return (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000


def pack_argmax_key(value: float, index: int) -> int:
    """(order_key(value) << 32) | (0xFFFFFFFF - index): max = best value,
    then lowest index, exactly what the device kernel all-reduces."""
    return (order_key(value) << 32) | (0xFFFFFFFF - index)


def unpack_argmax_index(key: int) -> int:
    return 0 if key == 0 else 0xFFFFFFFF - (key & 0xFFFFFFFF)
