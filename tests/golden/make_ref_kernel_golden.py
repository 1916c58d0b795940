"""Generates tests/golden/ref_kernels_order.npz: outputs of the REFERENCE'S
OWN CUDA decode kernels (src/cuda/kernels.cu gemv_bf16, gemv_w8a16,
lm_head_bf16, compiled unchanged for sm_100a into
oracle/_ref/libref_kernels.so by oracle/Makefile) on small seeded inputs.

They pin the CPU restatement of the reference kernels' summation order
(oracle_gemv_reference_order) bit for bit without a GPU
(tests/test_oracle.py).  Needs a CUDA device and the built
oracle/_ref/libref_kernels.so:

    python tests/golden/make_ref_kernel_golden.py

Inputs are regenerated from the seeds by ref_order_inputs() (numpy's
default_rng is deterministic across platforms), so only outputs are stored.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

# (name, kind, rows, in_features); kind: w8 / bf16 GEMV or bf16 LM head.
# in_features 896 and 1024 take the reference's one-warp-per-row kernels,
# 4864 and 1088 the four-warps-per-row ones (the LM head is always one warp).
REF_ORDER_CASES = [
    ("w8_896", "w8", 96, 896), ("w8_4864", "w8", 40, 4864), ("w8_1088", "w8", 24, 1088),
    ("bf16_896", "bf16", 96, 896), ("bf16_4864", "bf16", 40, 4864),
    ("bf16_1024", "bf16", 24, 1024), ("lm_896", "lm", 104, 896),
    ("lm_1152", "lm", 24, 1152),
]


def ref_order_inputs(kind, n, k, seed):
    """(weight, scales or None, bias bits, x bits) for one case."""
    from oracle import oracle as O
    rng = np.random.default_rng(seed)
    w = rng.normal(0.0, 0.02, (n, k)).astype(np.float32)
    x = O.f32_to_bf16(rng.standard_normal(k).astype(np.float32))
    b = O.f32_to_bf16(rng.normal(0.0, 0.02, n).astype(np.float32))
    if kind == "w8":
        q, s = O.quantize_groupwise(w)
        return q, s, b, x
    return O.f32_to_bf16(w), None, b, x


def main():
    import torch
    from oracle import oracle as O
    ref = O.ref_cuda()
    if ref is None:
        raise SystemExit("oracle/_ref/libref_kernels.so is not built")
    dev = torch.device("cuda:0")
    st = torch.cuda.current_stream().cuda_stream

    def dev_u16(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).to(dev)

    out = {}
    for i, (name, kind, n, k) in enumerate(REF_ORDER_CASES):
        w, s, b, x = ref_order_inputs(kind, n, k, 100 + i)
        dw = torch.from_numpy(w).to(dev) if kind == "w8" else dev_u16(w)
        db, dx = dev_u16(b), dev_u16(x)
        y = torch.empty(n, dtype=torch.int16, device=dev)
        if kind == "w8":
            ds = dev_u16(s)
            rc = ref.ref_gemv_w8a16(dw.data_ptr(), ds.data_ptr(), 64, db.data_ptr(),
                                    dx.data_ptr(), y.data_ptr(), n, k, st)
        elif kind == "bf16":
            rc = ref.ref_gemv_bf16(dw.data_ptr(), db.data_ptr(), dx.data_ptr(),
                                   y.data_ptr(), n, k, st)
        else:
            blocks = (n + 7) // 8
            bv = torch.empty(blocks, dtype=torch.float32, device=dev)
            bi = torch.empty(blocks, dtype=torch.int32, device=dev)
            am = torch.empty(1, dtype=torch.int32, device=dev)
            rc = ref.ref_lm_head_bf16(dw.data_ptr(), db.data_ptr(), dx.data_ptr(),
                                      y.data_ptr(), bv.data_ptr(), bi.data_ptr(),
                                      am.data_ptr(), n, k, st)
        assert rc == 0, name
        torch.cuda.synchronize()
        out[name] = y.cpu().numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "ref_kernels_order.npz"), **out)
    print("wrote", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
