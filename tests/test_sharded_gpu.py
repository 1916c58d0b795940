"""Sharded Linear on the GPU: the single-rank communicator on any box, and a
torchrun job over every visible GPU (2..8) when the box has several."""
import os
import re
import socket
import subprocess
import sys

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def sh(b200):
    import importlib
    return importlib.import_module("qwen25_b200.sharded")


def test_single_rank_comm_matches_unsharded(b200, sh, cuda):
    import torch
    comm = sh.Comm(sh.new_unique_id(), 1, 0)
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    m, k, n = 300, 896, 4864
    w = torch.randn(n, k, generator=g, device=cuda) * 0.02
    q, s = b200.quantize_groupwise(w)
    x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    ref = torch.empty_like(y)
    ws = sh.gemm_workspace(m, n, 1, cuda)
    sh.gemm_w8a16_allgather(comm, q, s, None, x, y, ws, m, n, k)
    b200.gemm_w8a16(q, s, 64, None, x, ref, m, n, k)
    v = 151936
    wl = (torch.randn(v, k, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
    xl = torch.randn(k, generator=g, device=cuda).to(torch.bfloat16)
    logits = torch.empty(v, dtype=torch.bfloat16, device=cuda)
    full = torch.empty_like(logits)
    am = torch.empty(1, dtype=torch.int32, device=cuda)
    am_ref = torch.empty_like(am)
    sh.lm_head_bf16(comm, wl, None, xl, logits, sh.lm_head_workspace(v, 1, cuda), am, v, k)
    bv, bi = b200.lm_head_workspace(v, cuda)
    b200.lm_head_bf16(wl, None, xl, full, bv, bi, am_ref, v, k)
    torch.cuda.synchronize()
    assert torch.equal(y, ref)
    assert torch.equal(logits, full)
    assert int(am.item()) == int(am_ref.item())
    comm.close()



def test_single_rank_window_gemm_matches_unsharded(b200, sh, cuda):
    """The fused form on one rank: the window holds Y, bit-identical to the
    plain GEMM (same tiles; the peer list is empty)."""
    import torch
    comm = sh.Comm(sh.new_unique_id(), 1, 0)
    g = torch.Generator(device=cuda)
    g.manual_seed(6)
    for m, k, n in ((300, 896, 4864), (1024, 896, 1024)):
        w = torch.randn(n, k, generator=g, device=cuda) * 0.02
        q, s = b200.quantize_groupwise(w)
        bias = (torch.randn(n, generator=g, device=cuda) * 0.02).to(torch.bfloat16)
        x = torch.randn(m, k, generator=g, device=cuda).to(torch.bfloat16)
        win = sh.Window(comm, m * n * 2)
        sh.gemm_w8a16_p2p(comm, win, q, s, bias, x, m, n, k)
        ref = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
        b200.gemm_w8a16(q, s, 64, bias, x, ref, m, n, k)
        torch.cuda.synchronize()
        assert torch.equal(win.tensor((m, n)), ref)
        with pytest.raises(Exception):
            sh.gemm_w8a16_p2p(comm, win, q, s, bias, x, m + 1, n, k)  # window too small
        win.close()
    comm.close()

def test_sharded_rejects_bad_splits(b200, sh, cuda):
    import torch
    comm = sh.Comm(sh.new_unique_id(), 1, 0)
    with pytest.raises(b200.Error):  # out_features not a multiple of 8 * nranks
        sh.gemm_w8a16_allgather(comm, torch.empty(1, device=cuda), torch.empty(1, device=cuda),
                                None, torch.empty(1, device=cuda), torch.empty(1, device=cuda),
                                torch.empty(1, device=cuda), 4, 12, 64)
    comm.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_worker(nproc, shapes):
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={nproc}", "--master-addr=127.0.0.1",
           f"--master-port={_free_port()}",
           os.path.join(REPO, "tests", "sharded_worker.py"), "--shapes", shapes]
    proc = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    assert proc.returncode == 0, proc.stdout[-3000:] + proc.stderr[-3000:]
    done = re.findall(r"^rank \d+ ok$", proc.stdout, flags=re.M)
    assert len(done) == nproc, proc.stdout[-3000:]
    return proc.stdout


def test_sharded_full_shapes_one_rank(b200, cuda):
    """configs[4] shapes (M=8192, 8192->28672 and 28672->8192; the 151936
    LM head) on a one-rank communicator, checked against the oracle."""
    _run_worker(1, "full")


def test_multi_gpu_sharded_linear(b200, cuda):
    """Every visible GPU (2..8): small shapes, then the configs[4] shapes,
    gathered outputs and the cross-GPU argmax checked against the oracle."""
    import torch
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs 2 or more GPUs")
    n = min(n, 8)
    _run_worker(n, "small")
    _run_worker(n, "full")
