"""One rank of the multi-GPU sharded-Linear check (launched by torchrun from
tests/test_sharded_gpu.py).  Every rank builds the same seeded full weights,
keeps its shard, runs the sharded W8A16 GEMM + all-gather, its fused form
(tiles stored into every rank's window over NVLink) and the
vocabulary-sharded LM head, and compares with the single-GPU kernels on the
full matrices.  Exit code 0 = all checks passed."""
import os
import sys

import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from conftest import load_package  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo")
    b200 = load_package()
    import importlib
    sh = importlib.import_module("qwen25_b200.sharded")
    comm = sh.Comm.from_process_group()
    g = torch.Generator(device=dev)
    g.manual_seed(1234)
    failures = []
    # --- sharded W8A16 GEMM, M=512, K=1024, N=2048
    m, k, n = 512, 1024, 256 * world * 2
    w = torch.randn(n, k, generator=g, device=dev) * 0.02
    q, s = b200.quantize_groupwise(w)
    bias = (torch.randn(n, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, generator=g, device=dev).to(torch.bfloat16)
    r0, nr = sh.shard_range(n, world, rank)
    y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = sh.gemm_workspace(m, n, world, dev)
    sh.gemm_w8a16_allgather(comm, q[r0:r0 + nr].contiguous(), s[r0:r0 + nr].contiguous(),
                            bias[r0:r0 + nr].contiguous(), x, y, ws, m, n, k)
    ref = torch.empty_like(y)
    b200.gemm_w8a16(q, s, 64, bias, x, ref, m, n, k)
    torch.cuda.synchronize()
    diff = (y.float() - ref.float()).abs()
    tol = ref.float().abs() * 2.0 ** -7 * 1.01 + 1e-4
    if not bool((diff <= tol).all()):
        failures.append(f"gemm max diff {diff.max().item()}")
    # --- the fused form: tiles stored into every rank's window by the GEMM
    win = sh.Window(comm, m * n * 2)
    sh.gemm_w8a16_p2p(comm, win, q[r0:r0 + nr].contiguous(), s[r0:r0 + nr].contiguous(),
                      bias[r0:r0 + nr].contiguous(), x, m, n, k)
    torch.cuda.synchronize()
    yw = win.tensor((m, n)).clone()
    if not torch.equal(yw, y):
        failures.append(f"p2p gemm differs from all-gather: max "
                        f"{(yw.float() - y.float()).abs().max().item()}")
    # two-pass path (tokens >= 1024), bias-free, and a second call on the
    # same window
    m2 = 1024
    x2 = torch.randn(m2, k, generator=g, device=dev).to(torch.bfloat16)
    win2 = sh.Window(comm, m2 * n * 2)
    for _ in range(2):
        sh.gemm_w8a16_p2p(comm, win2, q[r0:r0 + nr].contiguous(), s[r0:r0 + nr].contiguous(),
                          None, x2, m2, n, k)
    ref2 = torch.empty(m2, n, dtype=torch.bfloat16, device=dev)
    b200.gemm_w8a16(q, s, 64, None, x2, ref2, m2, n, k)
    torch.cuda.synchronize()
    y2 = win2.tensor((m2, n)).clone()
    d2 = (y2.float() - ref2.float()).abs()
    tol2 = ref2.float().abs() * 2.0 ** -7 * 1.01 + 1e-4
    if not bool((d2 <= tol2).all()):
        failures.append(f"p2p gemm (two-pass) max diff {d2.max().item()}")
    win.close()
    win2.close()
    # --- vocabulary-sharded LM head with a tie across the shard boundary
    v, kk = 4096 * world, 896
    wl = (torch.randn(v, kk, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    a, b_ = v // world - 1, v // world  # last row of shard 0, first of shard 1
    wl[a] = 2.0
    wl[b_] = 2.0
    xl = torch.randn(kk, generator=g, device=dev)
    xl[0] = 100.0
    xl = xl.to(torch.bfloat16)
    v0, vn = sh.shard_range(v, world, rank)
    logits = torch.empty(vn, dtype=torch.bfloat16, device=dev)
    wsl = sh.lm_head_workspace(v, world, dev)
    am = torch.full((1,), -1, dtype=torch.int32, device=dev)
    sh.lm_head_bf16(comm, wl[v0:v0 + vn].contiguous(), None, xl, logits, wsl, am, v, kk)
    full = torch.empty(v, dtype=torch.bfloat16, device=dev)
    bv, bi = b200.lm_head_workspace(v, dev)
    am_ref = torch.empty(1, dtype=torch.int32, device=dev)
    b200.lm_head_bf16(wl, None, xl, full, bv, bi, am_ref, v, kk)
    torch.cuda.synchronize()
    if int(am.item()) != int(am_ref.item()) or int(am.item()) != a:
        failures.append(f"lm head argmax {am.item()} vs {am_ref.item()} (tie at {a})")
    if not torch.equal(logits, full[v0:v0 + vn]):
        failures.append("lm head logits differ")
    comm.close()
    dist.destroy_process_group()
    if failures:
        print(f"rank {rank} FAILED: {failures}", flush=True)
        sys.exit(1)
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
