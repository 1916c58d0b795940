"""One rank of the multi-GPU sharded-Linear check (launched by torchrun from
tests/test_sharded_gpu.py, one process per GPU; world size 1 works too).

Every rank builds the same seeded full weights, keeps its shard and runs:
  * the column-sharded W8A16 GEMM in both forms -- NCCL all-gather
    (b200_sharded_gemm_w8a16_allgather) and fused (tiles stored into every
    rank's window over NVLink, b200_sharded_gemm_w8a16_p2p);
  * the fused form three times on ONE window with different inputs (a window
    reused call after call, one rank's stream stalled between calls);
  * the vocabulary-sharded LM head at the full 151936 vocabulary, once with a
    tie across a shard boundary and then back to back with one rank's stream
    stalled between calls.
The gathered outputs are checked against the CPU oracle (reference
tests/test_cuda.cpp:494-517 arithmetic, dequantise-to-BF16 form of
src/cuda/kernels.cu:1075-1094) on sampled rows x sampled columns of every
shard; the LM head's argmax against the oracle's fused LM head
(src/cuda/kernels.cu:492-603).

``--shapes full`` runs the BASELINE configs[4] sizes (M=8192, K=8192 ->
N=28672 and K=28672 -> N=8192); ``--shapes small`` a quick M=512 case.
Exit code 0 = every check passed on this rank."""
import argparse
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
from conftest import load_package, to_bits, REPO  # noqa: E402

sys.path.insert(0, REPO)
from oracle import oracle as O  # noqa: E402  (test infrastructure)

# north_star tolerance for a Linear output: |a - b| <= 2e-2 + 1e-2 |b|
ATOL, RTOL = 2e-2, 1e-2


def sample_rows(m, count, seed):
    rng = np.random.default_rng(seed)
    rows = set(rng.choice(m, size=min(count, m), replace=False).tolist())
    rows.update({0, m - 1})
    return np.array(sorted(rows))


def sample_cols(n, world, per_shard, seed):
    """Columns from every rank's shard, including both shard edges."""
    rng = np.random.default_rng(seed)
    ns = n // world
    out = []
    for r in range(world):
        lo = r * ns
        cols = set((lo + rng.choice(ns, size=min(per_shard, ns), replace=False)).tolist())
        cols.update({lo, lo + ns - 1})
        out.extend(sorted(cols))
    return np.array(out)


def oracle_check(name, y_bits, q, s, bias, x, rows, cols, failures, log):
    """y_bits: gathered output rows [len(rows), n] (BF16 bits); q, s, bias:
    the weight rows of the sampled columns `cols`, in that order."""
    exp = O.bf16_to_f32(O.linear_w8a16(q, s, bias, x[rows], gemm=True))
    got = O.bf16_to_f32(y_bits[:, cols])
    err = np.abs(got - exp)
    bad = err > ATOL + RTOL * np.abs(exp)
    if bad.any():
        i = np.argwhere(bad)[0]
        failures.append(f"{name}: {int(bad.sum())} of {bad.size} sampled outputs off; "
                        f"first at row {rows[i[0]]} col {cols[i[1]]}: {got[tuple(i)]} vs "
                        f"{exp[tuple(i)]}")
    exact = float((err == 0).mean())
    log.append(f"{name}: max |err| {err.max():.3g}, {exact:.1%} bit-equal to the oracle")


def gemm_case(b200, sh, comm, rank, world, dev, m, k, n, seed, failures, log):
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    w = torch.randn(n, k, generator=gen, device=dev) * 0.02
    q, s = b200.quantize_groupwise(w)
    del w
    bias = (torch.randn(n, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    r0, nr = sh.shard_range(n, world, rank)
    qs, ss, bs = q[r0:r0 + nr].contiguous(), s[r0:r0 + nr].contiguous(), \
        bias[r0:r0 + nr].contiguous()
    rows = sample_rows(m, 10, seed + 1)
    cols = sample_cols(n, world, 48 if world <= 4 else 24, seed + 2)
    csel = torch.from_numpy(cols).to(dev)
    q_h = q[csel].cpu().numpy()
    s_h = to_bits(s[csel])
    b_h = to_bits(bias[csel])
    del q, s
    torch.cuda.empty_cache()

    xs = []
    for i in range(3):
        xs.append(torch.randn(m, k, generator=gen, device=dev).to(torch.bfloat16))
    tag = f"{k}->{n} M={m}"

    # NCCL all-gather form
    y = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    ws = sh.gemm_workspace(m, n, world, dev)
    sh.gemm_w8a16_allgather(comm, qs, ss, bs, xs[0], y, ws, m, n, k)
    torch.cuda.synchronize()
    y_ag = y.clone()
    sel = torch.from_numpy(rows).to(dev)
    oracle_check(f"allgather {tag}", to_bits(y_ag[sel]), q_h, s_h, b_h,
                 to_bits(xs[0]), rows, cols, failures, log)
    del ws
    torch.cuda.empty_cache()

    # fused form: one window, three calls with different inputs, enqueued
    # back to back.  Before reading each call's result one rank stalls its
    # stream (a device-side sleep), so the other ranks reach the next call
    # while that rank has not read the window yet.
    win = sh.Window(comm, m * n * 2)
    yw = win.tensor((m, n))
    got, first = [], None
    for i, x in enumerate(xs):
        sh.gemm_w8a16_p2p(comm, win, qs, ss, bs, x, m, n, k)
        if world > 1 and rank == (i % world):
            torch.cuda._sleep(40_000_000)
        got.append(yw[sel].clone())
        if i == 0:
            first = yw.clone()
    torch.cuda.synchronize()
    if not torch.equal(first, y_ag):
        d = (first.float() - y_ag.float()).abs().max().item()
        failures.append(f"p2p {tag}: differs from the all-gather form (max {d})")
    del first
    for i, x in enumerate(xs):
        oracle_check(f"p2p {tag} call {i}", to_bits(got[i]), q_h, s_h, b_h,
                     to_bits(x), rows, cols, failures, log)
    win.close()
    log.append(f"gemm {tag}: {len(rows)} rows x {len(cols)} cols checked, 1+3 calls")


def lm_head_case(b200, sh, comm, rank, world, dev, failures, log):
    v, k = 151936, 896
    gen = torch.Generator(device=dev)
    gen.manual_seed(77)
    wl = (torch.randn(v, k, generator=gen, device=dev) * 0.02).to(torch.bfloat16)
    v0, vn = sh.shard_range(v, world, rank)
    wsl = sh.lm_head_workspace(v, world, dev)
    logits = torch.empty(vn, dtype=torch.bfloat16, device=dev)
    am = torch.full((1,), -1, dtype=torch.int32, device=dev)
    w_h = to_bits(wl)

    def run(wshard, x):
        sh.lm_head_bf16(comm, wshard, None, x, logits, wsl, am, v, k)
        torch.cuda.synchronize()
        return int(am.item())

    # 1. plain random input: argmax vs the oracle (exact when the top two
    #    logits differ by more than one BF16 ulp), logits vs oracle within 1 ulp
    x = torch.randn(k, generator=gen, device=dev).to(torch.bfloat16)
    got = run(wl[v0:v0 + vn].contiguous(), x)
    exp_logits, exp_am = O.lm_head(w_h, None, to_bits(x))
    ef = O.bf16_to_f32(exp_logits)
    top2 = np.sort(ef)[-2:]
    gf = O.bf16_to_f32(to_bits(logits))
    if (np.abs(gf - ef[v0:v0 + vn]) > np.maximum(0.008, 0.01 * np.abs(ef[v0:v0 + vn]))).any():
        failures.append("lm head: logits off the oracle")
    if got != exp_am and not (top2[1] - top2[0] <= np.abs(top2[1]) * 2.0 ** -7):
        failures.append(f"lm head argmax {got} vs oracle {exp_am}")
    log.append(f"lm head 151936: argmax {got} (oracle {exp_am})")

    # 2. a tie across a shard boundary (or vocab end when world == 1): the
    #    lowest index wins
    a = v // world - 1 if world > 1 else v - 2
    b = a + 1
    wt = wl.clone()
    wt[a] = 2.0
    wt[b] = 2.0
    xt = x.float().clone()
    xt[0] = 100.0
    xt = xt.to(torch.bfloat16)
    got = run(wt[v0:v0 + vn].contiguous(), xt)
    _, exp_am = O.lm_head(to_bits(wt), None, to_bits(xt))
    if got != a or exp_am != a:
        failures.append(f"lm head tie: {got} (oracle {exp_am}, expected {a})")
    del wt

    # 3. back-to-back calls, inputs changing every call, one rank delayed on
    #    the device: each call's argmax must be that call's
    shard = wl[v0:v0 + vn].contiguous()
    hot = [int(i) for i in np.random.default_rng(5).choice(v, size=12, replace=False)]
    xs, exp = [], []
    for i, h in enumerate(hot):
        xi = wl[h].float() * 40.0  # makes row h the clear winner
        xs.append(xi.to(torch.bfloat16))
    torch.cuda.synchronize()
    ams = torch.full((len(hot),), -1, dtype=torch.int32, device=dev)
    for i, xi in enumerate(xs):
        if world > 1 and rank == 1 and i % 3 == 0:
            torch.cuda._sleep(20_000_000)  # this rank's stream falls behind
        sh.lm_head_bf16(comm, shard, None, xi, logits, wsl, ams[i:i + 1], v, k)
    torch.cuda.synchronize()
    got_all = ams.cpu().tolist()
    for i, xi in enumerate(xs):
        _, e = O.lm_head(w_h, None, to_bits(xi))
        exp.append(e)
    if got_all != exp:
        failures.append(f"lm head back-to-back: {got_all} vs oracle {exp}")
    log.append(f"lm head back-to-back x{len(hot)}: ok={got_all == exp}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--shapes", default="small", choices=["small", "full"])
    args = ap.parse_args()
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("gloo")
    b200 = load_package()
    import importlib
    sh = importlib.import_module("qwen25_b200.sharded")
    comm = sh.Comm.from_process_group()
    failures, log = [], []
    if args.shapes == "full":
        cases = [(8192, 8192, 28672), (8192, 28672, 8192)]
    else:
        cases = [(512, 1024, 512 * world), (1024, 896, 256 * world)]
    for i, (m, k, n) in enumerate(cases):
        gemm_case(b200, sh, comm, rank, world, dev, m, k, n, 1000 + i, failures, log)
    lm_head_case(b200, sh, comm, rank, world, dev, failures, log)
    status = b200.device_status()
    if status != 0:
        failures.append(f"device status {status}")
    comm.close()
    dist.destroy_process_group()
    for line in log:
        print(f"rank {rank}: {line}", flush=True)
    if failures:
        print(f"rank {rank} FAILED: {failures}", flush=True)
        sys.exit(1)
    print(f"rank {rank} ok", flush=True)


if __name__ == "__main__":
    main()
