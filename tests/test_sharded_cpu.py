"""Host logic of the sharded Linear on CPU ranks (gloo, world size 2):
unique-id exchange, shard ranges, the cross-rank argmax key, and a rank that
dies before the exchange (the survivor must fail on the host, not hang)."""
import datetime
import multiprocessing as mp
import os
import socket

import numpy as np
import pytest

from conftest import REPO, load_package


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _sharded_module():
    import importlib
    import sys
    sys.path.insert(0, os.path.join(REPO, "tests"))
    load_package()
    return importlib.import_module("qwen25_b200.sharded")


def _worker_exchange(rank, world, port, out):
    dist = _init(rank, world, port)
    sh = _sharded_module()
    uid = sh.exchange_unique_id(rank)
    gathered = [None] * world
    dist.all_gather_object(gathered, uid)
    out.put((rank, len(uid), all(g == gathered[0] for g in gathered)))
    dist.destroy_process_group()


def _worker_argmax(rank, world, port, out):
    dist = _init(rank, world, port)
    sh = _sharded_module()
    from oracle import oracle as O
    v = 64 * world
    rng = np.random.default_rng(0)  # same logits on every rank
    vals = O.f32_to_bf16(rng.standard_normal(v).astype(np.float32))
    top = O.f32_to_bf16(np.array([7.0], np.float32))[0]
    vals[63] = vals[64] = vals[v - 1] = top  # tie straddling the shard boundary
    start, count = sh.shard_range(v, world, rank)
    local = O.bf16_to_f32(vals[start:start + count])
    best = int(np.argmax(local))  # numpy argmax: first (lowest) maximum
    key = sh.pack_argmax_key(float(local[best]), start + best)
    keys = [None] * world
    dist.all_gather_object(keys, key)
    out.put((rank, sh.unpack_argmax_index(max(keys)), O.argmax_bf16(vals)))
    dist.destroy_process_group()


def _worker_dies(rank, world, port, out):
    if rank == 1:
        _init(rank, world, port, timeout_s=5)
        os._exit(3)  # leaves before the unique-id exchange
    try:
        _init(rank, world, port, timeout_s=5)
        sh = _sharded_module()
        sh.exchange_unique_id(rank, make_id=lambda: b"x" * 128)
        import torch.distributed as dist
        dist.barrier()
        out.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any host-side failure is the point
        out.put((rank, "error: " + type(e).__name__))


def _run(target, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            pytest.fail("a rank hung")
    res = []
    while not out.empty():
        res.append(out.get())
    return sorted(res), [p.exitcode for p in procs]


def test_unique_id_exchange_gloo():
    res, codes = _run(_worker_exchange)
    assert codes == [0, 0]
    assert res == [(0, 128, True), (1, 128, True)]


def test_cross_rank_argmax_key_gloo():
    res, codes = _run(_worker_argmax)
    assert codes == [0, 0]
    for rank, got, want in res:
        assert got == want == 63


def test_rank_leaving_before_exchange_fails_on_host():
    res, codes = _run(_worker_dies)
    assert codes[1] == 3
    assert len(res) == 1 and res[0][0] == 0 and res[0][1].startswith("error")


def test_shard_range_and_key_order():
    sh = _sharded_module()
    assert sh.shard_range(151936, 8, 7) == (132944, 18992)
    with pytest.raises(ValueError):
        sh.shard_range(10, 4, 0)
    assert sh.pack_argmax_key(1.0, 5) > sh.pack_argmax_key(1.0, 6)  # lower index wins
    assert sh.pack_argmax_key(2.0, 9) > sh.pack_argmax_key(1.0, 0)
    assert sh.pack_argmax_key(-1.0, 0) > sh.pack_argmax_key(-2.0, 0)
    assert sh.unpack_argmax_index(sh.pack_argmax_key(-3.5, 1234)) == 1234
