"""The multi-GPU host logic on CPU: shard ranges, and the verification gather
run as two gloo ranks (world_size 2, 127.0.0.1), including a rank whose
output is wrong (detected) and a rank that never joins (times out, no hang)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from akili_bench_b200 import shard
from akili_bench_b200.parity import parity

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_unit_and_row_ranges_cover_exactly():
    for M in (8, 64, 8192, 8200, 16384):
        for world in (1, 2, 3, 4, 8):
            spans = [shard.row_range(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
                assert a1 == b0
            assert all(a % 8 == 0 for a, _ in spans)
    assert shard.unit_range(256, 8, 3) == (96, 128)  # flash: 8*32 heads over 8 GPUs
    assert shard.sample_rows(8192) == [0, 1, 4096, 8191]
    assert shard.sample_rows(1) == [0]
    with pytest.raises(ValueError):
        shard.row_range(64, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, bad_rank, q):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle_py
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    rng = np.random.default_rng(7)  # W, b shared by all ranks
    K, N = 64, 40
    w = (rng.standard_normal((K, N)) * K ** -0.5).astype(np.float32)
    b = (rng.standard_normal(N) * 0.1).astype(np.float32)
    x = np.random.default_rng(100 + rank).standard_normal((16, K)).astype(np.float32)
    rows = shard.sample_rows(16)
    y = oracle_py.kbt_gemm_add_relu(x, w, b, 16, N, K)  # stands in for this rank's device output
    if rank == bad_rank:
        y = y * 1.1
    outs, ins = shard.gather_rows([torch.from_numpy(y[rows]), torch.from_numpy(x[rows])], world)
    if rank == 0:
        res = shard.check_gathered(outs, ins, lambda xr: oracle_py.kbt_gemm_add_relu(
            np.ascontiguousarray(xr), w, b, xr.shape[0], N, K), parity)
        q.put(res)
    dist.destroy_process_group()


def _run(bad_rank):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, bad_rank, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = q.get(timeout=120)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    return res


def test_gather_and_check_two_gloo_ranks():
    res = _run(bad_rank=-1)
    assert res["ok"], res


def test_gather_detects_a_wrong_rank():
    res = _run(bad_rank=1)
    assert not res["ok"] and res["rank"] == 1


def _lonely(port, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        dist.init_process_group("gloo", rank=0, world_size=2, timeout=datetime.timedelta(seconds=3))
        shard.gather_rows([torch.zeros(4)], 2)
        q.put("returned")
    except Exception as e:  # the missing rank surfaces as an error, not a hang
        q.put(type(e).__name__)


def test_missing_rank_times_out_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    res = q.get(timeout=90)
    p.join(30)
    if p.is_alive():
        p.kill()
    assert res != "returned"
