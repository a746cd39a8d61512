"""Multi-GPU sharding plan and the D all-gather, run as world_size-2 gloo ranks
on the CPU.  Each rank computes its shard with the oracle (standing in for the
single-GPU kernel), the shards are gathered with gather_d, and every rank checks
the result against the full gold bit for bit."""
import os
import socket

import numpy as np
import pytest

from mix_precision_kernel_b200 import sharding as S


def test_plan_m_slabs_cover_rows():
    for M, world in [(4096, 8), (4100, 8), (7, 4), (1, 2)]:
        sh = S.plan(M, 512, world, "m")
        assert sh[0].m0 == 0 and sh[-1].m1 == M
        assert all(a.m1 == b.m0 for a, b in zip(sh, sh[1:]))
        assert all(s.n0 == 0 and s.n1 == 512 for s in sh)
        assert max(s.rows for s in sh) - min(s.rows for s in sh) <= 1


def test_plan_n_slabs_are_mx_aligned():
    for N, world in [(28672, 8), (1000, 3), (96, 2), (33, 2)]:
        sh = S.plan(2048, N, world, "n")
        assert sh[0].n0 == 0 and sh[-1].n1 == N
        assert all(a.n1 == b.n0 for a, b in zip(sh, sh[1:]))
        assert all(s.n0 % 32 == 0 for s in sh)
        assert all(s.n1 % 32 == 0 for s in sh[:-1])


def test_auto_mode():
    assert S.choose_mode(4096, 12288, 8) == "m"
    assert S.choose_mode(2048, 28672, 8) == "n"  # 2048 rows < 8 pair tiles of 256
    assert S.choose_mode(512, 4096, 1) == "m"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cases, q):
    import torch
    import torch.distributed as dist

    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        for M, N, K, mode in cases:
            inp = O.make_gemm_inputs(M, N, K, seed=M + N + K)
            _, gd, gs, _ = O.gold_mx(inp)
            shards = S.plan(M, N, world, mode)
            m = S.mode_of(shards, M, N)
            sh = shards[rank]
            # the rank's shard of the dequantized operands, computed with the oracle
            if m == "m":
                Aq = inp["A_deq"][sh.m0:sh.m1]
                Bq = inp["B_f32"]
                Cq = inp["C_deq"][sh.m0:sh.m1]
            else:
                Aq = inp["A_deq"]
                Bq = inp["B_f32"][:, sh.n0:sh.n1]
                Cq = inp["C_deq"][:, sh.n0:sh.n1]
            d, s = O.quantize(O.gemm_gold(Aq, Bq, Cq, threads=1), threads=1)
            D, Ds = S.gather_d(torch.from_numpy(d), torch.from_numpy(s), shards, m)
            ok = np.array_equal(D.numpy(), gd) and np.array_equal(Ds.numpy(), gs)
            q.put((rank, (M, N, K, mode), ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("cases", [
    [(64, 96, 64, "m"), (66, 96, 32, "m"), (64, 160, 32, "n"), (40, 200, 48, "n")],
])
def test_gloo_two_ranks_gather(cases):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    for p in procs:
        if p.is_alive():
            p.kill()
    results = [q.get(timeout=5) for _ in range(2 * len(cases))]
    assert all(ok for _, _, ok in results), results
    assert all(p.exitcode == 0 for p in procs)
