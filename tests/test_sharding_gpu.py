"""The sharded GEMM on two GPUs: each rank runs its M- or N-slab with the library
kernel on its own GPU, NCCL all-gathers D and its scales (gather_d), and every
rank compares the gathered result with the whole GEMM run on its own GPU, bit
for bit (rows and MX-aligned column slabs are computed independently, so the
shards must reproduce the unsharded D exactly).  Skipped with fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

CASES = [(1024, 512, 256, "m"), (1000, 768, 512, "m"), (256, 2048, 512, "n"), (128, 1000, 64, "n")]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import datetime

    import torch
    import torch.distributed as dist

    import mix_precision_kernel_b200 as mpk
    import oracle as O
    from mix_precision_kernel_b200 import sharding as S

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    try:
        for M, N, K, mode in CASES:
            inp = O.make_gemm_inputs(M, N, K, seed=M + N + K)

            def t(a):
                a = np.ascontiguousarray(a)
                if a.dtype == np.uint16:
                    return torch.from_numpy(a.view(np.int16)).to(dev).view(torch.bfloat16)
                return torch.from_numpy(a).to(dev)

            A, As, B = t(inp["A_data"]), t(inp["A_scales"]), t(inp["B_bf16"])
            C, Cs = t(inp["C_data"]), t(inp["C_scales"])
            full_d, full_s = mpk.gemm(A, As, B, C, Cs)
            shards = S.plan(M, N, world, mode)
            m = S.mode_of(shards, M, N)
            d, s = S.sharded_gemm(A, As, B, C, Cs, shards, rank, m)
            D, Ds = S.gather_d(d, s, shards, m)
            torch.cuda.synchronize()
            ok = bool(torch.equal(D, full_d)) and bool(torch.equal(Ds, full_s))
            q.put((rank, (M, N, K, mode), ok, mpk.device_status()))
            # the same slabs through the fused GEMM + all-gather, twice (epochs)
            gg = S.GatherGemm(M, N, K, shards, None)
            a, a_s, b, c, c_s = (x.contiguous() for x in S.slice_inputs(shards[rank], m, A, As, B, C, Cs))
            for _ in range(2):
                Dg, Dsg = gg(a, a_s, b, c, c_s)
                torch.cuda.synchronize()
                okg = bool(torch.equal(Dg, full_d)) and bool(torch.equal(Dsg, full_s))
                q.put((rank, (M, N, K, "fused-gather-" + m), okg, mpk.device_status()))
            gg.close()
            del gg
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nccl_two_ranks_sharded_gemm(mpk_lib, cuda):
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs)
    results = [q.get(timeout=10) for _ in range(world * 3 * len(CASES))]
    for rank, case, ok, status in results:
        assert ok, (rank, case)
        assert status == 0, (rank, case)
