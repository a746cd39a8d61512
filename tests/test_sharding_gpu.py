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


# The configurations' shapes split over two GPUs as the strong-scaling bench splits
# them: M-row slabs, or N-column slabs of 32-column multiples for the wide shape.
CONFIG_CASES = [(4096, 12288, 4096, 43, "m"), (4096, 4096, 11008, 44, "m"), (131072, 2048, 2048, 45, "m"),
                (2048, 28672, 8192, 46, "n")]


def _config_worker(rank, world, port, q):
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
                            timeout=datetime.timedelta(seconds=120))

    def host(t):
        t = t.detach().cpu()
        return t.view(torch.int16).numpy().view(np.uint16) if t.dtype == torch.bfloat16 else t.numpy()

    try:
        for M, N, K, seed, mode in CONFIG_CASES:
            # the same full inputs on both ranks (same seeded device generator)
            g = torch.Generator(device=dev).manual_seed(seed)
            A = torch.randn((M, K), generator=g, device=dev) * 0.02
            B = (torch.randn((K, N), generator=g, device=dev) * 0.02).to(torch.bfloat16)
            C = torch.randn((M, N), generator=g, device=dev) * 0.02
            Ad, As = mpk.quantize(A)
            Cd, Cs = mpk.quantize(C)
            del A, C
            shards = S.plan(M, N, world, mode)
            a, a_s, b, c, c_s = (x.contiguous() for x in S.slice_inputs(shards[rank], mode, Ad, As, B, Cd, Cs))
            sh = shards[rank]
            rows, cols = (sh.rows, N) if mode == "m" else (M, sh.cols)
            results = {}
            for name, sched in (("tiles", mpk.SCHEDULE_TILES), ("auto", mpk.SCHEDULE_AUTO)):
                prev = mpk.set_gemm_schedule(sched)
                try:
                    d, s = mpk.gemm(a, a_s, b, c, c_s)
                    Dg, Sg = S.gather_d(d, s, shards, mode)
                    full = mpk.gemm(Ad, As, B, Cd, Cs) if name == "tiles" else None
                    torch.cuda.synchronize()
                finally:
                    mpk.set_gemm_schedule(prev)
                results[name] = (Dg, Sg, full, mpk.gemm_plan(rows, cols, K))
            Dt, St, (Df, Sf), _ = results["tiles"]
            same = bool(torch.equal(Dt, Df)) and bool(torch.equal(St, Sf))
            q.put((rank, (M, N, K, mode, "whole tiles: gathered slabs == one GPU"), same, mpk.device_status()))
            if rank == 0:
                # the default schedule (stream-K where the slab's plan has it) against the
                # FP32 gold on a sample of rows, and within one E4M3 step of whole tiles
                Da, Sa, _, plan = results["auto"]
                rs = np.array(sorted({0, 127, 128, 255, M // 4, M // 2, M - 129, M - 1} |
                                     set(int(r) for r in np.random.default_rng(M).integers(0, M, 16))), np.int64)
                rt = torch.from_numpy(rs).to(dev)
                A_deq = O.dequantize(host(Ad[rt]), host(As[rt]))
                C_deq = O.dequantize(host(Cd[rt]), host(Cs[rt]))
                D_gold = O.gemm_gold(A_deq, O.bf16_bits_to_float(host(B)), C_deq)
                gd, gs = O.quantize(D_gold)
                hist = O.mx_ulp_hist(host(Da[rt]), host(Sa[rt]), gd, gs)
                vs_tiles = O.mx_ulp_hist(host(Da), host(Sa), host(Dt), host(St))
                ok = (hist[3] == 0 and hist[0] + hist[1] >= 0.999 * sum(hist) and vs_tiles[2] == 0
                      and vs_tiles[3] == 0)
                q.put((rank, (M, N, K, mode, f"default schedule {plan}: gold {hist}, vs tiles {vs_tiles}"), ok,
                       mpk.device_status()))
            del Ad, As, B, Cd, Cs, a, a_s, b, c, c_s, results, Dt, St, Df, Sf
            torch.cuda.empty_cache()
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_nccl_two_ranks_config_shapes(mpk_lib, cuda):
    """The configurations' GEMMs split over two GPUs: each rank's slab through the
    library, gathered over NCCL, equals the whole GEMM on one GPU bit for bit under
    the whole-tile schedule; under the default schedule (which may split a slab's
    last wave by K range) the gathered D meets the parity bar against the FP32
    gold on sampled rows and is within one E4M3 step of whole tiles."""
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_config_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=600) for _ in range(world * len(CONFIG_CASES) + len(CONFIG_CASES))]
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank did not finish"
    assert all(p.exitcode == 0 for p in procs)
    for rank, case, ok, status in results:
        print(rank, case, ok)
        assert ok, (rank, case)
        assert status == 0, (rank, case)
