"""Stream-K on the GPU: the tiles of a last, partial wave split across SM pairs by
K-step ranges, each split tile finished by the pair holding its last K-steps after
adding the other pairs' FP32 partial sums.

Each case is held to the parity bar against the oracle's FP32 gold, compared with
the whole-tile schedule of the same kernel (the two differ only in summation order:
no code more than one E4M3 step apart), and run twice to check that the
hand-off counters are reset between calls (the A pre-pass zeroes them)."""
import numpy as np
import pytest

import oracle as O
from gpu_util import run_gemm, to_dev, to_host
from test_gemm_gpu import check_parity

pytestmark = pytest.mark.gpu


def _schedule(mpk, mode):
    class _Ctx:
        def __enter__(self):
            self.prev = mpk.set_gemm_schedule(mode)

        def __exit__(self, *a):
            mpk.set_gemm_schedule(self.prev)

    return _Ctx()


def _sample_rows(M):
    rows = {0, 1, 127, 128, 255, 256, M // 2, M - 129, M - 128, M - 1}
    rng = np.random.default_rng(M)
    rows |= set(int(r) for r in rng.integers(0, M, 54))
    return np.array(sorted(r for r in rows if 0 <= r < M), np.int64)


def _against_tiles(mpk, inp, label, with_c=True, rows=None):
    d0, s0 = run_gemm(mpk, inp, with_c=with_c)
    d0b, s0b = run_gemm(mpk, inp, with_c=with_c)
    assert np.array_equal(d0, d0b) and np.array_equal(s0, s0b), "second call differs"
    with _schedule(mpk, mpk.SCHEDULE_TILES):
        dt, st = run_gemm(mpk, inp, with_c=with_c)
    hist = O.mx_ulp_hist(d0, s0, dt, st)
    print(f"{label}: vs whole tiles {hist}")
    assert hist[2] == 0 and hist[3] == 0
    if rows is None:
        check_parity(d0, s0, O.gold_mx(inp), label)
    else:  # exact gold for a sample of rows (row i of D depends on rows i of A and C only)
        check_parity(d0[rows], s0[rows], O.gold_mx(inp, rows=rows), label, ref_pass_mark=False)
    assert mpk.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1024, 10240, 4096), (768, 7680, 8192), (1024, 12288, 4096),
                                   (2048, 3584, 8192), (2048, 7168, 8192)])
def test_default_schedule_split_wave(mpk_lib, cuda, M, N, K):
    """Shapes whose default plan spreads the last wave's tiles over the SM pairs,
    among them the per-GPU slabs of the dense projection on 4 GPUs and of the wide
    shape on 8 and 4 GPUs."""
    tiles, sk_tiles, pairs = mpk_lib.gemm_plan(M, N, K)
    assert sk_tiles > 0 and pairs > sk_tiles, (tiles, sk_tiles, pairs)
    inp = O.make_gemm_inputs(M, N, K, seed=M + N + K)
    rows = _sample_rows(M) if M * N * K > 4e9 else None
    _against_tiles(mpk_lib, inp, f"stream-K {M}x{N}x{K} ({sk_tiles} tiles on {pairs} pairs)", rows=rows)


@pytest.mark.parametrize("M,N,K", [(256, 256, 2048), (1, 8, 16), (65, 7, 17), (200, 264, 80),
                                   (384, 256, 4112), (2048, 2404, 64), (600, 700, 1000)])
@pytest.mark.parametrize("with_c", [True, False])
def test_forced_stream_k(mpk_lib, cuda, M, N, K, with_c):
    """Every tile's K-steps spread over the pairs: one tile of 32 K-steps over 32
    pairs (the owner adds 31 partials), a single K-step, ragged M, N and K, a B copy
    (N % 8 != 0), right-edge tiles with few columns, no C."""
    with _schedule(mpk_lib, mpk_lib.SCHEDULE_STREAM_K):
        tiles, sk_tiles, pairs = mpk_lib.gemm_plan(M, N, K)
        assert sk_tiles == tiles
        inp = O.make_gemm_inputs(M, N, K, seed=3 * M + N + K, with_c=with_c)
        _against_tiles(mpk_lib, inp, f"forced stream-K {M}x{N}x{K} C={with_c} ({pairs} pairs)", with_c)


def test_forced_stream_k_exotic_scales_and_nan(mpk_lib, cuda):
    """Partial sums carry NaN and large values through the hand-off: A scale bytes
    over the whole range with NaN codes, C with NaN codes."""
    M, N, K = 256, 512, 1024
    inp = O.make_gemm_inputs(M, N, K, seed=5)
    rng = np.random.default_rng(5)
    inp["A_scales"] = rng.integers(100, 140, inp["A_scales"].shape, dtype=np.uint8)
    a = inp["A_data"].copy()
    a[rng.integers(0, M, 20), rng.integers(0, K, 20)] = 0x7F
    inp["A_data"] = a
    inp["A_deq"] = O.dequantize(inp["A_data"], inp["A_scales"])
    c = inp["C_data"].copy()
    c[rng.integers(0, M, 20), rng.integers(0, N, 20)] = 0xFF
    inp["C_data"] = c
    inp["C_deq"] = O.dequantize(inp["C_data"], inp["C_scales"])
    with _schedule(mpk_lib, mpk_lib.SCHEDULE_STREAM_K):
        d0, s0 = run_gemm(mpk_lib, inp)
        with _schedule(mpk_lib, mpk_lib.SCHEDULE_TILES):
            dt, st = run_gemm(mpk_lib, inp)
    gold = O.gold_mx(inp)
    for d, s_, tag in ((d0, s0, "stream-K"), (dt, st, "tiles")):
        hist = O.mx_ulp_hist(d, s_, gold[1], gold[2])
        print(f"exotic {tag}: {hist}")
        assert hist[3] == 0 and hist[0] + hist[1] >= 0.999 * sum(hist)
    assert O.mx_ulp_hist(d0, s0, dt, st)[3] == 0


@pytest.fixture
def forced_stream_k(mpk_lib):
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_STREAM_K)
    yield mpk_lib
    mpk_lib.set_gemm_schedule(prev)


def test_graph_replay_resets_the_hand_off(forced_stream_k, cuda):
    """A captured call replays with fresh counters each time (the captured pre-pass
    zeroes them), giving the eager call's D bit for bit."""
    import torch

    mpk_lib = forced_stream_k
    M, N, K = 512, 1024, 4096
    assert mpk_lib.gemm_plan(M, N, K)[1] > 0
    inp = O.make_gemm_inputs(M, N, K, seed=77)
    want_d, want_s = run_gemm(mpk_lib, inp)
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    D = torch.zeros((M, N), dtype=torch.uint8, device="cuda")
    S = torch.zeros((M, N // 32), dtype=torch.uint8, device="cuda")
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    torch.cuda.synchronize()
    with torch.cuda.graph(g, stream=s):
        for _ in range(3):
            mpk_lib.gemm_fp8_tensorcore(A, As, B, C, Cs, D, S, M, N, K, s)
    for _ in range(3):
        D.zero_(); S.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert np.array_equal(to_host(D), want_d) and np.array_equal(to_host(S), want_s)
    del g
    assert mpk_lib.device_status() == 0


def test_concurrent_streams_and_threads(forced_stream_k, cuda):
    """Stream-K calls in flight on several streams at once from several host
    threads: the pairs of one call may not all be resident while another call
    runs, and a pair waits only for pairs that started before it, so every call
    completes, each D equal to the same call made alone."""
    import threading

    import torch

    mpk_lib = forced_stream_k
    shapes = [(512, 1024, 4096), (256, 2048, 2048), (1024, 768, 2048), (128, 4096, 4096)]
    cases = []
    for i, (M, N, K) in enumerate(shapes):
        assert mpk_lib.gemm_plan(M, N, K)[1] > 0
        inp = O.make_gemm_inputs(M, N, K, seed=500 + i)
        want = run_gemm(mpk_lib, inp)
        dev = [to_dev(inp[k]) for k in ("A_data", "A_scales", "B_bf16", "C_data", "C_scales")]
        D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
        Ds = torch.empty((M, N // 32), dtype=torch.uint8, device="cuda")
        cases.append(((M, N, K), dev, D, Ds, want, torch.cuda.Stream()))
    torch.cuda.synchronize()
    errors = []

    def worker(case):
        (M, N, K), (A, As, B, C, Cs), D, Ds, _, st = case
        try:
            for _ in range(6):
                mpk_lib.gemm_fp8_tensorcore(A, As, B, C, Cs, D, Ds, M, N, K, st)
        except Exception as e:  # reported below
            errors.append(e)

    ths = [threading.Thread(target=worker, args=(c,)) for c in cases]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    for _, _, D, Ds, (wd, ws_), _ in cases:
        assert np.array_equal(to_host(D), wd) and np.array_equal(to_host(Ds), ws_)
    assert mpk_lib.device_status() == 0


def test_small_workspace_falls_back_to_whole_tiles(forced_stream_k, cuda):
    """A caller workspace with room for the operands but not for the partials runs
    whole tiles: D equals the whole-tile schedule's bit for bit."""
    import torch

    mpk_lib = forced_stream_k
    M, N, K = 256, 1024, 4096
    assert mpk_lib.gemm_plan(M, N, K)[1] > 0
    inp = O.make_gemm_inputs(M, N, K, seed=9)
    with _schedule(mpk_lib, mpk_lib.SCHEDULE_TILES):
        want_d, want_s = run_gemm(mpk_lib, inp)
        small = mpk_lib.gemm_workspace_size(M, N, K)
    assert small < mpk_lib.gemm_workspace_size(M, N, K)
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    S = torch.empty((M, N // 32), dtype=torch.uint8, device="cuda")
    ws = torch.empty((small,), dtype=torch.uint8, device="cuda")
    mpk_lib.gemm_fp8_tensorcore_ws(A, As, B, C, Cs, D, S, M, N, K, ws)
    torch.cuda.synchronize()
    assert np.array_equal(to_host(D), want_d) and np.array_equal(to_host(S), want_s)
