"""The three GEMM paths give the same D, bit for bit:

- mpk_gemm_mxfp8_bf16: A dequantized exactly to BF16 by a bandwidth pre-pass
  into a pooled workspace, then the TMA-fed BF16 x BF16 tensor-core kernel;
- mpk_gemm_mxfp8_bf16_ws with a caller workspace: the same kernels;
- mpk_gemm_mxfp8_bf16_ws with no workspace: A converted to BF16 on chip by the
  GEMM kernel's own transform warps.

All feed the same BF16 values to the same MMA sequence, so each meets the parity
bar against the oracle that the default path is held to.  The on-chip kernel runs
whole tiles only, so it is compared with the pre-pass path under the whole-tile
schedule; under the default schedule the pre-pass path may split the last wave's
tiles by K range (stream-K), which sums them in another order."""
import numpy as np
import pytest

import oracle as O
from gpu_util import run_gemm, to_dev, to_host
from test_gemm_gpu import check_parity

pytestmark = pytest.mark.gpu


def _both(mpk_lib, inp, with_c=True):
    """D of the default path (default schedule), after checking it against the
    caller-workspace path (same kernels and schedule: bit for bit) and the on-chip
    kernel against the pre-pass path under whole tiles (bit for bit)."""
    d0, s0 = run_gemm(mpk_lib, inp, with_c=with_c)
    d1, s1 = run_gemm(mpk_lib, inp, with_c=with_c, path="workspace")
    assert np.array_equal(d0, d1) and np.array_equal(s0, s1), "workspace"
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    try:
        dt, st = run_gemm(mpk_lib, inp, with_c=with_c)
        do, so = run_gemm(mpk_lib, inp, with_c=with_c, path="onchip")
    finally:
        mpk_lib.set_gemm_schedule(prev)
    assert np.array_equal(dt, do) and np.array_equal(st, so), "onchip"
    hist = O.mx_ulp_hist(d0, s0, dt, st)
    assert hist[2] == 0 and hist[3] == 0, hist  # schedules differ by summation order only
    return d0, s0


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (512, 512, 512), (256, 512, 1024),
                                   (1024, 1024, 1024)])
def test_ws_reference_shapes(mpk_lib, cuda, M, N, K):
    inp = O.make_gemm_inputs(M, N, K, seed=42)
    Dd, Ds = _both(mpk_lib, inp)
    check_parity(Dd, Ds, O.gold_mx(inp), f"ws {M}x{N}x{K}")


@pytest.mark.parametrize("M,N,K", [(200, 264, 80), (130, 136, 48), (1, 8, 16), (129, 520, 1104),
                                   (64, 2056, 192), (384, 256, 4112)])
@pytest.mark.parametrize("with_c", [True, False])
def test_ws_ragged(mpk_lib, cuda, M, N, K, with_c):
    """K % 32 != 0 takes the element-wise pre-pass; ragged M/N/K tiles are
    zero-filled by TMA."""
    inp = O.make_gemm_inputs(M, N, K, seed=M + N + K, with_c=with_c)
    Dd, Ds = _both(mpk_lib, inp, with_c=with_c)
    check_parity(Dd, Ds, O.gold_mx(inp), f"ws ragged {M}x{N}x{K} C={with_c}")


@pytest.mark.parametrize("M,N,K", [(100, 100, 100), (65, 7, 17), (64, 2050, 96)])
def test_ws_any_shape(mpk_lib, cuda, M, N, K):
    """Shapes outside TMA's stride rules need the padded workspace, whose size
    mpk_gemm_workspace_size reports; the on-chip kernel refuses them."""
    inp = O.make_gemm_inputs(M, N, K, seed=M + 2 * N + K)
    d0, s0 = run_gemm(mpk_lib, inp)
    d1, s1 = run_gemm(mpk_lib, inp, path="workspace")
    assert np.array_equal(d0, d1) and np.array_equal(s0, s1)
    check_parity(d1, s1, O.gold_mx(inp), f"ws any shape {M}x{N}x{K}")
    with pytest.raises(mpk_lib.MpkError) as e:
        run_gemm(mpk_lib, inp, path="onchip")
    assert e.value.status == mpk_lib.MPK_ERR_UNSUPPORTED


@pytest.mark.parametrize("with_nan", [False, True])
def test_ws_exotic_scales_and_nan_codes(mpk_lib, cuda, with_nan):
    """Scale bytes 0-2, 134/135 and 247-255 and NaN codes take the pre-pass's
    general conversion; results equal the fused kernel's."""
    M, N, K = 256, 256, 256
    inp = O.make_gemm_inputs(M, N, K, seed=78)
    rng = np.random.default_rng(78)
    pool = np.array([0, 1, 2, 3, 114, 134, 135, 200, 246, 247, 254, 255], np.uint8)
    sc = inp["A_scales"].copy()
    rows = rng.choice(M, 48, replace=False)
    sc[rows] = rng.choice(pool, (48, sc.shape[1]))
    inp["A_scales"] = sc
    if with_nan:
        d = inp["A_data"].copy()
        idx = rng.choice(M * K, 20, replace=False)
        d.ravel()[idx] = rng.choice(np.array([0x7F, 0xFF], np.uint8), 20)
        inp["A_data"] = d
    inp["A_deq"] = O.dequantize(inp["A_data"], inp["A_scales"])
    Dd, Ds = _both(mpk_lib, inp)
    gold = O.gold_mx(inp)
    hist = O.mx_ulp_hist(Dd, Ds, gold[1], gold[2])
    assert hist[3] == 0
    assert hist[0] + hist[1] >= 0.999 * sum(hist)


@pytest.mark.parametrize("M,N,K", [(131072, 2048, 2048), (65536, 1024, 4096), (262144, 512, 1024),
                                   (100003, 1000, 2048)])
def test_default_path_takes_the_onchip_kernel_for_tall_products(mpk_lib, cuda, M, N, K):
    """Tall products with few columns go straight to the on-chip conversion kernel
    from the default entry point; D equals the pre-pass kernel's (caller workspace)
    bit for bit, and the default call allocates no workspace.  The last shape has a
    ragged last row tile, a partial last column chunk and C/D rows too short for
    16-byte stores."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    Ad, As = mpk_lib.quantize(torch.randn((M, K), generator=g, device="cuda") * 0.02)
    Cd, Cs = mpk_lib.quantize(torch.randn((M, N), generator=g, device="cuda") * 0.02)
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    assert mpk_lib.gemm_path(Ad, B, M, N, K) == mpk_lib.PATH_ONCHIP
    D0 = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    S0 = torch.empty((M, (N + 31) // 32), dtype=torch.uint8, device="cuda")
    mpk_lib.release_workspace_pool()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    mpk_lib.gemm_fp8_tensorcore(Ad, As, B, Cd, Cs, D0, S0, M, N, K)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0 - (2 << 20)  # no workspace reserved
    D1, S1 = torch.empty_like(D0), torch.empty_like(S0)
    ws = torch.empty((mpk_lib.gemm_workspace_size(M, N, K),), dtype=torch.uint8, device="cuda")
    mpk_lib.gemm_fp8_tensorcore_ws(Ad, As, B, Cd, Cs, D1, S1, M, N, K, ws)
    torch.cuda.synchronize()
    assert torch.equal(D0, D1) and torch.equal(S0, S1)
    assert mpk_lib.device_status() == 0


@pytest.mark.parametrize("M,N,K,offset", [(512, 512, 2048, 1), (512, 512, 2048, 0), (384, 256, 1600, 0),
                                          (256, 512, 4096, 8), (512, 512, 1152, 0), (256, 768, 11008, 4)])
def test_onchip_scale_byte_placement(whole_tiles, cuda, M, N, K, offset):
    """The on-chip kernel reads each row's A scale bytes 16 at a time when they are
    16-byte aligned and K is a multiple of 512, 4 at a time when they are 4-byte
    aligned and K is a multiple of 128 (the row's last group cut short), else byte by
    byte: each placement gives the same D as the pre-pass path."""
    import torch

    mpk_lib = whole_tiles
    inp = O.make_gemm_inputs(M, N, K, seed=M + K + offset)
    want_d, want_s = run_gemm(mpk_lib, inp)
    A, B = to_dev(inp["A_data"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    sc = inp["A_scales"]
    buf = torch.zeros((sc.size + 64,), dtype=torch.uint8, device="cuda")
    As = buf[offset:offset + sc.size].view(sc.shape)
    As.copy_(to_dev(sc))
    D = torch.full((M, N), 0xEE, dtype=torch.uint8, device="cuda")
    Ds = torch.full((M, N // 32), 0xEE, dtype=torch.uint8, device="cuda")
    mpk_lib.gemm_fp8_tensorcore_ws(A, As, B, C, Cs, D, Ds, M, N, K, None)
    torch.cuda.synchronize()
    assert np.array_equal(to_host(D), want_d) and np.array_equal(to_host(Ds), want_s)
    assert mpk_lib.device_status() == 0


def test_ws_prepass_is_exact_bf16(mpk_lib, cuda):
    """The workspace holds code x 2^(s-127) rounded to BF16 (exact for s >= 3)."""
    import torch

    M, N, K = 96, 64, 256
    inp = O.make_gemm_inputs(M, N, K, seed=5)
    rng = np.random.default_rng(5)
    inp["A_scales"] = rng.integers(0, 256, inp["A_scales"].shape, dtype=np.uint8)
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    Ds = torch.empty((M, N // 32), dtype=torch.uint8, device="cuda")
    ws = torch.zeros((mpk_lib.gemm_workspace_size(M, N, K),), dtype=torch.uint8, device="cuda")
    mpk_lib.gemm_fp8_tensorcore_ws(A, As, B, None, None, D, Ds, M, N, K, ws)
    torch.cuda.synchronize()
    got = to_host(ws).view(np.uint16).reshape(M, K)
    want = O.to_bf16_bits(O.dequantize(inp["A_data"], inp["A_scales"]))
    nan = np.isnan(O.dequantize(inp["A_data"], inp["A_scales"]))
    got_nan = ((got & 0x7F80) == 0x7F80) & ((got & 0x7F) != 0)
    assert np.array_equal(nan, got_nan)
    assert np.array_equal(got[~nan], want[~nan])


def test_ws_argument_checks(mpk_lib, cuda):
    import torch

    M, N, K = 128, 128, 128
    inp = O.make_gemm_inputs(M, N, K, seed=1)
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    Ds = torch.empty((M, N // 32), dtype=torch.uint8, device="cuda")
    need = mpk_lib.gemm_workspace_size(M, N, K)
    assert need == M * K * 2
    assert mpk_lib.gemm_workspace_size(100, 100, 100) == 100 * 104 * 2 + (256 - 100 * 104 * 2 % 256) + 100 * 104 * 2
    small = torch.empty((need - 16,), dtype=torch.uint8, device="cuda")
    with pytest.raises(mpk_lib.MpkError) as e:
        mpk_lib.gemm_fp8_tensorcore_ws(A, As, B, None, None, D, Ds, M, N, K, small)
    assert e.value.status == mpk_lib.MPK_ERR_INVALID_VALUE
    big = torch.empty((need + 32,), dtype=torch.uint8, device="cuda")
    with pytest.raises(mpk_lib.MpkError) as e:
        mpk_lib.gemm_fp8_tensorcore_ws(A, As, B, None, None, D, Ds, M, N, K, big[8:].data_ptr(),
                                       workspace_bytes=need + 24)
    assert e.value.status == mpk_lib.MPK_ERR_MISALIGNED


def test_pool_release_and_reuse(mpk_lib, cuda):
    """The pooled workspace can be handed back between calls; later calls take a
    fresh one and give the same D."""
    inp = O.make_gemm_inputs(256, 512, 512, seed=3)
    d0, s0 = run_gemm(mpk_lib, inp)
    mpk_lib.release_workspace_pool()
    d1, s1 = run_gemm(mpk_lib, inp)
    mpk_lib.release_workspace_pool()
    mpk_lib.release_workspace_pool()
    assert np.array_equal(d0, d1) and np.array_equal(s0, s1)


@pytest.mark.parametrize("M,N,K", [(1024, 5120, 256), (2048, 2816, 192)])
def test_split_tail_tiles_match_onchip(whole_tiles, cuda, M, N, K):
    """When the last wave would run at most half full, the pre-pass kernel cuts the
    last raster tiles into 256 x 128 halves; D equals the on-chip kernel's (which
    never splits) bit for bit."""
    inp = O.make_gemm_inputs(M, N, K, seed=M + N)
    d0, s0 = run_gemm(whole_tiles, inp)
    d1, s1 = run_gemm(whole_tiles, inp, path="onchip")
    assert np.array_equal(d0, d1) and np.array_equal(s0, s1)


def test_split_tail_with_empty_half(whole_tiles, cuda):
    """N = 2404: the last column of tiles has 100 columns, so the second half of each
    split tile lies past N (no columns to store, accumulator phase still consumed)."""
    M, N, K = 2048, 2404, 64
    inp = O.make_gemm_inputs(M, N, K, seed=7)
    Dd, Ds = run_gemm(whole_tiles, inp)
    check_parity(Dd, Ds, O.gold_mx(inp), f"split tail {M}x{N}x{K}")
    assert whole_tiles.device_status() == 0


def test_concurrent_streams_and_threads(mpk_lib, cuda):
    """Calls in flight on several streams at once, issued from several host
    threads, each with its own pooled workspace: every D equals the same call made
    alone."""
    import threading

    import torch

    shapes = [(512, 768, 256), (1024, 512, 384), (256, 2048, 128), (768, 1024, 512)]
    cases = []
    for i, (M, N, K) in enumerate(shapes):
        inp = O.make_gemm_inputs(M, N, K, seed=300 + i)
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
            for _ in range(5):
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
