"""mpk_gemm_mxfp8_bf16_noalloc: the GEMM with its A workspace in the library's
fixed per-device array instead of an allocation.  It runs the same kernels as
mpk_gemm_mxfp8_bf16, so its D is held to the same parity bar against the oracle
and compared with the existing entry point's D on the same inputs, over two
calls in a row with different A (the second call must not see the first call's
workspace contents).  This file is collected last so that it also runs after
every other GPU test in one process; it passes alone as well."""
import numpy as np
import pytest

import oracle as O
from gpu_util import run_gemm, to_dev, to_host
from test_gemm_gpu import WITHIN_ONE_STEP, check_parity

pytestmark = pytest.mark.gpu


def _noalloc(mpk, inp, stream=None):
    import torch

    M, N, K = inp["M"], inp["N"], inp["K"]
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C = Cs = None
    if inp.get("C_data") is not None:
        C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    D = torch.full((M, N), 0xEE, dtype=torch.uint8, device="cuda")
    Ds = torch.full((M, (N + 31) // 32), 0xEE, dtype=torch.uint8, device="cuda")
    mpk.gemm_fp8_tensorcore_noalloc(A, As, B, C, Cs, D, Ds, M, N, K, stream)
    return D, Ds


def _close(d1, s1, d2, s2):
    """Within the GEMM parity tolerance of each other: no NaN mismatch and at least
    WITHIN_ONE_STEP of the codes within one E4M3 step."""
    hist = O.mx_ulp_hist(d1, s1, d2, s2)
    return hist[3] == 0 and hist[0] + hist[1] >= WITHIN_ONE_STEP * sum(hist), hist


@pytest.mark.parametrize("M,N,K", [(512, 512, 512), (200, 264, 80), (1024, 768, 2048)])
def test_two_calls_in_a_row_match_existing_entry_point(mpk_lib, cuda, M, N, K):
    import torch

    first = O.make_gemm_inputs(M, N, K, seed=100 + M)
    second = O.make_gemm_inputs(M, N, K, seed=200 + M, std=0.05)
    want1 = run_gemm(mpk_lib, first)
    want2 = run_gemm(mpk_lib, second)
    stream = torch.cuda.current_stream()
    D1, S1 = _noalloc(mpk_lib, first, stream)
    D2, S2 = _noalloc(mpk_lib, second, stream)
    torch.cuda.synchronize()
    for (Dd, Ds), want, inp, tag in (((D1, S1), want1, first, "first"), ((D2, S2), want2, second, "second")):
        got_d, got_s = to_host(Dd), to_host(Ds)
        ok, hist = _close(got_d, got_s, *want)
        print(f"noalloc {M}x{N}x{K} {tag} call vs mpk_gemm_mxfp8_bf16: {hist}")
        assert ok
        check_parity(got_d, got_s, O.gold_mx(inp), f"noalloc {M}x{N}x{K} {tag}")
    assert mpk_lib.device_status() == 0


def test_largest_size_that_fits(mpk_lib, cuda):
    """M*K*2 exactly MPK_NOALLOC_SCRATCH_BYTES (4096 x 4096) is accepted."""
    import torch

    M, K, N = 4096, 4096, 256
    assert M * K * 2 == mpk_lib.NOALLOC_SCRATCH_BYTES
    g = torch.Generator(device="cuda").manual_seed(7)
    Ad, As = mpk_lib.quantize(torch.randn((M, K), generator=g, device="cuda") * 0.02)
    Cd, Cs = mpk_lib.quantize(torch.randn((M, N), generator=g, device="cuda") * 0.02)
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    D0, S0 = mpk_lib.gemm(Ad, As, B, Cd, Cs)
    D1 = torch.empty_like(D0)
    S1 = torch.empty_like(S0)
    mpk_lib.gemm_fp8_tensorcore_noalloc(Ad, As, B, Cd, Cs, D1, S1, M, N, K)
    torch.cuda.synchronize()
    ok, hist = _close(to_host(D1), to_host(S1), to_host(D0), to_host(S0))
    print(f"noalloc 4096x256x4096 vs mpk_gemm_mxfp8_bf16: {hist}")
    assert ok


def test_oversize_is_rejected_before_any_launch(mpk_lib, cuda):
    """M*K*2 above the fixed scratch, with a K the on-chip kernel cannot take
    (K % 16 != 0), returns MPK_ERR_UNSUPPORTED with a message naming the limit, and
    leaves D untouched.  The buffers are real and full size, so nothing could be read
    out of bounds even if a launch happened."""
    import torch

    M, K, N = 4096, 4104, 64
    assert M * K * 2 > mpk_lib.NOALLOC_SCRATCH_BYTES
    A = torch.zeros((M, K), dtype=torch.uint8, device="cuda")
    As = torch.full((M, (K + 31) // 32), 127, dtype=torch.uint8, device="cuda")
    B = torch.zeros((K, N), dtype=torch.bfloat16, device="cuda")
    D = torch.full((M, N), 0xEE, dtype=torch.uint8, device="cuda")
    Ds = torch.full((M, N // 32), 0xEE, dtype=torch.uint8, device="cuda")
    with pytest.raises(mpk_lib.MpkError) as e:
        mpk_lib.gemm_fp8_tensorcore_noalloc(A, As, B, None, None, D, Ds, M, N, K)
    assert e.value.status == mpk_lib.MPK_ERR_UNSUPPORTED
    assert "scratch" in str(e.value)
    torch.cuda.synchronize()
    assert bool((D == 0xEE).all()) and bool((Ds == 0xEE).all())
    assert mpk_lib.device_status() == 0


def test_oversize_runs_the_onchip_kernel(mpk_lib, cuda):
    """A product whose BF16 A would not fit the scratch, within the on-chip kernel's
    limits, runs on that kernel: D equals the default entry point's under whole
    tiles, bit for bit, and no device memory is taken."""
    import torch

    M, N, K = 8192, 768, 4096  # BF16 A of 64 MiB
    assert M * K * 2 > mpk_lib.NOALLOC_SCRATCH_BYTES
    inp = O.make_gemm_inputs(M, N, K, seed=17)
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    try:
        want_d, want_s = run_gemm(mpk_lib, inp)
    finally:
        mpk_lib.set_gemm_schedule(prev)
    _noalloc(mpk_lib, inp)  # first call on the device loads the array
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    D, Ds = _noalloc(mpk_lib, inp)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0 - (2 << 20)
    assert np.array_equal(to_host(D), want_d) and np.array_equal(to_host(Ds), want_s)
    assert mpk_lib.device_status() == 0


def test_second_call_takes_no_device_memory(mpk_lib, cuda):
    """After the first call on a device (which loads the library's device code that
    holds the array), further calls leave the device's free memory unchanged."""
    import torch

    inp = O.make_gemm_inputs(512, 512, 512, seed=9)
    D, S = _noalloc(mpk_lib, inp)  # first call: the array is reserved here at the latest
    torch.cuda.synchronize()
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        mpk_lib.gemm_fp8_tensorcore_noalloc(A, As, B, C, Cs, D, S, 512, 512, 512)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    assert mpk_lib.device_status() == 0
