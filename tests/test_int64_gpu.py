"""Tensors with more than 2^31 elements: the library indexes with 64-bit
arithmetic (the reference indexes with int).  Rows near the end of the
tensors are checked against the oracle, which is exact for sampled rows (row i of
D depends only on row i of A and C)."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_host
from test_gemm_gpu import check_parity

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("path", ["default", "onchip"])
def test_gemm_d_beyond_2_31_elements(mpk_lib, cuda, path):
    """Both GEMM kernels: the pre-pass path (the default entry point at this width)
    and the on-chip conversion kernel (no workspace)."""
    import torch

    M, N, K = 65536, 36864, 64          # D: 2.4e9 elements
    assert M * N > 2**31
    g = torch.Generator(device="cuda").manual_seed(31)
    Ad, As = mpk_lib.quantize(torch.randn((M, K), generator=g, device="cuda") * 0.02)
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    C = torch.empty((M, N), dtype=torch.float32, device="cuda")
    C.normal_(0.0, 0.02, generator=g)
    Cd, Cs = mpk_lib.quantize(C)
    del C
    if path == "default":
        D, Ds = mpk_lib.gemm(Ad, As, B, Cd, Cs)
    else:
        D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
        Ds = torch.empty((M, N // 32), dtype=torch.uint8, device="cuda")
        mpk_lib.gemm_fp8_tensorcore_ws(Ad, As, B, Cd, Cs, D, Ds, M, N, K, None)
    torch.cuda.synchronize()
    rows = np.array([0, 32767, 58254, M - 2, M - 1])
    A_h, As_h = to_host(Ad[rows]), to_host(As[rows])
    C_h, Cs_h = to_host(Cd[rows]), to_host(Cs[rows])
    B_h = to_host(B)
    inp = {"M": len(rows), "N": N, "K": K, "A_data": A_h, "A_scales": As_h, "B_bf16": B_h,
           "C_data": C_h, "C_scales": Cs_h, "A_deq": O.dequantize(A_h, As_h),
           "B_f32": O.bf16_bits_to_float(B_h), "C_deq": O.dequantize(C_h, Cs_h)}
    check_parity(to_host(D[rows]), to_host(Ds[rows]), O.gold_mx(inp), f"D > 2^31 elements ({path})",
                 ref_pass_mark=False)
    assert mpk_lib.device_status() == 0


def test_codec_beyond_2_31_elements(mpk_lib, cuda):
    import torch

    M, K = 65536, 36864                  # 2.4e9 elements
    x = torch.empty((M, K), dtype=torch.float32, device="cuda")
    x.normal_(0.0, 0.02, generator=torch.Generator(device="cuda").manual_seed(5))
    d, s = mpk_lib.quantize(x)
    torch.cuda.synchronize()
    rows = np.array([0, 40000, M - 1])
    xr = to_host(x[rows])
    wd, ws = O.quantize(xr)
    assert np.array_equal(to_host(d[rows]), wd) and np.array_equal(to_host(s[rows]), ws)
    del x
    y = mpk_lib.dequantize(d, s)
    torch.cuda.synchronize()
    assert np.array_equal(to_host(y[rows]).view(np.uint32), O.dequantize(wd, ws).view(np.uint32))
