"""Every element of D at full size, not a row sample: the gold is the reference's
own GPU gold GEMM (gemm_reference_gpu, src/reference/gemm_reference.cu:61-66, FP32 on
CUDA cores, rebuilt for sm_100a in oracle/_ref) on the exactly dequantized operands,
quantized to MXFP8 with the reference's rule (the library's quantizer, bit-exact with
it).  Both sides accumulate in FP32 in different orders (the gold with FMA
contraction), so the bar is the parity bar: no NaN mismatch and at least 99.9 % of
the codes within one E4M3 step."""
import numpy as np
import pytest

import oracle as O
from gpu_util import to_host
from test_gemm_gpu import WITHIN_ONE_STEP

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")]


@pytest.mark.parametrize("M,N,K,seed", [
    (4096, 12288, 4096, 43),      # dense projection
    (131072, 2048, 2048, 45),     # tall-skinny
    (2048, 28672, 8192, 46),      # wide
])
def test_full_matrix_against_reference_gpu_gold(mpk_lib, cuda, M, N, K, seed):
    import torch

    g = torch.Generator(device="cuda").manual_seed(seed)
    Ad, As = mpk_lib.quantize(torch.randn((M, K), generator=g, device="cuda") * 0.02)
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    Cd, Cs = mpk_lib.quantize(torch.randn((M, N), generator=g, device="cuda") * 0.02)
    D, Ds = mpk_lib.gemm(Ad, As, B, Cd, Cs)

    A32 = mpk_lib.dequantize(Ad, As)
    C32 = mpk_lib.dequantize(Cd, Cs)
    B32 = B.float()
    G = torch.empty((M, N), dtype=torch.float32, device="cuda")
    rc = O.ref().ref_gemm_reference_gpu(A32.data_ptr(), B32.data_ptr(), C32.data_ptr(), G.data_ptr(),
                                        M, N, K, torch.cuda.current_stream().cuda_stream)
    assert rc == 0
    del A32, C32, B32
    gd, gs = mpk_lib.quantize(G)
    torch.cuda.synchronize()
    del G
    hist = O.mx_ulp_hist(to_host(D), to_host(Ds), to_host(gd), to_host(gs))
    total = sum(hist)
    print(f"full matrix {M}x{N}x{K}: exact={hist[0] / total:.6f} one-step={hist[1] / total:.6f} "
          f"more={hist[2]} nan-mismatch={hist[3]}")
    assert hist[3] == 0
    assert hist[0] + hist[1] >= WITHIN_ONE_STEP * total
    assert mpk_lib.device_status() == 0
