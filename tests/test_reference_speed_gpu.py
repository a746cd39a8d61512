"""The reference's own GPU kernels, rebuilt for sm_100a (oracle/_ref), timed beside
the library on the same B200 and the same inputs: its GEMM launcher
gemm_fp8_tensorcore (WMMA fp16, FP32 temporary, separate quantize;
src/kernels/gemm_fp8_tensorcore.cu:231-249) and its quantize/dequantize kernels
(src/quantize/mxfp8_quantize.cu:82-88, src/quantize/mxfp8_dequantize.cu:22-29).
The library must be faster on every one; the figures are printed for the record."""
import pytest

import oracle as O

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")]


def _time(fn, reps):
    import torch

    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


@pytest.mark.parametrize("M,N,K", [(4096, 12288, 4096), (4096, 4096, 11008), (131072, 2048, 2048),
                                   (2048, 28672, 8192)])
def test_gemm_faster_than_reference_kernel(mpk_lib, cuda, M, N, K):
    import torch

    g = torch.Generator(device="cuda").manual_seed(M + N)
    Ad, As = mpk_lib.quantize(torch.randn((M, K), generator=g, device="cuda") * 0.02)
    B = (torch.randn((K, N), generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    Cd, Cs = mpk_lib.quantize(torch.randn((M, N), generator=g, device="cuda") * 0.02)
    D = torch.empty((M, N), dtype=torch.uint8, device="cuda")
    Ds = torch.empty((M, (N + 31) // 32), dtype=torch.uint8, device="cuda")
    R = O.ref()
    s = torch.cuda.current_stream().cuda_stream
    args = (Ad.data_ptr(), As.data_ptr(), B.data_ptr(), Cd.data_ptr(), Cs.data_ptr(), D.data_ptr(),
            Ds.data_ptr(), M, N, K, s)
    ref_ms = _time(lambda: R.ref_gemm_fp8_tensorcore(*args), 3)
    ours_ms = _time(lambda: mpk_lib.gemm_fp8_tensorcore(Ad, As, B, Cd, Cs, D, Ds, M, N, K), 20)
    fl = 2.0 * M * N * K
    print(f"{M}x{N}x{K}: reference gemm_fp8_tensorcore {ref_ms:.3f} ms ({fl / ref_ms / 1e9:.1f} TFLOPS), "
          f"library {ours_ms:.4f} ms ({fl / ours_ms / 1e9:.1f} TFLOPS), {ref_ms / ours_ms:.1f}x")
    assert ours_ms < ref_ms


def test_codec_faster_than_reference_kernels(mpk_lib, cuda):
    import torch

    M, K = 131072, 2048
    x = torch.randn((M, K), generator=torch.Generator(device="cuda").manual_seed(3), device="cuda") * 0.02
    d = torch.empty((M, K), dtype=torch.uint8, device="cuda")
    s_ = torch.empty((M, K // 32), dtype=torch.uint8, device="cuda")
    y = torch.empty_like(x)
    R = O.ref()
    st = torch.cuda.current_stream().cuda_stream
    nbytes = M * K * (4 + 1) + M * K // 32
    rq = _time(lambda: R.ref_mxfp8_quantize_gpu(x.data_ptr(), d.data_ptr(), s_.data_ptr(), M, K, st), 5)
    oq = _time(lambda: mpk_lib.mxfp8_quantize_gpu(x, d, s_, M, K), 20)
    rd = _time(lambda: R.ref_mxfp8_dequantize_gpu(d.data_ptr(), s_.data_ptr(), y.data_ptr(), M, K, st), 5)
    od = _time(lambda: mpk_lib.mxfp8_dequantize_gpu(d, s_, y, M, K), 20)
    print(f"quantize: reference {nbytes / rq / 1e6:.0f} GB/s, library {nbytes / oq / 1e6:.0f} GB/s; "
          f"dequantize: reference {nbytes / rd / 1e6:.0f} GB/s, library {nbytes / od / 1e6:.0f} GB/s")
    assert oq < rq and od < rd
