"""The fused GEMM + all-gather entry point on one GPU: the epilogue's
multi-destination stores (every destination a local buffer here; across GPUs they
are peer-mapped buffers, covered by tests/test_sharding_gpu.py), the row offset,
and the bounded cross-GPU barrier -- including its timeout, driven by a flag that
nothing sets."""
import numpy as np
import pytest

import oracle as O
from gpu_util import run_gemm, to_dev, to_host

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K,row_offset,M_total", [(256, 512, 256, 100, 600), (130, 100, 64, 7, 140),
                                                      (64, 96, 0, 3, 70)])
def test_every_destination_gets_the_slab_rows(mpk_lib, cuda, M, N, K, row_offset, M_total):
    import torch

    inp = O.make_gemm_inputs(M, N, max(K, 16), seed=M + N + K)
    if K == 0:
        inp = dict(inp, K=0)
    want_d, want_s = run_gemm(mpk_lib, inp)
    nb = (N + 31) // 32
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    ndest = 3
    Ds = [torch.full((M_total, N), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(ndest)]
    Ss = [torch.full((M_total, nb), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(ndest)]
    ws = torch.empty(mpk_lib.gemm_workspace_size(M, N, max(K, 1)) + 2 * max(K, 1) * (N + 8) + 256,
                     dtype=torch.uint8, device="cuda")
    mpk_lib.gemm_fp8_tensorcore_gather(A, As, B, C, Cs, M, N, K, row_offset, M_total, Ds, Ss, ws)
    torch.cuda.synchronize()
    for d, s in zip(Ds, Ss):
        d, s = to_host(d), to_host(s)
        assert np.array_equal(d[row_offset:row_offset + M], want_d)
        assert np.array_equal(s[row_offset:row_offset + M], want_s)
        assert (d[:row_offset] == 0xEE).all() and (d[row_offset + M:] == 0xEE).all()
        assert (s[:row_offset] == 0xEE).all() and (s[row_offset + M:] == 0xEE).all()
    assert mpk_lib.device_status() == 0


@pytest.mark.parametrize("M,N,K,col_offset,N_total", [(256, 512, 256, 128, 1024), (130, 100, 64, 64, 164),
                                                      (96, 96, 32, 0, 192)])
def test_column_slab_lands_at_its_offset(mpk_lib, cuda, M, N, K, col_offset, N_total):
    """A column slab's D goes to columns [col_offset, col_offset + N) of every
    destination (rows N_total bytes apart), its scales to the matching blocks."""
    import torch

    inp = O.make_gemm_inputs(M, N, K, seed=M + N + col_offset)
    want_d, want_s = run_gemm(mpk_lib, inp)
    nb, nbt = (N + 31) // 32, (N_total + 31) // 32
    A, As, B = to_dev(inp["A_data"]), to_dev(inp["A_scales"]), to_dev(inp["B_bf16"])
    C, Cs = to_dev(inp["C_data"]), to_dev(inp["C_scales"])
    Ds = [torch.full((M, N_total), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(2)]
    Ss = [torch.full((M, nbt), 0xEE, dtype=torch.uint8, device="cuda") for _ in range(2)]
    ws = torch.empty(mpk_lib.gemm_workspace_size(M, N, K) + 2 * K * (N + 8) + 256, dtype=torch.uint8,
                     device="cuda")
    mpk_lib.gemm_fp8_tensorcore_gather(A, As, B, C, Cs, M, N, K, 0, M, Ds, Ss, ws, col_offset=col_offset,
                                       N_total=N_total)
    torch.cuda.synchronize()
    c0, b0 = col_offset, col_offset // 32
    for d, s in zip(Ds, Ss):
        d, s = to_host(d), to_host(s)
        assert np.array_equal(d[:, c0:c0 + N], want_d)
        assert np.array_equal(s[:, b0:b0 + nb], want_s)
        assert (d[:, :c0] == 0xEE).all() and (d[:, c0 + N:] == 0xEE).all()
        assert (s[:, :b0] == 0xEE).all() and (s[:, b0 + nb:] == 0xEE).all()


def test_gather_argument_checks(mpk_lib, cuda):
    import torch

    buf = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    b16 = torch.zeros(1 << 14, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(mpk_lib.MpkError) as e:   # rows past M_total
        mpk_lib.gemm_fp8_tensorcore_gather(buf, buf, b16, None, None, 64, 64, 64, 10, 70, [buf], [buf], buf)
    assert e.value.status == mpk_lib.MPK_ERR_INVALID_VALUE
    with pytest.raises(mpk_lib.MpkError) as e:   # workspace too small
        mpk_lib.gemm_fp8_tensorcore_gather(buf, buf, b16, None, None, 64, 64, 64, 0, 64, [buf], [buf],
                                           buf[:1024])
    assert e.value.status == mpk_lib.MPK_ERR_INVALID_VALUE


def test_barrier_single_gpu_and_timeout(mpk_lib, cuda):
    """world 1 passes at once.  With world 2 on one GPU the second flag array is
    local and no second GPU ever arrives: the wait expires after its budget, the
    status word records site 0x17E, and the context stays usable."""
    import torch

    f0 = torch.zeros(64, dtype=torch.int32, device="cuda")
    f1 = torch.zeros(64, dtype=torch.int32, device="cuda")
    mpk_lib.peer_barrier([f0], 0, 1, 1)
    torch.cuda.synchronize()
    assert mpk_lib.device_status() == 0
    assert int(f0[0]) == 1
    mpk_lib.set_wait_timeout_ns(2_000_000)
    try:
        mpk_lib.peer_barrier([f0, f1], 0, 2, 2)
        assert mpk_lib.device_status() == 0x100 + 0x7E
    finally:
        mpk_lib.set_wait_timeout_ns(2_000_000_000)
    assert int(f1[0]) == 2  # this GPU's arrival reached the other array
    x = torch.ones((4, 32), device="cuda")
    d, s = mpk_lib.quantize(x)
    torch.cuda.synchronize()
    assert int(s[0, 0]) == 119
