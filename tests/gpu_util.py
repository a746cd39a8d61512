"""Helpers shared by the GPU parity tests: move oracle inputs to the device,
run the library through its C ABI, and bring results back."""
from __future__ import annotations

import numpy as np


def to_dev(a: np.ndarray, device="cuda"):
    import torch

    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:  # bf16 bit patterns
        return torch.from_numpy(a.view(np.int16)).to(device).view(torch.bfloat16)
    return torch.from_numpy(a).to(device)


def to_host(t) -> np.ndarray:
    import torch

    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def run_gemm(mpk, inp: dict, device="cuda", with_c: bool = True, stream=None, path="default"):
    """D = A*B + C; returns (D_data, D_scales) on the host.  path: "default"
    (mpk_gemm_mxfp8_bf16, pooled workspace), "workspace" (mpk_gemm_mxfp8_bf16_ws
    with a fresh caller workspace) or "onchip" (mpk_gemm_mxfp8_bf16_ws with no
    workspace: A converted inside the GEMM kernel)."""
    import torch

    M, N, K = inp["M"], inp["N"], inp["K"]
    A = to_dev(inp["A_data"], device)
    As = to_dev(inp["A_scales"], device)
    B = to_dev(inp["B_bf16"], device)
    C = Cs = None
    if with_c and inp.get("C_data") is not None:
        C = to_dev(inp["C_data"], device)
        Cs = to_dev(inp["C_scales"], device)
    D = torch.full((M, N), 0xEE, dtype=torch.uint8, device=device)
    Ds = torch.full((M, (N + 31) // 32), 0xEE, dtype=torch.uint8, device=device)
    if path == "workspace":
        ws = torch.full((max(mpk.gemm_workspace_size(M, N, K), 16),), 0xEE, dtype=torch.uint8,
                        device=device)
        mpk.gemm_fp8_tensorcore_ws(A, As, B, C, Cs, D, Ds, M, N, K, ws, stream)
    elif path == "onchip":
        mpk.gemm_fp8_tensorcore_ws(A, As, B, C, Cs, D, Ds, M, N, K, None, stream)
    else:
        assert path == "default"
        mpk.gemm_fp8_tensorcore(A, As, B, C, Cs, D, Ds, M, N, K, stream)
    torch.cuda.synchronize()
    return to_host(D), to_host(Ds)


def run_ref_k7(inp: dict, device="cuda", with_c: bool = True):
    """The reference's own gemm_fp8_tensorcore (WMMA fp16, rebuilt for sm_100a)."""
    import torch

    import oracle

    R = oracle.ref()
    M, N, K = inp["M"], inp["N"], inp["K"]
    A = to_dev(inp["A_data"], device)
    As = to_dev(inp["A_scales"], device)
    B = to_dev(inp["B_bf16"], device)
    C = Cs = None
    if with_c and inp.get("C_data") is not None:
        C = to_dev(inp["C_data"], device)
        Cs = to_dev(inp["C_scales"], device)
    D = torch.zeros((M, N), dtype=torch.uint8, device=device)
    Ds = torch.zeros((M, (N + 31) // 32), dtype=torch.uint8, device=device)
    torch.cuda.synchronize()
    rc = R.ref_gemm_fp8_tensorcore(A.data_ptr(), As.data_ptr(), B.data_ptr(),
                                   C.data_ptr() if C is not None else None,
                                   Cs.data_ptr() if Cs is not None else None,
                                   D.data_ptr(), Ds.data_ptr(), M, N, K, None)
    torch.cuda.synchronize()
    assert rc == 0, rc
    return to_host(D), to_host(Ds)


def same_f32(a, b) -> bool:
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))
