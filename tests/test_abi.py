"""The C ABI without a GPU: every entry point declared in include/mpk.h is
exported by libmpk.so, the host-side codec utilities match the oracle bit for
bit, argument validation answers before any device work, and the drop-in C++
headers compile against the library."""
import ctypes
import os
import re
import shutil
import subprocess

import numpy as np
import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mpk.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(mpk_\w+)\s*\(", text, re.M)))


def test_header_declares_the_reference_replacements():
    names = declared_symbols()
    for n in ("mpk_gemm_mxfp8_bf16", "mpk_mxfp8_quantize", "mpk_mxfp8_dequantize",
              "mpk_mxfp8_quantize_host", "mpk_mxfp8_dequantize_host", "mpk_status_string",
              "mpk_last_error", "mpk_last_error_string", "mpk_device_status", "mpk_mxfp8_quantize_cols",
              "mpk_mxfp8_quantize_bf16_cols", "mpk_set_gemm_schedule", "mpk_gemm_plan", "mpk_gemm_path"):
        assert n in names, names


def test_library_exports_every_declared_symbol(mpk_lib):
    lib = ctypes.CDLL(mpk_lib.library_path())
    missing = [n for n in declared_symbols() if not hasattr(lib, n)]
    assert not missing, missing


def test_status_strings(mpk_lib):
    L = mpk_lib.lib()
    for code in (0, 1001, 1002, 1003, 1004, 1005, 1006):
        assert L.mpk_status_string(code)
    assert L.mpk_version() >= 100


def _host_quantize(mpk, x):
    M, K = x.shape
    d = np.empty((M, K), np.uint8)
    s = np.empty((M, (K + 31) // 32), np.uint8)
    mpk.mxfp8_quantize_host(np.ascontiguousarray(x), d, s, M, K)
    return d, s


@pytest.mark.parametrize("kind", ["normal", "wide", "bits", "special"])
@pytest.mark.parametrize("M,K", [(33, 100), (8, 4096), (5, 1), (64, 64)])
def test_host_quantize_matches_oracle(mpk_lib, kind, M, K):
    rng = np.random.default_rng(M * 31 + K)
    if kind == "normal":
        x = rng.standard_normal((M, K)).astype(np.float32)
    elif kind == "wide":
        x = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-80, 80, (M, K)))).astype(np.float32)
    elif kind == "bits":
        x = rng.integers(0, 1 << 32, (M, K), dtype=np.uint64).astype(np.uint32).view(np.float32)
    else:
        pool = np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 448, 449, 464, 1e-40, 3e38, -5.0],
                        np.float32)
        x = rng.choice(pool, (M, K))
    d, s = _host_quantize(mpk_lib, x)
    d0, s0 = O.quantize(x)
    assert np.array_equal(d, d0) and np.array_equal(s, s0)
    y = np.empty((M, K), np.float32)
    mpk_lib.mxfp8_dequantize_host(d, s, y, M, K)
    y0 = O.dequantize(d0, s0)
    assert np.all((np.isnan(y) & np.isnan(y0)) | (y.view(np.uint32) == y0.view(np.uint32)))


def test_host_quantize_sweeps_the_e4m3_range(mpk_lib):
    """Float bit patterns with |x| <= 448 in steps of 997 patterns, each block led
    by a 448 so that its scale is exactly 1 and the codes are the scalar E4M3
    encoding of the values themselves."""
    u = np.arange(0, 0x43E00001, 997, dtype=np.uint64).astype(np.uint32)
    vals = np.concatenate([u, u | 0x80000000]).view(np.float32)
    n = (len(vals) + 30) // 31 * 31
    vals = np.pad(vals, (0, n - len(vals)))
    blocks = vals.reshape(-1, 31)
    x = np.ascontiguousarray(np.concatenate([np.full((len(blocks), 1), 448.0, np.float32), blocks], axis=1))
    d, s = _host_quantize(mpk_lib, x)
    assert np.all(s == 127)
    d0, s0 = O.quantize(x)
    assert np.array_equal(d, d0) and np.array_equal(s, s0)


def test_argument_validation_without_a_device(mpk_lib):
    from mix_precision_kernel_b200 import (MPK_ERR_ARCH, MPK_ERR_INVALID_VALUE, MPK_SUCCESS)

    L = mpk_lib.lib()
    assert L.mpk_gemm_mxfp8_bf16(None, None, None, None, None, None, None, -1, 8, 16, None) == \
        MPK_ERR_INVALID_VALUE
    assert L.mpk_gemm_mxfp8_bf16(None, None, None, None, None, None, None, 0, 8, 16, None) == MPK_SUCCESS
    assert L.mpk_gemm_mxfp8_bf16(None, None, None, None, None, None, None, 8, 8, 16, None) == \
        MPK_ERR_INVALID_VALUE
    assert L.mpk_mxfp8_quantize(None, None, None, 4, -2, None) == MPK_ERR_INVALID_VALUE
    assert L.mpk_mxfp8_dequantize(None, None, None, 4, 0, None) == MPK_SUCCESS
    assert L.mpk_set_wait_timeout_ns(0) == MPK_ERR_INVALID_VALUE
    assert L.mpk_mxfp8_quantize_cols(None, None, None, -1, 4, None) == MPK_ERR_INVALID_VALUE
    assert L.mpk_mxfp8_quantize_cols(None, None, None, 0, 4, None) == MPK_SUCCESS
    assert L.mpk_mxfp8_quantize_bf16_cols(None, None, None, 4, 4, None) == MPK_ERR_INVALID_VALUE
    assert L.mpk_mxfp8_quantize_bf16_cols(3, 1 << 20, 1 << 20, 4, 4, None) == mpk_lib.MPK_ERR_MISALIGNED
    assert L.mpk_last_error_string() == L.mpk_last_error() and b"aligned" in L.mpk_last_error_string()
    import torch
    if not torch.cuda.is_available():
        # well-formed arguments, but no sm_100 device: refused before any launch
        fake = 1 << 20
        rc = L.mpk_gemm_mxfp8_bf16(fake, fake, fake, None, None, fake, fake, 256, 256, 256, None)
        assert rc == MPK_ERR_ARCH


@pytest.mark.skipif(shutil.which("nvcc") is None and not os.path.exists("/usr/local/cuda/bin/nvcc"),
                    reason="nvcc not available")
def test_dropin_headers_compile(mpk_lib, tmp_path):
    """A program written against the reference's header names builds against
    include/ and links to libmpk.so (run on a GPU by test_dropin_gpu)."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    lib_dir = os.path.dirname(mpk_lib.library_path())
    out = tmp_path / "test_dropin"
    cmd = [nvcc, "-std=c++17", "-O2", "-gencode", "arch=compute_100a,code=sm_100a",
           f"-I{os.path.join(ROOT, 'include')}", os.path.join(ROOT, "tests", "cpp", "test_dropin.cu"),
           f"-L{lib_dir}", "-lmpk", "-Xlinker", "-rpath", "-Xlinker", lib_dir, "-o", str(out)]
    subprocess.run(cmd, check=True, capture_output=True)
    assert out.exists()


def test_raw_workspace_address_needs_a_size(mpk_lib):
    """A workspace passed as a raw device address must come with its size, so the
    library can check it (no GPU call is made: the check is in the binding)."""
    import pytest

    with pytest.raises(ValueError):
        mpk_lib.gemm_fp8_tensorcore_ws(0, 0, 0, None, None, 0, 0, 16, 16, 16, 4096)


def test_collective_entry_points_validate_without_a_device(mpk_lib):
    """The fused all-gather, the cross-GPU barrier and the IPC helpers refuse bad
    arguments before touching a device."""
    import ctypes

    from mix_precision_kernel_b200 import MPK_ERR_INVALID_VALUE

    L = mpk_lib.lib()
    one = (ctypes.c_void_p * 1)(1 << 20)
    nine = (ctypes.c_void_p * 9)(*([1 << 20] * 9))
    g = L.mpk_gemm_mxfp8_bf16_gather
    # no destinations / too many destinations
    assert g(None, None, None, None, None, 8, 8, 16, 0, 0, 8, 8, one, one, 0, None, 0, None) == \
        MPK_ERR_INVALID_VALUE
    assert g(None, None, None, None, None, 8, 8, 16, 0, 0, 8, 8, nine, nine, 9, None, 0, None) == \
        MPK_ERR_INVALID_VALUE
    # slab rows past the full D; a column slab past it, or not starting on an MX block
    assert g(None, None, None, None, None, 8, 8, 16, 4, 0, 8, 8, one, one, 1, None, 0, None) == \
        MPK_ERR_INVALID_VALUE
    assert g(None, None, None, None, None, 8, 32, 16, 0, 32, 8, 48, one, one, 1, None, 0, None) == \
        MPK_ERR_INVALID_VALUE
    assert g(None, None, None, None, None, 8, 32, 16, 0, 16, 8, 64, one, one, 1, None, 0, None) == \
        MPK_ERR_INVALID_VALUE
    # barrier: epoch 0, rank outside the world, world above 8
    flags = (ctypes.c_void_p * 2)(1 << 20, 1 << 21)
    assert L.mpk_peer_barrier(flags, 0, 2, 0, None) == MPK_ERR_INVALID_VALUE
    assert L.mpk_peer_barrier(flags, 2, 2, 1, None) == MPK_ERR_INVALID_VALUE
    assert L.mpk_peer_barrier(nine, 0, 9, 1, None) == MPK_ERR_INVALID_VALUE
    # IPC: offset outside the allocation, closing a pointer that was never imported
    handle = ctypes.create_string_buffer(64)
    out = ctypes.c_void_p(0)
    assert L.mpk_ipc_import(handle, 4096, 4096, ctypes.byref(out)) == MPK_ERR_INVALID_VALUE
    assert L.mpk_ipc_close(1 << 20) == MPK_ERR_INVALID_VALUE


def test_default_path_routing(mpk_lib):
    """mpk_gemm_mxfp8_bf16 sends tall products with few columns (N <= 2048 and a BF16
    copy of A of at least 256 MiB) to the on-chip conversion kernel when the plan has
    whole tiles only and the operands meet that kernel's TMA limits; everything else
    takes the pre-pass path.  Host logic only (aligned fake addresses)."""
    on, pre = mpk_lib.PATH_ONCHIP, mpk_lib.PATH_PREPASS
    a, b = 1 << 20, 1 << 21  # 16-byte aligned addresses
    path = lambda M, N, K, A=a, B=b: mpk_lib.gemm_path(A, B, M, N, K)
    assert path(131072, 2048, 2048) == on      # the tall-skinny projection
    assert path(262144, 512, 1024) == on
    assert path(65536, 2048, 4096) == on
    assert path(32768, 2048, 2048) == pre      # BF16 A of 128 MiB: fits L2 about once
    assert path(131072, 4096, 2048) == pre     # more columns to amortise the pre-pass
    assert path(4096, 12288, 4096) == pre
    assert path(131072, 2048, 2056) == pre     # K % 16 != 0: TMA row stride
    assert path(131072, 2044, 2048) == pre     # N % 8 != 0
    assert path(131072, 2048, 2048, A=a + 8) == pre  # misaligned A codes
    assert path(131072, 2048, 2048, B=b + 2) == pre  # misaligned B
    assert path(0, 2048, 2048) == pre and path(131072, 2048, 0) == pre
    prev = mpk_lib.set_gemm_schedule(mpk_lib.SCHEDULE_TILES)
    try:
        assert path(131072, 2048, 2048) == pre  # a forced schedule keeps the pre-pass kernel
    finally:
        mpk_lib.set_gemm_schedule(prev)
    with pytest.raises(mpk_lib.MpkError):
        mpk_lib.gemm_path(a, b, -1, 8, 16)
