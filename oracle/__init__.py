"""CPU oracle for the MXFP8 x BF16 GEMM path.  TEST INFRASTRUCTURE ONLY.

Only the test suite, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this package; it checks results and is never the thing measured or
shipped.  The product library (``mix_precision_kernel_b200``) has no CPU path.

Two shared libraries back it:

* ``_build/libmpk_oracle.so`` -- ``mpk_oracle.c``, a plain-C restatement of the
  reference's host algorithm (each function cites the reference file:line it
  follows), plus ``inputs.cpp``, the libstdc++ ``mt19937`` input generator.
* ``_ref/libmpk_ref.so`` -- the reference's own sources compiled in place by
  ``Makefile`` (present when the reference checkout was available at build
  time).  It pins the restatement and provides the reference's GPU launchers for
  on-device comparisons.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import threading

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libmpk_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libmpk_ref.so")
MX_BLOCK = 32

_lock = threading.Lock()
_lib = None
_ref = None

_f32p = ctypes.POINTER(ctypes.c_float)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_i64 = ctypes.c_int64


def build(ref_dir: str | None = None) -> None:
    """Compile the oracle (and the reference, when its sources are present)."""
    cmd = ["make", "-s", "-C", HERE, "all"]
    if ref_dir:
        cmd.append(f"REF_DIR={ref_dir}")
    subprocess.run(cmd, check=True)


def _ptr(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def lib() -> ctypes.CDLL:
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(ORACLE_SO):
                build()
            L = ctypes.CDLL(ORACLE_SO)
            L.orc_e4m3_to_float.restype = ctypes.c_float
            L.orc_e4m3_to_float.argtypes = [ctypes.c_uint8]
            L.orc_float_to_e4m3.restype = ctypes.c_uint8
            L.orc_float_to_e4m3.argtypes = [ctypes.c_float]
            L.orc_e8m0_to_float.restype = ctypes.c_float
            L.orc_e8m0_to_float.argtypes = [ctypes.c_uint8]
            L.orc_float_to_e8m0.restype = ctypes.c_uint8
            L.orc_float_to_e8m0.argtypes = [ctypes.c_float]
            L.orc_float_to_bf16.restype = ctypes.c_uint16
            L.orc_float_to_bf16.argtypes = [ctypes.c_float]
            L.orc_mxfp8_quantize.argtypes = [_f32p, _u8p, _u8p, _i64, _i64, ctypes.c_int]
            L.orc_mxfp8_dequantize.argtypes = [_u8p, _u8p, _f32p, _i64, _i64, ctypes.c_int]
            L.orc_gemm_gold.argtypes = [_f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, ctypes.c_int]
            L.orc_gemm_gold_rows.argtypes = [_f32p, _f32p, _f32p, _f32p,
                                             ctypes.POINTER(ctypes.c_int64), _i64, _i64, _i64,
                                             ctypes.c_int]
            L.orc_error_stats.argtypes = [_f32p, _f32p, _i64] + [ctypes.POINTER(ctypes.c_double)] * 3
            L.orc_compute_relative_error.restype = ctypes.c_float
            L.orc_compute_relative_error.argtypes = [_f32p, _f32p, _i64]
            L.orc_mx_ulp_hist.argtypes = [_u8p, _u8p, _u8p, _u8p, _i64, _i64,
                                          ctypes.POINTER(ctypes.c_int64)]
            L.orc_sweep_float_to_e4m3.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _u8p]
            L.orc_fill_normal.argtypes = [ctypes.c_uint32, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                          ctypes.POINTER(_f32p), ctypes.POINTER(ctypes.c_int64)]
            L.orc_fill_uniform.argtypes = L.orc_fill_normal.argtypes
            _lib = L
    return _lib


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref() -> ctypes.CDLL:
    """The reference's own code (oracle/_ref/libmpk_ref.so)."""
    global _ref
    with _lock:
        if _ref is None:
            if not os.path.exists(REF_SO):
                raise FileNotFoundError(f"{REF_SO} not built (reference sources absent)")
            R = ctypes.CDLL(REF_SO)
            R.ref_fp8_e4m3_to_float.restype = ctypes.c_float
            R.ref_fp8_e4m3_to_float.argtypes = [ctypes.c_uint8]
            R.ref_float_to_fp8_e4m3.restype = ctypes.c_uint8
            R.ref_float_to_fp8_e4m3.argtypes = [ctypes.c_float]
            R.ref_e8m0_to_float.restype = ctypes.c_float
            R.ref_e8m0_to_float.argtypes = [ctypes.c_uint8]
            R.ref_float_to_e8m0.restype = ctypes.c_uint8
            R.ref_float_to_e8m0.argtypes = [ctypes.c_float]
            R.ref_float_to_bf16.restype = ctypes.c_uint16
            R.ref_float_to_bf16.argtypes = [ctypes.c_float]
            R.ref_sweep_float_to_e4m3.argtypes = [ctypes.c_uint64, ctypes.c_uint64, _u8p]
            R.ref_mxfp8_quantize_host.argtypes = [_f32p, _u8p, _u8p, ctypes.c_int, ctypes.c_int]
            R.ref_mxfp8_dequantize_host.argtypes = [_u8p, _u8p, _f32p, ctypes.c_int, ctypes.c_int]
            R.ref_gemm_reference_host.argtypes = [_f32p, _f32p, _f32p, _f32p,
                                                  ctypes.c_int, ctypes.c_int, ctypes.c_int]
            vp = ctypes.c_void_p
            ci = ctypes.c_int
            for name, args in {
                "ref_mxfp8_quantize_gpu": [vp, vp, vp, ci, ci, vp],
                "ref_mxfp8_dequantize_gpu": [vp, vp, vp, ci, ci, vp],
                "ref_gemm_reference_gpu": [vp, vp, vp, vp, ci, ci, ci, vp],
                "ref_gemm_fp8_tensorcore": [vp, vp, vp, vp, vp, vp, vp, ci, ci, ci, vp],
            }.items():
                f = getattr(R, name)
                f.argtypes = args
                f.restype = ci
            _ref = R
    return _ref


def default_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1)


# ---------------------------------------------------------------------------
# Inputs
# ---------------------------------------------------------------------------

def fill_normal(seed: int, std: float, sizes, mean: float = 0.0):
    """Arrays drawn in order from one mt19937(seed) + normal_distribution<float>."""
    arrs = [np.empty(int(n), dtype=np.float32) for n in sizes]
    ptrs = (_f32p * len(arrs))(*[_ptr(a, _f32p) for a in arrs])
    szs = (ctypes.c_int64 * len(arrs))(*[int(n) for n in sizes])
    lib().orc_fill_normal(seed, mean, std, len(arrs), ptrs, szs)
    return arrs


def fill_uniform(seed: int, lo: float, hi: float, sizes):
    """Arrays drawn in order from one mt19937(seed) + uniform_real_distribution<float>."""
    arrs = [np.empty(int(n), dtype=np.float32) for n in sizes]
    ptrs = (_f32p * len(arrs))(*[_ptr(a, _f32p) for a in arrs])
    szs = (ctypes.c_int64 * len(arrs))(*[int(n) for n in sizes])
    lib().orc_fill_uniform(seed, lo, hi, len(arrs), ptrs, szs)
    return arrs


# ---------------------------------------------------------------------------
# Codec and gold
# ---------------------------------------------------------------------------

def nblk(k: int) -> int:
    return (k + MX_BLOCK - 1) // MX_BLOCK


def quantize(x: np.ndarray, threads: int | None = None):
    """float32 [M, K] -> (codes u8 [M, K], scales u8 [M, ceil(K/32)])."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    M, K = x.shape
    d = np.empty((M, K), np.uint8)
    s = np.empty((M, nblk(K)), np.uint8)
    lib().orc_mxfp8_quantize(_ptr(x, _f32p), _ptr(d, _u8p), _ptr(s, _u8p), M, K,
                             threads or default_threads())
    return d, s


def dequantize(d: np.ndarray, s: np.ndarray, threads: int | None = None) -> np.ndarray:
    d = np.ascontiguousarray(d, dtype=np.uint8)
    s = np.ascontiguousarray(s, dtype=np.uint8)
    M, K = d.shape
    assert s.shape == (M, nblk(K)), (s.shape, M, K)
    out = np.empty((M, K), np.float32)
    lib().orc_mxfp8_dequantize(_ptr(d, _u8p), _ptr(s, _u8p), _ptr(out, _f32p), M, K,
                               threads or default_threads())
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit patterns (uint16), round-to-nearest-even, NaN -> 0x7FFF."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = 0x7FFF
    return r


def bf16_bits_to_float(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def gemm_gold(A: np.ndarray, B: np.ndarray, C: np.ndarray | None, threads: int | None = None):
    """FP32 D = A @ B + C, bit-identical to the reference's host gold."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    M, K = A.shape
    K2, N = B.shape
    assert K == K2
    D = np.empty((M, N), np.float32)
    cp = None
    if C is not None:
        C = np.ascontiguousarray(C, dtype=np.float32)
        cp = _ptr(C, _f32p)
    lib().orc_gemm_gold(_ptr(A, _f32p), _ptr(B, _f32p), cp, _ptr(D, _f32p), M, N, K,
                        threads or default_threads())
    return D


def gemm_gold_rows(A, B, C, rows, threads: int | None = None):
    """Gold for the listed rows only (exact for those rows)."""
    A = np.ascontiguousarray(A, dtype=np.float32)
    B = np.ascontiguousarray(B, dtype=np.float32)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    M, K = A.shape
    N = B.shape[1]
    D = np.empty((len(rows), N), np.float32)
    cp = None
    if C is not None:
        C = np.ascontiguousarray(C, dtype=np.float32)
        cp = _ptr(C, _f32p)
    lib().orc_gemm_gold_rows(_ptr(A, _f32p), _ptr(B, _f32p), cp, _ptr(D, _f32p),
                             rows.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), len(rows), N, K,
                             threads or default_threads())
    return D


def error_stats(res: np.ndarray, ref_: np.ndarray):
    """(max_rel, avg_rel, rmse) with denominator max(|ref|, 1e-6)."""
    res = np.ascontiguousarray(res, dtype=np.float32).ravel()
    ref_ = np.ascontiguousarray(ref_, dtype=np.float32).ravel()
    mx, av, rm = ctypes.c_double(), ctypes.c_double(), ctypes.c_double()
    lib().orc_error_stats(_ptr(res, _f32p), _ptr(ref_, _f32p), res.size,
                          ctypes.byref(mx), ctypes.byref(av), ctypes.byref(rm))
    return mx.value, av.value, rm.value


def compute_relative_error(res, ref_) -> float:
    res = np.ascontiguousarray(res, dtype=np.float32).ravel()
    ref_ = np.ascontiguousarray(ref_, dtype=np.float32).ravel()
    return float(lib().orc_compute_relative_error(_ptr(res, _f32p), _ptr(ref_, _f32p), res.size))


def mx_ulp_hist(d1, s1, d2, s2):
    """[exact, within 1 E4M3 step, more, NaN mismatch] counts between two MXFP8 tensors."""
    d1 = np.ascontiguousarray(d1, np.uint8); s1 = np.ascontiguousarray(s1, np.uint8)
    d2 = np.ascontiguousarray(d2, np.uint8); s2 = np.ascontiguousarray(s2, np.uint8)
    M, N = d1.shape
    h = (ctypes.c_int64 * 4)()
    lib().orc_mx_ulp_hist(_ptr(d1, _u8p), _ptr(s1, _u8p), _ptr(d2, _u8p), _ptr(s2, _u8p), M, N, h)
    return [int(v) for v in h]


def make_gemm_inputs(M: int, N: int, K: int, seed: int, std: float = 0.02, order: str = "ABC",
                     with_c: bool = True):
    """Inputs in the reference's recipe (tests/test_gemm_correctness.cu:23-54).

    Returns a dict with the FP32 draws, the MXFP8 A and C, the BF16 B (uint16 bits)
    and their exact FP32 dequantizations.
    """
    sizes = {"A": M * K, "B": K * N, "C": M * N}
    names = [c for c in order if with_c or c != "C"]
    arrs = dict(zip(names, fill_normal(seed, std, [sizes[c] for c in names])))
    A_f = arrs["A"].reshape(M, K)
    B_f = arrs["B"].reshape(K, N)
    A_d, A_s = quantize(A_f)
    B_h = to_bf16_bits(B_f)
    out = {
        "M": M, "N": N, "K": K,
        "A_data": A_d, "A_scales": A_s, "B_bf16": B_h,
        "A_deq": dequantize(A_d, A_s), "B_f32": bf16_bits_to_float(B_h),
        "C_data": None, "C_scales": None, "C_deq": None,
    }
    if with_c:
        C_d, C_s = quantize(arrs["C"].reshape(M, N))
        out.update(C_data=C_d, C_scales=C_s, C_deq=dequantize(C_d, C_s))
    return out


def gold_mx(inp: dict, rows=None):
    """The reference's gold: FP32 GEMM then the MXFP8 round trip along N.

    Returns (D_fp32, D_data, D_scales, D_deq) for all rows or for ``rows``.
    """
    if rows is None:
        D = gemm_gold(inp["A_deq"], inp["B_f32"], inp["C_deq"])
    else:
        D = gemm_gold_rows(inp["A_deq"], inp["B_f32"], inp["C_deq"], rows)
    d, s = quantize(D)
    return D, d, s, dequantize(d, s)
