"""Generates the golden fixtures in this directory from the reference itself.

    python tests/golden/make_golden.py

Requires oracle/_ref/libmpk_ref.so, i.e. the reference project's own sources
compiled in place by ``make -C oracle ref`` (the reference checkout must be
present).  Inputs come from oracle/inputs.cpp (libstdc++ std::mt19937 with
std::normal_distribution / uniform_real_distribution, as the reference's tests
draw them); every output is produced by the reference's functions:

  codec_golden.npz
    q128x100_*   tests/test_mxfp8_quantize.cu:142-144 round-trip case (uniform(-10,10),
                 mt19937(42), K=100 ragged): reference mxfp8_quantize_host/dequantize_host
    q128x256_*   :45-102 GPU-vs-host case (uniform(-5,5), mt19937(123)): host quantize
    q512x1024_*  same recipe at 512x1024
    special_*    hand-made blocks: zeros, 400.0, +-448/449/464, NaN/inf, FLT_MIN-scale,
                 subnormals, mixed signs and a ragged tail
    lut_*        reference dequantize of all 256 codes x scale bytes
                 {0,1,2,3,114,127,246,247,254,255}
  gemm_golden.npz
    g64x96x128_* a small GEMM in the tests/test_gemm_correctness.cu:23-65 recipe
                 (mt19937(42), N(0, 0.02^2), A then B then C): MXFP8 inputs, the
                 FP32 gold of gemm_reference_host and its MXFP8 round trip
    c0_*         config M=N=K=512 (the same recipe): SHA-256 of every input and
                 output array plus the first entries (known answers)
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

F32 = ctypes.POINTER(ctypes.c_float)
U8 = ctypes.POINTER(ctypes.c_uint8)


def p(a, t):
    return a.ctypes.data_as(t)


def ref_quantize(R, x):
    M, K = x.shape
    d = np.empty((M, K), np.uint8)
    s = np.empty((M, (K + 31) // 32), np.uint8)
    R.ref_mxfp8_quantize_host(p(x, F32), p(d, U8), p(s, U8), M, K)
    return d, s


def ref_dequantize(R, d, s):
    M, K = d.shape
    out = np.empty((M, K), np.float32)
    R.ref_mxfp8_dequantize_host(p(d, U8), p(s, U8), p(out, F32), M, K)
    return out


def ref_gemm(R, A, B, C):
    M, K = A.shape
    N = B.shape[1]
    D = np.empty((M, N), np.float32)
    R.ref_gemm_reference_host(p(A, F32), p(B, F32), p(C, F32) if C is not None else None, p(D, F32),
                              M, N, K)
    return D


def special_rows() -> np.ndarray:
    f = np.float32
    rows = []
    rows.append(np.zeros(32, f))
    rows.append(np.full(32, 400.0, f))
    r = np.linspace(-448, 448, 32).astype(f); rows.append(r)
    r = np.array([448, 449, 464, 465, -449, -464, -465, 480] + [1.0] * 24, f); rows.append(r)
    r = np.array([np.nan, 1.0, -2.0, np.inf] + [0.5] * 28, f); rows.append(r)
    r = np.array([-np.inf, 3.0] + [np.nan] * 30, f); rows.append(r)
    r = np.full(32, np.nan, f); rows.append(r)
    r = np.full(32, 1e-40, f); r[::2] = -1e-41; rows.append(r)                 # subnormals
    r = np.full(32, 1.1754944e-38, f); rows.append(r)                            # FLT_MIN
    r = (np.arange(32, dtype=f) - 16) * f(1e-3); rows.append(r)                 # mixed signs
    r = np.array([2.0 ** e for e in range(-20, 12)], f); rows.append(r)          # wide range
    r = np.array([-0.0] * 16 + [0.0] * 16, f); rows.append(r)                    # signed zeros
    r = np.full(32, 3.0e38, f); rows.append(r)
    r = np.array([1.0 + i / 16.0 for i in range(32)], f) * f(448.0 / 2.9375); rows.append(r)
    return np.stack(rows)


def main() -> None:
    R = oracle.ref()
    out = {}
    # --- codec ---------------------------------------------------------------
    for name, seed, lo, hi, M, K in [("q128x100", 42, -10.0, 10.0, 128, 100),
                                     ("q128x256", 123, -5.0, 5.0, 128, 256),
                                     ("q512x1024", 123, -5.0, 5.0, 512, 1024)]:
        x = oracle.fill_uniform(seed, lo, hi, [M * K])[0].reshape(M, K)
        d, s = ref_quantize(R, x)
        out[f"{name}_data"], out[f"{name}_scales"] = d, s
        if M * K <= 128 * 256:
            out[f"{name}_deq"] = ref_dequantize(R, d, s)
        out[f"{name}_seed"] = np.array([seed, M, K], np.int64)
        out[f"{name}_range"] = np.array([lo, hi], np.float32)
    sp = special_rows()
    d, s = ref_quantize(R, sp)
    out["special_in"], out["special_data"], out["special_scales"] = sp, d, s
    out["special_deq"] = ref_dequantize(R, d, s)
    sp_tail = np.ascontiguousarray(sp[:, :21])                                  # ragged K = 21
    d, s = ref_quantize(R, sp_tail)
    out["special21_in"], out["special21_data"], out["special21_scales"] = sp_tail, d, s
    scales = np.array([0, 1, 2, 3, 114, 127, 246, 247, 254, 255], np.uint8)
    codes = np.tile(np.arange(256, dtype=np.uint8), (len(scales), 1))          # [10][256]
    lut_s = np.repeat(scales[:, None], 256 // 32, axis=1)
    out["lut_scales"] = scales
    out["lut_deq"] = ref_dequantize(R, codes, np.ascontiguousarray(lut_s))
    np.savez_compressed(os.path.join(HERE, "codec_golden.npz"), **out)

    # --- gemm ----------------------------------------------------------------
    g = {}
    M, N, K = 64, 96, 128
    A, B, C = oracle.fill_normal(42, 0.02, [M * K, K * N, M * N])
    A, B, C = A.reshape(M, K), B.reshape(K, N), C.reshape(M, N)
    Ad, As = ref_quantize(R, A)
    Bh = np.array([R.ref_float_to_bf16(float(v)) for v in B.ravel()], np.uint16).reshape(K, N)
    Cd, Cs = ref_quantize(R, C)
    Adq, Cdq = ref_dequantize(R, Ad, As), ref_dequantize(R, Cd, Cs)
    Bf = (Bh.astype(np.uint32) << 16).view(np.float32)
    D = ref_gemm(R, Adq, Bf, Cdq)
    Dd, Ds = ref_quantize(R, D)
    g.update(g64x96x128_A_data=Ad, g64x96x128_A_scales=As, g64x96x128_B_bf16=Bh,
             g64x96x128_C_data=Cd, g64x96x128_C_scales=Cs, g64x96x128_D_fp32=D,
             g64x96x128_D_data=Dd, g64x96x128_D_scales=Ds,
             g64x96x128_D_noC_fp32=ref_gemm(R, Adq, Bf, None))
    M = N = K = 512
    A, B, C = oracle.fill_normal(42, 0.02, [M * K, K * N, M * N])
    A, B, C = A.reshape(M, K), B.reshape(K, N), C.reshape(M, N)
    Ad, As = ref_quantize(R, A)
    Bh = oracle.to_bf16_bits(B)
    Cd, Cs = ref_quantize(R, C)
    D = ref_gemm(R, ref_dequantize(R, Ad, As), (Bh.astype(np.uint32) << 16).view(np.float32),
                 ref_dequantize(R, Cd, Cs))
    Dd, Ds = ref_quantize(R, D)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    g["c0_sha256"] = np.array([sha(a) for a in (Ad, As, Bh, Cd, Cs, D, Dd, Ds)])
    g["c0_first"] = np.array([Ad[0, 0], As[0, 0], Dd[0, 0], Ds[0, 0]], np.int64)
    g["c0_D00"] = np.array([D[0, 0]], np.float32)
    np.savez_compressed(os.path.join(HERE, "gemm_golden.npz"), **g)
    print("wrote", os.listdir(HERE))


if __name__ == "__main__":
    main()
