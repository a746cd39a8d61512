"""Pins the CPU oracle: against the golden fixtures generated from the reference
(tests/golden/make_golden.py) and, where oracle/_ref was built, against the
reference's own compiled code directly.  CPU only."""
import concurrent.futures as cf
import ctypes
import hashlib
import os

import numpy as np
import pytest

import oracle as O

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
needs_ref = pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")


@pytest.fixture(scope="module")
def codec_gold():
    return np.load(os.path.join(GOLD, "codec_golden.npz"))


@pytest.fixture(scope="module")
def gemm_gold():
    return np.load(os.path.join(GOLD, "gemm_golden.npz"))


def same_f32(a, b):
    """Bit equality with every NaN equal to every NaN."""
    a = np.asarray(a, np.float32)
    b = np.asarray(b, np.float32)
    nan = np.isnan(a) & np.isnan(b)
    return bool(np.all(nan | (a.view(np.uint32) == b.view(np.uint32))))


# ------------------------------- golden vectors -------------------------------

@pytest.mark.parametrize("name", ["q128x100", "q128x256", "q512x1024"])
def test_quantize_matches_reference_golden(codec_gold, name):
    seed, M, K = codec_gold[f"{name}_seed"]
    lo, hi = codec_gold[f"{name}_range"]
    x = O.fill_uniform(int(seed), float(lo), float(hi), [int(M * K)])[0].reshape(M, K)
    d, s = O.quantize(x)
    assert np.array_equal(d, codec_gold[f"{name}_data"])
    assert np.array_equal(s, codec_gold[f"{name}_scales"])
    if f"{name}_deq" in codec_gold:
        assert same_f32(O.dequantize(d, s), codec_gold[f"{name}_deq"])


@pytest.mark.parametrize("tag", ["special", "special21"])
def test_quantize_special_values_golden(codec_gold, tag):
    d, s = O.quantize(codec_gold[f"{tag}_in"])
    assert np.array_equal(d, codec_gold[f"{tag}_data"])
    assert np.array_equal(s, codec_gold[f"{tag}_scales"])
    if f"{tag}_deq" in codec_gold:
        assert same_f32(O.dequantize(d, s), codec_gold[f"{tag}_deq"])


def test_dequantize_all_codes_golden(codec_gold):
    scales = codec_gold["lut_scales"]
    codes = np.tile(np.arange(256, dtype=np.uint8), (len(scales), 1))
    s = np.repeat(scales[:, None], 8, axis=1)
    assert same_f32(O.dequantize(codes, s), codec_gold["lut_deq"])


def test_gemm_gold_small_golden(gemm_gold):
    g = {k[len("g64x96x128_"):]: gemm_gold[k] for k in gemm_gold.files if k.startswith("g64x96x128_")}
    inp = O.make_gemm_inputs(64, 96, 128, seed=42)
    for k in ("A_data", "A_scales", "C_data", "C_scales"):
        assert np.array_equal(inp[k], g[k]), k
    assert np.array_equal(inp["B_bf16"], g["B_bf16"])
    D, Dd, Ds, _ = O.gold_mx(inp)
    assert np.array_equal(D.view(np.uint32), g["D_fp32"].view(np.uint32))
    assert np.array_equal(Dd, g["D_data"]) and np.array_equal(Ds, g["D_scales"])
    D0 = O.gemm_gold(inp["A_deq"], inp["B_f32"], None)
    assert np.array_equal(D0.view(np.uint32), g["D_noC_fp32"].view(np.uint32))


def test_config0_known_answers(gemm_gold):
    """M=N=K=512, mt19937(42): every array hashes to the reference's output."""
    inp = O.make_gemm_inputs(512, 512, 512, seed=42)
    D, Dd, Ds, _ = O.gold_mx(inp)
    sha = lambda a: hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
    got = [sha(a) for a in (inp["A_data"], inp["A_scales"], inp["B_bf16"], inp["C_data"],
                            inp["C_scales"], D, Dd, Ds)]
    assert got == list(gemm_gold["c0_sha256"])
    assert [inp["A_data"][0, 0], inp["A_scales"][0, 0], Dd[0, 0], Ds[0, 0]] == [0x75, 114, 0x69, 114]
    assert np.float32(D[0, 0]) == gemm_gold["c0_D00"][0]


# --------------------- the reference's own host tests, replayed ---------------------

@pytest.mark.parametrize("M,K", [(64, 128), (256, 512), (128, 100)])
def test_roundtrip_tolerance(M, K):
    """tests/test_mxfp8_quantize.cu:9-43: host round trip, max rel err < 0.25."""
    x = O.fill_uniform(42, -10.0, 10.0, [M * K])[0].reshape(M, K)
    y = O.dequantize(*O.quantize(x))
    m = np.abs(x) > 1e-4
    assert np.max(np.abs(y[m] - x[m]) / np.abs(x[m])) < 0.25


def test_edge_cases():
    """tests/test_mxfp8_quantize.cu:104-135."""
    z = np.zeros((1, 32), np.float32)
    assert np.all(O.dequantize(*O.quantize(z)) == 0.0)
    v = np.full((1, 32), 400.0, np.float32)
    assert abs(O.dequantize(*O.quantize(v))[0, 0] - 400.0) / 400.0 <= 0.1


# ------------------------ direct comparison with oracle/_ref ------------------------

@needs_ref
def test_exhaustive_float_to_e4m3_against_reference():
    """All 2^32 float bit patterns through the scalar E4M3 encoder (fp8_types.h:14-21)."""
    L, R = O.lib(), O.ref()
    u8 = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint8))
    CH = 1 << 24

    def chunk(i):
        lo, hi = i * CH, (i + 1) * CH
        a = np.empty(CH, np.uint8)
        b = np.empty(CH, np.uint8)
        L.orc_sweep_float_to_e4m3(lo, hi, u8(a))
        R.ref_sweep_float_to_e4m3(lo, hi, u8(b))
        return int(np.count_nonzero(a != b))

    with cf.ThreadPoolExecutor(O.default_threads()) as ex:
        assert sum(ex.map(chunk, range(1 << 8))) == 0


@needs_ref
def test_scalars_against_reference():
    L, R = O.lib(), O.ref()
    for v in range(256):
        a, b = L.orc_e4m3_to_float(v), R.ref_fp8_e4m3_to_float(v)
        assert a == b or (a != a and b != b)
        a, b = L.orc_e8m0_to_float(v), R.ref_e8m0_to_float(v)
        assert a == b
    rng = np.random.default_rng(1)
    bits = rng.integers(0, 1 << 32, 200000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    for x in bits[:50000]:
        assert L.orc_float_to_e8m0(float(x)) == R.ref_float_to_e8m0(float(x))
        assert L.orc_float_to_bf16(float(x)) == R.ref_float_to_bf16(float(x))


@needs_ref
@pytest.mark.parametrize("M,K,dist", [(33, 100, "normal"), (7, 1, "normal"), (64, 4096, "wide"),
                                      (5, 31, "special"), (16, 64, "normal")])
def test_codec_against_reference(M, K, dist):
    R = O.ref()
    rng = np.random.default_rng(M * 1000 + K)
    if dist == "normal":
        x = rng.standard_normal((M, K)).astype(np.float32)
    elif dist == "wide":
        x = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-60, 60, (M, K)))).astype(np.float32)
    else:
        x = rng.choice(np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 448, 449, 1e-40, 3e38, -5.0],
                                np.float32), (M, K))
    d, s = O.quantize(x)
    d2 = np.empty_like(d)
    s2 = np.empty_like(s)
    f32 = ctypes.POINTER(ctypes.c_float)
    u8 = ctypes.POINTER(ctypes.c_uint8)
    R.ref_mxfp8_quantize_host(x.ctypes.data_as(f32), d2.ctypes.data_as(u8), s2.ctypes.data_as(u8), M, K)
    assert np.array_equal(d, d2) and np.array_equal(s, s2)
    y = O.dequantize(d, s)
    y2 = np.empty_like(y)
    R.ref_mxfp8_dequantize_host(d.ctypes.data_as(u8), s.ctypes.data_as(u8), y2.ctypes.data_as(f32), M, K)
    assert same_f32(y, y2)


@needs_ref
@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (96, 200, 160), (512, 512, 512)])
def test_gemm_gold_bit_identical_to_reference(M, N, K):
    R = O.ref()
    inp = O.make_gemm_inputs(M, N, K, seed=7)
    D = O.gemm_gold(inp["A_deq"], inp["B_f32"], inp["C_deq"])
    D2 = np.empty_like(D)
    f32 = lambda a: a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    R.ref_gemm_reference_host(f32(inp["A_deq"]), f32(inp["B_f32"]), f32(inp["C_deq"]), f32(D2), M, N, K)
    assert np.array_equal(D.view(np.uint32), D2.view(np.uint32))


def test_row_sampled_gold_equals_full_gold():
    inp = O.make_gemm_inputs(96, 64, 96, seed=3)
    full = O.gemm_gold(inp["A_deq"], inp["B_f32"], inp["C_deq"])
    rows = np.array([0, 5, 63, 95], np.int64)
    part = O.gemm_gold_rows(inp["A_deq"], inp["B_f32"], inp["C_deq"], rows)
    assert np.array_equal(full[rows].view(np.uint32), part.view(np.uint32))


def test_ulp_histogram_semantics():
    d = np.array([[0x40, 0x41, 0x3F, 0xC1]], np.uint8)
    s = np.array([[127]], np.uint8)
    d2 = np.array([[0x40, 0x40, 0x41, 0xC3]], np.uint8)
    h = O.mx_ulp_hist(d, s, d2, s)
    assert h == [1, 1, 2, 0]  # (0x40,0x40) exact; (0x41,0x40) one step; (0x3F,0x41), (0xC1,0xC3) two
