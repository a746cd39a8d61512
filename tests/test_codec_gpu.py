"""MXFP8 quantize / dequantize on the GPU, bit-exact against the oracle and the
reference's golden vectors (reference tests/test_mxfp8_quantize.cu)."""
import os

import numpy as np
import pytest

import oracle as O
from gpu_util import same_f32, to_dev, to_host

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def gpu_quantize(mpk, x):
    import torch

    M, K = x.shape
    xd = to_dev(x)
    d = torch.full((M, K), 0xEE, dtype=torch.uint8, device="cuda")
    s = torch.full((M, (K + 31) // 32), 0xEE, dtype=torch.uint8, device="cuda")
    mpk.mxfp8_quantize_gpu(xd, d, s, M, K)
    torch.cuda.synchronize()
    return to_host(d), to_host(s)


def gpu_dequantize(mpk, d, s):
    import torch

    M, K = d.shape
    out = torch.full((M, K), float("nan"), dtype=torch.float32, device="cuda")
    mpk.mxfp8_dequantize_gpu(to_dev(d), to_dev(s), out, M, K)
    torch.cuda.synchronize()
    return to_host(out)


def inputs(kind, M, K, seed):
    rng = np.random.default_rng(seed)
    if kind == "normal":
        return (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    if kind == "wide":
        return (rng.standard_normal((M, K)) * np.exp(rng.uniform(-80, 80, (M, K)))).astype(np.float32)
    if kind == "bits":  # arbitrary float bit patterns: NaN, inf, subnormals, everything
        return rng.integers(0, 1 << 32, (M, K), dtype=np.uint64).astype(np.uint32).view(np.float32)
    if kind == "special":
        pool = np.array([0.0, -0.0, np.nan, -np.nan, np.inf, -np.inf, 448, -448, 449, 464, 465,
                         1e-40, -1e-45, 1.1754944e-38, 3e38, -5.0, 0.015625, 2.0 ** -9], np.float32)
        return rng.choice(pool, (M, K))
    raise ValueError(kind)


SHAPES = [(1, 32), (3, 33), (128, 100), (7, 1), (64, 4096), (257, 96), (2, 8192), (1000, 64)]


@pytest.mark.parametrize("kind", ["normal", "wide", "bits", "special"])
@pytest.mark.parametrize("M,K", SHAPES)
def test_quantize_bit_exact(mpk_lib, cuda, kind, M, K):
    x = inputs(kind, M, K, seed=M * 7919 + K)
    d, s = gpu_quantize(mpk_lib, x)
    d0, s0 = O.quantize(x)
    assert np.array_equal(s, s0)
    assert np.array_equal(d, d0)


@pytest.mark.parametrize("kind", ["normal", "wide", "bits"])
@pytest.mark.parametrize("M,K", SHAPES)
def test_dequantize_bit_exact(mpk_lib, cuda, kind, M, K):
    rng = np.random.default_rng(M + K)
    if kind == "bits":
        d = rng.integers(0, 256, (M, K), dtype=np.uint8)
        s = rng.integers(0, 256, (M, (K + 31) // 32), dtype=np.uint8)
    else:
        d, s = O.quantize(inputs(kind, M, K, seed=M * 31 + K))
    assert same_f32(gpu_dequantize(mpk_lib, d, s), O.dequantize(d, s))


def test_dequantize_all_codes_all_scales(mpk_lib, cuda):
    """Every E4M3 code under every E8M0 byte (0 -> 0.0 and 255 -> inf included)."""
    codes = np.tile(np.arange(256, dtype=np.uint8), (256, 1))
    s = np.repeat(np.arange(256, dtype=np.uint8)[:, None], 8, axis=1)
    assert same_f32(gpu_dequantize(mpk_lib, codes, s), O.dequantize(codes, s))
    g = np.load(os.path.join(GOLD, "codec_golden.npz"))
    sc = g["lut_scales"]
    codes = np.tile(np.arange(256, dtype=np.uint8), (len(sc), 1))
    out = gpu_dequantize(mpk_lib, codes, np.ascontiguousarray(np.repeat(sc[:, None], 8, axis=1)))
    assert same_f32(out, g["lut_deq"])


@pytest.mark.parametrize("name", ["q128x100", "q128x256", "q512x1024"])
def test_reference_quantize_cases(mpk_lib, cuda, name):
    """tests/test_mxfp8_quantize.cu:45-102 and :142-146, held to bit-exactness
    (the reference allows codes to differ by one)."""
    g = np.load(os.path.join(GOLD, "codec_golden.npz"))
    seed, M, K = g[f"{name}_seed"]
    lo, hi = g[f"{name}_range"]
    x = O.fill_uniform(int(seed), float(lo), float(hi), [int(M * K)])[0].reshape(M, K)
    d, s = gpu_quantize(mpk_lib, x)
    assert np.array_equal(d, g[f"{name}_data"]) and np.array_equal(s, g[f"{name}_scales"])
    if f"{name}_deq" in g:
        assert same_f32(gpu_dequantize(mpk_lib, d, s), g[f"{name}_deq"])


@pytest.mark.parametrize("tag", ["special", "special21"])
def test_special_value_golden(mpk_lib, cuda, tag):
    g = np.load(os.path.join(GOLD, "codec_golden.npz"))
    d, s = gpu_quantize(mpk_lib, np.ascontiguousarray(g[f"{tag}_in"]))
    assert np.array_equal(d, g[f"{tag}_data"]) and np.array_equal(s, g[f"{tag}_scales"])


def test_unaligned_pointers_take_general_path(mpk_lib, cuda):
    """Offsets that break 16-byte alignment must still be exact."""
    import torch

    M, K = 9, 64
    x = inputs("normal", M, K, 5)
    big = torch.zeros(M * K + 1, dtype=torch.float32, device="cuda")
    big[1:] = to_dev(x.ravel())
    xv = big[1:].view(M, K)
    d = torch.zeros(M * K + 3, dtype=torch.uint8, device="cuda")[3:].view(M, K)
    s = torch.zeros((M, 2), dtype=torch.uint8, device="cuda")
    mpk_lib.mxfp8_quantize_gpu(xv, d, s, M, K)
    torch.cuda.synchronize()
    d0, s0 = O.quantize(x)
    assert np.array_equal(to_host(d), d0) and np.array_equal(to_host(s), s0)
    out = torch.zeros(M * K + 1, dtype=torch.float32, device="cuda")[1:].view(M, K)
    mpk_lib.mxfp8_dequantize_gpu(d, s, out, M, K)
    torch.cuda.synchronize()
    assert same_f32(to_host(out), O.dequantize(d0, s0))


@pytest.mark.skipif(not O.ref_available(), reason="oracle/_ref not built")
def test_matches_reference_gpu_kernels(mpk_lib, cuda):
    """Same inputs through the reference's own K1/K2 kernels rebuilt for sm_100a."""
    import torch

    R = O.ref()
    M, K = 512, 1024
    x = inputs("normal", M, K, 11)
    xd = to_dev(x)
    d = torch.zeros((M, K), dtype=torch.uint8, device="cuda")
    s = torch.zeros((M, K // 32), dtype=torch.uint8, device="cuda")
    assert R.ref_mxfp8_quantize_gpu(xd.data_ptr(), d.data_ptr(), s.data_ptr(), M, K, None) == 0
    out = torch.zeros((M, K), dtype=torch.float32, device="cuda")
    assert R.ref_mxfp8_dequantize_gpu(d.data_ptr(), s.data_ptr(), out.data_ptr(), M, K, None) == 0
    torch.cuda.synchronize()
    d1, s1 = gpu_quantize(mpk_lib, x)
    assert np.array_equal(d1, to_host(d)) and np.array_equal(s1, to_host(s))
    assert same_f32(gpu_dequantize(mpk_lib, d1, s1), to_host(out))


def test_full_size_against_oracle_and_value_idempotence(mpk_lib, cuda):
    """131072 x 2048 (the codec benchmark shape): the whole tensor matches the
    oracle bit for bit, and dequantize(quantize(dequantize(q))) == dequantize(q).
    (Code-level idempotence does not hold for this format: a block whose largest
    value rounds to exactly 224 * scale re-quantizes with half the scale and twice
    the codes -- same values.)"""
    import torch

    M, K = 131072, 2048
    g = torch.Generator(device="cuda").manual_seed(45)
    x = torch.randn((M, K), generator=g, device="cuda", dtype=torch.float32) * 0.02
    d, s = mpk_lib.quantize(x)
    y = mpk_lib.dequantize(d, s)
    y2 = mpk_lib.dequantize(*mpk_lib.quantize(y))
    assert torch.equal(y.view(torch.int32), y2.view(torch.int32))
    xh = to_host(x)
    del x, y2
    d0, s0 = O.quantize(xh)
    assert np.array_equal(to_host(d), d0) and np.array_equal(to_host(s), s0)
    assert same_f32(to_host(y), O.dequantize(d0, s0))
    del y, d, s
    torch.cuda.empty_cache()


# ------------------------------ MXFP8 -> BF16 ------------------------------

def _bf16_expected(d, s):
    """Oracle dequantization rounded to BF16 (RNE); NaN positions returned apart."""
    f = O.dequantize(d, s)
    return O.to_bf16_bits(f), np.isnan(f)


def _gpu_dequantize_bf16(mpk, d, s, offset=0):
    import torch

    M, K = d.shape
    out = torch.full((M * K + offset,), 0x5555, dtype=torch.int16, device="cuda")
    view = out[offset:]
    mpk.mxfp8_dequantize_bf16_gpu(to_dev(d), to_dev(s), view.data_ptr(), M, K)
    torch.cuda.synchronize()
    return to_host(view).view(np.uint16).reshape(M, K)


@pytest.mark.parametrize("M,K,offset", [(256, 256, 0), (37, 96, 0), (64, 100, 0), (33, 64, 3)])
def test_dequantize_bf16_all_codes_all_scales(mpk_lib, cuda, M, K, offset):
    """Every code under every scale byte: BF16 bits equal the oracle's value
    rounded to nearest even (exact for scale >= 3), NaN exactly where the oracle
    has NaN.  K % 32 != 0 or an unaligned output takes the element-wise kernel."""
    rng = np.random.default_rng(M * K + offset)
    d = (np.arange(M * K) % 256).astype(np.uint8).reshape(M, K)
    rng.shuffle(d, axis=1)
    s = rng.integers(0, 256, (M, (K + 31) // 32), dtype=np.uint8)
    s.ravel()[:256] = np.arange(256, dtype=np.uint8)[: s.size]
    got = _gpu_dequantize_bf16(mpk_lib, d, s, offset)
    want, nan = _bf16_expected(d, s)
    got_nan = ((got & 0x7F80) == 0x7F80) & ((got & 0x7F) != 0)
    assert np.array_equal(nan, got_nan)
    assert np.array_equal(got[~nan], want[~nan])


# ------------------------------ BF16 -> MXFP8 ------------------------------

def _gpu_quantize_bf16(mpk, bits, offset=0):
    import torch

    M, K = bits.shape
    src = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).reshape(-1)).to("cuda")
    buf = torch.empty(src.numel() + offset, dtype=torch.int16, device="cuda")
    buf[offset:].copy_(src)
    d = torch.full((M, K), 0xEE, dtype=torch.uint8, device="cuda")
    s = torch.full((M, (K + 31) // 32), 0xEE, dtype=torch.uint8, device="cuda")
    mpk.mxfp8_quantize_bf16_gpu(buf.data_ptr() + 2 * offset, d, s, M, K)
    torch.cuda.synchronize()
    return to_host(d), to_host(s)


@pytest.mark.parametrize("kind", ["normal", "bits"])
@pytest.mark.parametrize("M,K,offset", [(256, 2048, 0), (64, 100, 0), (33, 256, 3), (7, 32, 0)])
def test_quantize_bf16_bit_exact(mpk_lib, cuda, kind, M, K, offset):
    """Equal to the FP32 quantizer of the oracle on the exactly widened values, for
    N(0, 0.02^2) data and for arbitrary BF16 bit patterns (NaN, inf, subnormals),
    on the flat path and on the general path (ragged K, unaligned input)."""
    rng = np.random.default_rng(M * K + offset)
    if kind == "normal":
        bits = O.to_bf16_bits((rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    else:
        bits = rng.integers(0, 1 << 16, (M, K), dtype=np.uint32).astype(np.uint16)
        bits[0, :32] = 0x7FC0  # an all-NaN block
    d, s = _gpu_quantize_bf16(mpk_lib, bits, offset)
    wd, ws = O.quantize(O.bf16_bits_to_float(bits))
    assert np.array_equal(d, wd) and np.array_equal(s, ws)


# ------------------------- quantize along the rows -------------------------

def _cols_expected(xf):
    """The row quantizer of the oracle on the transposed tensor, transposed back:
    codes [M][K], scales [ceil(M/32)][K]."""
    dT, sT = O.quantize(np.ascontiguousarray(xf.T))
    return np.ascontiguousarray(dT.T), np.ascontiguousarray(sT.T)


def _gpu_quantize_cols(mpk, x, offset=0):
    """x: float32 array or bf16 bit patterns (uint16); offset in elements from an
    aligned allocation, to exercise the general path."""
    import torch

    M, K = x.shape
    flat = to_dev(np.ascontiguousarray(x).reshape(-1))
    big = torch.empty(flat.numel() + offset, dtype=flat.dtype, device="cuda")
    big[offset:].copy_(flat)
    d = torch.full((M, K), 0xEE, dtype=torch.uint8, device="cuda")
    s = torch.full(((M + 31) // 32, K), 0xEE, dtype=torch.uint8, device="cuda")
    fn = mpk.mxfp8_quantize_cols_gpu if x.dtype == np.float32 else mpk.mxfp8_quantize_bf16_cols_gpu
    fn(big.data_ptr() + offset * big.element_size(), d, s, M, K)
    torch.cuda.synchronize()
    return to_host(d), to_host(s)


@pytest.mark.parametrize("kind", ["normal", "wide", "bits", "special"])
@pytest.mark.parametrize("M,K,offset", [(256, 1024, 0), (100, 37, 0), (33, 4096, 0), (1, 5, 0), (131, 260, 1),
                                        (64, 96, 3), (4096, 512, 0)])
def test_quantize_cols_bit_exact(mpk_lib, cuda, kind, M, K, offset):
    """Blocks of 32 rows per column: ragged M (a partial last block), K not a
    multiple of 4 or an unaligned input (the one-column-per-thread path), NaN,
    infinities and the saturation range."""
    rng = np.random.default_rng(M * 7 + K)
    if kind == "normal":
        x = (rng.standard_normal((M, K)) * 0.02).astype(np.float32)
    elif kind == "wide":
        x = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-60, 60, (M, K)))).astype(np.float32)
    elif kind == "bits":
        x = rng.integers(0, 1 << 32, (M, K), dtype=np.uint64).astype(np.uint32).view(np.float32)
    else:
        pool = np.array([0.0, -0.0, np.nan, np.inf, -np.inf, 448, 449, 464, 1e-40, 3e38, -5.0], np.float32)
        x = rng.choice(pool, (M, K))
    d, s = _gpu_quantize_cols(mpk_lib, x, offset)
    wd, ws = _cols_expected(x)
    assert np.array_equal(d, wd) and np.array_equal(s, ws)


@pytest.mark.parametrize("M,K,offset", [(256, 2048, 0), (100, 37, 0), (65, 260, 1)])
def test_quantize_bf16_cols_bit_exact(mpk_lib, cuda, M, K, offset):
    """BF16 source: the column quantizer of each value widened exactly to FP32."""
    rng = np.random.default_rng(M + K)
    normal = O.to_bf16_bits((rng.standard_normal((M, K)) * 0.02).astype(np.float32))
    any_bits = rng.integers(0, 1 << 16, (M, K), dtype=np.uint32).astype(np.uint16)
    bits = np.where(rng.random((M, K)) < 0.5, normal, any_bits).astype(np.uint16)
    d, s = _gpu_quantize_cols(mpk_lib, bits, offset)
    wd, ws = _cols_expected(O.bf16_bits_to_float(bits))
    assert np.array_equal(d, wd) and np.array_equal(s, ws)


def test_quantize_cols_large_matches_row_quantizer_of_transpose(mpk_lib, cuda):
    """16384 x 2048 N(0, 0.02^2): the column quantizer equals the library's own row
    quantizer applied to the transposed tensor on the device, bit for bit."""
    import torch

    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.randn((16384, 2048), generator=g, device="cuda") * 0.02
    d, s = mpk_lib.quantize_cols(x)
    dT, sT = mpk_lib.quantize(x.t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(d, dT.t()) and torch.equal(s, sT.t())
    d16, s16 = mpk_lib.quantize_cols(x.to(torch.bfloat16))
    dT16, sT16 = mpk_lib.quantize(x.to(torch.bfloat16).float().t().contiguous())
    torch.cuda.synchronize()
    assert torch.equal(d16, dT16.t()) and torch.equal(s16, sT16.t())
