// MXFP8 quantize / dequantize as HBM-bandwidth kernels (sm_100a).
//
// Format (reference include/mxfp8_utils.h:24-47, src/quantize/*.cu):
//   data   u8 [M][K] row-major, E4M3 codes
//   scales u8 [M][ceil(K/32)] row-major, E8M0 bytes, one per 32 elements along K
//
// Both directions are bit-exact against the reference's host functions.
//
// Fast path (K % 32 == 0, aligned pointers): the tensor is a flat run of 32-element
// blocks whose scale index equals the flat block index.  Each warp instruction
// touches one contiguous span (512 B of FP32, 128 B of codes), lanes issue several
// loads before any arithmetic, and the grid covers every SM with 2048 threads.
// General path (ragged K, e.g. K = 100, or unaligned pointers): one warp per
// (row, block), one element per lane.
#include <cuda_runtime.h>
#include <cstdint>
#include <cuda_bf16.h>

#include "mpk_ptx.cuh"
#include "mpk_internal.h"

namespace mpk {

constexpr int kCodecThreads = 256;

// ------------------------------- quantize ----------------------------------

// Flat quantize: lane l of a warp holds float4 number base + 32j + l for j < kQuantU,
// so every load instruction reads 512 contiguous bytes and every code store writes
// 128; an MX block (8 float4) sits in 8 consecutive lanes, whose amax is three
// xor-shuffles.  kQuantU loads are issued before any arithmetic (64 B in flight per
// thread).
constexpr int kQuantU = 4;

__global__ void __launch_bounds__(kCodecThreads)
mxfp8_quantize_flat_kernel(const float* __restrict__ in, uint8_t* __restrict__ data,
                           uint8_t* __restrict__ scales, int64_t n_f4)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const float4* i4 = reinterpret_cast<const float4*>(in);
    uint32_t* d32 = reinterpret_cast<uint32_t*>(data);
    // base is warp-uniform, so the full-mask shuffles are legal; lanes past the end
    // compute on zeros and store nothing.
    for (int64_t base = warp * 32 * kQuantU; base < n_f4; base += nwarps * 32 * kQuantU) {
        float4 v[kQuantU];
#pragma unroll
        for (int j = 0; j < kQuantU; ++j) {
            const int64_t f = base + 32 * j + lane;
            v[j] = f < n_f4 ? __ldcs(i4 + f) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
#pragma unroll
        for (int j = 0; j < kQuantU; ++j) {
            const int64_t f = base + 32 * j + lane;
            // The reference folds its max from 0 (src/quantize/mxfp8_quantize.cu:125-128), so
            // NaN elements are ignored and an all-NaN block has amax 0: the final
            // fmaxf with 0 turns the tree's NaN (every operand NaN) into that 0.
            float amax = fmaxf(fmaxf(fabsf(v[j].x), fabsf(v[j].y)), fmaxf(fabsf(v[j].z), fabsf(v[j].w)));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 4));
            amax = fmaxf(amax, 0.0f);
            float inv;
            const uint32_t s = mx_block_scale(amax, inv);
            if (f < n_f4) {
                const uint32_t c0 = f32x2_to_e4m3x2(v[j].x * inv, v[j].y * inv);
                const uint32_t c1 = f32x2_to_e4m3x2(v[j].z * inv, v[j].w * inv);
                __stcs(d32 + f, c0 | (c1 << 16));
                if ((lane & 7) == 0) scales[f >> 3] = (uint8_t)s;
            }
        }
    }
}

// BF16 source of the quantizer: each element widened exactly to FP32.
__device__ __forceinline__ float load_elem(const float* p) { return *p; }
__device__ __forceinline__ float load_elem(const uint16_t* p) { return __uint_as_float((uint32_t)*p << 16); }

// BF16 [M][K] -> MXFP8 along K, flat path: lane l of a warp holds octet (8 BF16)
// base + 32j + l for j < kQuantBf16U, so every load instruction reads 512
// contiguous bytes; an MX block (4 octets) sits in 4 consecutive lanes.  Same
// arithmetic as the FP32 quantizer on the widened values.
constexpr int kQuantBf16U = 4;

__global__ void __launch_bounds__(kCodecThreads)
mxfp8_quantize_bf16_flat_kernel(const uint16_t* __restrict__ in, uint8_t* __restrict__ data,
                                uint8_t* __restrict__ scales, int64_t n_octets)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const uint4* i8 = reinterpret_cast<const uint4*>(in);
    for (int64_t base = warp * 32 * kQuantBf16U; base < n_octets; base += nwarps * 32 * kQuantBf16U) {
        uint4 v[kQuantBf16U];
#pragma unroll
        for (int j = 0; j < kQuantBf16U; ++j) {
            const int64_t o = base + 32 * j + lane;
            v[j] = o < n_octets ? __ldcs(i8 + o) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int j = 0; j < kQuantBf16U; ++j) {
            const int64_t o = base + 32 * j + lane;
            const uint32_t w[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
            float f[8];
            float amax = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                f[2 * i] = __uint_as_float(w[i] << 16);
                f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
                amax = fmaxf(amax, fmaxf(fabsf(f[2 * i]), fabsf(f[2 * i + 1])));
            }
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 1));
            amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, 2));
            amax = fmaxf(amax, 0.0f);  // all-NaN block: amax 0, as the reference's max folded from 0
            float inv;
            const uint32_t s = mx_block_scale(amax, inv);
            if (o < n_octets) {
                __stcs(reinterpret_cast<uint2*>(data) + o, quantize8(f, inv));
                if ((lane & 3) == 0) scales[o >> 2] = (uint8_t)s;
            }
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(kCodecThreads)
mxfp8_quantize_rowblock_kernel(const T* __restrict__ in, uint8_t* __restrict__ data,
                               uint8_t* __restrict__ scales, int64_t M, int64_t K, int64_t nblk)
{
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < M * nblk; w += warps) {
        const int64_t row = w / nblk, blk = w % nblk;
        const int64_t k = blk * 32 + lane;
        const bool valid = k < K;
        const float x = valid ? load_elem(in + row * K + k) : 0.0f;
        float amax = fmaxf(0.0f, fabsf(x));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        float inv;
        const uint32_t s = mx_block_scale(amax, inv);
        if (valid) data[row * K + k] = (uint8_t)(f32x2_to_e4m3x2(x * inv, 0.0f) & 0xFFu);
        if (lane == 0) scales[row * nblk + blk] = (uint8_t)s;
    }
}

// D = MXFP8(C) (or MXFP8(0) without C): the K == 0 case of the GEMM, where the
// product term is empty.  One warp per (row, block).
__global__ void __launch_bounds__(kCodecThreads)
mxfp8_requantize_kernel(const uint8_t* __restrict__ c_data, const uint8_t* __restrict__ c_scales,
                        uint8_t* __restrict__ d_data, uint8_t* __restrict__ d_scales, int64_t M,
                        int64_t N, int64_t nblk)
{
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t w = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < M * nblk; w += warps) {
        const int64_t row = w / nblk, blk = w % nblk;
        const int64_t k = blk * 32 + lane;
        const bool valid = k < N;
        float x = 0.0f;
        if (valid && c_data)
            x = e4m3x2_to_f32x2(c_data[row * N + k]).x * e8m0_to_f32(c_scales[row * nblk + blk]);
        float amax = fmaxf(0.0f, fabsf(x));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xFFFFFFFFu, amax, o));
        float inv;
        const uint32_t s = mx_block_scale(amax, inv);
        if (valid) d_data[row * N + k] = (uint8_t)(f32x2_to_e4m3x2(x * inv, 0.0f) & 0xFFu);
        if (lane == 0) d_scales[row * nblk + blk] = (uint8_t)s;
    }
}

// ------------------------------ dequantize ---------------------------------

// Flat dequantize: lane l of a warp converts code quad base + 32j + l for j <
// kDequantU, so every code load reads 128 contiguous bytes and every float4 store
// writes 512; the kDequantU loads are issued first.
constexpr int kDequantU = 8;

__global__ void __launch_bounds__(kCodecThreads)
mxfp8_dequantize_flat_kernel(const uint8_t* __restrict__ data, const uint8_t* __restrict__ scales,
                             float* __restrict__ out, int64_t n_quads)
{
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    const uint32_t* d32 = reinterpret_cast<const uint32_t*>(data);
    float4* o4 = reinterpret_cast<float4*>(out);
    for (int64_t base = warp * 32 * kDequantU; base < n_quads; base += nwarps * 32 * kDequantU) {
        uint32_t c[kDequantU], sb[kDequantU];
#pragma unroll
        for (int j = 0; j < kDequantU; ++j) {
            const int64_t q = base + 32 * j + lane;
            c[j] = q < n_quads ? __ldcs(d32 + q) : 0u;
            sb[j] = q < n_quads ? __ldg(scales + (q >> 3)) : 0u;
        }
#pragma unroll
        for (int j = 0; j < kDequantU; ++j) {
            const int64_t q = base + 32 * j + lane;
            if (q < n_quads) {
                const float sc = e8m0_to_f32(sb[j]);
                const float2 a = e4m3x2_to_f32x2(c[j]), b = e4m3x2_to_f32x2(c[j] >> 16);
                __stcs(o4 + q, make_float4(a.x * sc, a.y * sc, b.x * sc, b.y * sc));
            }
        }
    }
}

__global__ void __launch_bounds__(kCodecThreads)
mxfp8_dequantize_elem_kernel(const uint8_t* __restrict__ data, const uint8_t* __restrict__ scales,
                             float* __restrict__ out, int64_t M, int64_t K, int64_t nblk)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * K; i += stride) {
        const int64_t row = i / K, k = i % K;
        const float s = e8m0_to_f32(scales[row * nblk + k / 32]);
        out[i] = e4m3x2_to_f32x2(data[i]).x * s;
    }
}


// ------------------------- dequantize to BF16 (GEMM A) -------------------------
//
// MXFP8 [M][K] -> BF16 [M][K], exact: code x 2^(s-127) has at most 4 significant
// bits and BF16 keeps FP32's exponent range, so the product is representable for
// every scale byte except 1 and 2 (whose smallest products sit below BF16's
// subnormal range and are rounded to nearest even, as cvt.rn does).  Byte 0 gives
// 0 and byte 255 gives +-inf (NaN for code 0), as the reference's e8m0_to_float.
//
// Fast path per 8 codes sharing a scale byte in 3..134 with no NaN code: integer
// bit placement of each code as BF16 code x 2^-120, then one exact mul.rn.bf16x2
// by 2^(s-7).  Anything else: E4M3 -> f32 hardware conversion, FP32 multiply,
// cvt.rn to BF16.
__device__ __forceinline__ uint32_t prmt_b32(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t bf16x2_mul(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint4 e4m3x8_to_bf16x8(uint2 c, uint32_t s)
{
    const uint32_t in[2] = {c.x, c.y};
    uint32_t out[4];
    const uint32_t wm0 = in[0] & 0x7F7F7F7Fu, wm1 = in[1] & 0x7F7F7F7Fu;
    const uint32_t nan_probe = ((wm0 + 0x01010101u) | (wm1 + 0x01010101u)) & 0x80808080u;
    if ((s - 3u) <= 131u && nan_probe == 0u) {
        uint32_t f = (s + 120u) << 7;
        f |= f << 16;
        const uint32_t wm[2] = {wm0, wm1};
#pragma unroll
        for (int w = 0; w < 2; ++w) {
            const uint32_t ws = in[w] & 0x80808080u;
            out[2 * w] = bf16x2_mul(prmt_b32(wm[w], 0u, 0x4140u) * 16u + prmt_b32(ws, 0u, 0x1404u), f);
            out[2 * w + 1] = bf16x2_mul(prmt_b32(wm[w], 0u, 0x4342u) * 16u + prmt_b32(ws, 0u, 0x3424u), f);
        }
    } else {
        const float sc = e8m0_to_f32(s);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const float2 f = e4m3x2_to_f32x2(in[w] >> (16 * h));
                uint32_t packed;
                asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(f.y * sc), "f"(f.x * sc));
                out[2 * w + h] = packed;
            }
        }
    }
    return make_uint4(out[0], out[1], out[2], out[3]);
}

// K % 32 == 0, 8-byte aligned codes, 16-byte aligned output: flat run of blocks.
// Lane l of a warp converts octet base + 32j + l for j < kPrepassU (loads first).
// The BF16 output is stored with the default policy so that it stays in L2 for
// the GEMM that reads it next.
constexpr int kPrepassU = 2;

// Block 0 of the A pre-pass zeroes the GEMM's stream-K counters (n_zero words).
__device__ __forceinline__ void zero_words_block0(uint32_t* words, int n)
{
    if (blockIdx.x == 0)
        for (int i = threadIdx.x; i < n; i += blockDim.x) words[i] = 0u;
}

__global__ void __launch_bounds__(kCodecThreads)
mxfp8_dequantize_bf16_flat_kernel(const uint8_t* __restrict__ data, const uint8_t* __restrict__ scales,
                                  uint16_t* __restrict__ out, int64_t n_octets, uint32_t* zero_words,
                                  int n_zero)
{
    allow_dependent_launch();
    zero_words_block0(zero_words, n_zero);
    const int lane = threadIdx.x & 31;
    const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
    for (int64_t base = warp * 32 * kPrepassU; base < n_octets; base += nwarps * 32 * kPrepassU) {
        uint2 c[kPrepassU];
        uint32_t sb[kPrepassU];
#pragma unroll
        for (int j = 0; j < kPrepassU; ++j) {
            const int64_t o = base + 32 * j + lane;
            c[j] = o < n_octets ? __ldcs(reinterpret_cast<const uint2*>(data) + o) : make_uint2(0u, 0u);
            sb[j] = o < n_octets ? __ldg(scales + (o >> 2)) : 127u;
        }
#pragma unroll
        for (int j = 0; j < kPrepassU; ++j) {
            const int64_t o = base + 32 * j + lane;
            if (o < n_octets) reinterpret_cast<uint4*>(out)[o] = e4m3x8_to_bf16x8(c[j], sb[j]);
        }
    }
}

// Any shape and alignment, output rows ld_out elements apart: one element per thread.
__global__ void __launch_bounds__(kCodecThreads)
mxfp8_dequantize_bf16_elem_kernel(const uint8_t* __restrict__ data, const uint8_t* __restrict__ scales,
                                  uint16_t* __restrict__ out, int64_t M, int64_t K, int64_t nblk,
                                  int64_t ld_out, uint32_t* zero_words, int n_zero)
{
    allow_dependent_launch();
    zero_words_block0(zero_words, n_zero);
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < M * K; i += stride) {
        const int64_t row = i / K, k = i % K;
        const float v = e4m3x2_to_f32x2(data[i]).x * e8m0_to_f32(scales[row * nblk + k / 32]);
        out[row * ld_out + k] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

// ------------------------- quantize along the rows --------------------------
// MXFP8 with the block axis along the strided dimension: each column of a
// row-major [M][K] tensor is cut into blocks of 32 consecutive rows, each with one
// E8M0 scale; codes keep the input's layout ([M][K]) and the scales are
// [ceil(M/32)][K] row-major.  The arithmetic is the reference's per-block rule
// (src/quantize/mxfp8_quantize.cu:7-42: amax with NaN ignored, E8M0 = round-up
// power of two of amax / 448, RNE E4M3 of x / scale), so the result is the row
// quantizer's on the transposed tensor, transposed back.
//
// One thread per (32-row block, group of kCols columns); consecutive threads take
// consecutive column groups, so each of the 32 row loads of a warp reads one
// contiguous span (512 B of FP32 with 4 columns per thread) and each code store
// writes one (128 B).  All 32 rows are loaded before any arithmetic.
constexpr int kColsThreads = 128;

template <typename T, int kCols>
__device__ __forceinline__ void load_cols(const T* p, float (&v)[kCols])
{
    if constexpr (kCols == 4 && sizeof(T) == 4) {
        const float4 x = __ldcs(reinterpret_cast<const float4*>(p));
        v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
    } else if constexpr (kCols == 4) {
        const uint2 x = __ldcs(reinterpret_cast<const uint2*>(p));
        v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xFFFF0000u);
        v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xFFFF0000u);
    } else {
#pragma unroll
        for (int c = 0; c < kCols; ++c) v[c] = load_elem(p + c);
    }
}

template <typename T, int kCols>
__global__ void __launch_bounds__(kColsThreads)
mxfp8_quantize_cols_kernel(const T* __restrict__ in, uint8_t* __restrict__ data, uint8_t* __restrict__ scales,
                           int64_t M, int64_t K, int64_t ngroups, int64_t nblocks)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < ngroups * nblocks; w += stride) {
        const int64_t k0 = (w % ngroups) * kCols;
        const int64_t r0 = (w / ngroups) * 32;
        const int rows = (int)min((int64_t)32, M - r0);
        float v[32][kCols];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (i < rows) {
                load_cols<T, kCols>(in + (r0 + i) * K + k0, v[i]);
            } else {
#pragma unroll
                for (int c = 0; c < kCols; ++c) v[i][c] = 0.0f;
            }
        }
        float inv[kCols];
        uint32_t sc = 0u;
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
            float amax = 0.0f;  // NaN elements ignored; rows past M contribute 0
#pragma unroll
            for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i][c]));
            sc |= mx_block_scale(amax, inv[c]) << (8 * c);
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (i >= rows) break;
            uint8_t* dst = data + (r0 + i) * K + k0;
            if constexpr (kCols == 4) {
                const uint32_t c01 = f32x2_to_e4m3x2(v[i][0] * inv[0], v[i][1] * inv[1]);
                const uint32_t c23 = f32x2_to_e4m3x2(v[i][2] * inv[2], v[i][3] * inv[3]);
                __stcs(reinterpret_cast<uint32_t*>(dst), c01 | (c23 << 16));
            } else {
#pragma unroll
                for (int c = 0; c < kCols; ++c) dst[c] = (uint8_t)f32x2_to_e4m3x2(v[i][c] * inv[c], 0.0f);
            }
        }
        uint8_t* sdst = scales + (r0 / 32) * K + k0;
        if constexpr (kCols == 4) {
            *reinterpret_cast<uint32_t*>(sdst) = sc;
        } else {
#pragma unroll
            for (int c = 0; c < kCols; ++c) sdst[c] = (uint8_t)(sc >> (8 * c));
        }
    }
}

// BF16 source, 8 columns per thread: the 32 rows are held as packed BF16 (one
// 16-byte load per row, 512 B per warp instruction) and widened where they are
// used, so the registers hold the block twice as densely as FP32 would.
__global__ void __launch_bounds__(kColsThreads)
mxfp8_quantize_bf16_cols8_kernel(const uint16_t* __restrict__ in, uint8_t* __restrict__ data,
                                 uint8_t* __restrict__ scales, int64_t M, int64_t K, int64_t ngroups,
                                 int64_t nblocks)
{
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t w = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; w < ngroups * nblocks; w += stride) {
        const int64_t k0 = (w % ngroups) * 8;
        const int64_t r0 = (w / ngroups) * 32;
        const int rows = (int)min((int64_t)32, M - r0);
        uint4 v[32];
        const uint4* src = reinterpret_cast<const uint4*>(in + r0 * K + k0);
        const int64_t step = K / 8;  // one row, in 16-byte units
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = i < rows ? __ldcs(src + i * step) : make_uint4(0u, 0u, 0u, 0u);
        // Block amax on the packed BF16 bits: a magnitude's bits order like its value
        // (non-negative floats), NaN magnitudes (above 0x7F80) are dropped as fmaxf
        // drops them, and rows past M are zeros.
        uint32_t amax2[4] = {0u, 0u, 0u, 0u};
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            const uint32_t wd[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                const uint32_t m = wd[h] & 0x7FFF7FFFu;
                amax2[h] = __vmaxu2(amax2[h], m & __vcmpleu2(m, 0x7F807F80u));
            }
        }
        float inv[8];
        uint32_t sc[2] = {0u, 0u};
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            const float amax = __uint_as_float(c & 1 ? amax2[c >> 1] & 0xFFFF0000u : amax2[c >> 1] << 16);
            sc[c >> 2] |= mx_block_scale(amax, inv[c]) << (8 * (c & 3));
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) {
            if (i >= rows) break;
            const uint32_t wd[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
            uint32_t q[4];
#pragma unroll
            for (int h = 0; h < 4; ++h)
                q[h] = f32x2_to_e4m3x2(__uint_as_float(wd[h] << 16) * inv[2 * h],
                                       __uint_as_float(wd[h] & 0xFFFF0000u) * inv[2 * h + 1]);
            __stcs(reinterpret_cast<uint2*>(data + r0 * K + k0) + i * step,
                   make_uint2(q[0] | (q[1] << 16), q[2] | (q[3] << 16)));
        }
        *reinterpret_cast<uint2*>(scales + (r0 / 32) * K + k0) = make_uint2(sc[0], sc[1]);
    }
}

// ------------------------------- launchers ---------------------------------

static int codec_grid(int64_t work_items)
{
    const int64_t per_block = kCodecThreads;
    int64_t blocks = (work_items + per_block - 1) / per_block;
    const int64_t cap = (int64_t)device_sm_count() * 8;  // 2048 threads per SM
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (int)blocks;
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_mxfp8_quantize(const float* in, uint8_t* data, uint8_t* scales, int64_t M,
                                  int64_t K, cudaStream_t stream)
{
    const int64_t nblk = (K + 31) / 32;
    if (M == 0 || K == 0) return cudaSuccess;
    if (K % 32 == 0 && aligned16(in) && (reinterpret_cast<uintptr_t>(data) & 3u) == 0) {
        const int64_t nf4 = M * K / 4;
        mxfp8_quantize_flat_kernel<<<codec_grid(nf4 / kQuantU), kCodecThreads, 0, stream>>>(in, data, scales,
                                                                                         nf4);
    } else {
        mxfp8_quantize_rowblock_kernel<float><<<codec_grid(M * nblk * 32), kCodecThreads, 0, stream>>>(
            in, data, scales, M, K, nblk);
    }
    return cudaGetLastError();
}

cudaError_t launch_mxfp8_quantize_bf16(const void* in, uint8_t* data, uint8_t* scales, int64_t M,
                                       int64_t K, cudaStream_t stream)
{
    const int64_t nblk = (K + 31) / 32;
    if (M == 0 || K == 0) return cudaSuccess;
    const uint16_t* x = static_cast<const uint16_t*>(in);
    if (K % 32 == 0 && aligned16(in) && (reinterpret_cast<uintptr_t>(data) & 7u) == 0) {
        const int64_t no = M * K / 8;
        mxfp8_quantize_bf16_flat_kernel<<<codec_grid(no / kQuantBf16U), kCodecThreads, 0, stream>>>(
            x, data, scales, no);
    } else {
        mxfp8_quantize_rowblock_kernel<uint16_t><<<codec_grid(M * nblk * 32), kCodecThreads, 0, stream>>>(
            x, data, scales, M, K, nblk);
    }
    return cudaGetLastError();
}

template <typename T>
static cudaError_t launch_quantize_cols(const T* in, uint8_t* data, uint8_t* scales, int64_t M, int64_t K,
                                        cudaStream_t stream)
{
    if (M == 0 || K == 0) return cudaSuccess;
    const int64_t nblocks = (M + 31) / 32;
    const uintptr_t ia = reinterpret_cast<uintptr_t>(in), da = reinterpret_cast<uintptr_t>(data),
                    sa = reinterpret_cast<uintptr_t>(scales);
    const bool vec = K % 4 == 0 && ia % (4 * sizeof(T)) == 0 && da % 4 == 0 && sa % 4 == 0;
    const int64_t ngroups = vec ? K / 4 : K;
    int64_t blocks = (ngroups * nblocks + kColsThreads - 1) / kColsThreads;
    const int64_t cap = (int64_t)device_sm_count() * 32;
    if (blocks > cap) blocks = cap;
    if (vec)
        mxfp8_quantize_cols_kernel<T, 4><<<(int)blocks, kColsThreads, 0, stream>>>(in, data, scales, M, K, ngroups,
                                                                                  nblocks);
    else
        mxfp8_quantize_cols_kernel<T, 1><<<(int)blocks, kColsThreads, 0, stream>>>(in, data, scales, M, K, ngroups,
                                                                                  nblocks);
    return cudaGetLastError();
}

cudaError_t launch_mxfp8_quantize_cols(const float* in, uint8_t* data, uint8_t* scales, int64_t M, int64_t K,
                                       cudaStream_t stream)
{
    return launch_quantize_cols<float>(in, data, scales, M, K, stream);
}

cudaError_t launch_mxfp8_quantize_bf16_cols(const void* in, uint8_t* data, uint8_t* scales, int64_t M,
                                            int64_t K, cudaStream_t stream)
{
    const uint16_t* x = static_cast<const uint16_t*>(in);
    if (M == 0 || K == 0) return cudaSuccess;
    if (K % 8 == 0 && aligned16(in) && (reinterpret_cast<uintptr_t>(data) & 7u) == 0 &&
        (reinterpret_cast<uintptr_t>(scales) & 7u) == 0) {
        const int64_t nblocks = (M + 31) / 32, ngroups = K / 8;
        int64_t blocks = (ngroups * nblocks + kColsThreads - 1) / kColsThreads;
        const int64_t cap = (int64_t)device_sm_count() * 32;
        if (blocks > cap) blocks = cap;
        mxfp8_quantize_bf16_cols8_kernel<<<(int)blocks, kColsThreads, 0, stream>>>(x, data, scales, M, K, ngroups,
                                                                                  nblocks);
        return cudaGetLastError();
    }
    return launch_quantize_cols<uint16_t>(x, data, scales, M, K, stream);
}

cudaError_t launch_mxfp8_dequantize(const uint8_t* data, const uint8_t* scales, float* out,
                                    int64_t M, int64_t K, cudaStream_t stream)
{
    const int64_t nblk = (K + 31) / 32;
    if (M == 0 || K == 0) return cudaSuccess;
    if (K % 32 == 0 && aligned16(out) && (reinterpret_cast<uintptr_t>(data) & 3u) == 0) {
        const int64_t nq = M * K / 4;
        mxfp8_dequantize_flat_kernel<<<codec_grid(nq / kDequantU), kCodecThreads, 0, stream>>>(data, scales,
                                                                                            out, nq);
    } else {
        mxfp8_dequantize_elem_kernel<<<codec_grid(M * K), kCodecThreads, 0, stream>>>(
            data, scales, out, M, K, nblk);
    }
    return cudaGetLastError();
}

cudaError_t launch_mxfp8_dequantize_bf16(const uint8_t* data, const uint8_t* scales, void* out,
                                         int64_t M, int64_t K, int64_t ld_out, cudaStream_t stream,
                                         uint32_t* zero_words, int n_zero)
{
    const int64_t nblk = (K + 31) / 32;
    if (M == 0 || K == 0) return cudaSuccess;
    uint16_t* o = static_cast<uint16_t*>(out);
    if (K % 32 == 0 && ld_out == K && aligned16(out) && (reinterpret_cast<uintptr_t>(data) & 7u) == 0) {
        const int64_t no = M * K / 8;
        mxfp8_dequantize_bf16_flat_kernel<<<codec_grid(no / kPrepassU), kCodecThreads, 0, stream>>>(
            data, scales, o, no, zero_words, n_zero);
    } else {
        mxfp8_dequantize_bf16_elem_kernel<<<codec_grid(M * K), kCodecThreads, 0, stream>>>(
            data, scales, o, M, K, nblk, ld_out, zero_words, n_zero);
    }
    return cudaGetLastError();
}

cudaError_t launch_mxfp8_requantize(const uint8_t* c_data, const uint8_t* c_scales, uint8_t* d_data,
                                    uint8_t* d_scales, int64_t M, int64_t N, cudaStream_t stream)
{
    const int64_t nblk = (N + 31) / 32;
    if (M == 0 || N == 0) return cudaSuccess;
    mxfp8_requantize_kernel<<<codec_grid(M * nblk * 32), kCodecThreads, 0, stream>>>(
        c_data, c_scales, d_data, d_scales, M, N, nblk);
    return cudaGetLastError();
}

}  // namespace mpk
