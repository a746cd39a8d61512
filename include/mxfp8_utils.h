// Drop-in replacement for the reference's include/mxfp8_utils.h and the E4M3/BF16
// part of include/fp8_types.h (chcoliang/mix_precision_kernel
// include/mxfp8_utils.h:8-47, include/fp8_types.h:8-21, :34-40).
//
// The scalar helpers are header-inline with the reference's semantics; the
// quantize/dequantize entry points forward to libmpk's C ABI (include/mpk.h).
// As in the reference, a failing call prints a message and exits; use the C ABI
// directly to receive the status code instead.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "gemm_common.h"
#include "mpk.h"

// ---- include/fp8_types.h:8-21, :34-40 ----------------------------------------

// E4M3 code -> float, exact (0x7F / 0xFF -> NaN).
__host__ __device__ inline float fp8_e4m3_to_float(uint8_t val)
{
    __nv_fp8_e4m3 f;
    f.__x = val;
    return static_cast<float>(f);
}

// float -> E4M3 code: NaN -> 0x7F, clamp to +-448, round to nearest even.
__host__ __device__ inline uint8_t float_to_fp8_e4m3(float val)
{
    if (val != val) return 0x7F;
    if (val > 448.0f) val = 448.0f;
    if (val < -448.0f) val = -448.0f;
    return static_cast<uint8_t>(__nv_cvt_float_to_fp8(val, __NV_SATFINITE, __NV_E4M3));
}

__host__ __device__ inline float bf16_to_float(__nv_bfloat16 val) { return __bfloat162float(val); }
__host__ __device__ inline __nv_bfloat16 float_to_bf16(float val) { return __float2bfloat16(val); }

// ---- include/mxfp8_utils.h:8-22 -----------------------------------------------

// E8M0 byte -> float with bit pattern byte << 23 (byte 0 -> 0.0, 255 -> +inf).
__host__ __device__ inline float e8m0_to_float(uint8_t e8m0)
{
    const uint32_t bits = static_cast<uint32_t>(e8m0) << 23;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
}

// float -> E8M0 byte, rounded up to a power of two (x <= 0 -> 0).
__host__ __device__ inline uint8_t float_to_e8m0(float val)
{
    if (val <= 0.0f) return 0;
    uint32_t bits;
    memcpy(&bits, &val, sizeof(bits));
    uint32_t e = (bits >> 23) & 0xFFu;
    if ((bits & 0x007FFFFFu) && e < 255u) ++e;
    return static_cast<uint8_t>(e);
}

struct MxFp8Data {
    uint8_t* data;     // E4M3 codes
    uint8_t* scales;   // E8M0 scales, one per 32 elements along K
    int M;
    int K;
    int num_blocks_k;  // ceil(K / 32)
};

// ---- include/mxfp8_utils.h:34-47 ----------------------------------------------

namespace mpk_compat {
inline void check(int status, const char* what)
{
    if (status != MPK_SUCCESS) {
        fprintf(stderr, "%s failed: %s (%s)\n", what, mpk_status_string(status), mpk_last_error_string());
        exit(EXIT_FAILURE);
    }
}
}  // namespace mpk_compat

// float [M][K] -> MXFP8 along K, host (reference src/quantize/mxfp8_quantize.cu:116-144).
inline void mxfp8_quantize_host(const float* input, uint8_t* output_data, uint8_t* output_scales,
                                int M, int K)
{
    mpk_compat::check(mpk_mxfp8_quantize_host(input, output_data, output_scales, M, K),
                      "mxfp8_quantize_host");
}

// float [M][K] -> MXFP8 along K on the GPU (src/quantize/mxfp8_quantize.cu:82-88).
inline void mxfp8_quantize_gpu(const float* d_input, uint8_t* d_output_data, uint8_t* d_output_scales,
                               int M, int K, cudaStream_t stream = 0)
{
    mpk_compat::check(mpk_mxfp8_quantize(d_input, d_output_data, d_output_scales, M, K, stream),
                      "mxfp8_quantize_gpu");
}

// MXFP8 -> float [M][K], host (src/quantize/mxfp8_dequantize.cu:32-47).
inline void mxfp8_dequantize_host(const uint8_t* input_data, const uint8_t* input_scales,
                                  float* output, int M, int K)
{
    mpk_compat::check(mpk_mxfp8_dequantize_host(input_data, input_scales, output, M, K),
                      "mxfp8_dequantize_host");
}

// MXFP8 -> float [M][K] on the GPU (src/quantize/mxfp8_dequantize.cu:22-29).
inline void mxfp8_dequantize_gpu(const uint8_t* d_input_data, const uint8_t* d_input_scales,
                                 float* d_output, int M, int K, cudaStream_t stream = 0)
{
    mpk_compat::check(mpk_mxfp8_dequantize(d_input_data, d_input_scales, d_output, M, K, stream),
                      "mxfp8_dequantize_gpu");
}
