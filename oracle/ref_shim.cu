// C-ABI wrappers around the reference project's own functions.  TEST
// INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file together with the reference's unmodified
// sources (src/quantize/mxfp8_quantize.cu, src/quantize/mxfp8_dequantize.cu,
// src/reference/gemm_reference.cu, src/kernels/gemm_fp8_tensorcore.cu), read in
// place from the reference checkout, into oracle/_ref/libmpk_ref.so.  The
// reference's functions are C++ (mangled) free functions; these wrappers give
// them plain C names so the tests can load them with ctypes.  Nothing here
// changes what the reference computes.
#include <cstdint>
#include <cstring>

#include "gemm_kernels.h"     // include/gemm_kernels.h:12-16
#include "gemm_reference.h"   // include/gemm_reference.h:7-12
#include "mxfp8_utils.h"      // include/mxfp8_utils.h:8-47

extern "C" {

// Scalar conversions (include/fp8_types.h:8-21, :34-40; include/mxfp8_utils.h:8-22).
float ref_fp8_e4m3_to_float(uint8_t v) { return fp8_e4m3_to_float(v); }
uint8_t ref_float_to_fp8_e4m3(float x) { return float_to_fp8_e4m3(x); }
float ref_e8m0_to_float(uint8_t b) { return e8m0_to_float(b); }
uint8_t ref_float_to_e8m0(float x) { return float_to_e8m0(x); }
uint16_t ref_float_to_bf16(float x)
{
    __nv_bfloat16 h = float_to_bf16(x);
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
}

void ref_sweep_float_to_e4m3(uint64_t lo, uint64_t hi, uint8_t* out)
{
    for (uint64_t u = lo; u < hi; ++u) {
        uint32_t b = (uint32_t)u;
        float f;
        std::memcpy(&f, &b, 4);
        out[u - lo] = float_to_fp8_e4m3(f);
    }
}

// Host functions (src/quantize/mxfp8_quantize.cu:116-144,
// src/quantize/mxfp8_dequantize.cu:32-47, src/reference/gemm_reference.cu:68-80).
void ref_mxfp8_quantize_host(const float* in, uint8_t* data, uint8_t* scales, int M, int K)
{
    mxfp8_quantize_host(in, data, scales, M, K);
}
void ref_mxfp8_dequantize_host(const uint8_t* data, const uint8_t* scales, float* out, int M, int K)
{
    mxfp8_dequantize_host(data, scales, out, M, K);
}
void ref_gemm_reference_host(const float* A, const float* B, const float* C, float* D,
                             int M, int N, int K)
{
    gemm_reference_host(A, B, C, D, M, N, K);
}

// GPU launchers of the reference, rebuilt for sm_100a, for on-device
// comparisons (device pointers; stream 0 when the stream argument is null).
int ref_mxfp8_quantize_gpu(const float* in, uint8_t* data, uint8_t* scales, int M, int K, void* stream)
{
    mxfp8_quantize_gpu(in, data, scales, M, K, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}
int ref_mxfp8_dequantize_gpu(const uint8_t* data, const uint8_t* scales, float* out, int M, int K,
                             void* stream)
{
    mxfp8_dequantize_gpu(data, scales, out, M, K, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}
int ref_gemm_reference_gpu(const float* A, const float* B, const float* C, float* D,
                           int M, int N, int K, void* stream)
{
    gemm_reference_gpu(A, B, C, D, M, N, K, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}
int ref_gemm_fp8_tensorcore(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                            const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                            uint8_t* D_scales, int M, int N, int K, void* stream)
{
    gemm_fp8_tensorcore(A_data, A_scales, (const __nv_bfloat16*)B, C_data, C_scales, D_data,
                        D_scales, M, N, K, (cudaStream_t)stream);
    return (int)cudaGetLastError();
}

}  // extern "C"
