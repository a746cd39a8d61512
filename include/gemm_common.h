// Drop-in replacement for the reference's include/gemm_common.h
// (chcoliang/mix_precision_kernel include/gemm_common.h:8-53): the CUDA_CHECK
// macro, the timing/FLOP helper, the relative-error metric and the MX block
// size, with the reference's meaning.  Header-only.
#pragma once

#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>

// Print and exit on a CUDA error (include/gemm_common.h:8-16).
#define CUDA_CHECK(call)                                                                      \
    do {                                                                                      \
        cudaError_t mpk_cuda_check_err_ = (call);                                             \
        if (mpk_cuda_check_err_ != cudaSuccess) {                                             \
            fprintf(stderr, "CUDA error at %s:%d: %s\n", __FILE__, __LINE__,                  \
                    cudaGetErrorString(mpk_cuda_check_err_));                                 \
            exit(EXIT_FAILURE);                                                               \
        }                                                                                     \
    } while (0)

struct GemmDims {
    int M;
    int N;
    int K;
};

struct TimingResult {
    float elapsed_ms;
    float tflops;
    float bandwidth_gb_s;
};

// FLOPs = 2*M*N*K (include/gemm_common.h:30-37).
inline TimingResult time_kernel(int M, int N, int K, float elapsed_ms)
{
    TimingResult r;
    r.elapsed_ms = elapsed_ms;
    r.tflops = static_cast<float>(2.0 * M * N * K / (elapsed_ms * 1e9));
    r.bandwidth_gb_s = 0.0f;
    return r;
}

// Maximum relative error over entries with |reference| > 1e-6
// (include/gemm_common.h:39-50).
inline float compute_relative_error(const float* result, const float* reference, int size)
{
    float worst = 0.0f;
    for (int i = 0; i < size; ++i) {
        const float ref = reference[i];
        if (fabsf(ref) > 1e-6f) {
            const float rel = fabsf(result[i] - ref) / fabsf(ref);
            if (rel > worst) worst = rel;
        }
    }
    return worst;
}

constexpr int WARP_SIZE = 32;
constexpr int MXFP8_BLOCK_SIZE = 32;
