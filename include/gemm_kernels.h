// Drop-in replacement for the reference's include/gemm_kernels.h
// (chcoliang/mix_precision_kernel include/gemm_kernels.h:7-16).
//
//   D = A * B + C
//   A [M,K] MXFP8, B [K,N] bf16, C [M,N] MXFP8 (optional), D [M,N] MXFP8
//   (FP8 E4M3 data, E8M0 scales, block_size = 32; A along K, C and D along N)
//
// Only the reference's fastest variant, gemm_fp8_tensorcore, is provided; it runs
// libmpk's sm_100a kernel (include/mpk.h).  The other four reference variants
// (CUDA-core, mixed-tiled, native-MMA, cuBLASLt) are alternative backends with the
// same contract and are not part of this library.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>

#include "mpk.h"

// Same signature and argument meaning as the reference (include/gemm_kernels.h:12-16),
// any M, N, K.  Differences: no per-call cudaMalloc/cudaFree or implicit device
// synchronization.  The workspace (A's BF16 copy, M*K*2 bytes, plus the stream-K
// partials when the schedule uses them, mpk_gemm_workspace_size) comes from a
// library-owned stream-ordered pool that keeps what it has reserved: the first call
// of each larger workspace size on a device grows the pool (the driver maps new
// device memory inside that call); calls of that size or smaller afterwards reuse
// it without any driver allocation, until mpk_release_workspace_pool.  A caller
// that must know its footprint before its first request makes one call of its
// largest size at set-up.  Any failure (no sm_100 device, out of memory, a shape the
// on-chip kernel cannot take while the stream is being captured) prints a message
// and exits, as the reference's CUDA_CHECK does.
inline void gemm_fp8_tensorcore(const uint8_t* d_A_data, const uint8_t* d_A_scales,
                                const __nv_bfloat16* d_B, const uint8_t* d_C_data,
                                const uint8_t* d_C_scales, uint8_t* d_D_data, uint8_t* d_D_scales,
                                int M, int N, int K, cudaStream_t stream = 0)
{
    const int st = mpk_gemm_mxfp8_bf16(d_A_data, d_A_scales, d_B, d_C_data, d_C_scales, d_D_data,
                                       d_D_scales, M, N, K, stream);
    if (st != MPK_SUCCESS) {
        fprintf(stderr, "gemm_fp8_tensorcore failed: %s (%s)\n", mpk_status_string(st), mpk_last_error_string());
        exit(EXIT_FAILURE);
    }
}
