// Internal interfaces between the translation units of libmpk (not installed).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mpk {

// Device properties of the current device (cached per device).
int device_sm_count();
int device_cc_major();
int device_cc_minor();

// Codec launchers (codec.cu).  Arguments are validated by the ABI layer.
cudaError_t launch_mxfp8_quantize(const float* in, uint8_t* data, uint8_t* scales, int64_t M,
                                  int64_t K, cudaStream_t stream);
cudaError_t launch_mxfp8_dequantize(const uint8_t* data, const uint8_t* scales, float* out,
                                    int64_t M, int64_t K, cudaStream_t stream);
// MXFP8 [M][K] -> BF16 [M][K] (exact for scale bytes other than 1 and 2).
cudaError_t launch_mxfp8_quantize_bf16(const void* in, uint8_t* data, uint8_t* scales, int64_t M,
                                       int64_t K, cudaStream_t stream);
// The GEMM's A pre-pass also zeroes zero_words[0 .. n_zero) (the stream-K ticket and
// arrival counters of the GEMM kernel launched after it).
cudaError_t launch_mxfp8_dequantize_bf16(const uint8_t* data, const uint8_t* scales, void* out,
                                         int64_t M, int64_t K, int64_t ld_out, cudaStream_t stream,
                                         uint32_t* zero_words = nullptr, int n_zero = 0);
// float / BF16 [M][K] -> MXFP8 with blocks of 32 rows in each column: codes [M][K],
// scales [ceil(M/32)][K].
cudaError_t launch_mxfp8_quantize_cols(const float* in, uint8_t* data, uint8_t* scales, int64_t M, int64_t K,
                                       cudaStream_t stream);
cudaError_t launch_mxfp8_quantize_bf16_cols(const void* in, uint8_t* data, uint8_t* scales, int64_t M,
                                            int64_t K, cudaStream_t stream);
// D = MXFP8(dequant(C)) along N (C may be null: D = MXFP8(0)).  The K == 0 GEMM.
cudaError_t launch_mxfp8_requantize(const uint8_t* c_data, const uint8_t* c_scales, uint8_t* d_data,
                                    uint8_t* d_scales, int64_t M, int64_t N, cudaStream_t stream);

// GEMM launcher (gemm.cu).  Returns an MPK status code (0 on success).
int launch_gemm_mxfp8_bf16(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                           const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                           uint8_t* D_scales, int M, int N, int K, cudaStream_t stream);

// The on-chip conversion kernel's requirements: K % 16 == 0, N % 8 == 0, A_data and B
// 16-byte aligned (TMA row strides and base addresses).  Returns 0 or an MPK status
// with the detail set.
int check_onchip_gemm_shape(const uint8_t* A_data, const void* B, int N, int K);

// GEMM with the A operand dequantized to BF16 by a pre-pass into `workspace`, then
// streamed by TMA.  Any M, N, K and alignment: A's BF16 copy has rows padded to a
// multiple of 8 elements, and B is copied into the workspace with padded rows when
// N % 8 != 0 or B is not 16-byte aligned (gemm_b_needs_copy).  `workspace` must be
// 16-byte aligned and hold gemm_workspace_bytes(M, N, K, gemm_b_needs_copy(B, N)).
// Extra destinations of the fused all-gather: element (r, c) of the product goes to
// (row_offset + r, col_offset + c) of D_data and of every D_extra[i] (other GPUs' full
// buffers), rows ldd bytes apart; col_offset is a multiple of 32.
struct GatherDest {
    int n_extra;
    int64_t row_offset, col_offset, ldd;
    uint8_t* D_extra[7];
    uint8_t* Ds_extra[7];
};
// True when mpk_gemm_mxfp8_bf16 runs the on-chip conversion kernel for these
// operands (tall products with few columns; see gemm.cu).
bool gemm_default_onchip(const void* A_data, const void* B, int M, int N, int K);
bool gemm_b_needs_copy(const void* B, int N);
// 0 if `bytes` bytes at ptr lie in memory the current device may store to (an
// allocation of this device, or a buffer imported on it with mpk_ipc_import).
int check_store_target(const void* ptr, size_t bytes, const char* what);
// Workspace of the pre-pass path: gemm_workspace_bytes_min holds A's BF16 copy and
// B's padded copy; gemm_workspace_bytes adds the stream-K partials when the current
// schedule uses stream-K for this shape (with less than that the kernel runs whole
// tiles only).
size_t gemm_workspace_bytes_min(int M, int N, int K, bool copy_b);
size_t gemm_workspace_bytes(int M, int N, int K, bool copy_b);
int launch_gemm_mxfp8_bf16_prepass(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                                   const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                                   uint8_t* D_scales, int M, int N, int K, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream,
                                   const GatherDest* gather = nullptr);

// Stream-K plan of an M x N x K product on the current device under the current
// schedule: `tiles` tiles (the first of the raster) spread over `clusters` clusters;
// tiles == 0 means whole tiles only.
struct SkPlan {
    int tiles, clusters;
};
SkPlan gemm_sk_plan(int M, int N, int K);
int gemm_set_schedule(int mode);
int gemm_schedule();
// Cross-GPU barrier over flag arrays (flags[i]: GPU i's array, at least `world`
// uint32 slots, peer-accessible); bounded wait, expiry recorded in the status word.
int launch_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t epoch, cudaStream_t stream);

// Device-side status word of the GEMM kernels (gemm.cu): read and clear.
int read_and_clear_device_status(int* value);
// Bounded-wait self test: one CTA waits on an mbarrier that nothing arrives on.
int launch_wait_selftest(uint64_t timeout_ns, cudaStream_t stream);

// Wait budget for device-side spin waits, in nanoseconds.
uint64_t wait_timeout_ns();
void set_wait_timeout_ns(uint64_t ns);

// Thread-local detail message for the last failing call.
void set_last_error(const char* fmt, ...);

}  // namespace mpk
