/*
 * libmpk -- C ABI of the B200 (sm_100a) MXFP8 x BF16 GEMM and MXFP8 codec.
 *
 * Drop-in boundary for the hot path of chcoliang/mix_precision_kernel:
 *
 *     D = A * B + C
 *     A  [M][K]  MXFP8: E4M3 codes (u8, row-major) + E8M0 scales (u8 [M][ceil(K/32)])
 *     B  [K][N]  BF16, row-major (N contiguous)
 *     C  [M][N]  MXFP8 with blocks along N (optional: both C pointers may be NULL)
 *     D  [M][N]  MXFP8 with blocks along N
 *
 * Conventions (the reference's, include/gemm_kernels.h:7-9 and
 * include/mxfp8_utils.h:24-47): scales are row-major [rows][ceil(cols/32)]
 * indexed row*nblk + col/32; data is row-major with leading dimension cols; no
 * padding or swizzle.  All pointers are device pointers owned by the caller.
 * `stream` is a cudaStream_t (NULL = the legacy default stream).
 *
 * Differences from the reference, by design:
 *   - every entry point returns a status code (0 = success) instead of calling
 *     exit() on failure; a detail message is available from mpk_last_error_string();
 *   - no call synchronizes the device; every launch is stream-ordered;
 *   - mpk_gemm_mxfp8_bf16 does not cudaMalloc/cudaFree per call: the workspace of
 *     its A pre-pass (about M*K*2 bytes, mpk_gemm_workspace_size) comes from a
 *     library-owned stream-ordered pool that stays reserved for reuse
 *     (mpk_release_workspace_pool returns it);
 *   - indexing is 64-bit.
 */
#ifndef MPK_H_
#define MPK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  Values below 1000 are cudaError_t values passed through. */
enum {
    MPK_SUCCESS = 0,
    MPK_ERR_INVALID_VALUE = 1001,   /* null pointer, negative size, size overflow */
    MPK_ERR_UNSUPPORTED = 1002,     /* shape or size an entry point does not handle (see mpk_last_error) */
    MPK_ERR_MISALIGNED = 1003,      /* pointer alignment an entry point requires is not met */
    MPK_ERR_DEVICE_TIMEOUT = 1004,  /* a bounded device-side wait expired (read by mpk_device_status) */
    MPK_ERR_ARCH = 1005,            /* current device is not sm_100 */
    MPK_ERR_DRIVER = 1006           /* CUDA driver entry point or tensor-map encoding failed */
};

/* D = A*B + C.  Replaces gemm_fp8_tensorcore (reference include/gemm_kernels.h:12-16,
 * src/kernels/gemm_fp8_tensorcore.cu:231-249).  Any M, N, K >= 0 and any pointer
 * alignment, as in the reference.  C_data/C_scales may both be NULL (no C term).
 *
 * A is dequantized exactly to BF16 by a bandwidth pre-pass into a workspace taken
 * from the library's pool on `stream` (rows padded to a multiple of 8 elements; B is
 * also copied there with padded rows when N % 8 != 0 or B is not 16-byte aligned),
 * then the tensor-core kernel streams both operands by TMA.  While `stream` is
 * being captured into a CUDA graph the workspace is a stream-ordered allocation
 * (cudaMallocAsync), which the capture records as the graph's own allocation and
 * free nodes.  If no workspace can be had, the kernel that converts A on chip runs
 * instead: it needs no workspace and gives a bit-identical D, but needs K % 16 == 0,
 * N % 8 == 0 and 16-byte aligned A_data and B (else MPK_ERR_UNSUPPORTED /
 * MPK_ERR_MISALIGNED).
 *
 * Tall products with few columns -- N <= 2048 and M * K * 2 >= 256 MiB, under the
 * default schedule, when the plan has no stream-K split and the operands meet the
 * on-chip kernel's limits above -- take the on-chip kernel directly: there the extra
 * pass of the pre-pass over A in HBM costs more than converting A inside the GEMM,
 * and D is the same bit for bit.  mpk_gemm_path reports which path a call takes. */
int mpk_gemm_mxfp8_bf16(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                        const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                        uint8_t* D_scales, int M, int N, int K, void* stream);

/* Same computation with a caller-provided workspace: 16-byte aligned, at least
 * mpk_gemm_workspace_size() bytes (plus K*N*2 when B is not 16-byte aligned), and
 * not used by other work in flight until this call's kernels have finished on
 * `stream`.  With workspace == NULL the on-chip conversion kernel runs (no
 * workspace at all; its shape and alignment limits apply).  No counterpart in the
 * reference (its launcher allocates its own temporary). */
int mpk_gemm_mxfp8_bf16_ws(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                           const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                           uint8_t* D_scales, int M, int N, int K, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Workspace bytes mpk_gemm_mxfp8_bf16_ws needs for an M x N x K product with a
 * 16-byte aligned B: M * roundup(K, 8) * 2, rounded up to 256, plus
 * K * roundup(N, 8) * 2 when N % 8 != 0, plus, when the current schedule spreads the
 * last partial wave of tiles over the SMs (stream-K, see mpk_gemm_plan), 256 KiB per
 * participating SM pair and a few hundred bytes of counters (at most 18.5 MiB +
 * 1 KiB on a 148-SM B200).  A workspace with room for the operands but not for the
 * stream-K partials is accepted; the kernel then runs whole tiles only.  The size
 * depends on the current device's SM count and on mpk_set_gemm_schedule. */
int mpk_gemm_workspace_size(int M, int N, int K, size_t* bytes);

/* Work schedule of the tensor-core kernel of mpk_gemm_mxfp8_bf16 and its _ws and
 * _noalloc forms (process-wide; the fused all-gather always runs whole tiles).
 *   MPK_SCHEDULE_AUTO      (default) whole 256x256 tiles in waves over the SM pairs;
 *                          the tiles of a last, partial wave are spread over all
 *                          pairs by K-step ranges (stream-K): each pair computes a
 *                          contiguous range of K-steps, a tile split across pairs is
 *                          finished by the pair holding its last K-steps after adding
 *                          the others' FP32 partial sums.  Used when it keeps more
 *                          pairs busy than whole tiles would and gives each pair at
 *                          least 8 K-steps of 64; otherwise a partial wave of at most
 *                          half the pairs is cut into 256x128 tiles.
 *   MPK_SCHEDULE_TILES     whole tiles only (the split last wave as above).  D is
 *                          then the same for any schedule of the same tiles (every
 *                          element summed in one K order).
 *   MPK_SCHEDULE_STREAM_K  every tile's K-steps spread over the SM pairs (testing).
 * Split tiles sum their K ranges in a different order than whole tiles, so D may
 * differ between schedules by one E4M3 step in rare elements; for a given shape,
 * device and schedule it is deterministic.  No counterpart in the reference. */
enum { MPK_SCHEDULE_AUTO = 0, MPK_SCHEDULE_TILES = 1, MPK_SCHEDULE_STREAM_K = 2 };
int mpk_set_gemm_schedule(int schedule);
int mpk_gemm_schedule(void);

/* The schedule an M x N x K product gets on the current device: *stream_k_tiles
 * tiles (the first of the tile raster) spread over *stream_k_pairs SM pairs, the rest
 * whole tiles; *tiles is the total number of 256x256 tiles.  No counterpart in the
 * reference. */
int mpk_gemm_plan(int M, int N, int K, int* tiles, int* stream_k_tiles, int* stream_k_pairs);

/* Kernel path of mpk_gemm_mxfp8_bf16 for these operands (*path):
 *   MPK_PATH_PREPASS  A dequantized to BF16 by the pre-pass, then the BF16-A tensor-core
 *                     kernel (two launches; falls back to MPK_PATH_ONCHIP only when
 *                     no workspace can be had);
 *   MPK_PATH_ONCHIP   the kernel that converts A on chip (one launch, no workspace).
 * Depends on the shape, on A_data's and B's alignment and on the current schedule.
 * No counterpart in the reference. */
enum { MPK_PATH_PREPASS = 0, MPK_PATH_ONCHIP = 1 };
int mpk_gemm_path(const void* A_data, const void* B_bf16, int M, int N, int K, int* path);

/* Returns the current device's pooled GEMM workspace to the driver, once the
 * work queued on it has finished.  No counterpart in the reference. */
int mpk_release_workspace_pool(void);

/* Fixed size of the device array behind mpk_gemm_mxfp8_bf16_noalloc: 32 MiB per
 * device, enough for the BF16 copy of an A with M*K <= 16,777,216 (4096 x 4096) when
 * K % 8 == 0, N % 8 == 0 and B is 16-byte aligned (other shapes need the workspace
 * that mpk_gemm_mxfp8_bf16_ws describes, or run on the on-chip conversion kernel). */
#define MPK_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* Same computation as mpk_gemm_mxfp8_bf16, for callers that may not allocate
 * device memory once running (a caching allocator that has reserved the device, a
 * latency-bound loop, a fixed memory budget).  The A workspace is a fixed array in
 * the library's device image (MPK_NOALLOC_SCRATCH_BYTES per device, held until the
 * process exits); after the first call on a device, calls allocate nothing.  With
 * CUDA's default lazy module loading the array is reserved by that first call on
 * each device (when it loads the image holding the array), so make one call during
 * set-up, before a caching allocator reserves the device's memory and before any
 * stream capture (or run with CUDA_MODULE_LOADING=EAGER, which reserves it when the
 * context is created).  The array's address is looked up on every call, so calls
 * stay valid after cudaDeviceReset (whose next first call reserves it again).
 * Shapes the default entry point sends to the on-chip conversion kernel take it here
 * too, and so do shapes whose workspace would exceed the array when K % 16 == 0,
 * N % 8 == 0 and A_data and B are 16-byte aligned (that kernel needs no workspace;
 * D is the whole-tile result); other sizes whose workspace exceeds the array return
 * MPK_ERR_UNSUPPORTED.  Nothing in
 * the array needs to start at zero.  When the array also has room for the
 * stream-K partials (see mpk_set_gemm_schedule) the call uses them, otherwise it
 * runs whole tiles.  All calls on a device share the array: calls that can run at
 * the same time (different streams without an event between them, or unordered
 * host threads) race, so issue them on one stream or order them.  No counterpart
 * in the reference. */
int mpk_gemm_mxfp8_bf16_noalloc(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                                const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                                uint8_t* D_scales, int M, int N, int K, void* stream);

/* Fused GEMM + all-gather of D over NVLink, for one slab of a GEMM whose D
 * (M_total x N_total) every GPU keeps whole: an M-row slab (A and C the slab's rows,
 * B whole) or an N-column slab (A whole, B and C the slab's columns, col_offset a
 * multiple of 32).  Computes the slab's D = A*B + C (M x N) and writes element (r, c)
 * at (row_offset + r, col_offset + c) of every destination: D_dest[0] / Ds_dest[0] is
 * this GPU's full D / D scales, the others are the other GPUs' full buffers mapped
 * into this process (peer pointers), written while later tiles are still computing
 * (each must be this GPU's memory or imported with mpk_ipc_import, and hold the
 * M_total x N_total D; else MPK_ERR_INVALID_VALUE before any launch).  The A
 * workspace is the caller's, as for mpk_gemm_mxfp8_bf16_ws (must be non-NULL).  The
 * other GPUs' parts are in this GPU's buffer only after mpk_peer_barrier with the same
 * epoch has completed on every GPU.  No counterpart in the reference (its path has
 * no collective). */
int mpk_gemm_mxfp8_bf16_gather(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                               const uint8_t* C_data, const uint8_t* C_scales, int M, int N, int K,
                               int64_t row_offset, int64_t col_offset, int M_total, int N_total,
                               uint8_t* const* D_dest, uint8_t* const* Ds_dest, int ndest, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Stream-ordered barrier across `world` GPUs: flags[i] is GPU i's array of at least
 * `world` uint32 slots (zeroed before first use, peer-mapped); every GPU calls it
 * with the same epoch, which must increase by one from 1 on each use.  A GPU that
 * does not arrive within the wait budget makes the others record site 0x17E in
 * their device status word (mpk_device_status) and continue.  No counterpart in
 * the reference. */
int mpk_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t epoch, void* stream);

/* Sharing a device buffer with the other processes of a node (CUDA IPC), for the
 * destinations and flag arrays above.  mpk_ipc_export describes the allocation
 * holding dev_ptr: a 64-byte handle, dev_ptr's offset in it and its size.
 * mpk_ipc_import, called in another process with ITS OWN device current, maps that
 * allocation for the current device (enabling peer access to the owner) and
 * returns the address of the exported pointer; the gather and barrier entry points
 * accept only pointers of the current device's allocations or of buffers imported
 * on it.  mpk_ipc_close releases an import (reference counted).  No counterpart in
 * the reference. */
int mpk_ipc_export(const void* dev_ptr, void* handle, uint64_t* offset, uint64_t* alloc_bytes);
int mpk_ipc_import(const void* handle, uint64_t offset, uint64_t alloc_bytes, void** dev_ptr);
int mpk_ipc_close(void* dev_ptr);

/* float [M][K] -> MXFP8 along K.  Replaces mxfp8_quantize_gpu (reference
 * include/mxfp8_utils.h:38-40, src/quantize/mxfp8_quantize.cu:82-88).  Bit-exact
 * with the reference's host and device quantizers.  Any K >= 1. */
int mpk_mxfp8_quantize(const float* input, uint8_t* data, uint8_t* scales, int M, int K,
                       void* stream);

/* MXFP8 [M][K] -> float.  Replaces mxfp8_dequantize_gpu (reference
 * include/mxfp8_utils.h:46-47, src/quantize/mxfp8_dequantize.cu:22-29).  Bit-exact. */
int mpk_mxfp8_dequantize(const uint8_t* data, const uint8_t* scales, float* output, int M, int K,
                         void* stream);

/* BF16 [M][K] (bit patterns, 2-byte aligned) -> MXFP8 along K: the quantizer of
 * mpk_mxfp8_quantize applied to each value widened exactly to FP32, for producers of
 * A that hold BF16 activations.  No counterpart in the reference (its quantizer
 * takes FP32 only). */
int mpk_mxfp8_quantize_bf16(const void* input, uint8_t* data, uint8_t* scales, int M, int K,
                            void* stream);

/* float [M][K] (row-major) -> MXFP8 with the blocks along the rows: each column is
 * cut into blocks of 32 consecutive rows (the last one partial when M % 32 != 0),
 * each with one E8M0 scale.  data is [M][K] (the input's layout), scales are
 * [ceil(M/32)][K] row-major, scale of rows [32b, 32b+32) of column k at b*K + k.
 * The reference's quantize rule (src/quantize/mxfp8_quantize.cu:7-42) with the
 * block axis chosen: bit-exact with mpk_mxfp8_quantize applied to the transposed
 * tensor, transposed back.  For producers whose blocks run along the strided axis
 * (an activation stored [K][M] for an A operand, or a C built column-wise).  Any
 * M, K >= 0; input 4-byte aligned.  No counterpart in the reference (its quantizer
 * blocks along the contiguous axis only). */
int mpk_mxfp8_quantize_cols(const float* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream);

/* BF16 [M][K] (bit patterns, 2-byte aligned) -> MXFP8 with the blocks along the
 * rows, as mpk_mxfp8_quantize_cols on each value widened exactly to FP32.  No
 * counterpart in the reference. */
int mpk_mxfp8_quantize_bf16_cols(const void* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream);

/* MXFP8 [M][K] -> BF16 [M][K] (bit patterns, 2-byte aligned output): code x
 * 2^(scale-127) rounded to nearest even, which is exact for scale bytes >= 3.
 * This is the A pre-pass of mpk_gemm_mxfp8_bf16.  No counterpart in the reference
 * (its dequantizer produces FP32 only). */
int mpk_mxfp8_dequantize_bf16(const uint8_t* data, const uint8_t* scales, void* output, int M, int K,
                              void* stream);

/* Host-side utilities with the reference's semantics, for building inputs and
 * checking results on the CPU (reference include/mxfp8_utils.h:34-35, :43-44;
 * src/quantize/mxfp8_quantize.cu:116-144, src/quantize/mxfp8_dequantize.cu:32-47).
 * Host pointers.  They are never used by the device entry points above. */
int mpk_mxfp8_quantize_host(const float* input, uint8_t* data, uint8_t* scales, int M, int K);
int mpk_mxfp8_dequantize_host(const uint8_t* data, const uint8_t* scales, float* output, int M,
                              int K);

/* Reads and clears the device-side status word of the current device after
 * synchronizing it.  *device_status receives 0 when no bounded wait expired since
 * the last read, else a nonzero site code; returns MPK_ERR_DEVICE_TIMEOUT in that
 * case.  (The reference has no equivalent: its waits cannot fail.) */
int mpk_device_status(int* device_status);

/* Budget of every device-side spin wait, in nanoseconds (default 2e9). */
int mpk_set_wait_timeout_ns(uint64_t ns);

/* Launches one CTA that waits on an mbarrier nothing will arrive on, with the
 * given budget; the wait must expire and record MPK_ERR_DEVICE_TIMEOUT in the
 * device status word.  Exercises the timeout path without faulting the GPU. */
int mpk_wait_selftest(uint64_t timeout_ns, void* stream);

/* Static description of a status code, and the detail of the last failure on
 * the calling thread (mpk_last_error_string; mpk_last_error is the same function
 * under its earlier name). */
const char* mpk_status_string(int status);
const char* mpk_last_error_string(void);
const char* mpk_last_error(void);

/* Library version (major*10000 + minor*100 + patch). */
int mpk_version(void);

#ifdef __cplusplus
}
#endif

#endif /* MPK_H_ */
