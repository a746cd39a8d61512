// extern "C" entry points of libmpk (declared in include/mpk.h): argument
// validation, status codes, device checks and the host-side codec utilities.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "mpk.h"
#include "mpk_internal.h"

namespace mpk {

namespace {
thread_local char t_last_error[512] = "";
std::mutex g_prop_mu;
struct DevProps { bool init = false; int sms = 0, major = 0, minor = 0; };
DevProps g_props[64];
uint64_t g_timeout_ns = 2000000000ull;

const DevProps& props()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) dev = 0;
    std::lock_guard<std::mutex> lk(g_prop_mu);
    DevProps& p = g_props[dev];
    if (!p.init) {
        cudaDeviceGetAttribute(&p.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&p.major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&p.minor, cudaDevAttrComputeCapabilityMinor, dev);
        if (p.sms <= 0) p.sms = 148;
        p.init = true;
    }
    return p;
}
}  // namespace

void set_last_error(const char* fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
    va_end(ap);
}

int device_sm_count() { return props().sms; }
int device_cc_major() { return props().major; }
int device_cc_minor() { return props().minor; }
uint64_t wait_timeout_ns() { return g_timeout_ns; }
void set_wait_timeout_ns(uint64_t ns) { g_timeout_ns = ns; }

static int check_arch()
{
    const DevProps& p = props();
    if (p.major != 10 || p.minor != 0) {
        set_last_error("libmpk is built for sm_100a; current device is sm_%d%d", p.major, p.minor);
        return MPK_ERR_ARCH;
    }
    return MPK_SUCCESS;
}

static int from_cuda(cudaError_t e, const char* what)
{
    if (e == cudaSuccess) return MPK_SUCCESS;
    set_last_error("%s: %s", what, cudaGetErrorString(e));
    return (int)e;
}

// ---------------------------------------------------------------------------
// Host-side codec (reference semantics; see include/mpk.h)
// ---------------------------------------------------------------------------
static inline uint32_t fbits(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
static inline float bitsf(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }

static float host_e8m0_to_f32(uint8_t b) { return bitsf((uint32_t)b << 23); }

static uint8_t host_e8m0_roundup(float x)
{
    if (x <= 0.0f) return 0;
    const uint32_t u = fbits(x);
    uint32_t e = (u >> 23) & 0xFFu;
    if ((u & 0x7FFFFFu) && e < 255u) ++e;
    return (uint8_t)e;
}

// Round-to-nearest-even into E4M3 after the reference's NaN test and clamp
// (include/fp8_types.h:14-21).  Normal range: round the FP32 mantissa to 3 bits
// with integer arithmetic; below 2^-6 the quantum is the fixed 2^-9.
static uint8_t host_f32_to_e4m3(float x)
{
    if (std::isnan(x)) return 0x7F;
    if (x > 448.0f) x = 448.0f;
    if (x < -448.0f) x = -448.0f;
    const uint32_t u = fbits(x);
    const uint8_t sign = (uint8_t)((u >> 24) & 0x80u);
    const uint32_t a = u & 0x7FFFFFFFu;
    if (a >= 0x3C800000u) {  // |x| >= 2^-6
        const uint32_t r = a + 0x7FFFFu + ((a >> 20) & 1u);
        const uint32_t e = (r >> 23) - 120u;  // rebias 127 -> 7
        return sign | (uint8_t)((e << 3) | ((r >> 20) & 7u));
    }
    const float q = std::nearbyint(bitsf(a) * 512.0f);  // exact scaling, RNE
    return sign | (uint8_t)q;
}

static float host_e4m3_to_f32(uint8_t v)
{
    const uint32_t e = (v >> 3) & 15u, m = v & 7u;
    float mag;
    if (e == 15u && m == 7u) mag = NAN;
    else if (e == 0u) mag = std::ldexp((float)m, -9);
    else mag = bitsf(((e + 120u) << 23) | (m << 20));
    return (v & 0x80u) ? -mag : mag;
}

}  // namespace mpk

using namespace mpk;

extern "C" {

int mpk_version(void) { return 100; }

const char* mpk_last_error_string(void) { return t_last_error; }
const char* mpk_last_error(void) { return t_last_error; }

int mpk_set_gemm_schedule(int schedule) { return gemm_set_schedule(schedule); }
int mpk_gemm_schedule(void) { return gemm_schedule(); }

int mpk_gemm_plan(int M, int N, int K, int* tiles, int* stream_k_tiles, int* stream_k_pairs)
{
    if (!tiles || !stream_k_tiles || !stream_k_pairs || M < 0 || N < 0 || K < 0) {
        set_last_error("mpk_gemm_plan: null output or negative size");
        return MPK_ERR_INVALID_VALUE;
    }
    const SkPlan plan = gemm_sk_plan(M, N, K);
    *tiles = (int)((((int64_t)M + 255) / 256) * (((int64_t)N + 255) / 256));
    *stream_k_tiles = plan.tiles;
    *stream_k_pairs = plan.clusters;
    return MPK_SUCCESS;
}

int mpk_gemm_path(const void* A_data, const void* B_bf16, int M, int N, int K, int* path)
{
    if (!path || M < 0 || N < 0 || K < 0) {
        set_last_error("mpk_gemm_path: null output or negative size");
        return MPK_ERR_INVALID_VALUE;
    }
    *path = K > 0 && M > 0 && N > 0 && gemm_default_onchip(A_data, B_bf16, M, N, K) ? MPK_PATH_ONCHIP
                                                                                  : MPK_PATH_PREPASS;
    return MPK_SUCCESS;
}

const char* mpk_status_string(int status)
{
    switch (status) {
    case MPK_SUCCESS: return "success";
    case MPK_ERR_INVALID_VALUE: return "invalid value (null pointer or negative size)";
    case MPK_ERR_UNSUPPORTED: return "shape or size not supported by this entry point";
    case MPK_ERR_MISALIGNED: return "pointer alignment not supported by this entry point";
    case MPK_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait expired";
    case MPK_ERR_ARCH: return "current device is not sm_100";
    case MPK_ERR_DRIVER: return "CUDA driver entry point or tensor-map encoding failed";
    default: return status < 1000 ? cudaGetErrorString((cudaError_t)status) : "unknown status";
    }
}

int mpk_set_wait_timeout_ns(uint64_t ns)
{
    if (ns == 0) {
        set_last_error("wait timeout must be positive");
        return MPK_ERR_INVALID_VALUE;
    }
    set_wait_timeout_ns(ns);
    return MPK_SUCCESS;
}

static int validate_gemm(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                         const uint8_t*& C_data, const uint8_t*& C_scales, uint8_t* D_data,
                         uint8_t* D_scales, int M, int N, int K, bool& nothing_to_do)
{
    nothing_to_do = false;
    if (M < 0 || N < 0 || K < 0) {
        set_last_error("negative size M=%d N=%d K=%d", M, N, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || N == 0) {
        nothing_to_do = true;
        return MPK_SUCCESS;
    }
    if (!D_data || !D_scales || (K > 0 && (!A_data || !A_scales || !B_bf16))) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    // The reference adds C only when both C pointers are set
    // (src/kernels/gemm_fp8_tensorcore.cu:188).
    if (!C_data || !C_scales) C_data = nullptr, C_scales = nullptr;
    return check_arch();
}

// Stream-ordered pool of one device for the A workspace of mpk_gemm_mxfp8_bf16.
// Its release threshold is unbounded, so after the first call of a given size the
// workspace is reused without any driver allocation; mpk_release_workspace_pool
// hands the reserve back.
namespace {
std::mutex g_pool_mu;
cudaMemPool_t g_pools[64] = {};
}  // namespace

static cudaMemPool_t workspace_pool(bool create)
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_pool_mu);
    if (!g_pools[dev] && create) {
        cudaMemPoolProps pp;
        std::memset(&pp, 0, sizeof(pp));
        pp.allocType = cudaMemAllocationTypePinned;
        pp.location.type = cudaMemLocationTypeDevice;
        pp.location.id = dev;
        cudaMemPool_t pool = nullptr;
        if (cudaMemPoolCreate(&pool, &pp) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        uint64_t keep = UINT64_MAX;
        cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
        g_pools[dev] = pool;
    }
    return g_pools[dev];
}

// Drops the current device's pool handle (after its context was destroyed).
static void forget_workspace_pool()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return;
    }
    std::lock_guard<std::mutex> lk(g_pool_mu);
    g_pools[dev] = nullptr;
}

int mpk_gemm_mxfp8_bf16(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                        const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                        uint8_t* D_scales, int M, int N, int K, void* stream)
{
    bool done = false;
    if (int rc = validate_gemm(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N, K, done))
        return rc;
    if (done) return MPK_SUCCESS;
    const cudaStream_t st = (cudaStream_t)stream;
    if (K == 0) {
        // A*B is empty: D = MXFP8(C), or MXFP8(0) without C.
        return from_cuda(launch_mxfp8_requantize(C_data, C_scales, D_data, D_scales, M, N, st),
                         "requantize launch");
    }
    // Tall products with few columns: the on-chip conversion kernel is faster than
    // the pre-pass path and needs no workspace (gemm_default_onchip).
    if (gemm_default_onchip(A_data, B_bf16, M, N, K))
        return launch_gemm_mxfp8_bf16(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N,
                                      K, st);
    // Pre-pass path.  Eager calls take the workspace from the library's pool on
    // `stream`.  While `stream` is being captured into a CUDA graph, the workspace
    // is a stream-ordered allocation of the device's default pool, which the
    // capture turns into the graph's own memory allocation and free nodes.  If no
    // workspace can be had (or the capture state cannot be read), the in-kernel
    // conversion runs instead: it needs no workspace and gives the same D.
    const size_t need = gemm_workspace_bytes(M, N, K, gemm_b_needs_copy(B_bf16, N));
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusInvalidated;
    if (cudaStreamIsCapturing(st, &cs) != cudaSuccess) {
        cudaGetLastError();
        cs = cudaStreamCaptureStatusInvalidated;
    }
    void* ws = nullptr;
    cudaError_t ae = cudaErrorNotReady;
    if (cs == cudaStreamCaptureStatusNone) {
        if (cudaMemPool_t pool = workspace_pool(true)) ae = cudaMallocFromPoolAsync(&ws, need, pool, st);
        if (ae == cudaErrorInvalidValue) {
            // The pool belonged to a context that cudaDeviceReset destroyed: make a
            // new one and try once more.
            cudaGetLastError();
            forget_workspace_pool();
            if (cudaMemPool_t pool = workspace_pool(true)) ae = cudaMallocFromPoolAsync(&ws, need, pool, st);
        }
    } else if (cs == cudaStreamCaptureStatusActive) {
        ae = cudaMallocAsync(&ws, need, st);
    }
    if (ae == cudaSuccess) {
        const int rc = launch_gemm_mxfp8_bf16_prepass(A_data, A_scales, B_bf16, C_data, C_scales, D_data,
                                                      D_scales, M, N, K, ws, need, st);
        const cudaError_t fe = cudaFreeAsync(ws, st);
        return rc ? rc : from_cuda(fe, "workspace release");
    }
    if (ae != cudaErrorNotReady) cudaGetLastError();
    if (int rc = check_onchip_gemm_shape(A_data, B_bf16, N, K)) return rc;
    return launch_gemm_mxfp8_bf16(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N,
                                  K, st);
}

int mpk_release_workspace_pool(void)
{
    cudaMemPool_t pool = workspace_pool(false);
    if (!pool) return MPK_SUCCESS;
    return from_cuda(cudaMemPoolTrimTo(pool, 0), "workspace pool trim");
}

int mpk_gemm_workspace_size(int M, int N, int K, size_t* bytes)
{
    if (!bytes || M < 0 || N < 0 || K < 0) return MPK_ERR_INVALID_VALUE;
    *bytes = gemm_workspace_bytes(M, N, K, N % 8 != 0);
    return MPK_SUCCESS;
}

int mpk_gemm_mxfp8_bf16_ws(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                           const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                           uint8_t* D_scales, int M, int N, int K, void* workspace,
                           size_t workspace_bytes, void* stream)
{
    bool done = false;
    if (int rc = validate_gemm(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N, K, done))
        return rc;
    if (done) return MPK_SUCCESS;
    if (K == 0)
        return from_cuda(launch_mxfp8_requantize(C_data, C_scales, D_data, D_scales, M, N,
                                                 (cudaStream_t)stream),
                         "requantize launch");
    if (!workspace) {
        if (int rc = check_onchip_gemm_shape(A_data, B_bf16, N, K)) return rc;
        return launch_gemm_mxfp8_bf16(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M,
                                      N, K, (cudaStream_t)stream);
    }
    const bool copy_b = gemm_b_needs_copy(B_bf16, N);
    const size_t need = gemm_workspace_bytes_min(M, N, K, copy_b);
    if (workspace_bytes < need) {
        set_last_error("workspace of %zu bytes needed%s, got %zu", need,
                       copy_b && N % 8 == 0 ? " (B is not 16-byte aligned, so a padded copy of B is "
                                              "included)" : "",
                       workspace_bytes);
        return MPK_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 15u) {
        set_last_error("workspace must be 16-byte aligned");
        return MPK_ERR_MISALIGNED;
    }
    return launch_gemm_mxfp8_bf16_prepass(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales,
                                          M, N, K, workspace, workspace_bytes, (cudaStream_t)stream);
}

int mpk_gemm_mxfp8_bf16_gather(const uint8_t* A_data, const uint8_t* A_scales, const void* B_bf16,
                               const uint8_t* C_data, const uint8_t* C_scales, int M, int N, int K,
                               int64_t row_offset, int64_t col_offset, int M_total, int N_total,
                               uint8_t* const* D_dest, uint8_t* const* Ds_dest, int ndest, void* workspace,
                               size_t workspace_bytes, void* stream)
{
    if (ndest < 1 || ndest > 8 || !D_dest || !Ds_dest) {
        set_last_error("fused all-gather needs 1..8 destinations, got %d", ndest);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M < 0 || N < 0 || M_total < 0 || row_offset < 0 || row_offset + M > (int64_t)M_total) {
        set_last_error("rows [%lld, %lld) do not fit in M_total=%d", (long long)row_offset,
                       (long long)row_offset + M, M_total);
        return MPK_ERR_INVALID_VALUE;
    }
    if (N_total < 0 || col_offset < 0 || col_offset % 32 != 0 || col_offset + N > (int64_t)N_total) {
        set_last_error("columns [%lld, %lld) do not fit in N_total=%d or do not start on an MX block",
                       (long long)col_offset, (long long)col_offset + N, N_total);
        return MPK_ERR_INVALID_VALUE;
    }
    if (N != N_total && N % 32 != 0 && col_offset + N != N_total) {
        set_last_error("a column slab must be a whole number of MX blocks unless it ends the row");
        return MPK_ERR_INVALID_VALUE;
    }
    for (int d = 0; d < ndest; ++d) {
        if (!D_dest[d] || !Ds_dest[d]) {
            set_last_error("null destination %d", d);
            return MPK_ERR_INVALID_VALUE;
        }
    }
    bool done = false;
    if (M > 0 && N > 0) {
        // Every buffer the epilogue stores into must be mapped for this GPU and hold
        // the whole M_total x N_total D (or its scales).
        const size_t d_bytes = (size_t)M_total * (size_t)N_total;
        const size_t s_bytes = (size_t)M_total * (size_t)((N_total + 31) / 32);
        for (int d = 0; d < ndest; ++d) {
            if (int rc = check_store_target(D_dest[d], d_bytes, "a D destination")) return rc;
            if (int rc = check_store_target(Ds_dest[d], s_bytes, "a D-scales destination")) return rc;
        }
    }
    if (int rc = validate_gemm(A_data, A_scales, B_bf16, C_data, C_scales, D_dest[0], Ds_dest[0], M, N, K,
                               done))
        return rc;
    if (done) return MPK_SUCCESS;
    const cudaStream_t st = (cudaStream_t)stream;
    const int64_t nblkN = (N + 31) / 32;
    if (K == 0) {
        if (N != N_total) {
            set_last_error("K == 0 with a column slab is not supported by the fused all-gather");
            return MPK_ERR_UNSUPPORTED;
        }
        for (int d = 0; d < ndest; ++d) {
            if (int rc = from_cuda(launch_mxfp8_requantize(C_data, C_scales, D_dest[d] + row_offset * N,
                                                           Ds_dest[d] + row_offset * nblkN, M, N, st),
                                   "requantize launch"))
                return rc;
        }
        return MPK_SUCCESS;
    }
    const size_t need = gemm_workspace_bytes_min(M, N, K, gemm_b_needs_copy(B_bf16, N));
    if (!workspace || workspace_bytes < need) {
        set_last_error("fused all-gather needs a workspace of %zu bytes, got %zu", need, workspace_bytes);
        return MPK_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(workspace) & 15u) {
        set_last_error("workspace must be 16-byte aligned");
        return MPK_ERR_MISALIGNED;
    }
    GatherDest g;
    std::memset(&g, 0, sizeof(g));
    g.n_extra = ndest - 1;
    g.row_offset = row_offset;
    g.col_offset = col_offset;
    g.ldd = N_total;
    for (int d = 1; d < ndest; ++d) {
        g.D_extra[d - 1] = D_dest[d];
        g.Ds_extra[d - 1] = Ds_dest[d];
    }
    return launch_gemm_mxfp8_bf16_prepass(A_data, A_scales, B_bf16, C_data, C_scales, D_dest[0], Ds_dest[0],
                                          M, N, K, workspace, workspace_bytes, st, &g);
}

int mpk_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t epoch, void* stream)
{
    if (!flags || world < 1 || world > 8 || rank < 0 || rank >= world || epoch == 0) {
        set_last_error("peer barrier: bad arguments (rank %d, world %d, epoch %u)", rank, world, epoch);
        return MPK_ERR_INVALID_VALUE;
    }
    for (int i = 0; i < world; ++i) {
        if (!flags[i] || (reinterpret_cast<uintptr_t>(flags[i]) & 3u)) {
            set_last_error("peer barrier: flag array %d is null or not 4-byte aligned", i);
            return MPK_ERR_INVALID_VALUE;
        }
        if (int rc = check_store_target(flags[i], (size_t)world * 4u, "a barrier flag array")) return rc;
    }
    if (int rc = check_arch()) return rc;
    return launch_peer_barrier(flags, rank, world, epoch, (cudaStream_t)stream);
}

int mpk_mxfp8_quantize(const float* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream)
{
    if (M < 0 || K < 0) {
        set_last_error("negative size M=%d K=%d", M, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!input || !data || !scales) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    if (int rc = check_arch()) return rc;
    return from_cuda(launch_mxfp8_quantize(input, data, scales, M, K, (cudaStream_t)stream),
                     "quantize launch");
}

int mpk_mxfp8_dequantize(const uint8_t* data, const uint8_t* scales, float* output, int M, int K,
                         void* stream)
{
    if (M < 0 || K < 0) {
        set_last_error("negative size M=%d K=%d", M, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!data || !scales || !output) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    if (int rc = check_arch()) return rc;
    return from_cuda(launch_mxfp8_dequantize(data, scales, output, M, K, (cudaStream_t)stream),
                     "dequantize launch");
}

int mpk_mxfp8_quantize_bf16(const void* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream)
{
    if (M < 0 || K < 0) {
        set_last_error("negative size M=%d K=%d", M, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!input || !data || !scales) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(input) & 1u) {
        set_last_error("BF16 input must be 2-byte aligned");
        return MPK_ERR_MISALIGNED;
    }
    if (int rc = check_arch()) return rc;
    return from_cuda(launch_mxfp8_quantize_bf16(input, data, scales, M, K, (cudaStream_t)stream),
                     "quantize-bf16 launch");
}

static int validate_cols(const void* input, const uint8_t* data, const uint8_t* scales, int M, int K,
                         size_t elem_bytes, bool& nothing_to_do)
{
    nothing_to_do = false;
    if (M < 0 || K < 0) {
        set_last_error("negative size M=%d K=%d", M, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || K == 0) {
        nothing_to_do = true;
        return MPK_SUCCESS;
    }
    if (!input || !data || !scales) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(input) % elem_bytes) {
        set_last_error("input must be %zu-byte aligned", elem_bytes);
        return MPK_ERR_MISALIGNED;
    }
    return check_arch();
}

int mpk_mxfp8_quantize_cols(const float* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream)
{
    bool done = false;
    if (int rc = validate_cols(input, data, scales, M, K, 4, done)) return rc;
    if (done) return MPK_SUCCESS;
    return from_cuda(launch_mxfp8_quantize_cols(input, data, scales, M, K, (cudaStream_t)stream),
                     "column quantize launch");
}

int mpk_mxfp8_quantize_bf16_cols(const void* input, uint8_t* data, uint8_t* scales, int M, int K, void* stream)
{
    bool done = false;
    if (int rc = validate_cols(input, data, scales, M, K, 2, done)) return rc;
    if (done) return MPK_SUCCESS;
    return from_cuda(launch_mxfp8_quantize_bf16_cols(input, data, scales, M, K, (cudaStream_t)stream),
                     "column quantize-bf16 launch");
}

int mpk_mxfp8_dequantize_bf16(const uint8_t* data, const uint8_t* scales, void* output, int M, int K,
                              void* stream)
{
    if (M < 0 || K < 0) {
        set_last_error("negative size M=%d K=%d", M, K);
        return MPK_ERR_INVALID_VALUE;
    }
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!data || !scales || !output) {
        set_last_error("null device pointer");
        return MPK_ERR_INVALID_VALUE;
    }
    if (reinterpret_cast<uintptr_t>(output) & 1u) {
        set_last_error("BF16 output must be 2-byte aligned");
        return MPK_ERR_MISALIGNED;
    }
    if (int rc = check_arch()) return rc;
    return from_cuda(launch_mxfp8_dequantize_bf16(data, scales, output, M, K, K, (cudaStream_t)stream),
                     "dequantize-bf16 launch");
}

int mpk_mxfp8_quantize_host(const float* input, uint8_t* data, uint8_t* scales, int M, int K)
{
    if (M < 0 || K < 0) return MPK_ERR_INVALID_VALUE;
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!input || !data || !scales) return MPK_ERR_INVALID_VALUE;
    const int64_t nblk = (K + 31) / 32;
    for (int64_t r = 0; r < M; ++r) {
        for (int64_t b = 0; b < nblk; ++b) {
            const int64_t k0 = b * 32, k1 = (k0 + 32 < K) ? k0 + 32 : K;
            const float* x = input + r * K;
            float amax = 0.0f;
            for (int64_t k = k0; k < k1; ++k) {
                const float a = std::fabs(x[k]);
                if (a > amax) amax = a;
            }
            float sv = amax / 448.0f;
            if (sv < 1.1754944e-38f) sv = 1.1754944e-38f;
            const uint8_t s = host_e8m0_roundup(sv);
            const float actual = host_e8m0_to_f32(s);
            const float inv = actual > 0.0f ? 1.0f / actual : 0.0f;
            scales[r * nblk + b] = s;
            for (int64_t k = k0; k < k1; ++k) data[r * K + k] = host_f32_to_e4m3(x[k] * inv);
        }
    }
    return MPK_SUCCESS;
}

int mpk_mxfp8_dequantize_host(const uint8_t* data, const uint8_t* scales, float* output, int M, int K)
{
    if (M < 0 || K < 0) return MPK_ERR_INVALID_VALUE;
    if (M == 0 || K == 0) return MPK_SUCCESS;
    if (!data || !scales || !output) return MPK_ERR_INVALID_VALUE;
    const int64_t nblk = (K + 31) / 32;
    for (int64_t r = 0; r < M; ++r)
        for (int64_t k = 0; k < K; ++k)
            output[r * K + k] = host_e4m3_to_f32(data[r * K + k]) * host_e8m0_to_f32(scales[r * nblk + k / 32]);
    return MPK_SUCCESS;
}

int mpk_device_status(int* device_status)
{
    int v = 0;
    const int rc = read_and_clear_device_status(&v);
    if (device_status) *device_status = v;
    if (rc == MPK_ERR_DEVICE_TIMEOUT) set_last_error("device wait expired at site 0x%x", v);
    return rc;
}

int mpk_wait_selftest(uint64_t timeout_ns, void* stream)
{
    if (int rc = check_arch()) return rc;
    return launch_wait_selftest(timeout_ns, (cudaStream_t)stream);
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free GEMM: mpk_gemm_mxfp8_bf16_noalloc
// ---------------------------------------------------------------------------
// Who needs it: callers that may not allocate device memory once they are running.
// A serving loop whose framework's caching allocator has reserved (nearly) all of
// HBM at start-up would see a driver or pool allocation fail or fragment memory it
// does not own; a latency-bound loop cannot afford the first-use cost of growing a
// pool (an OS mapping of new device memory) in the middle of a request; a process
// running under a fixed device-memory budget must know its footprint before its
// first request.  For them this entry point runs the same two kernels as
// mpk_gemm_mxfp8_bf16 (A pre-pass, then the tensor-core kernel) with the BF16 copy
// of A in the fixed array below, which is part of the library's device image: it
// takes MPK_NOALLOC_SCRATCH_BYTES of device memory on each device from the moment
// the image is loaded there, and the call path itself allocates nothing.  With
// CUDA's default lazy loading, the image that holds the array (this file's device
// code, which has no kernels) is loaded on a device by the first
// mpk_gemm_mxfp8_bf16_noalloc call there, when that call looks up the array's
// address: that first call is when the device memory is taken, so callers that
// reserve the device's memory for a caching allocator make one call before they do
// (or set CUDA_MODULE_LOADING=EAGER, which loads it when the CUDA context is
// created).
//
// Contents: nothing in the array has to start at zero or hold anything between
// calls.  Each call's pre-pass writes all M*K*2 bytes that the call's GEMM kernel
// then reads (rows and columns outside M x K are never read; the tensor-map loads
// fill them with zeros).
//
// Ordering: one array per device, shared by every call on that device.  Two calls
// whose kernels can be in flight at the same time (different streams without an
// event between them, or different host threads without ordering) race: one call's
// pre-pass can overwrite A while the other's GEMM reads it.  Issue the calls on one
// stream, or order them with events.
static __device__ __align__(256) uint8_t g_noalloc_scratch[MPK_NOALLOC_SCRATCH_BYTES];

// Device address of g_noalloc_scratch in the current device's context.  In host
// code the array's name is only a stand-in, so the address is asked of the runtime,
// with the device current, on every call: it is valid only for the context that
// loaded this device code, and is not kept across calls, so a context re-created
// after cudaDeviceReset gets its own array's address.  Once the code is loaded the
// lookup is a table search; the first lookup on a device (or on a re-created
// context) loads it, which is when the array is reserved.
static int noalloc_scratch(void** out)
{
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress((void**)&ptr, g_noalloc_scratch);
    if (e != cudaSuccess) return from_cuda(e, "cudaGetSymbolAddress of the no-alloc scratch");
    *out = ptr;
    return MPK_SUCCESS;
}

extern "C" int mpk_gemm_mxfp8_bf16_noalloc(const uint8_t* A_data, const uint8_t* A_scales,
                                           const void* B_bf16, const uint8_t* C_data,
                                           const uint8_t* C_scales, uint8_t* D_data,
                                           uint8_t* D_scales, int M, int N, int K, void* stream)
{
    bool done = false;
    if (int rc = validate_gemm(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N, K, done))
        return rc;
    if (done) return MPK_SUCCESS;
    const cudaStream_t st = (cudaStream_t)stream;
    if (K == 0)
        return from_cuda(launch_mxfp8_requantize(C_data, C_scales, D_data, D_scales, M, N, st),
                         "requantize launch");
    // The on-chip conversion kernel needs no workspace: it serves the shapes the
    // default entry point routes to it, and any shape whose workspace would not fit
    // the fixed scratch when the operands meet its limits.
    if (gemm_default_onchip(A_data, B_bf16, M, N, K))
        return launch_gemm_mxfp8_bf16(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N,
                                      K, st);
    const size_t need = gemm_workspace_bytes_min(M, N, K, gemm_b_needs_copy(B_bf16, N));
    if (need > (size_t)MPK_NOALLOC_SCRATCH_BYTES) {
        if (check_onchip_gemm_shape(A_data, B_bf16, N, K) == MPK_SUCCESS)
            return launch_gemm_mxfp8_bf16(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales, M, N,
                                          K, st);
        set_last_error("mpk_gemm_mxfp8_bf16_noalloc: the workspace of %zu bytes exceeds its fixed scratch "
                       "of %zu bytes (M*K <= %zu for K %% 8 == 0, N %% 8 == 0 and 16-byte aligned B), and "
                       "the on-chip conversion kernel needs K %% 16 == 0, N %% 8 == 0 and 16-byte aligned "
                       "A_data and B; use mpk_gemm_mxfp8_bf16 or mpk_gemm_mxfp8_bf16_ws",
                       need, (size_t)MPK_NOALLOC_SCRATCH_BYTES, (size_t)MPK_NOALLOC_SCRATCH_BYTES / 2);
        return MPK_ERR_UNSUPPORTED;
    }
    void* scratch = nullptr;
    if (int rc = noalloc_scratch(&scratch)) return rc;
    return launch_gemm_mxfp8_bf16_prepass(A_data, A_scales, B_bf16, C_data, C_scales, D_data, D_scales,
                                          M, N, K, scratch, (size_t)MPK_NOALLOC_SCRATCH_BYTES, st);
}
