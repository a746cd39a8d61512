// Inline-PTX building blocks for sm_100a: mbarriers with bounded waits, TMA
// tensor loads, tcgen05 (TMEM allocation, MMA, commit, loads) and the scalar
// MXFP8 numerics shared by the codec and the GEMM epilogue.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace mpk {

// ---------------------------------------------------------------------------
// MXFP8 scalar numerics, device side.
//
// Semantics follow the reference's header-inline helpers:
//   include/mxfp8_utils.h:8-11   e8m0 byte b -> float with bit pattern b<<23
//                                (b=0 -> 0.0, b=255 -> +inf)
//   include/mxfp8_utils.h:13-22  float -> e8m0, rounding up to a power of two
//   include/fp8_types.h:8-12     E4M3 -> float, exact
//   include/fp8_types.h:14-21    float -> E4M3: NaN -> 0x7F, clamp +-448, RNE
// ---------------------------------------------------------------------------
__device__ __forceinline__ float e8m0_to_f32(uint32_t b) { return __uint_as_float(b << 23); }

// Programmatic dependent launch.  A kernel that calls allow_dependent_launch lets
// the next kernel on its stream, if launched with programmatic stream
// serialization, start once all of this grid's blocks have called it; that
// dependent kernel calls wait_for_prerequisite_grid before touching anything this
// grid writes, which returns when this grid has completed and its memory is
// visible.  Without the launch attribute both are no-ops.
__device__ __forceinline__ void allow_dependent_launch()
{
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_for_prerequisite_grid()
{
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Two E4M3 codes (low byte = first element) -> two floats, exact.
__device__ __forceinline__ float2 e4m3x2_to_f32x2(uint32_t two_codes)
{
    uint32_t h2;
    asm("{\n\t.reg .b16 c;\n\tcvt.u16.u32 c, %1;\n\tcvt.rn.f16x2.e4m3x2 %0, c;\n\t}"
        : "=r"(h2) : "r"(two_codes));
    float lo, hi;
    asm("{\n\t.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.f32.f16 %0, l;\n\tcvt.f32.f16 %1, h;\n\t}"
        : "=f"(lo), "=f"(hi) : "r"(h2));
    return make_float2(lo, hi);
}

// The reference's clamp to +-448 followed by round-to-nearest-even into E4M3,
// with NaN -> 0x7F (include/fp8_types.h:14-21), is exactly one cvt.rn.satfinite on
// sm_100a: it saturates out-of-range values and infinities to +-448, and it turns
// every NaN, of either sign, into 0x7F.  Both were checked exhaustively on the GPU
// (all 2^32 inputs in either slot against the clamp-and-fix-up form; all NaN
// patterns give 0x7F).
// Returns two codes packed as (second << 8) | first.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float first, float second)
{
    uint32_t r;
    // cvt packs its first source into the upper byte.
    asm("{\n\t.reg .b16 c;\n\tcvt.rn.satfinite.e4m3x2.f32 c, %1, %2;\n\tcvt.u32.u16 %0, c;\n\t}"
        : "=r"(r) : "f"(second), "f"(first));
    return r;
}

// Block scale for one MX block from its amax (src/quantize/mxfp8_quantize.cu:26-37):
// the reference takes q = amax / 448 rounded to nearest, clamps it below at
// FLT_MIN, rounds it up to a power of two as an E8M0 byte s, and multiplies the
// elements by 1 / 2^(s-127).  The same bits without a division:
//   - 448 = 1.75 * 2^8 and the FP32 neighbours of 448 * 2^e lie further than half
//     an ulp of 2^e from it after the division, so for a normal quotient q is a
//     power of two exactly when amax = 448 * 2^e, and s = ceil(log2(amax / 448)) + 127
//     = (exponent field of amax) - 8 + (mantissa field of amax > 0x600000);
//   - quotients below FLT_MIN (amax < 448 * 2^-126, zero included) give s = 1;
//   - amax = +inf gives s = 255, whose scale is inf and whose inverse is 0;
//   - the inverse 2^(127-s) is exact: exponent field 254 - s, or the subnormal
//     2^-127 for s = 254.
// amax is never negative or NaN (fmaxf drops NaN).  This matches the division
// rule for every non-negative float amax (checked exhaustively, all 2^31 + 1).
__device__ __forceinline__ uint32_t mx_block_scale(float amax, float& inv)
{
    const uint32_t u = __float_as_uint(amax);
    const int t = (int)(u >> 23) - 8 + ((u & 0x7FFFFFu) > 0x600000u ? 1 : 0);
    uint32_t s = t < 1 ? 1u : (uint32_t)t;
    if (u >= 0x7F800000u) s = 255u;
    const uint32_t ib = s >= 255u ? 0u : (s == 254u ? 0x00400000u : (254u - s) << 23);
    inv = __uint_as_float(ib);
    return s;
}

// Quantize 8 floats with a precomputed 1/scale; returns 8 codes little-endian.
__device__ __forceinline__ uint2 quantize8(const float* v, float inv)
{
    uint32_t c0 = f32x2_to_e4m3x2(v[0] * inv, v[1] * inv);
    uint32_t c1 = f32x2_to_e4m3x2(v[2] * inv, v[3] * inv);
    uint32_t c2 = f32x2_to_e4m3x2(v[4] * inv, v[5] * inv);
    uint32_t c3 = f32x2_to_e4m3x2(v[6] * inv, v[7] * inv);
    return make_uint2(c0 | (c1 << 16), c2 | (c3 << 16));
}

// ---------------------------------------------------------------------------
// Shared-memory addresses and mbarriers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;"
                 :: "r"(bar), "r"(bytes) : "memory");
}

// One phase test.  If the phase is not complete the thread is suspended in
// hardware until it completes or `suspend_ns` elapses (no issue slots are spent
// spinning meanwhile).
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity, uint32_t suspend_ns = 0u)
{
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(bar), "r"(parity), "r"(suspend_ns) : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Error codes written to the device status word (see mpk.h MPK_ERR_DEVICE_TIMEOUT).
constexpr int kDevTimeoutBase = 0x100;  // + wait site id

// Bounded wait on an mbarrier phase.  Returns false (and raises the CTA's abort
// flag and the device status word) if the phase does not complete within
// timeout_ns, or if another warp of the CTA already aborted.  Each test parks the
// thread for up to 1 ms; no wait in this library can spin forever.
constexpr uint32_t kSuspendNs = 1000000u;

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, int site, uint64_t timeout_ns)
{
    if (mbar_try_wait(bar, parity, kSuspendNs)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity, kSuspendNs)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > timeout_ns) {
            *abort_flag = 1;
            if (status) atomicCAS(status, 0, kDevTimeoutBase + site);
            return false;
        }
    }
}

// ---------------------------------------------------------------------------
// TMA (tensor copies global -> shared, completion through an mbarrier)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar,
                                            int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(dst), "l"(tmap), "r"(bar), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap)
{
    asm volatile("prefetch.tensormap [%0];" :: "l"(tmap) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy (tensor core).
__device__ __forceinline__ void fence_proxy_async_smem()
{
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Order this thread's earlier generic-proxy accesses of global memory (an acquire of
// data other SMs stored) before the async-proxy accesses it issues next (bulk copies).
__device__ __forceinline__ void fence_proxy_async_global()
{
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Bulk copy (no tensor map, no multicast) of `bytes` from global memory into this
// CTA's shared memory, completing on an mbarrier of this CTA.  Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_load_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar)
{
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(dst), "l"(src), "r"(bytes), "r"(bar) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t holder_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(holder_smem), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (BF16 inputs, FP32 accumulate).
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives row
// (lane base + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
          "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr));
}

// Warp-collective load of 64 consecutive 32-bit columns of this warp's 32 TMEM lanes
// (lane i reads row i), the two-chunk form of tmem_ld_32x32b_x32.
__device__ __forceinline__ void tmem_ld_32x32b_x64(uint32_t taddr, uint32_t (&r)[64])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp-collective store of 16 consecutive 32-bit columns of this warp's 32 TMEM
// lanes (lane i writes row i).
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t* r)
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
           "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
           "r"(r[15])
        : "memory");
}

// Warp-collective store of 32 consecutive 32-bit columns of this warp's 32 TMEM
// lanes (lane i writes row i), the inverse of tmem_ld_32x32b_x32.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};"
        :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
           "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
           "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
           "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]),
           "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor for tcgen05 (sm_100 layout):
//   [0,14) start address >> 4, [16,30) leading byte offset >> 4,
//   [32,46) stride byte offset >> 4, [46,48) version = 1,
//   [49,52) base offset = 0, [52] LBO mode = 0, [61,64) layout (2 = 128-byte swizzle).
__device__ __forceinline__ uint64_t umma_smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                         uint32_t sbo_bytes)
{
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor for kind::f16: FP32 accumulator, BF16 A and B,
// A K-major, B MN-major (the reference's B is [K][N] with N contiguous).
__host__ __device__ constexpr uint32_t umma_idesc_bf16_f32(int m, int n, bool b_mn_major)
{
    return (1u << 4)                         // D format: F32
         | (1u << 7)                         // A format: BF16
         | (1u << 10)                        // B format: BF16
         | ((b_mn_major ? 1u : 0u) << 16)    // B major
         | ((uint32_t)(n >> 3) << 17)        // N / 8
         | ((uint32_t)(m >> 4) << 24);       // M / 16
}


// ---------------------------------------------------------------------------
// Thread-block clusters and the 2-CTA (cta_group::2) forms
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t cluster_id_x()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

__device__ __forceinline__ uint32_t nclusters_x()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}

// Arrive on an mbarrier that may live in a peer CTA (shared::cluster address).
// Default (release, CTA-scope) semantics: the data it publishes is shared memory
// read by the tensor core, which the writer has already made visible to the
// async proxy with fence.proxy.async.  A cluster-scope release here would also
// wait for this thread's outstanding global loads (about a microsecond).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];"
                 :: "r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                 :: "r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA load whose completion is signalled on an mbarrier of either CTA of the pair
// (`bar` is a shared::cluster address).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const void* tmap, uint32_t bar_cluster,
                                                 int32_t x, int32_t y)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];"
        :: "r"(dst), "l"(tmap), "r"(bar_cluster), "r"(x), "r"(y) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t holder_smem, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(holder_smem), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;"
                 :: "r"(taddr), "r"(ncols) : "memory");
}

// Pair MMA (issued by the even CTA): D[tmem of both CTAs] (+)= A * B, M=256 split
// 128/128 across the pair, B's N columns split in halves across the pair.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Pair MMA with A in tensor memory: each CTA's M/2 rows of A at the same column
// address of its own tensor memory (lane = row, K-major, two 16-bit elements per
// 32-bit column), B from shared memory through its descriptor.
__device__ __forceinline__ void umma_bf16_pair_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                                      uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
                 :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
                 : "memory");
}

// Arrive on the mbarrier at the same offset in every CTA of `cta_mask` once the
// pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair_mc(uint32_t bar, uint16_t cta_mask)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
                 :: "r"(bar), "h"(cta_mask) : "memory");
}

// Arrive on a local mbarrier once the pair MMAs issued so far complete.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(bar) : "memory");
}

// Per-warpgroup register reallocation (all 128 threads of the warpgroup execute it).
template <int N>
__device__ __forceinline__ void setmaxnreg_dec()
{
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" :: "n"(N));
}
template <int N>
__device__ __forceinline__ void setmaxnreg_inc()
{
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" :: "n"(N));
}

// Named barrier over a subset of warps.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads)
{
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(nthreads) : "memory");
}

// 32-bit store into a CTA of this cluster (shared::cluster address from mapa_shared).
__device__ __forceinline__ void st_shared_cluster_u32(uint32_t cluster_addr, uint32_t v)
{
    asm volatile("st.shared::cluster.u32 [%0], %1;" :: "r"(cluster_addr), "r"(v) : "memory");
}

// Cross-SM hand-off of data in global memory: the writer's red_release_gpu_add
// makes its earlier stores visible to any thread whose ld_acquire_gpu then reads
// the counter value that includes it.
__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v)
{
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

}  // namespace mpk
