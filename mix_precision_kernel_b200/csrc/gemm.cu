// D = A*B + C with A in MXFP8, B in BF16 and C/D in MXFP8 (blocks along N):
// a persistent, warp-specialised tcgen05 kernel for sm_100a.
//
// Replaces the reference's launcher gemm_fp8_tensorcore
// (src/kernels/gemm_fp8_tensorcore.cu:231-249), which runs a WMMA fp16 kernel
// into an FP32 temporary it allocates per call, then quantizes that temporary in
// a second kernel.  Here the whole path is one kernel and allocates nothing.
//
// Tile: 128 (M) x 256 (N) output per CTA, K stepped 64 at a time through a
// 4-stage shared-memory ring.  Per stage:
//   A codes  u8   128 x 64   8 KiB  TMA, 64-byte swizzle
//   A bf16        128 x 64  16 KiB  written by the transform warps, K-major,
//                                   128-byte swizzle (the UMMA canonical layout)
//   B bf16         64 x 256 32 KiB  TMA, four 64x64 boxes, 128-byte swizzle,
//                                   MN-major (B is [K][N] with N contiguous)
//   A scales      128 x 2  loaded by the transform warps from global memory
//
// Warp roles (10 warps):
//   warp 0      TMA producer (A codes + B), one elected lane
//   warp 1      TMEM owner and MMA issuer: tcgen05.mma.cta_group::1.kind::f16,
//               M=128 N=256 K=16, FP32 accumulators in TMEM, two accumulator
//               buffers of 256 columns so the epilogue of tile i overlaps the
//               mainloop of tile i+1
//   warps 2-5   transform: E4M3 code x 2^(scale-127) -> BF16, exact for scale
//               bytes 3..246 (E4M3 has 4 significant bits and BF16 8), written
//               in the swizzled K-major layout, then fence.proxy.async
//   warps 6-9   epilogue: tcgen05.ld (one thread per accumulator row, 32
//               consecutive columns = one MX block per load), + dequantized C,
//               block amax, E8M0 scale, RNE E4M3, 16-byte stores
//
// Every mbarrier wait is bounded (mpk::mbar_wait); on expiry the CTA raises an
// abort flag, records a status code, drains its in-flight TMA and MMA work with
// a second bounded wait, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "mpk.h"
#include "mpk_internal.h"
#include "mpk_ptx.cuh"

namespace mpk {
namespace gemm {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;
constexpr int STAGES = 4;
constexpr int UMMA_K = 16;
#ifndef MPK_TRANSFORM_WARPS
#define MPK_TRANSFORM_WARPS 4
#endif
constexpr int kTransformWarps = MPK_TRANSFORM_WARPS;  // 4 (one row per thread) or 8 (half rows)
constexpr int kRowParts = kTransformWarps / 4;        // transform threads per tile row
constexpr int kChunksPerThread = 4 / kRowParts;       // 16-element chunks per thread and stage
static_assert(kTransformWarps == 4 || kTransformWarps == 8, "4 or 8 transform warps");
constexpr int kEpilogueWarps = 4;
// C chunks (32 columns each) the epilogue prefetches per round: the whole 256-column
// row segment with 4 transform warps, half of it when registers are tighter.
constexpr int kCPrefetch = kTransformWarps == 4 ? 8 : 4;
constexpr int kThreads = 32 * (2 + kTransformWarps + kEpilogueWarps);
constexpr int kFirstTransformWarp = 2;
constexpr int kFirstEpilogueWarp = kFirstTransformWarp + kTransformWarps;

constexpr int A8_BYTES = BM * BK;           // 8192
constexpr int A16_BYTES = BM * BK * 2;      // 16384
constexpr int B_BOX_BYTES = 64 * BK * 2;    // one 64(N) x 64(K) box: 8192
constexpr int B_BYTES = BK * BN * 2;        // 32768
constexpr uint32_t kTxBytes = A8_BYTES + B_BYTES;
constexpr uint32_t kTmemCols = 2 * BN;      // two FP32 accumulators

constexpr int OFF_B = 0;
constexpr int OFF_A16 = OFF_B + STAGES * B_BYTES;
constexpr int OFF_A8 = OFF_A16 + STAGES * A16_BYTES;
constexpr int OFF_BAR = OFF_A8 + STAGES * A8_BYTES;
// barriers: full_tma[S], full_a16[S], empty[S], tfull[2], tempty[2], drain
constexpr int kNumBars = 3 * STAGES + 5;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int SMEM_USED = OFF_MISC + 16;
constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack for 1024-byte alignment
static_assert(SMEM_BYTES <= 232448, "exceeds the sm_100 per-block shared memory limit");

constexpr uint32_t kIdesc = umma_idesc_bf16_f32(BM, BN, /*b_mn_major=*/true);
constexpr uint64_t kDrainTimeoutNs = 200000000ull;  // teardown waits: 0.2 s

struct Params {
    const uint8_t* A_scales;
    const uint8_t* C_data;
    const uint8_t* C_scales;
    uint8_t* D_data;
    uint8_t* D_scales;
    int* status;
    uint64_t timeout_ns;
    int M, N, K;
    int nblkK, nblkN;
    int num_m_tiles, num_n_tiles, num_kb;
    int vec_cd;  // C/D rows are 16-byte aligned: vector path for full 32-column chunks
};

// Wait-site ids reported in the device status word.
enum { kSiteEmpty = 1, kSiteFullTma = 2, kSiteFullA16 = 3, kSiteTmemEmpty = 4, kSiteTmemFull = 5 };

__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& m0, int& n0)
{
    m0 = (tile % p.num_m_tiles) * BM;  // M fastest: consecutive CTAs share a B column band
    n0 = (tile / p.num_m_tiles) * BN;
}

// 16 scale bytes of one row starting at block index b0 (bytes past the row end
// or of an out-of-range row read as 0).  Issued one group of 8 k-steps ahead.
__device__ __forceinline__ uint4 load_scale_group(const uint8_t* __restrict__ row_scales, int b0,
                                                  int nblk, bool row_ok)
{
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (row_ok) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            const int b = b0 + i;
            const uint32_t v = (b < nblk) ? (uint32_t)__ldg(row_scales + b) : 0u;
            w[i >> 2] |= v << (8 * (i & 3));
        }
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

// 16 E4M3 codes with one E8M0 scale -> 16 BF16 (two 16-byte chunks), exact for
// scale bytes 3..246: code * 2^(s-127) is formed exactly in FP32 and rounded to
// BF16, where it is representable.
__device__ __forceinline__ void transform16(const uint4 q, float scale, uint4& o0, uint4& o1)
{
    uint32_t out[8];
    const uint32_t in[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int w = 0; w < 4; ++w) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const float2 f = e4m3x2_to_f32x2(in[w] >> (16 * h));
            uint32_t packed;
            asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(f.y * scale), "f"(f.x * scale));
            out[2 * w + h] = packed;
        }
    }
    o0 = make_uint4(out[0], out[1], out[2], out[3]);
    o1 = make_uint4(out[4], out[5], out[6], out[7]);
}

// Epilogue math for one MX block of 32 accumulator values of one row.
__device__ __forceinline__ uint32_t quantize_block32(float (&v)[32], uint4& c0, uint4& c1)
{
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));  // NaN ignored
    float inv;
    const uint32_t s = mx_block_scale(amax, inv);
    const uint2 q0 = quantize8(v + 0, inv), q1 = quantize8(v + 8, inv);
    const uint2 q2 = quantize8(v + 16, inv), q3 = quantize8(v + 24, inv);
    c0 = make_uint4(q0.x, q0.y, q1.x, q1.y);
    c1 = make_uint4(q2.x, q2.y, q3.x, q3.y);
    return s;
}

__global__ void __launch_bounds__(kThreads, 1)
gemm_mxfp8_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const Params p)
{
    extern __shared__ uint8_t smem_raw[];
    // Swizzled TMA destinations and UMMA descriptors need 1024-byte alignment of
    // the shared-memory address itself.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + OFF_BAR;
    auto full_tma = [&](int s) { return bar0 + 8u * s; };
    auto full_a16 = [&](int s) { return bar0 + 8u * (STAGES + s); };
    auto empty = [&](int s) { return bar0 + 8u * (2 * STAGES + s); };
    auto tfull = [&](int a) { return bar0 + 8u * (3 * STAGES + a); };
    auto tempty = [&](int a) { return bar0 + 8u * (3 * STAGES + 2 + a); };
    const uint32_t drain = bar0 + 8u * (3 * STAGES + 4);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    // Stays 0: the abort flag of the teardown waits, which must not be cut short.
    volatile int* never_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int num_tiles = p.num_m_tiles * p.num_n_tiles;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(full_tma(s), 1);
            mbar_init(full_a16(s), kTransformWarps);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), kEpilogueWarps);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        *never_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            prefetch_tmap(&tmap_a);
            prefetch_tmap(&tmap_b);
            int s = 0;
            uint32_t ph = 0;
            int issued = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x) {
                int m0, n0;
                tile_coords(p, tile, m0, n0);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status, kSiteEmpty, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
                                 :: "r"(full_tma(s)), "r"(kTxBytes) : "memory");
                    const int k0 = kb * BK;
                    tma_load_2d(sbase + OFF_A8 + s * A8_BYTES, &tmap_a, full_tma(s), k0, m0);
#pragma unroll
                    for (int j = 0; j < BN / 64; ++j)
                        tma_load_2d(sbase + OFF_B + s * B_BYTES + j * B_BOX_BYTES, &tmap_b, full_tma(s),
                                    n0 + 64 * j, k0);
                    ++issued;
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                // Let the copies already issued land before the CTA can exit.
                const int outstanding = issued < STAGES ? issued : STAGES;
                int ss = s;
                uint32_t pp = ph;
                for (int i = 0; i < outstanding; ++i) {
                    if (--ss < 0) { ss = STAGES - 1; pp ^= 1u; }
                    mbar_wait(full_tma(ss), pp, never_abort, nullptr, 0, kDrainTimeoutNs);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; ok && tile < num_tiles; tile += gridDim.x, ++it) {
                const int acc = it & 1;
                const uint32_t acc_ph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(tempty(acc), acc_ph ^ 1u, abort_flag, p.status, kSiteTmemEmpty,
                               p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = 0; kb < p.num_kb; ++kb) {
                    if (!mbar_wait(full_tma(s), ph, abort_flag, p.status, kSiteFullTma, p.timeout_ns) ||
                        !mbar_wait(full_a16(s), ph, abort_flag, p.status, kSiteFullA16, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = sbase + OFF_A16 + s * A16_BYTES;
                    const uint32_t b_addr = sbase + OFF_B + s * B_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        // A: K-major, 128-byte rows, 8-row groups 1024 B apart; a K step of
                        // 16 elements is 32 bytes inside the swizzle atom.
                        const uint64_t adesc = umma_smem_desc_sw128(a_addr + k * UMMA_K * 2, 16, 1024);
                        // B: MN-major, 64-column chunks 8 KiB apart (LBO), 8-row K groups
                        // 1024 B apart (SBO); a K step of 16 rows is 2 KiB.
                        const uint64_t bdesc = umma_smem_desc_sw128(b_addr + k * UMMA_K * 128, B_BOX_BYTES, 1024);
                        umma_bf16(d_tmem, adesc, bdesc, kIdesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    umma_commit(empty(s));
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit(tfull(acc));
            }
            // All MMAs issued by this thread complete before TMEM is released.
            umma_commit(drain);
            mbar_wait(drain, 0, never_abort, nullptr, 0, kDrainTimeoutNs);
        }
    } else if (warp < kFirstEpilogueWarp) {
        // ------------------------------- transform --------------------------------
        // Thread t owns tile row r = t % 128 and, with 8 transform warps, half of its
        // 64 K-elements per stage (one MX block).  A warp covers 32 consecutive rows,
        // which keeps the 64B-swizzled reads and 128B-swizzled writes conflict-free.
        const int t = threadIdx.x - 32 * kFirstTransformWarp;
        const int r = t & (BM - 1);
        const int part = t / BM;
        const int groups = (p.num_kb + 7) / 8;                 // 8 k-steps per scale group
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        int tile = blockIdx.x;
        int m0 = 0, n0 = 0;
        if (tile < num_tiles) tile_coords(p, tile, m0, n0);
        uint4 nxt = load_scale_group(p.A_scales + (int64_t)(m0 + r) * p.nblkK, 0, p.nblkK,
                                     tile < num_tiles && m0 + r < p.M);
        const uint32_t a8_row_off = (uint32_t)r * 64u;
        const uint32_t a8_xor = (uint32_t)((r >> 1) & 3);
        const uint32_t a16_row_off = (uint32_t)(r >> 3) * 1024u + (uint32_t)(r & 7) * 128u;
        const uint32_t a16_xor = (uint32_t)(r & 7);
        for (; ok && tile < num_tiles; tile += gridDim.x) {
            tile_coords(p, tile, m0, n0);
            for (int g = 0; ok && g < groups; ++g) {
                const uint4 cur = nxt;
                {   // prefetch the next scale group (same tile, or the first of the next tile)
                    int nt = tile, ng = g + 1;
                    if (ng == groups) { nt = tile + gridDim.x; ng = 0; }
                    int nm0 = m0, nn0;
                    if (nt < num_tiles) tile_coords(p, nt, nm0, nn0);
                    nxt = load_scale_group(p.A_scales + (int64_t)(nm0 + r) * p.nblkK, 16 * ng, p.nblkK,
                                           nt < num_tiles && nm0 + r < p.M);
                }
                const uint32_t cw[4] = {cur.x, cur.y, cur.z, cur.w};
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const int kb = g * 8 + j;
                    if (kb >= p.num_kb) break;
                    if (!mbar_wait(full_tma(s), ph, abort_flag, p.status, kSiteFullTma, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    const uint8_t* a8 = smem + OFF_A8 + s * A8_BYTES;
                    uint8_t* a16 = smem + OFF_A16 + s * A16_BYTES;
                    const uint32_t sc2 = (cw[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
                    uint4 q[kChunksPerThread];
#pragma unroll
                    for (int cc = 0; cc < kChunksPerThread; ++cc) {
                        const uint32_t c = (uint32_t)(part * kChunksPerThread + cc);
                        q[cc] = *reinterpret_cast<const uint4*>(a8 + a8_row_off + ((c ^ a8_xor) << 4));
                    }
#pragma unroll
                    for (int cc = 0; cc < kChunksPerThread; ++cc) {
                        const uint32_t c = (uint32_t)(part * kChunksPerThread + cc);
                        uint4 o0 = make_uint4(0u, 0u, 0u, 0u), o1 = o0;
                        if (kb * BK + 16 * (int)c < p.K)  // K % 16 == 0: chunks are all in or all out
                            transform16(q[cc], e8m0_to_f32((sc2 >> (8 * (c >> 1))) & 0xFFu), o0, o1);
                        *reinterpret_cast<uint4*>(a16 + a16_row_off + (((2 * c) ^ a16_xor) << 4)) = o0;
                        *reinterpret_cast<uint4*>(a16 + a16_row_off + (((2 * c + 1) ^ a16_xor) << 4)) = o1;
                    }
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(full_a16(s));
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
            }
        }
    } else {
        // -------------------------------- epilogue --------------------------------
        const int quad = warp & 3;                 // TMEM lanes this warp may access
        const int r = quad * 32 + lane;            // accumulator row within the tile
        const bool has_c = p.C_data != nullptr;
        bool aborted = false;
        int it = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++it) {
            int m0, n0;
            tile_coords(p, tile, m0, n0);
            const int acc = it & 1;
            const uint32_t acc_ph = (uint32_t)(it >> 1) & 1u;
            const int64_t grow = (int64_t)m0 + r;
            const bool row_ok = grow < p.M;
            const int nchunks = min(BN / 32, (p.N - n0 + 31) / 32);
            bool full_seen = false;
#pragma unroll
            for (int c0 = 0; c0 < BN / 32; c0 += kCPrefetch) {
                if (c0 >= nchunks) break;  // warp-uniform
                // Prefetch this row's C codes and scales for the next kCPrefetch chunks
                // (before the accumulator is ready, so the loads overlap the mainloop).
                uint4 cq[kCPrefetch][2];
                uint32_t cs[kCPrefetch];
#pragma unroll
                for (int ci = 0; ci < kCPrefetch; ++ci) {
                    const int c = c0 + ci;
                    cq[ci][0] = cq[ci][1] = make_uint4(0u, 0u, 0u, 0u);
                    cs[ci] = 0u;
                    const int col0 = n0 + 32 * c;
                    if (has_c && row_ok && c < nchunks) {
                        cs[ci] = __ldg(p.C_scales + grow * p.nblkN + col0 / 32);
                        if (p.vec_cd && col0 + 32 <= p.N) {
                            const uint4* src = reinterpret_cast<const uint4*>(p.C_data + grow * p.N + col0);
                            cq[ci][0] = __ldg(src);
                            cq[ci][1] = __ldg(src + 1);
                        }
                    }
                }
                if (!full_seen) {
                    if (!mbar_wait(tfull(acc), acc_ph, abort_flag, p.status, kSiteTmemFull, p.timeout_ns)) {
                        aborted = true;
                        break;
                    }
                    tc_fence_after();
                    full_seen = true;
                }
#pragma unroll
                for (int ci = 0; ci < kCPrefetch; ++ci) {
                    const int c = c0 + ci;
                    if (c >= nchunks) break;  // warp-uniform: tcgen05.ld is warp-collective
                    uint32_t raw[32];
                    tmem_ld_32x32b_x32(tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + 32 * c), raw);
                    tmem_ld_wait();
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
                    const int col0 = n0 + 32 * c;
                    const int valid = min(32, p.N - col0);
                    if (valid == 32 && p.vec_cd) {
                        if (has_c) {
                            const float sc = e8m0_to_f32(cs[ci]);
                            const uint32_t cw[8] = {cq[ci][0].x, cq[ci][0].y, cq[ci][0].z, cq[ci][0].w,
                                                    cq[ci][1].x, cq[ci][1].y, cq[ci][1].z, cq[ci][1].w};
#pragma unroll
                            for (int w = 0; w < 8; ++w) {
                                const float2 lo = e4m3x2_to_f32x2(cw[w]);
                                const float2 hi = e4m3x2_to_f32x2(cw[w] >> 16);
                                v[4 * w + 0] += lo.x * sc;
                                v[4 * w + 1] += lo.y * sc;
                                v[4 * w + 2] += hi.x * sc;
                                v[4 * w + 3] += hi.y * sc;
                            }
                        }
                        uint4 d0, d1;
                        const uint32_t sd = quantize_block32(v, d0, d1);
                        if (row_ok) {
                            uint4* dst = reinterpret_cast<uint4*>(p.D_data + grow * p.N + col0);
                            dst[0] = d0;
                            dst[1] = d1;
                            p.D_scales[grow * p.nblkN + col0 / 32] = (uint8_t)sd;
                        }
                    } else {
                        // Ragged or unaligned chunk: element-wise C loads and D stores.
                        if (has_c && row_ok) {
                            const float sc = e8m0_to_f32(cs[ci]);
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < valid)
                                    v[i] += e4m3x2_to_f32x2(p.C_data[grow * p.N + col0 + i]).x * sc;
                        }
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            if (i >= valid) v[i] = 0.0f;  // columns past N do not enter the amax
                        uint4 d0, d1;
                        const uint32_t sd = quantize_block32(v, d0, d1);
                        if (row_ok) {
                            const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                if (i < valid) p.D_data[grow * p.N + col0 + i] = (uint8_t)(dw[i >> 2] >> (8 * (i & 3)));
                            p.D_scales[grow * p.nblkN + col0 / 32] = (uint8_t)sd;
                        }
                    }
                }
            }
            if (aborted) break;
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty(acc));
        }
    }

    // ------------------------------- teardown -------------------------------------
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, kTmemCols);
    }
}

// Bounded-wait self test: waits on a barrier no one arrives on.
__global__ void wait_selftest_kernel(int* status, uint64_t timeout_ns)
{
    __shared__ alignas(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(smem_u32(&bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (threadIdx.x == 0) mbar_wait(smem_u32(&bar), 0, &abort_flag, status, 0x7F, timeout_ns);
}

}  // namespace gemm

// ----------------------------------------------------------------------------
// Host side
// ----------------------------------------------------------------------------

// Device status word: written only by a kernel whose bounded wait expired.
static __device__ int g_device_status;

namespace {

std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
int* g_status_ptr[64] = {};
bool g_smem_attr_set[64] = {};

int get_device(int& dev)
{
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_last_error("cudaGetDevice failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    if (dev < 0 || dev >= 64) {
        set_last_error("device ordinal %d out of range", dev);
        return MPK_ERR_INVALID_VALUE;
    }
    return MPK_SUCCESS;
}

int status_ptr(int dev, int** out)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_status_ptr[dev]) {
        void* ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_device_status);
        if (e != cudaSuccess) {
            set_last_error("cudaGetSymbolAddress(status) failed: %s", cudaGetErrorString(e));
            return (int)e;
        }
        g_status_ptr[dev] = static_cast<int*>(ptr);
    }
    *out = g_status_ptr[dev];
    return MPK_SUCCESS;
}

int get_encoder(PFN_cuTensorMapEncodeTiled_v12000* fn)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_encode) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q);
        if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !f) {
            set_last_error("cuTensorMapEncodeTiled entry point unavailable");
            return MPK_ERR_DRIVER;
        }
        g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }
    *fn = g_encode;
    return MPK_SUCCESS;
}

int encode_2d(PFN_cuTensorMapEncodeTiled_v12000 enc, CUtensorMap* map, CUtensorMapDataType dt,
              const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes, uint32_t box_inner,
              uint32_t box_outer, CUtensorMapSwizzle swz)
{
    const cuuint64_t dims[2] = {inner, outer};
    const cuuint64_t strides[1] = {row_bytes};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        set_last_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
        return MPK_ERR_DRIVER;
    }
    return MPK_SUCCESS;
}

}  // namespace

int launch_gemm_mxfp8_bf16(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                           const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                           uint8_t* D_scales, int M, int N, int K, cudaStream_t stream)
{
    using namespace gemm;
    int dev = 0, rc = get_device(dev);
    if (rc) return rc;
    int* status = nullptr;
    if ((rc = status_ptr(dev, &status))) return rc;
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    if ((rc = get_encoder(&enc))) return rc;

    CUtensorMap tmap_a, tmap_b;
    if ((rc = encode_2d(enc, &tmap_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, A_data, (uint64_t)K, (uint64_t)M,
                        (uint64_t)K, BK, BM, CU_TENSOR_MAP_SWIZZLE_64B)))
        return rc;
    if ((rc = encode_2d(enc, &tmap_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, B, (uint64_t)N, (uint64_t)K,
                        (uint64_t)N * 2, 64, BK, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;

    Params p;
    p.A_scales = A_scales;
    p.C_data = C_data;
    p.C_scales = C_scales;
    p.D_data = D_data;
    p.D_scales = D_scales;
    p.status = status;
    p.timeout_ns = wait_timeout_ns();
    p.M = M;
    p.N = N;
    p.K = K;
    p.nblkK = (K + 31) / 32;
    p.nblkN = (N + 31) / 32;
    p.num_m_tiles = (M + BM - 1) / BM;
    p.num_n_tiles = (N + BN - 1) / BN;
    p.num_kb = (K + BK - 1) / BK;
    const bool al_c = C_data == nullptr || (reinterpret_cast<uintptr_t>(C_data) & 15u) == 0;
    const bool al_d = (reinterpret_cast<uintptr_t>(D_data) & 15u) == 0;
    p.vec_cd = (N % 16 == 0 && al_c && al_d) ? 1 : 0;

    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_smem_attr_set[dev]) {
            cudaError_t e = cudaFuncSetAttribute(gemm_mxfp8_bf16_kernel,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
            if (e != cudaSuccess) {
                set_last_error("cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
                return (int)e;
            }
            g_smem_attr_set[dev] = true;
        }
    }
    const int num_tiles = p.num_m_tiles * p.num_n_tiles;
    const int grid = num_tiles < device_sm_count() ? num_tiles : device_sm_count();
    gemm_mxfp8_bf16_kernel<<<grid, kThreads, SMEM_BYTES, stream>>>(tmap_a, tmap_b, p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("GEMM launch failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    return MPK_SUCCESS;
}

int read_and_clear_device_status(int* value)
{
    int dev = 0, rc = get_device(dev);
    if (rc) return rc;
    int* status = nullptr;
    if ((rc = status_ptr(dev, &status))) return rc;
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        set_last_error("cudaDeviceSynchronize failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    int v = 0;
    e = cudaMemcpy(&v, status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) {
        const int zero = 0;
        e = cudaMemcpy(status, &zero, sizeof(int), cudaMemcpyHostToDevice);
    }
    if (e != cudaSuccess) {
        set_last_error("status copy failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    *value = v;
    return v ? MPK_ERR_DEVICE_TIMEOUT : MPK_SUCCESS;
}

int launch_wait_selftest(uint64_t timeout_ns, cudaStream_t stream)
{
    int dev = 0, rc = get_device(dev);
    if (rc) return rc;
    int* status = nullptr;
    if ((rc = status_ptr(dev, &status))) return rc;
    gemm::wait_selftest_kernel<<<1, 32, 0, stream>>>(status, timeout_ns);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("self-test launch failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    return MPK_SUCCESS;
}

}  // namespace mpk
