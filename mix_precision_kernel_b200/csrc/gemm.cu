// D = A*B + C with A in MXFP8, B in BF16 and C/D in MXFP8 (blocks along N):
// persistent, warp-specialised, 2-CTA tcgen05 kernels for sm_100a.
//
// Replaces the reference's launcher gemm_fp8_tensorcore
// (src/kernels/gemm_fp8_tensorcore.cu:231-249), which runs a WMMA fp16 kernel
// into an FP32 temporary it allocates per call, then quantizes that temporary in
// a second kernel.  Here the +C and the MXFP8 quantization of D are fused into the
// GEMM's epilogue.
//
// Two kernels share the work decomposition, the pair MMA and the epilogue:
//   gemm_bf16a_mxfp8_kernel  (the default path) A was dequantized exactly to BF16
//                            by a bandwidth pre-pass (codec.cu); both operands
//                            arrive by TMA.  Optionally forwards D tiles to other
//                            GPUs (the fused all-gather).
//   gemm_mxfp8_bf16_kernel   (the allocation-free variant) A arrives as E4M3 codes
//                            and transform warps convert it to BF16 in tensor memory.
//
// Work decomposition.  Clusters of two CTAs on neighbouring SMs own 256 x 256
// output tiles (persistent, work items strided by the number of clusters, in the
// panel raster of tile_coords; the last partial wave may be cut into 256 x 128
// items, item_coords).  CTA rank r of the pair owns output rows [m0 + 128 r, +128)
// and loads only its half of the tile's B columns, [n0 + 128 r, +128): the pair MMA
// (tcgen05.mma.cta_group::2, M=256 N=256 K=16, issued by rank 0) reads A rows from
// each CTA (its shared memory, or in the on-chip variant its tensor memory) and B
// columns from both CTAs' shared memory, and writes each CTA's 128 x 256 FP32
// accumulator into that CTA's tensor memory.  Versus one CTA per 128 x 256 tile
// this halves the B bytes each SM pulls from L2 per MMA.
//
// On-chip variant, per CTA and per K-step of 64:
//   A codes  u8   128 x 64   8 KiB  TMA (64-byte swizzle) into a ring of A8_STAGES,
//                                   completes on this CTA's a8_full
//   B bf16         64 x 128 16 KiB  TMA, two 64x64 boxes, 128-byte swizzle, MN-major,
//                                   into a ring of STAGES (.cta_group::2: completes on
//                                   rank 0's full)
//   A bf16        128 x 64  32 TMEM columns (lane = row, two BF16 per column), written
//                                   by the transform warps with tcgen05.st into the
//                                   stage of the same ring; arrives on rank 0's full
// Warp roles of the on-chip variant (per CTA):
//   warp 0   B producer (one lane); warp 2 A-code producer (one lane)
//   warp 1   TMEM owner (cta_group::2 allocation); on rank 0 also the MMA issuer
//   warps 4-11 transform, two groups of 4 alternating K-steps: E4M3 code x
//            2^(scale-127) -> BF16 (exact for scale bytes 3..246), tcgen05.st, then
//            an arrive on rank 0's full
//   last 4   epilogue: tcgen05.ld of this CTA's accumulator rows, + dequantized C,
//            per-32-column amax, E8M0 scale, RNE E4M3, 16-byte stores
// (The BF16-A kernel's ring and roles are described at its definition.)
//
// Every mbarrier wait is bounded (mpk::mbar_wait*); on expiry the CTA raises an
// abort flag, records a status code, drains the copies and MMAs it has in
// flight with a second bounded wait, frees TMEM and exits.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "mpk.h"
#include "mpk_internal.h"
#include "mpk_ptx.cuh"

namespace mpk {
namespace gemm {

constexpr int BM = 128;        // rows per CTA; the pair covers 2*BM
constexpr int PAIR_M = 2 * BM;
#ifndef MPK_PANEL_M
#define MPK_PANEL_M 8
#endif
constexpr int kPanelM = MPK_PANEL_M;  // M tiles per raster panel (tile_coords)
constexpr int kMaxGatherDest = 8;      // destinations of the fused all-gather (GPUs)
constexpr int BN = 256;        // output columns per tile (each CTA loads BN/2 of B)
constexpr int BN_HALF = BN / 2;
constexpr int BK = 64;
// On-chip variant: a stage is a K block of OC_BK = 2 K-steps (one barrier wait and
// one commit per 8 MMAs); ring of STAGES blocks consumed by the MMA (B halves in
// shared memory and the converted BF16 A tile in tensor memory per stage) and ring
// of A8_STAGES A-code blocks consumed by the transform.
constexpr int OC_KSTEPS = 2;
constexpr int OC_BK = OC_KSTEPS * 64;
#ifndef MPK_STAGES
#define MPK_STAGES 4
#endif
constexpr int STAGES = MPK_STAGES;
#ifndef MPK_A8_STAGES
#define MPK_A8_STAGES 4
#endif
constexpr int A8_STAGES = MPK_A8_STAGES;
constexpr int UMMA_K = 16;

#ifndef MPK_TRANSFORM_GROUPS
#define MPK_TRANSFORM_GROUPS 2
#endif
// Transform warps come in groups of 4 (one thread per tile row).  Group g converts
// the K-steps kb with kb % G == g, so G stages are in conversion at once and each
// group's per-stage latencies (fence, arrive, waits) overlap the others' work.
constexpr int kTransformGroups = MPK_TRANSFORM_GROUPS;
static_assert(kTransformGroups == 1 || kTransformGroups == 2 || kTransformGroups == 4, "1, 2 or 4");
constexpr int kTransformWarps = 4 * kTransformGroups;
constexpr int kEpilogueWarps = 4;
// Warpgroup-aligned layout: warps 0-3 control (B producer, MMA/TMEM, A-code
// producer, one idle), then the transform groups, then the epilogue warpgroup.
constexpr int kFirstTransformWarp = 4;
#ifndef MPK_B_PRODUCER_WARP
#define MPK_B_PRODUCER_WARP 0
#endif
constexpr int kBProducerWarp = MPK_B_PRODUCER_WARP;  // 0 or 3 (the other one idles)
static_assert(kBProducerWarp == 0 || kBProducerWarp == 3, "warp 0 or 3");
constexpr int kFirstEpilogueWarp = kFirstTransformWarp + kTransformWarps;
constexpr int kThreads = 32 * (kFirstEpilogueWarp + kEpilogueWarps);
// Register split per warpgroup (setmaxnreg): the launch gives every thread
// kLaunchRegs; control warps drop to kCtrlRegs, transform warps to kXformRegs and
// the epilogue rises to kEpiRegs.  The sum never exceeds the launch allocation
// (checked below), and the launcher verifies the compiled register count before
// it launches, so setmaxnreg.inc can always be satisfied.
constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8 > 255 ? 248 : (65536 / kThreads) / 8 * 8;
constexpr int kCtrlRegs = 48;
constexpr int kXformRegs = kTransformGroups == 4 ? 72 : kLaunchRegs;
constexpr int kEpiRegs = (kThreads * kLaunchRegs - 128 * kCtrlRegs - 32 * kTransformWarps * kXformRegs) /
                         128 / 8 * 8 > 248 ? 248
                       : (kThreads * kLaunchRegs - 128 * kCtrlRegs - 32 * kTransformWarps * kXformRegs) / 128 / 8 * 8;
static_assert(128 * kCtrlRegs + 32 * kTransformWarps * kXformRegs + 128 * kEpiRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
#ifndef MPK_C_PREFETCH
#define MPK_C_PREFETCH (kEpiRegs >= 160 ? 8 : 4)
#endif
constexpr int kCPrefetch = MPK_C_PREFETCH;  // C chunks (32 columns) prefetched per round

constexpr int A8_BYTES = BM * OC_BK;            // on-chip A codes per CTA and stage: 16384
constexpr int A16_BYTES = BM * BK * 2;          // 16384
constexpr int B_BOX_BYTES = 64 * BK * 2;        // one 64(N) x 64(K) box: 8192
constexpr int B_BYTES = BK * BN_HALF * 2;       // 16384 per CTA
constexpr uint32_t kTmemCols = 2 * BN;          // all 512 columns of tensor memory

// On-chip variant's tensor memory (per CTA, 128 lanes = the CTA's 128 tile rows):
// one FP32 accumulator of BN columns, then the BF16 A ring: one stage per K block,
// 64 columns (128 BF16 of a row, two per 32-bit column).  Pair MMAs of N = 128 (two
// per K slice into two half accumulators) run at about two thirds of the rate of
// N = 256 on B200, so the tile keeps one N = 256 accumulator and the epilogue's
// drain is not overlapped with the next tile's MMAs.
constexpr uint32_t kTmemACol = BN;
constexpr uint32_t kTmemAStageCols = OC_BK / 2;
static_assert(kTmemACol + STAGES * kTmemAStageCols <= kTmemCols, "tensor memory holds 512 columns");

constexpr int OC_B_BYTES = OC_KSTEPS * B_BYTES;  // on-chip B per CTA and stage: 32768
constexpr int OFF_B = 0;
constexpr int OFF_A8 = OFF_B + STAGES * OC_B_BYTES;
constexpr int OFF_BAR = OFF_A8 + A8_STAGES * A8_BYTES;
// barriers: a8_full[S8], a8_empty[S8], full[S], empty[S], tfull, tempty, drain
constexpr int kNumBars = 2 * A8_STAGES + 2 * STAGES + 3;
constexpr int OFF_MISC = OFF_BAR + kNumBars * 8;
constexpr int SMEM_USED = OFF_MISC + 16;
constexpr int SMEM_BYTES = SMEM_USED + 1024;  // slack for 1024-byte alignment
static_assert(SMEM_BYTES <= 232448, "exceeds the sm_100 per-block shared memory limit");
static_assert(A8_STAGES >= STAGES, "the transform's phase waits assume A8_STAGES >= STAGES");

// Pair MMA: M = 256 across the two CTAs, N = 256 (N = 128 for split tail tiles),
// B MN-major.
constexpr uint32_t kIdesc = umma_idesc_bf16_f32(PAIR_M, BN, /*b_mn_major=*/true);
constexpr uint32_t kIdescHalf = umma_idesc_bf16_f32(PAIR_M, BN / 2, /*b_mn_major=*/true);
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
    int num_kb2;  // on-chip kernel: K blocks of OC_BK (two K-steps)
    // Work items (item_coords): items below split_from are whole tiles in raster
    // order; the remaining raster tiles are each cut into two 256 x 128 items.
    int num_items, split_from;
    int panel_m;  // M tiles per raster panel (tile_coords)
    int vec_cd;   // C/D rows are 16-byte aligned: vector path for full 32-column chunks
    // Fused all-gather (kernels instantiated with kGather only): element (r, c) of
    // this product is written at (row_offset + r, col_offset + c) of D_data and of
    // every D_extra[i] (other GPUs' full-D buffers, reached by peer stores over
    // NVLink), whose rows are ldd bytes apart (scale rows lds apart); col_offset is
    // a multiple of 32.  C is read at (r, c) of this product.
    int n_extra;
    int64_t row_offset, col_offset, ldd, lds;
    uint8_t* D_extra[kMaxGatherDest - 1];
    uint8_t* Ds_extra[kMaxGatherDest - 1];
    // Stream-K (BF16-A kernel; sk_tiles == 0 disables it).  The first sk_tiles tiles
    // of the raster are not whole work items: their sk_iters = sk_tiles * num_kb
    // K-steps, taken in raster order, are cut into sk_clusters contiguous ranges,
    // one per cluster (sk_range_start).  A tile whose K-steps fall into several
    // ranges is finished by the cluster holding its last K-steps (the owner); the
    // others (contributors) store their FP32 partial sums into sk_partial (one slot
    // of kSkSlotFloats per contributing CTA) and count their arrival in sk_sync.
    // sk_sync[0] hands out the clusters' logical indices in start order; the A
    // pre-pass zeroes sk_sync[0 .. 1 + 2 * sk_clusters) before the kernel reads it.
    int sk_tiles, sk_clusters;
    int64_t sk_iters;
    float* sk_partial;
    uint32_t* sk_sync;
};

// Wait-site ids reported in the device status word.
enum { kSiteEmpty = 1, kSiteFullB = 2, kSiteFullA16 = 3, kSiteTmemEmpty = 4, kSiteTmemFull = 5,
       kSiteFullA8 = 6, kSiteEmptyA8 = 7, kSiteEmptyT = 8, kSiteEpiDone = 9, kSiteCopy = 10,
       kSitePartials = 11 };

// One stream-K partial: a CTA's 128 x 256 FP32 accumulator, stored as
// [chunk of 32 columns][quad of 4 columns][row][4], so that thread r (row r) of a
// warp stores and loads consecutive 16-byte pieces.
constexpr int kSkSlotFloats = BM * BN;
constexpr uint32_t kSkArrivals = kEpilogueWarps * 32;  // every epilogue thread of a contributing CTA arrives

// Tile order for L2 reuse.  The tile grid is cut into panels of panel_m M tiles;
// within a panel tiles go M fastest, then N.  The tiles in flight at once (one per
// cluster, consecutive indices) then form a panel_m x (clusters / panel_m)
// rectangle, so each A row band and each B column band they read is fetched from
// HBM about once per wave and shared through L2 -- rather than once per tile, as
// in a single row or column of 74 tiles (A or B re-read per tile column/row).
__device__ __forceinline__ void tile_coords(const Params& p, int tile, int& m0, int& n0)
{
    const int per_panel = p.panel_m * p.num_n_tiles;
    const int panel = tile / per_panel;
    const int r = tile - panel * per_panel;
    const int rows = min(p.panel_m, p.num_m_tiles - panel * p.panel_m);  // last panel may be short
    m0 = (panel * p.panel_m + r % rows) * PAIR_M;
    n0 = (r / rows) * BN;
}

// Work item -> tile origin; returns the item's width (BN, or BN / 2 for the halves
// of a split tail tile).  With 768 tiles on 74 clusters the eleventh wave would run
// 28 tiles on 74 clusters; as 56 half tiles it takes half as long.
__device__ __forceinline__ int item_coords(const Params& p, int item, int& m0, int& n0)
{
    if (item < p.split_from) {
        tile_coords(p, item, m0, n0);
        return BN;
    }
    const int j = item - p.split_from;
    tile_coords(p, p.split_from + (j >> 1), m0, n0);
    n0 += (j & 1) * (BN / 2);
    return BN / 2;
}

// ---------------------------------------------------------------------------
// Work units of the BF16-A kernel.  Every role of a CTA (producer, MMA issuer,
// epilogue, copy warps) walks the same sequence: first this cluster's stream-K
// range, from its last K-step down (so the partial sums other clusters wait for
// are computed first and the unit this cluster finishes comes last), then whole
// items strided across the clusters.
// ---------------------------------------------------------------------------
enum { kUnitWhole = 0, kUnitContrib = 1, kUnitOwner = 2 };

struct Unit {
    int m0, n0, bn;     // tile origin and width
    int kb0, kb1;       // K-steps [kb0, kb1)
    int kind;           // kUnitWhole: all K-steps; kUnitContrib: store a partial; kUnitOwner: finish the tile
    int first_contrib;  // owner: clusters first_contrib .. (this cluster - 1) hold the tile's other partials
};

__device__ __forceinline__ int64_t sk_range_start(const Params& p, int c)
{
    return (int64_t)c * p.sk_iters / p.sk_clusters;
}

struct UnitWalk {
    int64_t lo, hi;  // stream-K K-steps still to do: [lo, hi), taken from the top
    int item, stride, cluster;

    __device__ __forceinline__ UnitWalk(const Params& p, int c, int nclusters)
        : lo(0), hi(0), item(p.sk_tiles + c), stride(nclusters), cluster(c)
    {
        if (c < p.sk_clusters) {
            lo = sk_range_start(p, c);
            hi = sk_range_start(p, c + 1);
        }
    }

    __device__ __forceinline__ bool next(const Params& p, Unit& u)
    {
        if (hi > lo) {
            const int t = (int)((hi - 1) / p.num_kb);
            const int64_t t0 = (int64_t)t * p.num_kb;  // the tile's first K-step
            const int64_t b = lo > t0 ? lo : t0;
            tile_coords(p, t, u.m0, u.n0);
            u.bn = BN;
            u.kb0 = (int)(b - t0);
            u.kb1 = (int)(hi - t0);
            u.kind = u.kb1 < p.num_kb ? kUnitContrib : (u.kb0 > 0 ? kUnitOwner : kUnitWhole);
            u.first_contrib = cluster;
            if (u.kind == kUnitOwner) {
                // Ranges are contiguous and non-empty: the tile's earlier K-steps lie in
                // the ranges of clusters cluster-1, cluster-2, ... down to the one whose
                // range contains t0.  Each of them computes this tile first.
                int c = cluster - 1;
                while (c > 0 && sk_range_start(p, c) > t0) --c;
                u.first_contrib = c;
            }
            hi = b;
            return true;
        }
        if (item < p.num_items) {
            u.bn = item_coords(p, item, u.m0, u.n0);
            u.kb0 = 0;
            u.kb1 = p.num_kb;
            u.kind = kUnitWhole;
            u.first_contrib = cluster;
            item += stride;
            return true;
        }
        return false;
    }
};

// Partial slot of CTA `rank` of cluster `cluster`.
__device__ __forceinline__ float4* sk_slot(const Params& p, int cluster, uint32_t rank)
{
    return reinterpret_cast<float4*>(p.sk_partial + (size_t)(cluster * 2 + (int)rank) * kSkSlotFloats);
}

// Owner side: wait until every contributor CTA of this rank has arrived (bounded).
__device__ __forceinline__ bool sk_wait_partials(const Params& p, int c_first, int c_last, uint32_t rank,
                                                 volatile int* abort_flag)
{
    for (int c = c_last; c >= c_first; --c) {
        const uint32_t* cnt = p.sk_sync + 1 + 2 * c + (int)rank;
        if (ld_acquire_gpu(cnt) >= kSkArrivals) continue;
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu(cnt) < kSkArrivals) {
            if (*abort_flag) return false;
            if (globaltimer_ns() - t0 > p.timeout_ns) {
                *abort_flag = 1;
                atomicCAS(p.status, 0, kDevTimeoutBase + kSitePartials);
                return false;
            }
            __nanosleep(128);
        }
    }
    return true;
}

// Owner side.  The contributors' partials reach the owner through a staging area
// of `slots` pieces of 16 KiB in shared memory (one contributor's 32 columns x
// 128 rows, contiguous in its partial): piece i = 32-column chunk i / n of
// contributor c_last - i % n (n contributors, highest K range first) goes to slot
// i % slots.  Warp 2 (idle otherwise) waits for the contributors' arrivals, then
// streams the pieces in by bulk copies, refilling a slot once all 128 epilogue
// threads have read it; it starts as soon as the partials are there, so the first
// pieces are usually in shared memory before the owner's own accumulator is done.
// The epilogue adds them chunk by chunk while it finishes the tile.  Reading the
// partials through bulk copies keeps `slots` x 16 KiB in flight without spending
// registers, which is what the merge needs: it is bound by the latency of L2.
constexpr uint32_t kSkPieceBytes = BM * 32 * 4;

struct MergeStage {
    const uint8_t* stage;      // slots x kSkPieceBytes of shared memory
    int slots;
    uint32_t pfull0, pempty0;  // slots' full (1 arrival + bytes) and empty (128 arrivals) barriers
    volatile int* never_abort;
};

// Warp 2, one lane: the bulk copies of this cluster's owner unit's partials (if
// the cluster has an owner unit and this CTA has rows of it).
__device__ __noinline__ void sk_issue_merge(const Params& p, int cluster, int nclusters, uint32_t rank,
                                            const MergeStage ms, volatile int* abort_flag)
{
    UnitWalk walk(p, cluster, nclusters);
    Unit u;
    bool found = false;
    while (walk.hi > walk.lo && walk.next(p, u))
        if (u.kind == kUnitOwner) {
            found = true;
            break;
        }
    if (!found || (int64_t)u.m0 + BM * (int)rank >= p.M) return;
    const int c_first = u.first_contrib, c_last = cluster - 1, n = c_last - c_first + 1;
    const int nchunks = min(BN / 32, (p.N - u.n0 + 31) / 32);
    if (!sk_wait_partials(p, c_first, c_last, rank, abort_flag)) return;
    fence_proxy_async_global();  // the bulk copies read what the acquires made visible
    const uint32_t stage_s = smem_u32(ms.stage);
    const int npieces = n * nchunks;
    int issued = 0;
    bool ok = true;
    for (int i = 0; i < npieces; ++i) {
        const int slot = i % ms.slots;
        if (i >= ms.slots) {  // the slot's previous piece must have been read by every thread
            ok = mbar_wait(ms.pempty0 + 8u * slot, (uint32_t)(i / ms.slots - 1) & 1u, abort_flag, p.status,
                           kSitePartials, p.timeout_ns);
            if (!ok) break;
        }
        const float4* src = sk_slot(p, c_last - i % n, rank) + (size_t)(i / n) * 8 * BM;
        mbar_arrive_expect_tx(ms.pfull0 + 8u * slot, kSkPieceBytes);
        bulk_load_g2s(stage_s + (uint32_t)slot * kSkPieceBytes, src, kSkPieceBytes, ms.pfull0 + 8u * slot);
        ++issued;
    }
    if (!ok) {
        // Copies in flight land before shared memory can be released.
        for (int i = issued > ms.slots ? issued - ms.slots : 0; i < issued; ++i)
            mbar_wait(ms.pfull0 + 8u * (i % ms.slots), (uint32_t)(i / ms.slots) & 1u, ms.never_abort, nullptr, 0,
                      kDrainTimeoutNs);
    }
}

// Epilogue side: add the n pieces of 32-column chunk `chunk` to this thread's row
// (v), releasing their slots.  Returns false if a bounded wait gave up.
__device__ __forceinline__ bool sk_add_pieces(const Params& p, const MergeStage& ms, int n, int chunk, int r,
                                              bool row_ok, float (&v)[32], volatile int* abort_flag)
{
    for (int j = 0; j < n; ++j) {
        const int i = chunk * n + j;
        const int slot = i % ms.slots;
        if (!mbar_wait(ms.pfull0 + 8u * slot, (uint32_t)(i / ms.slots) & 1u, abort_flag, p.status, kSitePartials,
                       p.timeout_ns))
            return false;
        if (row_ok) {
            const float4* x = reinterpret_cast<const float4*>(ms.stage + (size_t)slot * kSkPieceBytes) + r;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const float4 y = x[q * BM];
                v[4 * q + 0] += y.x;
                v[4 * q + 1] += y.y;
                v[4 * q + 2] += y.z;
                v[4 * q + 3] += y.w;
            }
        }
        mbar_arrive(ms.pempty0 + 8u * slot);
    }
    return true;
}

// Contributor side: store this CTA's accumulator (this warp's lane quarter `tacc`)
// as its partial, rows past M skipped; warp-collective.
__device__ __noinline__ void sk_store_partial(float4* slot_row, uint32_t tacc, bool row_ok, int nchunks)
{
#pragma unroll 1
    for (int c = 0; c < nchunks; c += 2) {  // two chunks per tensor-memory wait
        const bool two = c + 1 < nchunks;
        uint32_t raw[2][32];
        tmem_ld_32x32b_x32(tacc + 32u * c, raw[0]);
        if (two) tmem_ld_32x32b_x32(tacc + 32u * (c + 1), raw[1]);
        tmem_ld_wait();
        if (row_ok) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (h == 1 && !two) break;
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    __stcg(slot_row + (size_t)((c + h) * 8 + q) * BM,
                           make_float4(__uint_as_float(raw[h][4 * q]), __uint_as_float(raw[h][4 * q + 1]),
                                       __uint_as_float(raw[h][4 * q + 2]), __uint_as_float(raw[h][4 * q + 3])));
            }
        }
    }
}

// 16 scale bytes of one row starting at block index b0 (bytes past the row end
// or of an out-of-range row read as 0).  Issued one group of 8 k-steps ahead, the
// result first used a group later, so the loads' latency overlaps the conversion
// of the current group: `width` 16 (the row's scale bytes 16-byte aligned and a
// whole number of groups long) one 16-byte load; 4 (4-byte aligned, a whole number
// of 4-byte words) four word loads, words past the row end skipped; otherwise byte
// loads packed on the spot (their latency exposed).
__device__ __forceinline__ uint4 load_scale_group(const uint8_t* __restrict__ row_scales, int b0,
                                                  int nblk, bool row_ok, int width)
{
    if (!row_ok) return make_uint4(0u, 0u, 0u, 0u);
    if (width == 16) return __ldg(reinterpret_cast<const uint4*>(row_scales + b0));
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    if (width == 4) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
            if (b0 + 4 * i < nblk) w[i] = __ldg(reinterpret_cast<const uint32_t*>(row_scales + b0 + 4 * i));
        return make_uint4(w[0], w[1], w[2], w[3]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int b = b0 + i;
        const uint32_t v = (b < nblk) ? (uint32_t)__ldg(row_scales + b) : 0u;
        w[i >> 2] |= v << (8 * (i & 3));
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel)
{
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b)
{
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

// One row of one K block of the on-chip variant: 128 E4M3 codes (eight 16-code
// chunks) with four E8M0 scale bytes packed in `scales` (byte q for codes
// 32q .. 32q+31) -> 128 BF16, packed two per 32-bit word in K order (word j = codes
// 2j, 2j+1, the lower one in the low half), which is the row's layout in a
// tensor-memory A operand (lane = row, 32-bit column j).
//
// Exact general path: E4M3 -> f16 -> f32 with hardware conversions, multiply by
// the FP32 scale (byte 0 -> 0.0 and 255 -> inf, as in the reference), round to
// BF16; codes at K offset >= kvalid become zeros.  Used for scale bytes outside
// 3..134, NaN codes and the K tail; kept out of line so the hot loop stays small.
__device__ __noinline__ void convert_block_exact(const uint8_t* a8row, uint32_t a8xr, uint32_t scales, int kvalid,
                                                 uint32_t* out)
{
#pragma unroll 1
    for (int c = 0; c < OC_BK / 16; ++c) {
        // Chunk c (codes 16c .. 16c+15), re-read from the 128-byte swizzled code row.
        const uint4 qc = *reinterpret_cast<const uint4*>(a8row + ((((uint32_t)c) ^ a8xr) << 4));
        const uint32_t in[4] = {qc.x, qc.y, qc.z, qc.w};
        const float scale = e8m0_to_f32((scales >> (8 * (c / 2))) & 0xFFu);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int k = 16 * c + 4 * w + 2 * h;  // K offset of the pair's first code
                const float2 f = e4m3x2_to_f32x2(in[w] >> (16 * h));
                const float lo = k < kvalid ? f.x * scale : 0.0f;
                const float hi = k + 1 < kvalid ? f.y * scale : 0.0f;
                uint32_t packed;
                asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(packed) : "f"(hi), "f"(lo));
                out[8 * c + 2 * w + h] = packed;
            }
        }
    }
}

// Fast path for one row of one K block (same contract as convert_block_exact),
// valid when the scale bytes of the 32-code blocks holding codes inside K are in
// 3..134 and no code is NaN (0x7F/0xFF): fast_block_ok checks this on the eight
// 16-code chunks q[0..7], and convert_half_fast converts 32 codes (two chunks, one
// scale byte s) to 16 words.  Codes past K are zeros (the TMA load fills them), and
// their scale bytes read 0 (2^-7 as a factor), so they convert to +0 as on the exact
// path.
// Each code's sign and 7 magnitude bits are moved into a BF16 bit pattern equal to
// code x 2^-120 (the E4M3 exponent bits land in the low BF16 exponent bits; E4M3
// subnormals become BF16 subnormals); one BF16 multiply by 2^(s-7) -- a power of
// two, so exact -- gives code x 2^(s-127).  Integer ops and mul.rn.bf16x2 only:
// per pair of codes one prmt puts each code byte in the low byte of a 16-bit lane
// with its sign bit replicated through the high byte, a shift by 4 moves the 7
// magnitude bits to bits 4..10 (the sign copies to bits 11..15, and the low lane's
// top nibble into the high lane's bits 0..3), and the mask 0x87F0 per lane keeps
// the magnitude and bit 15.
__device__ __forceinline__ bool fast_block_ok(const uint4 (&q)[OC_BK / 16], uint32_t scales, int kvalid)
{
    uint32_t nan_probe = 0u;
#pragma unroll
    for (int c = 0; c < OC_BK / 16; ++c) {
        const uint32_t in[4] = {q[c].x, q[c].y, q[c].z, q[c].w};
#pragma unroll
        for (int w = 0; w < 4; ++w) nan_probe |= (in[w] & 0x7F7F7F7Fu) + 0x01010101u;  // 0x7F -> 0x80
    }
    bool ok = (nan_probe & 0x80808080u) == 0u;
#pragma unroll
    for (int b = 0; b < OC_BK / 32; ++b)
        ok = ok && (32 * b >= kvalid || (((scales >> (8 * b)) & 0xFFu) - 3u) <= 131u);
    return ok;
}

__device__ __forceinline__ void convert_half_fast(uint4 qa, uint4 qb, uint32_t s, uint32_t (&out)[16])
{
    uint32_t f = (s + 120u) << 7;  // BF16 2^(s-7)
    f |= f << 16;
    const uint32_t in[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        const uint32_t b01 = prmt(in[w], 0u, 0x9180u);  // codes 0, 1: byte, sign fill
        const uint32_t b23 = prmt(in[w], 0u, 0xB3A2u);  // codes 2, 3
        out[2 * w] = mul_bf16x2((b01 << 4) & 0x87F087F0u, f);
        out[2 * w + 1] = mul_bf16x2((b23 << 4) & 0x87F087F0u, f);
    }
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

// Ragged or unaligned 32-column chunk of one accumulator row: loads the chunk
// from TMEM itself (warp-collective; every lane calls this together), element-wise
// C loads and D stores, columns past N kept out of the block amax.  Out of line to
// keep the epilogue's hot code small.
// A stream-K owner's chunk (n_merge > 0) also adds its contributors' pieces; returns
// false if that gave up waiting (the warp then leaves the tile together).
template <bool kGather>
__device__ __noinline__ bool epilogue_ragged_chunk(const Params& p, uint32_t taddr, uint32_t cscale,
                                                   bool has_c, bool row_ok, int64_t grow, int col0,
                                                   int valid, const MergeStage* ms, int n_merge, int chunk,
                                                   int r, volatile int* abort_flag)
{
    uint32_t raw[32];
    tmem_ld_32x32b_x32(taddr, raw);
    tmem_ld_wait();
    float v[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
    if (n_merge > 0) {
        const bool ok = sk_add_pieces(p, *ms, n_merge, chunk, r, row_ok, v, abort_flag);
        if (!__all_sync(0xFFFFFFFFu, ok)) return false;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = (i < valid) ? v[i] : 0.0f;
    if (has_c && row_ok) {
        const float sc = e8m0_to_f32(cscale);
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < valid) v[i] += e4m3x2_to_f32x2(p.C_data[grow * p.N + col0 + i]).x * sc;
    }
    uint4 d0, d1;
    const uint32_t sd = quantize_block32(v, d0, d1);
    if (row_ok) {
        const uint32_t dw[8] = {d0.x, d0.y, d0.z, d0.w, d1.x, d1.y, d1.z, d1.w};
        const int64_t doff = kGather ? (grow + p.row_offset) * p.ldd + p.col_offset + col0 : grow * p.N + col0;
        const int64_t soff = kGather ? (grow + p.row_offset) * p.lds + (p.col_offset + col0) / 32
                                     : grow * p.nblkN + col0 / 32;
#pragma unroll
        for (int i = 0; i < 32; ++i)
            if (i < valid) p.D_data[doff + i] = (uint8_t)(dw[i >> 2] >> (8 * (i & 3)));
        p.D_scales[soff] = (uint8_t)sd;
    }
    return true;
}

// Adds one full 32-column chunk of C (32 E4M3 codes in c0, c1 and their scale
// byte) to the accumulator values v.
__device__ __forceinline__ void add_c_chunk(float (&v)[32], uint4 c0, uint4 c1, uint32_t cscale)
{
    const float sc = e8m0_to_f32(cscale);
    const uint32_t cw[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
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

// One full 32-column D chunk (two 16-byte stores) and its scale byte, into this
// GPU's D (in the fused all-gather, at the slab's row offset of the full D; the
// copy warps forward it to the other GPUs).
template <bool kGather>
__device__ __forceinline__ void store_d_chunk(const Params& p, int64_t grow, int col0, uint4 d0, uint4 d1,
                                              uint32_t sd)
{
    const int64_t doff = kGather ? (grow + p.row_offset) * p.ldd + p.col_offset + col0 : grow * p.N + col0;
    const int64_t soff = kGather ? (grow + p.row_offset) * p.lds + (p.col_offset + col0) / 32
                                 : grow * p.nblkN + col0 / 32;
    uint4* dst = reinterpret_cast<uint4*>(p.D_data + doff);
    dst[0] = d0;
    dst[1] = d1;
    p.D_scales[soff] = (uint8_t)sd;
}

// Fused all-gather, copy warps: forward one finished tile's D rows of this CTA
// (128 rows x up to 256 columns, and their scale bytes) from this GPU's D to every
// other destination.  Lanes of the copying warps take consecutive 16-byte pieces of
// a row, so each store instruction writes whole row segments across NVLink;
// kForwardU loads are in flight per lane before the stores.  Reads go through L2
// (the tile was just written there).
constexpr int kForwardU = 16;

__device__ __forceinline__ void forward_tile(const Params& p, int64_t r0, int nrows, int n0, int ncols,
                                             int t, int nthreads)
{
    const int64_t base_row = p.row_offset + r0;
    const int64_t c0 = p.col_offset + n0;  // the tile's first column in the full D
    const bool vec = p.vec_cd && (ncols % 16 == 0);
    if (vec) {
        const int per_row = ncols / 16;
        const int units = nrows * per_row;
        for (int u0 = t; u0 < units; u0 += kForwardU * nthreads) {
            uint4 v[kForwardU];
            int64_t off[kForwardU];
#pragma unroll
            for (int j = 0; j < kForwardU; ++j) {
                const int u = u0 + j * nthreads;
                off[j] = -1;
                if (u < units) {
                    off[j] = (base_row + u / per_row) * p.ldd + c0 + 16 * (u % per_row);
                    v[j] = __ldcg(reinterpret_cast<const uint4*>(p.D_data + off[j]));
                }
            }
            for (int i = 0; i < p.n_extra; ++i) {
#pragma unroll
                for (int j = 0; j < kForwardU; ++j)
                    if (off[j] >= 0) *reinterpret_cast<uint4*>(p.D_extra[i] + off[j]) = v[j];
            }
        }
    } else {
        const int units = nrows * ncols;
        for (int u = t; u < units; u += nthreads) {
            const int64_t off = (base_row + u / ncols) * p.ldd + c0 + u % ncols;
            const uint8_t b = __ldcg(p.D_data + off);
            for (int i = 0; i < p.n_extra; ++i) p.D_extra[i][off] = b;
        }
    }
    // Scale bytes: a full tile row has 8, one 8-byte piece when the scale rows are
    // 8-byte aligned (one NVLink write instead of eight).
    const int nsc = (ncols + 31) / 32;
    bool sc_vec = nsc == 8 && p.lds % 8 == 0 && (c0 / 32) % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(p.D_scales) & 7u) == 0;
    for (int i = 0; i < p.n_extra; ++i) sc_vec = sc_vec && (reinterpret_cast<uintptr_t>(p.Ds_extra[i]) & 7u) == 0;
    if (sc_vec) {
        for (int r = t; r < nrows; r += nthreads) {
            const int64_t off = (base_row + r) * p.lds + c0 / 32;
            const uint2 v = __ldcg(reinterpret_cast<const uint2*>(p.D_scales + off));
            for (int i = 0; i < p.n_extra; ++i) *reinterpret_cast<uint2*>(p.Ds_extra[i] + off) = v;
        }
    } else {
        for (int u = t; u < nrows * nsc; u += nthreads) {
            const int64_t off = (base_row + u / nsc) * p.lds + c0 / 32 + u % nsc;
            const uint8_t b = __ldcg(p.D_scales + off);
            for (int i = 0; i < p.n_extra; ++i) p.Ds_extra[i][off] = b;
        }
    }
}

// Epilogue of one CTA (4 warps, one thread per accumulator row): for every work
// unit of this cluster (UnitWalk), wait for the accumulator, then
//   whole tile / stream-K owner: add the contributors' partials (owner), add the
//     dequantized C, quantize D to MXFP8 along N and store it;
//   stream-K contributor: store the FP32 accumulator as this CTA's partial and count
//     this thread's arrival;
// and release the accumulator on rank 0's tempty barrier.
template <bool kGather, bool kStreamK>
__device__ __forceinline__ void run_epilogue(const Params& p, uint32_t tmem_base, uint32_t tfull0,
                                         uint32_t tempty_base, int cluster, int nclusters,
                                         uint32_t rank, int warp, int lane, volatile int* abort_flag,
                                         uint32_t epi_done = 0u, volatile int* tiles_done = nullptr,
                                         MergeStage ms = MergeStage{nullptr, 0, 0u, 0u, nullptr})
{
    auto tfull = [&](int a) { return tfull0 + 8u * a; };
    const int quad = warp & 3;                 // TMEM lanes this warp may access
    const int r = quad * 32 + lane;            // accumulator row within this CTA's tile
    const bool has_c = p.C_data != nullptr;
    bool aborted = false;
    int it = 0;
    int published = 0;  // units published to the copy warps (contributor units are not)
    UnitWalk walk(p, cluster, nclusters);
    Unit u;
    for (; walk.next(p, u); ++it) {
        const int m0 = u.m0, n0 = u.n0, bn = u.bn;
        const int acc = it & 1;
        const uint32_t acc_ph = (uint32_t)(it >> 1) & 1u;
        const int64_t grow = (int64_t)m0 + BM * (int)rank + r;
        const bool row_ok = grow < p.M;
        const int nchunks = min(bn / 32, (p.N - n0 + 31) / 32);
        if (kStreamK && u.kind == kUnitContrib) {
            const uint32_t tacc = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN);
            if (!mbar_wait(tfull(acc), acc_ph, abort_flag, p.status, kSiteTmemFull, p.timeout_ns)) break;
            tc_fence_after();
            sk_store_partial(sk_slot(p, cluster, rank) + r, tacc, row_ok, nchunks);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_base + 8u * acc);
            red_release_gpu_add(p.sk_sync + 1 + 2 * cluster + (int)rank, 1u);
            continue;
        }
        // Stream-K owner: the tile's other K ranges are the partials of n_merge
        // clusters (first_contrib .. cluster-1), added chunk by chunk below (none when
        // this CTA has no rows of the tile: its issuer copies nothing).
        const int n_merge = kStreamK && u.kind == kUnitOwner && (int64_t)m0 + BM * (int)rank < p.M
                                ? cluster - u.first_contrib : 0;
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
                const int col0 = n0 + 32 * c;
                const int valid = min(32, p.N - col0);
                const uint32_t taddr = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * BN + 32 * c);
                if (valid == 32 && p.vec_cd) {
                    uint32_t raw[32];
                    tmem_ld_32x32b_x32(taddr, raw);
                    tmem_ld_wait();
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
                    if (kStreamK && n_merge > 0) {
                        const bool ok = sk_add_pieces(p, ms, n_merge, c, r, row_ok, v, abort_flag);
                        if (!__all_sync(0xFFFFFFFFu, ok)) {  // the warp leaves together
                            aborted = true;
                            break;
                        }
                    }
                    if (has_c) add_c_chunk(v, cq[ci][0], cq[ci][1], cs[ci]);
                    uint4 d0, d1;
                    const uint32_t sd = quantize_block32(v, d0, d1);
                    if (row_ok) store_d_chunk<kGather>(p, grow, col0, d0, d1, sd);
                } else if (!epilogue_ragged_chunk<kGather>(p, taddr, cs[ci], has_c, row_ok, grow, col0, valid,
                                                           &ms, n_merge, c, r, abort_flag)) {
                    aborted = true;
                    break;
                }
            }
            if (aborted) break;
        }
        if (aborted) break;
        // An item with no columns inside N (the second half of a split tile at the
        // right edge) still waits for its accumulator phase, so that phases pair up.
        if (!full_seen && !mbar_wait(tfull(acc), acc_ph, abort_flag, p.status, kSiteTmemFull, p.timeout_ns))
            break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_base + 8u * acc);
        if (kGather && tiles_done != nullptr) {
            // Publish "this unit's D rows are in this GPU's D" to the copy warps:
            // every epilogue thread arrives (release) after its stores; one thread
            // waits for all 128 (acquire) and bumps the counter the copy warps poll.
            mbar_arrive(epi_done);
            bool ok = true;
            if (quad == 0) {
                if (lane == 0) {
                    ok = mbar_wait(epi_done, (uint32_t)published & 1u, abort_flag, p.status, kSiteEpiDone,
                                   p.timeout_ns);
                    if (ok) {
                        __threadfence_block();
                        *tiles_done = published + 1;
                    }
                }
                ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;  // the warp leaves together
            }
            if (!ok) break;
            ++published;
        }
    }
}

// Epilogue of the on-chip variant (4 warps, one thread per accumulator row): for
// every tile of this cluster, wait for the accumulator, add the dequantized C,
// quantize D to MXFP8 along N, store it, and release the accumulator on rank 0's
// tempty barrier.
__device__ __forceinline__ void run_epilogue_onchip(const Params& p, uint32_t tmem_base, uint32_t tfull,
                                                    uint32_t tempty_rank0, int cluster, int nclusters,
                                                    uint32_t rank, int warp, int lane, volatile int* abort_flag)
{
    const int quad = warp & 3;       // TMEM lanes this warp may access
    const int r = quad * 32 + lane;  // accumulator row within this CTA's tile
    const bool has_c = p.C_data != nullptr;
    const int num_tiles = p.num_m_tiles * p.num_n_tiles;
    int it = 0;
    for (int tile = cluster; tile < num_tiles; tile += nclusters, ++it) {
        int m0, n0;
        tile_coords(p, tile, m0, n0);
        const int64_t grow = (int64_t)m0 + BM * (int)rank + r;
        const bool row_ok = grow < p.M;
        const int nchunks = min(BN / 32, (p.N - n0 + 31) / 32);
        // This row's C codes and scales for the whole tile, loaded before the
        // accumulator is ready so that the loads overlap the mainloop.
        uint4 cq[BN / 32][2];
        uint32_t cs[BN / 32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
            cq[c][0] = cq[c][1] = make_uint4(0u, 0u, 0u, 0u);
            cs[c] = 0u;
            const int col0 = n0 + 32 * c;
            if (has_c && row_ok && c < nchunks) {
                cs[c] = __ldg(p.C_scales + grow * p.nblkN + col0 / 32);
                if (p.vec_cd && col0 + 32 <= p.N) {
                    const uint4* src = reinterpret_cast<const uint4*>(p.C_data + grow * p.N + col0);
                    cq[c][0] = __ldg(src);
                    cq[c][1] = __ldg(src + 1);
                }
            }
        }
        if (!mbar_wait(tfull, (uint32_t)it & 1u, abort_flag, p.status, kSiteTmemFull, p.timeout_ns)) break;
        tc_fence_after();
        const uint32_t trow = tmem_base + ((uint32_t)(quad * 32) << 16);
        if (p.vec_cd && n0 + BN <= p.N) {
            // Whole tile inside N: two chunks per tensor-memory load, and the
            // accumulator is released as soon as the last two chunks are in registers,
            // so the next tile's MMAs start while their math and stores run.
#pragma unroll
            for (int pr = 0; pr < BN / 64; ++pr) {
                uint32_t raw[64];
                tmem_ld_32x32b_x64(trow + (uint32_t)(64 * pr), raw);
                tmem_ld_wait();
                if (pr == BN / 64 - 1) {
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(tempty_rank0);
                }
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int c = 2 * pr + h;
                    float v[32];
#pragma unroll
                    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[32 * h + i]);
                    if (has_c) add_c_chunk(v, cq[c][0], cq[c][1], cs[c]);
                    uint4 d0, d1;
                    const uint32_t sd = quantize_block32(v, d0, d1);
                    if (row_ok) store_d_chunk<false>(p, grow, n0 + 32 * c, d0, d1, sd);
                }
            }
            continue;
        }
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
            if (c >= nchunks) break;  // warp-uniform: tcgen05.ld is warp-collective
            const int col0 = n0 + 32 * c;
            const int valid = min(32, p.N - col0);
            const uint32_t taddr = trow + (uint32_t)(32 * c);
            if (valid == 32 && p.vec_cd) {
                uint32_t raw[32];
                tmem_ld_32x32b_x32(taddr, raw);
                tmem_ld_wait();
                float v[32];
#pragma unroll
                for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(raw[i]);
                if (has_c) add_c_chunk(v, cq[c][0], cq[c][1], cs[c]);
                uint4 d0, d1;
                const uint32_t sd = quantize_block32(v, d0, d1);
                if (row_ok) store_d_chunk<false>(p, grow, col0, d0, d1, sd);
            } else {
                // No partials to merge here: the chunk cannot give up.
                epilogue_ragged_chunk<false>(p, taddr, cs[c], has_c, row_ok, grow, col0, valid, nullptr, 0, c, r,
                                             abort_flag);
            }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(tempty_rank0);
    }
}

// On-chip variant.  Per CTA and K block of two K-steps: the A-code producer brings
// this CTA's 128 x 128 A codes (128-byte swizzle), the B producer its half of the
// tile's B columns for both K-steps (four 64 x 64 boxes, tile columns 128 rank ..
// +127); a transform group converts the codes to BF16 and stores them into the A
// stage in tensor memory (tcgen05.st, lane = row); rank 0 issues the pair MMAs
// (tcgen05.mma.cta_group::2, A from tensor memory, B from shared memory, M = 256,
// N = 256) into the accumulator.
__global__ void __maxnreg__(kLaunchRegs)
gemm_mxfp8_bf16_kernel(const __grid_constant__ CUtensorMap tmap_a,
                       const __grid_constant__ CUtensorMap tmap_b, const Params p)
{
    extern __shared__ uint8_t smem_raw[];
    // Swizzled TMA destinations and UMMA descriptors need 1024-byte alignment of
    // the shared-memory address itself; both CTAs of the pair get the same offsets.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + OFF_BAR;
    auto a8_full = [&](int j) { return bar0 + 8u * j; };
    auto a8_empty = [&](int j) { return bar0 + 8u * (A8_STAGES + j); };
    // Stage s of the MMA ring completes on rank 0's full(s) when both CTAs' B boxes
    // have landed (TMA transaction bytes) and both CTAs' transform groups have stored
    // the converted A; one MMA commit to empty(s) in both CTAs frees the B slot and
    // the A stage together.
    const uint32_t barS = bar0 + 8u * (2 * A8_STAGES);
    auto full = [&](int s) { return barS + 8u * s; };
    auto empty = [&](int s) { return barS + 8u * (STAGES + s); };
    const uint32_t tfull = barS + 8u * (2 * STAGES);
    const uint32_t tempty = tfull + 8u;
    const uint32_t drain = tfull + 16u;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + OFF_MISC + 4);
    // Stays 0: the abort flag of the teardown waits, which must not be cut short.
    volatile int* never_abort = reinterpret_cast<volatile int*>(smem + OFF_MISC + 8);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();     // 0 = MMA leader of the pair
    const int cluster = (int)cluster_id_x();
    const int nclusters = (int)nclusters_x();
    const int num_tiles = p.num_m_tiles * p.num_n_tiles;

    if (threadIdx.x == 0) {
        for (int j = 0; j < A8_STAGES; ++j) {
            mbar_init(a8_full(j), 1);
            mbar_init(a8_empty(j), 4);  // the 4 warps of the transform group that read it
        }
        for (int s = 0; s < STAGES; ++s) {
            // rank 0's B producer (expect_tx) + one transform group per stage, both CTAs
            mbar_init(full(s), 1 + 2 * 4);
            mbar_init(empty(s), 1);
        }
        mbar_init(tfull, 1);
        mbar_init(tempty, 2 * kEpilogueWarps);
        mbar_init(drain, 1);
        *abort_flag = 0;
        *never_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();  // barriers of both CTAs initialised, TMEM allocated in both
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    bool producer_aborted = false;

    if (warp < kFirstTransformWarp) {
    setmaxnreg_dec<kCtrlRegs>();
    if (warp == kBProducerWarp) {
        // ---------------------------- B producer (TMA) ----------------------------
        if (lane == 0) {
            prefetch_tmap(&tmap_b);
            int s = 0;
            uint32_t ph = 0;
            int issued = 0;
            bool ok = true;
            for (int tile = cluster; ok && tile < num_tiles; tile += nclusters) {
                int m0, n0;
                tile_coords(p, tile, m0, n0);
                for (int kb2 = 0; kb2 < p.num_kb2; ++kb2) {
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status, kSiteEmpty, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    // B boxes of both CTAs complete on rank 0's full: per K-step h of the
                    // block, this CTA's two 64-column boxes (rows past K read as zeros).
                    if (rank == 0) mbar_arrive_expect_tx(full(s), 2 * OC_B_BYTES);
                    const uint32_t fb = mapa_shared(full(s), 0);
#pragma unroll
                    for (int h = 0; h < OC_KSTEPS; ++h)
#pragma unroll
                        for (int j = 0; j < BN_HALF / 64; ++j)
                            tma_load_2d_pair(sbase + OFF_B + s * OC_B_BYTES + h * B_BYTES + j * B_BOX_BYTES, &tmap_b,
                                             fb, n0 + BN_HALF * (int)rank + 64 * j, (kb2 * OC_KSTEPS + h) * BK);
                    ++issued;
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                producer_aborted = true;
                // Let the copies already issued land before the CTA can exit.
                const int outstanding = issued < STAGES ? issued : STAGES;
                int ss = s;
                uint32_t pp = ph;
                for (int i = 0; i < outstanding; ++i) {
                    if (--ss < 0) { ss = STAGES - 1; pp ^= 1u; }
                    if (rank == 0) mbar_wait(full(ss), pp, never_abort, nullptr, 0, kDrainTimeoutNs);
                }
            }
        }
    } else if (warp == 2) {
        // -------------------------- A-code producer (TMA) --------------------------
        if (lane == 0) {
            prefetch_tmap(&tmap_a);
            int j = 0;
            uint32_t ph = 0;
            int issued = 0;
            bool ok = true;
            for (int tile = cluster; ok && tile < num_tiles; tile += nclusters) {
                int m0, n0;
                tile_coords(p, tile, m0, n0);
                const int row0 = m0 + BM * (int)rank;
                for (int kb2 = 0; kb2 < p.num_kb2; ++kb2) {
                    if (!mbar_wait(a8_empty(j), ph ^ 1u, abort_flag, p.status, kSiteEmptyA8, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(a8_full(j), A8_BYTES);
                    tma_load_2d(sbase + OFF_A8 + j * A8_BYTES, &tmap_a, a8_full(j), kb2 * OC_BK, row0);
                    ++issued;
                    if (++j == A8_STAGES) { j = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                producer_aborted = true;
                const int outstanding = issued < A8_STAGES ? issued : A8_STAGES;
                int jj = j;
                uint32_t pp = ph;
                for (int i = 0; i < outstanding; ++i) {
                    if (--jj < 0) { jj = A8_STAGES - 1; pp ^= 1u; }
                    mbar_wait(a8_full(jj), pp, never_abort, nullptr, 0, kDrainTimeoutNs);
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------- MMA issuer (rank 0) ---------------------------
        if (rank == 0 && lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            bool ok = true;
            for (int tile = cluster; ok && tile < num_tiles; tile += nclusters, ++it) {
                if (!mbar_wait(tempty, ((uint32_t)it & 1u) ^ 1u, abort_flag, p.status, kSiteTmemEmpty,
                               p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                for (int kb2 = 0; kb2 < p.num_kb2; ++kb2) {
                    if (!mbar_wait(full(s), ph, abort_flag, p.status, kSiteFullB, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_tmem = tmem_base + kTmemACol + (uint32_t)s * kTmemAStageCols;
                    const uint32_t b_addr = sbase + OFF_B + s * OC_B_BYTES;
                    // The block's second K-step lies past K when num_kb is odd: its MMAs
                    // are not issued (they would add zeros).
                    const int nslices = (kb2 * OC_KSTEPS + 1 < p.num_kb ? OC_KSTEPS : 1) * (BK / UMMA_K);
#pragma unroll
                    for (int k = 0; k < OC_KSTEPS * (BK / UMMA_K); ++k) {
                        if (k >= nslices) break;
                        // B: MN-major, per K-step two 64-column chunks 8 KiB apart (LBO),
                        // 8-row K groups 1024 B apart (SBO); a K slice of 16 rows is 2 KiB.
                        // A: a K slice of 16 BF16 is 8 tensor-memory columns.
                        const uint64_t bdesc = umma_smem_desc_sw128(
                            b_addr + (k / (BK / UMMA_K)) * B_BYTES + (k % (BK / UMMA_K)) * UMMA_K * 128, B_BOX_BYTES,
                            1024);
                        umma_bf16_pair_tmem_a(tmem_base, a_tmem + (uint32_t)(k * UMMA_K / 2), bdesc, kIdesc,
                                              (kb2 | k) != 0 ? 1u : 0u);
                    }
                    umma_commit_pair_mc(empty(s), 0x3);  // frees stage s in both CTAs
                    if (++s == STAGES) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit_pair_mc(tfull, 0x3);
            }
            // All pair MMAs issued by this thread complete before TMEM is released.
            umma_commit_pair(drain);
            mbar_wait(drain, 0, never_abort, nullptr, 0, kDrainTimeoutNs);
        }
    }
    // warp 3: idle (keeps the transform and epilogue warpgroups aligned)
    } else if (warp < kFirstEpilogueWarp) {
        if constexpr (kXformRegs < kLaunchRegs) setmaxnreg_dec<kXformRegs>();
        // ------------------------------- transform --------------------------------
        // Group g (4 warps, one thread per row of this CTA's A tile) converts the
        // K blocks kb2 with kb2 % G == g.  A warp covers 32 consecutive rows, which
        // keeps the 128B-swizzled code reads conflict-free and matches the
        // tensor-memory lanes the warp may write (warp % 4 = lanes 32 (warp % 4) ..).
        const int t = threadIdx.x - 32 * kFirstTransformWarp;
        const int r = t & (BM - 1);
        const int grp = t / BM;
        // A scale group is 16 scale bytes: 4 K blocks of a row.
        constexpr int kBlocksPerGroup = 16 * 32 / OC_BK;
        const int groups = (p.num_kb2 + kBlocksPerGroup - 1) / kBlocksPerGroup;
        const uint32_t full_base = mapa_shared(full(0), 0);
        const uint32_t a_tmem_row = tmem_base + ((uint32_t)((warp & 3) * 32) << 16) + kTmemACol;
        bool ok = true;
        int tile = cluster;
        int m0 = 0, n0 = 0;
        if (tile < num_tiles) tile_coords(p, tile, m0, n0);
        int grow = m0 + BM * (int)rank + r;
        const int sc_width = p.nblkK % 16 == 0 && (reinterpret_cast<uintptr_t>(p.A_scales) & 15u) == 0 ? 16
                             : p.nblkK % 4 == 0 && (reinterpret_cast<uintptr_t>(p.A_scales) & 3u) == 0 ? 4
                                                                                                      : 1;
        uint4 nxt = load_scale_group(p.A_scales + (int64_t)grow * p.nblkK, 0, p.nblkK,
                                     tile < num_tiles && grow < p.M, sc_width);
        const uint32_t a8_row_off = (uint32_t)r * (uint32_t)OC_BK;
        const uint32_t a8_xor = (uint32_t)(r & 7);
        int64_t base_stage = 0;  // global stage index of kb2 = 0 of the current tile
        for (; ok && tile < num_tiles; tile += nclusters, base_stage += p.num_kb2) {
            tile_coords(p, tile, m0, n0);
            for (int g = 0; ok && g < groups; ++g) {
                const uint4 cur = nxt;
                {   // prefetch the next scale group (same tile, or the first of the next tile)
                    int nt = tile, ng = g + 1;
                    if (ng == groups) { nt = tile + nclusters; ng = 0; }
                    int nm0 = m0, nn0;
                    if (nt < num_tiles) tile_coords(p, nt, nm0, nn0);
                    const int nrow = nm0 + BM * (int)rank + r;
                    nxt = load_scale_group(p.A_scales + (int64_t)nrow * p.nblkK, 16 * ng, p.nblkK,
                                           nt < num_tiles && nrow < p.M, sc_width);
                }
#pragma unroll 1
                for (int j = grp; j < kBlocksPerGroup; j += kTransformGroups) {
                    const int kb2 = g * kBlocksPerGroup + j;
                    if (kb2 >= p.num_kb2) break;
                    const int64_t i = base_stage + kb2;  // global stage index
                    const int s = (int)(i % STAGES);
                    const uint32_t ph = (uint32_t)((i / STAGES) & 1);
                    const int j8 = (int)(i % A8_STAGES);
                    const uint32_t ph8 = (uint32_t)((i / A8_STAGES) & 1);
                    // The A stage is free once the MMAs of its previous round completed.
                    // Waiting on it first also keeps every group within STAGES (<=
                    // A8_STAGES) stages of the MMA, so no parity wait below can match a
                    // phase one round too old.
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status, kSiteEmptyT, p.timeout_ns) ||
                        !mbar_wait(a8_full(j8), ph8, abort_flag, p.status, kSiteFullA8, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();  // the MMAs' reads of the stage come before the stores below
                    const uint8_t* a8 = smem + OFF_A8 + j8 * A8_BYTES;
                    uint4 q[OC_BK / 16];
#pragma unroll
                    for (int c = 0; c < OC_BK / 16; ++c)
                        q[c] = *reinterpret_cast<const uint4*>(a8 + a8_row_off + ((((uint32_t)c) ^ a8_xor) << 4));
                    // This block's 4 scale bytes: word j of the group.
                    const uint32_t sc4 = j < 2 ? (j == 0 ? cur.x : cur.y) : (j == 2 ? cur.z : cur.w);
                    const int kvalid = p.K - kb2 * OC_BK;
                    const uint32_t ta = a_tmem_row + (uint32_t)s * kTmemAStageCols;
                    // tcgen05.st is warp-collective: the warp takes one path together.
                    if (__all_sync(0xFFFFFFFFu, fast_block_ok(q, sc4, kvalid))) {
#pragma unroll
                        for (int h = 0; h < OC_BK / 32; ++h) {
                            uint32_t out[16];
                            convert_half_fast(q[2 * h], q[2 * h + 1], (sc4 >> (8 * h)) & 0xFFu, out);
                            tmem_st_32x32b_x16(ta + 16u * (uint32_t)h, out);
                        }
                    } else {
                        uint32_t ex[OC_BK / 2];
                        convert_block_exact(a8 + a8_row_off, a8_xor, sc4, kvalid, ex);
#pragma unroll
                        for (int h = 0; h < OC_BK / 32; ++h) tmem_st_32x32b_x16(ta + 16u * (uint32_t)h, ex + 16 * h);
                    }
                    // The codes are consumed: release the A-code slot to the producer.
                    __syncwarp();
                    if (lane == 0) mbar_arrive(a8_empty(j8));
                    tmem_st_wait();
                    tc_fence_before();
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cluster(full_base + 8u * s);
                }
            }
        }
    } else {
        setmaxnreg_inc<kEpiRegs>();
        // -------------------------------- epilogue --------------------------------
        run_epilogue_onchip(p, tmem_base, tfull, mapa_shared(tempty, 0), cluster, nclusters, rank, warp, lane,
                            abort_flag);
    }

    // ------------------------------- teardown -------------------------------------
    if (producer_aborted) {
        // A B copy of the peer may still be landing after rank 0 stopped expecting it;
        // give it time before this CTA's shared memory can be released.
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 100000ull) {
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();  // both CTAs done with TMEM, barriers and each other's smem
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
    }
}


// ============================================================================
// BF16-A variant: A is dequantized to BF16 in HBM by a bandwidth pre-pass
// (launch_mxfp8_dequantize_bf16, exact) and streamed by TMA like B, so the
// mainloop has no transform on its critical path.  Same clusters, tiles, pair
// MMA and epilogue as above; per CTA and K-step the ring holds the CTA's 128 x 64
// BF16 A rows (16 KiB, 128-byte swizzle = the UMMA K-major layout) and its 64 x 128
// B half (16 KiB), both completing on rank 0's full barrier.
//
// Warps: 0 TMA producer, 1 TMEM owner + MMA issuer (rank 0), 2-3 copy warps of the
// fused all-gather (otherwise warp 2 streams a stream-K owner's partials in), 4-7
// epilogue.  Launched after the A pre-pass with programmatic stream serialization:
// only the producer waits for the pre-pass.
//
// Shared memory: kStages ring stages, then kSlots 16 KiB stream-K staging pieces.
// Three variants: whole tiles (7 stages), stream-K (5 stages + 4 pieces: the
// merge's staging costs two stages, which the mainloop does not need at full speed)
// and the fused all-gather (7 stages, whole tiles).
// ============================================================================
constexpr int P_THREADS = 256;
constexpr int P_FIRST_EPI_WARP = 4;
constexpr int P_TILE_STAGES = 7;                      // whole-tile and all-gather variants
constexpr int P_SK_STAGES = 5, P_SK_SLOTS = 4;        // stream-K variant

template <int kStages, int kSlots>
struct PLayout {
    static constexpr int OFF_B = 0;
    static constexpr int OFF_A = OFF_B + kStages * B_BYTES;
    static constexpr int OFF_STAGE = OFF_A + kStages * A16_BYTES;
    static constexpr int OFF_BAR = OFF_STAGE + kSlots * (int)kSkPieceBytes;
    // barriers: full[S], empty[S], tfull[2], tempty[2], drain, epi_done, piece_full[P],
    // piece_empty[P]
    static constexpr int NUM_BARS = 2 * kStages + 6 + 2 * kSlots;
    static constexpr int OFF_MISC = OFF_BAR + NUM_BARS * 8;
    // misc: TMEM address, abort flag, teardown flag, units done (all-gather), cluster ticket
    static constexpr int SMEM_BYTES = OFF_MISC + 32 + 1024;
    static_assert(SMEM_BYTES <= 232448, "exceeds the sm_100 per-block shared memory limit");
};
static_assert(BK * BN == B_BYTES, "per-stage B bytes of one CTA are BK * item width");

template <bool kGather, int kStages, int kSlots>
__global__ void __launch_bounds__(P_THREADS, 1)
gemm_bf16a_mxfp8_kernel(const __grid_constant__ CUtensorMap tmap_a16,
                        const __grid_constant__ CUtensorMap tmap_b, const Params p)
{
    using Lay = PLayout<kStages, kSlots>;
    constexpr bool kStreamK = kSlots > 0;
    static_assert(!(kGather && kStreamK), "the fused all-gather runs whole tiles");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = sbase + Lay::OFF_BAR;
    auto full = [&](int s) { return bar0 + 8u * s; };
    auto empty = [&](int s) { return bar0 + 8u * (kStages + s); };
    auto tfull = [&](int a) { return bar0 + 8u * (2 * kStages + a); };
    auto tempty = [&](int a) { return bar0 + 8u * (2 * kStages + 2 + a); };
    const uint32_t drain = bar0 + 8u * (2 * kStages + 4);
    const uint32_t epi_done = bar0 + 8u * (2 * kStages + 5);  // fused all-gather only
    const uint32_t piece_full0 = bar0 + 8u * (2 * kStages + 6);  // stream-K only
    const uint32_t piece_empty0 = piece_full0 + 8u * kSlots;
    const MergeStage ms{smem + Lay::OFF_STAGE, kSlots, piece_full0, piece_empty0,
                        reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC + 8)};
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Lay::OFF_MISC);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC + 4);
    volatile int* never_abort = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC + 8);
    volatile int* tiles_done = reinterpret_cast<volatile int*>(smem + Lay::OFF_MISC + 12);
    volatile uint32_t* ticket = reinterpret_cast<volatile uint32_t*>(smem + Lay::OFF_MISC + 16);
    const bool forward = kGather && p.n_extra > 0;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    int cluster = (int)cluster_id_x();
    const int nclusters = (int)nclusters_x();

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(tfull(a), 1);
            mbar_init(tempty(a), 2 * kEpilogueWarps);
        }
        mbar_init(drain, 1);
        mbar_init(epi_done, 4 * 32);
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(piece_full0 + 8u * i, 1);
            mbar_init(piece_empty0 + 8u * i, kEpilogueWarps * 32);
        }
        *abort_flag = 0;
        *never_abort = 0;
        *tiles_done = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc_pair(smem_u32(tmem_holder), kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    cluster_sync_all();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    bool producer_aborted = false;
    if (p.sk_tiles > 0) {
        // Stream-K: a cluster waits only for partials of clusters with a lower
        // logical index, and logical indices are handed out in the order the
        // clusters start, so every cluster waited for is already running.  The
        // counter is zeroed by the A pre-pass, which has completed once
        // wait_for_prerequisite_grid returns.
        if (rank == 0 && threadIdx.x == 0) {
            wait_for_prerequisite_grid();
            const uint32_t tk = atomicAdd(p.sk_sync, 1u);
            const uint32_t a = smem_u32(const_cast<uint32_t*>(ticket));
            st_shared_cluster_u32(mapa_shared(a, 0), tk);
            st_shared_cluster_u32(mapa_shared(a, 1), tk);
        }
        cluster_sync_all();
        cluster = (int)*ticket;
    }

    if (warp == 0) {
        // ------------------------ TMA producer (A and B) -------------------------
        if (lane == 0) {
            prefetch_tmap(&tmap_a16);
            prefetch_tmap(&tmap_b);
            // The A pre-pass may still be running (programmatic dependent launch):
            // BF16 A is read only after it has completed.
            wait_for_prerequisite_grid();
            int s = 0;
            uint32_t ph = 0;
            int issued = 0;
            bool ok = true;
            UnitWalk walk(p, cluster, nclusters);
            Unit u;
            while (ok && walk.next(p, u)) {
                const int row0 = u.m0 + BM * (int)rank;
                const int col0 = u.n0 + (u.bn / 2) * (int)rank;
                // both CTAs' A rows and B columns for one K-step
                const uint32_t tx = 2u * (uint32_t)(A16_BYTES + BK * u.bn);
                for (int kb = u.kb0; kb < u.kb1; ++kb) {
                    if (!mbar_wait(empty(s), ph ^ 1u, abort_flag, p.status, kSiteEmpty, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(full(s), tx);
                    const uint32_t fb = mapa_shared(full(s), 0);
                    tma_load_2d_pair(sbase + Lay::OFF_A + s * A16_BYTES, &tmap_a16, fb, kb * BK, row0);
                    for (int j = 0; j < u.bn / 128; ++j)
                        tma_load_2d_pair(sbase + Lay::OFF_B + s * B_BYTES + j * B_BOX_BYTES, &tmap_b, fb,
                                         col0 + 64 * j, kb * BK);
                    ++issued;
                    if (++s == kStages) { s = 0; ph ^= 1u; }
                }
            }
            if (!ok) {
                producer_aborted = true;
                const int outstanding = issued < kStages ? issued : kStages;
                int ss = s;
                uint32_t pp = ph;
                for (int i = 0; i < outstanding; ++i) {
                    if (--ss < 0) { ss = kStages - 1; pp ^= 1u; }
                    if (rank == 0) mbar_wait(full(ss), pp, never_abort, nullptr, 0, kDrainTimeoutNs);
                }
            }
        }
    } else if (warp == 1) {
        // --------------------------- MMA issuer (rank 0) ---------------------------
        if (rank == 0 && lane == 0) {
            int s = 0;
            uint32_t ph = 0;
            int it = 0;
            bool ok = true;
            UnitWalk walk(p, cluster, nclusters);
            Unit u;
            for (; ok && walk.next(p, u); ++it) {
                const uint32_t idesc = u.bn == BN ? kIdesc : kIdescHalf;
                const int acc = it & 1;
                const uint32_t acc_ph = (uint32_t)(it >> 1) & 1u;
                if (!mbar_wait(tempty(acc), acc_ph ^ 1u, abort_flag, p.status, kSiteTmemEmpty,
                               p.timeout_ns)) {
                    ok = false;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
                for (int kb = u.kb0; kb < u.kb1; ++kb) {
                    if (!mbar_wait(full(s), ph, abort_flag, p.status, kSiteFullB, p.timeout_ns)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = sbase + Lay::OFF_A + s * A16_BYTES;
                    const uint32_t b_addr = sbase + Lay::OFF_B + s * B_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; ++k) {
                        const uint64_t adesc = umma_smem_desc_sw128(a_addr + k * UMMA_K * 2, 16, 1024);
                        const uint64_t bdesc = umma_smem_desc_sw128(b_addr + k * UMMA_K * 128, B_BOX_BYTES, 1024);
                        umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb != u.kb0 || k != 0) ? 1u : 0u);
                    }
                    umma_commit_pair_mc(empty(s), 0x3);
                    if (++s == kStages) { s = 0; ph ^= 1u; }
                }
                if (!ok) break;
                umma_commit_pair_mc(tfull(acc), 0x3);
            }
            umma_commit_pair(drain);
            mbar_wait(drain, 0, never_abort, nullptr, 0, kDrainTimeoutNs);
        }
    } else if (warp >= P_FIRST_EPI_WARP) {
        run_epilogue<kGather, kStreamK>(p, tmem_base, tfull(0), mapa_shared(tempty(0), 0), cluster, nclusters,
                                        rank, warp, lane, abort_flag, epi_done, forward ? tiles_done : nullptr, ms);
    } else if (kStreamK && warp == 2) {
        // ---------- stream-K: bulk copies of the partials an owner unit adds ----------
        if (lane == 0) sk_issue_merge(p, cluster, nclusters, rank, ms, abort_flag);
    } else if (forward) {
        // ---------------- fused all-gather: copy warps 2 and 3 ----------------
        // Forward every tile this CTA's epilogue has finished (tiles_done counts
        // them, in this cluster's tile order) to the other GPUs' full-D buffers.
        const int t = threadIdx.x - 64;
        int published = 0;
        UnitWalk walk(p, cluster, nclusters);
        Unit u;
        while (walk.next(p, u)) {
            if (u.kind == kUnitContrib) continue;  // no D rows: its owner forwards the tile
            const uint64_t t0 = globaltimer_ns();
            bool ok = true;
            while (*tiles_done <= published) {
                if (*abort_flag) { ok = false; break; }
                if (globaltimer_ns() - t0 > p.timeout_ns) {
                    *abort_flag = 1;
                    atomicCAS(p.status, 0, kDevTimeoutBase + kSiteCopy);
                    ok = false;
                    break;
                }
                __nanosleep(256);
            }
            if (!ok) break;
            __threadfence_block();
            ++published;
            const int64_t r0 = (int64_t)u.m0 + BM * (int)rank;
            const int nrows = (int)min((int64_t)BM, (int64_t)p.M - r0);
            const int ncols = min(u.bn, p.N - u.n0);
            if (nrows > 0 && ncols > 0) forward_tile(p, r0, nrows, u.n0, ncols, t, 64);
        }
    }

    if (producer_aborted) {
        const uint64_t t0 = globaltimer_ns();
        while (globaltimer_ns() - t0 < 100000ull) {
        }
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, kTmemCols);
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

// Cross-GPU barrier of the fused all-gather, one warp: lane t < world publishes
// `epoch` into slot `rank` of GPU t's flag array (a peer store, after a system-scope
// fence so that this GPU's earlier peer stores of D are visible first), then waits
// until slot t of this GPU's own array holds `epoch` or later.  Each wait is
// bounded: on expiry the site code 0x7E goes to the device status word and the
// lane stops waiting.
struct PeerFlags {
    uint32_t* f[kMaxGatherDest];
};

__global__ void peer_barrier_kernel(PeerFlags flags, int rank, int world, uint32_t epoch, int* status,
                                    uint64_t timeout_ns)
{
    const int t = threadIdx.x;
    if (t >= world) return;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(flags.f[t] + rank), "r"(epoch) : "memory");
    const uint32_t* mine = flags.f[rank] + t;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(mine) : "memory");
        if ((int32_t)(v - epoch) >= 0) break;
        if (globaltimer_ns() - t0 > timeout_ns) {
            atomicCAS(status, 0, kDevTimeoutBase + 0x7E);
            break;
        }
        __nanosleep(2000);
    }
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
bool g_smem_attr_set[64] = {};
bool g_regs_checked[64] = {};

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

// Address of the status word in the current device's context, looked up on every
// call (a table search once the device code is loaded), so that it is never an
// address of a context that cudaDeviceReset has destroyed.
int status_ptr(int dev, int** out)
{
    (void)dev;
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_device_status);
    if (e != cudaSuccess) {
        set_last_error("cudaGetSymbolAddress(status) failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    *out = static_cast<int*>(ptr);
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

namespace {

// Shared host setup of both GEMM kernels: device checks, status word, B tensor map
// and the kernel parameters.
// B's tensor map covers N x K elements with rows ldb elements apart (ldb >= N, a
// multiple of 8); columns past N read as zeros.
int gemm_setup(const uint8_t* A_scales, const void* B, int ldb, const uint8_t* C_data,
               const uint8_t* C_scales, uint8_t* D_data, uint8_t* D_scales, int M, int N, int K,
               int& dev, PFN_cuTensorMapEncodeTiled_v12000& enc, CUtensorMap& tmap_b, gemm::Params& p)
{
    using namespace gemm;
    int rc = get_device(dev);
    if (rc) return rc;
    int* status = nullptr;
    if ((rc = status_ptr(dev, &status))) return rc;
    if ((rc = get_encoder(&enc))) return rc;
    if ((rc = encode_2d(enc, &tmap_b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, B, (uint64_t)N, (uint64_t)K,
                        (uint64_t)ldb * 2, 64, BK, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
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
    p.num_m_tiles = (M + PAIR_M - 1) / PAIR_M;
    p.num_n_tiles = (N + BN - 1) / BN;
    p.num_kb = (K + BK - 1) / BK;
    p.num_kb2 = (p.num_kb + OC_KSTEPS - 1) / OC_KSTEPS;
    p.num_items = p.split_from = p.num_m_tiles * p.num_n_tiles;
    // About sqrt(74 clusters) rows per panel keeps the in-flight rectangle square;
    // up to 2 * kPanelM M tiles stay one panel (M fastest over all rows), which
    // timed slightly better there.
    p.panel_m = p.num_m_tiles <= 2 * kPanelM ? p.num_m_tiles : kPanelM;
    p.n_extra = 0;
    p.row_offset = p.col_offset = 0;
    p.ldd = N;
    p.lds = p.nblkN;
    for (int i = 0; i < kMaxGatherDest - 1; ++i) p.D_extra[i] = p.Ds_extra[i] = nullptr;
    p.sk_tiles = p.sk_clusters = 0;
    p.sk_iters = 0;
    p.sk_partial = nullptr;
    p.sk_sync = nullptr;
    const bool al_c = C_data == nullptr || (reinterpret_cast<uintptr_t>(C_data) & 15u) == 0;
    const bool al_d = (reinterpret_cast<uintptr_t>(D_data) & 15u) == 0;
    p.vec_cd = (N % 16 == 0 && al_c && al_d) ? 1 : 0;
    return MPK_SUCCESS;
}

// Grid: one cluster per work item up to one per SM pair; at least min_clusters (the
// stream-K clusters, which need not have whole items).
template <typename Kernel>
int launch_pair_kernel(Kernel kernel, int smem_bytes, int threads, const CUtensorMap& tmap_a,
                       const CUtensorMap& tmap_b, const gemm::Params& p, cudaStream_t stream,
                       bool after_prepass = false, int min_clusters = 0)
{
    const int max_clusters = device_sm_count() / 2;
    int clusters = p.num_items < max_clusters ? p.num_items : max_clusters;
    if (clusters < min_clusters) clusters = min_clusters;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // After the A pre-pass: launch while it finishes (it allows dependents at its
    // start); the producer waits for it before the first load of BF16 A.
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = after_prepass ? 2 : 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmap_a, tmap_b, p);
    if (e == cudaErrorInvalidValue || e == cudaErrorLaunchOutOfResources) {
        // The shared-memory attribute is set once per device; a context re-created
        // by cudaDeviceReset has lost it.  Set it again and retry once.
        cudaGetLastError();
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) == cudaSuccess)
            e = cudaLaunchKernelEx(&cfg, kernel, tmap_a, tmap_b, p);
    }
    if (e != cudaSuccess) {
        set_last_error("GEMM launch failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    return MPK_SUCCESS;
}

int ensure_smem_attr(const void* kernel, int bytes, bool* flag)
{
    std::lock_guard<std::mutex> lk(g_mu);
    if (!*flag) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
        if (e != cudaSuccess) {
            set_last_error("cudaFuncSetAttribute failed: %s", cudaGetErrorString(e));
            return (int)e;
        }
        *flag = true;
    }
    return MPK_SUCCESS;
}

bool g_smem_attr_bf16a[64] = {};
bool g_smem_attr_gather[64] = {};
bool g_smem_attr_sk[64] = {};

}  // namespace

namespace {
constexpr size_t kWsAlign = 256;
size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }
int64_t padded8(int x) { return ((int64_t)x + 7) / 8 * 8; }

// Work schedule of the BF16-A kernel (mpk_set_gemm_schedule).
std::atomic<int> g_schedule{MPK_SCHEDULE_AUTO};
// A stream-K range shorter than this many 64-wide K-steps costs more in partial
// traffic and hand-off than it saves.
constexpr int kSkMinIters = 8;

// Bytes of A's BF16 copy and of B's padded copy (when needed) at the start of the
// workspace.
size_t operand_bytes(int M, int N, int K, bool copy_b)
{
    size_t bytes = round_up((size_t)M * (size_t)padded8(K) * 2u, kWsAlign);
    if (copy_b) bytes += (size_t)K * (size_t)padded8(N) * 2u;
    return bytes;
}

// Stream-K region after the operands: one partial slot per CTA of the stream-K
// clusters, then the ticket and arrival counters.
size_t sk_region_bytes(int sk_clusters)
{
    if (sk_clusters <= 0) return 0;
    return (size_t)sk_clusters * 2u * (size_t)gemm::kSkSlotFloats * 4u +
           round_up(4u * (1u + 2u * (size_t)sk_clusters), kWsAlign);
}
}  // namespace

SkPlan gemm_sk_plan(int M, int N, int K)
{
    using namespace gemm;
    SkPlan plan{0, 0};
    const int mode = g_schedule.load(std::memory_order_relaxed);
    if (mode == MPK_SCHEDULE_TILES || M <= 0 || N <= 0 || K <= 0) return plan;
    const int64_t tiles = (int64_t)((M + PAIR_M - 1) / PAIR_M) * ((N + BN - 1) / BN);
    const int64_t kb = (K + BK - 1) / BK;
    const int64_t clusters = device_sm_count() / 2;
    if (mode == MPK_SCHEDULE_STREAM_K) {
        // every tile's K-steps spread over all clusters (for tests of the hand-off)
        plan.tiles = (int)tiles;
        plan.clusters = (int)std::min(clusters, tiles * kb);
        return plan;
    }
    // Auto: the tiles of the last, partial wave are spread over the clusters when
    // that gives each cluster at least kSkMinIters K-steps and more clusters than
    // whole tiles would keep busy, and when the partial wave is a large part of the
    // run: one to three full waves, at least 128 K-steps of whole tiles per cluster
    // after the spread ones, and a last wave at most 85 % full.  The contributors'
    // stores and the owners' merge of the partials share each SM's L2 port with the
    // whole tiles' loads; with fewer whole K-steps to hide behind, with many waves or
    // with a nearly full last wave they cost about what they save (measured on B200:
    // +4 to +20 % inside these bounds, -4 to -19 % outside them).
    const int64_t rem = tiles % clusters;
    const int64_t waves = tiles / clusters;
    if (rem == 0 || waves < 1 || waves > 3 || waves * kb < 128 || rem * 100 > clusters * 85) return plan;
    const int64_t csk = std::min(clusters, rem * kb / kSkMinIters);
    if (csk <= rem) return plan;
    plan.tiles = (int)rem;
    plan.clusters = (int)csk;
    return plan;
}

int gemm_set_schedule(int mode)
{
    if (mode != MPK_SCHEDULE_AUTO && mode != MPK_SCHEDULE_TILES && mode != MPK_SCHEDULE_STREAM_K) {
        set_last_error("unknown GEMM schedule %d", mode);
        return MPK_ERR_INVALID_VALUE;
    }
    g_schedule.store(mode);
    return MPK_SUCCESS;
}

int gemm_schedule() { return g_schedule.load(); }

int check_onchip_gemm_shape(const uint8_t* A_data, const void* B, int N, int K)
{
    if (K % 16 != 0 || N % 8 != 0) {
        set_last_error("the on-chip conversion kernel needs K %% 16 == 0 and N %% 8 == 0 (TMA row strides); "
                       "got N=%d K=%d -- pass a workspace (mpk_gemm_mxfp8_bf16_ws) for other shapes",
                       N, K);
        return MPK_ERR_UNSUPPORTED;
    }
    if ((reinterpret_cast<uintptr_t>(A_data) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u)) {
        set_last_error("the on-chip conversion kernel needs A_data and B 16-byte aligned (TMA) -- "
                       "pass a workspace (mpk_gemm_mxfp8_bf16_ws) for other pointers");
        return MPK_ERR_MISALIGNED;
    }
    return MPK_SUCCESS;
}

// Default entry point: run the on-chip conversion kernel instead of the pre-pass and
// the BF16-A kernel.  Measured on B200, the on-chip kernel is faster when N <= 2048
// and the BF16 copy of A (M * K * 2 bytes) is at least 256 MiB, about twice L2:
// the pre-pass then costs a whole extra pass over A in HBM (write 2 bytes, read 2
// bytes back per code) against a GEMM with few columns to amortise it over.  Only
// whole-tile plans (the default schedule with no stream-K split) are routed, so D
// is the same bit for bit as the pre-pass path's; the operands must meet the
// on-chip kernel's TMA limits.
bool gemm_default_onchip(const void* A_data, const void* B, int M, int N, int K)
{
    using namespace gemm;
    if (g_schedule.load(std::memory_order_relaxed) != MPK_SCHEDULE_AUTO) return false;
    if (N > 2048 || (int64_t)M * K * 2 < (int64_t(256) << 20)) return false;
    if (K % 16 != 0 || N % 8 != 0) return false;
    if ((reinterpret_cast<uintptr_t>(A_data) & 15u) || (reinterpret_cast<uintptr_t>(B) & 15u)) return false;
    return gemm_sk_plan(M, N, K).tiles == 0;
}

bool gemm_b_needs_copy(const void* B, int N)
{
    return N % 8 != 0 || (reinterpret_cast<uintptr_t>(B) & 15u) != 0;
}

size_t gemm_workspace_bytes_min(int M, int N, int K, bool copy_b) { return operand_bytes(M, N, K, copy_b); }

size_t gemm_workspace_bytes(int M, int N, int K, bool copy_b)
{
    const SkPlan plan = gemm_sk_plan(M, N, K);
    const size_t ops = operand_bytes(M, N, K, copy_b);
    return plan.tiles > 0 ? round_up(ops, kWsAlign) + sk_region_bytes(plan.clusters) : ops;
}

int launch_gemm_mxfp8_bf16(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                           const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                           uint8_t* D_scales, int M, int N, int K, cudaStream_t stream)
{
    using namespace gemm;
    int dev = 0;
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    CUtensorMap tmap_a, tmap_b;
    Params p;
    int rc = gemm_setup(A_scales, B, N, C_data, C_scales, D_data, D_scales, M, N, K, dev, enc, tmap_b, p);
    if (rc) return rc;
    if ((rc = encode_2d(enc, &tmap_a, CU_TENSOR_MAP_DATA_TYPE_UINT8, A_data, (uint64_t)K, (uint64_t)M,
                        (uint64_t)K, OC_BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if ((rc = ensure_smem_attr((const void*)gemm_mxfp8_bf16_kernel, SMEM_BYTES, &g_smem_attr_set[dev])))
        return rc;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_regs_checked[dev]) {
            cudaFuncAttributes fa;
            cudaError_t e = cudaFuncGetAttributes(&fa, gemm_mxfp8_bf16_kernel);
            if (e != cudaSuccess) {
                set_last_error("cudaFuncGetAttributes failed: %s", cudaGetErrorString(e));
                return (int)e;
            }
            // The setmaxnreg split assumes exactly kLaunchRegs per thread at launch.
            if (fa.numRegs != kLaunchRegs) {
                set_last_error("GEMM kernel compiled with %d registers per thread, expected %d",
                               fa.numRegs, kLaunchRegs);
                return MPK_ERR_UNSUPPORTED;
            }
            g_regs_checked[dev] = true;
        }
    }
    return launch_pair_kernel(gemm_mxfp8_bf16_kernel, SMEM_BYTES, kThreads, tmap_a, tmap_b, p, stream);
}

int launch_gemm_mxfp8_bf16_prepass(const uint8_t* A_data, const uint8_t* A_scales, const void* B,
                                   const uint8_t* C_data, const uint8_t* C_scales, uint8_t* D_data,
                                   uint8_t* D_scales, int M, int N, int K, void* workspace,
                                   size_t workspace_bytes, cudaStream_t stream, const GatherDest* gather)
{
    using namespace gemm;
    int dev = 0;
    PFN_cuTensorMapEncodeTiled_v12000 enc;
    CUtensorMap tmap_a16, tmap_b;
    Params p;
    // Workspace: A's BF16 copy [M][lda], then (when needed) B's padded copy [K][ldb].
    const int64_t lda = padded8(K);
    const bool copy_b = gemm_b_needs_copy(B, N);
    const int64_t ldb = copy_b ? padded8(N) : N;
    void* b_copy = static_cast<uint8_t*>(workspace) + round_up((size_t)M * (size_t)lda * 2u, kWsAlign);
    const void* b_used = copy_b ? b_copy : B;
    int rc = gemm_setup(A_scales, b_used, (int)ldb, C_data, C_scales, D_data, D_scales, M, N, K, dev, enc,
                        tmap_b, p);
    if (rc) return rc;
    if ((rc = encode_2d(enc, &tmap_a16, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, workspace, (uint64_t)K,
                        (uint64_t)M, (uint64_t)lda * 2, BK, BM, CU_TENSOR_MAP_SWIZZLE_128B)))
        return rc;
    if (gather) {
        if (gather->n_extra < 0 || gather->n_extra > kMaxGatherDest - 1) {
            set_last_error("fused all-gather: %d extra destinations (at most %d)", gather->n_extra,
                           kMaxGatherDest - 1);
            return MPK_ERR_INVALID_VALUE;
        }
        p.n_extra = gather->n_extra;
        p.row_offset = gather->row_offset;
        p.col_offset = gather->col_offset;
        p.ldd = gather->ldd;
        p.lds = (gather->ldd + 31) / 32;
        if (p.ldd % 16 != 0 || p.col_offset % 16 != 0) p.vec_cd = 0;
        for (int i = 0; i < gather->n_extra; ++i) {
            p.D_extra[i] = gather->D_extra[i];
            p.Ds_extra[i] = gather->Ds_extra[i];
            if (reinterpret_cast<uintptr_t>(p.D_extra[i]) & 15u) p.vec_cd = 0;
        }
    }
    if (copy_b) {
        const cudaError_t ce = cudaMemcpy2DAsync(b_copy, (size_t)ldb * 2, B, (size_t)N * 2, (size_t)N * 2,
                                                 (size_t)K, cudaMemcpyDeviceToDevice, stream);
        if (ce != cudaSuccess) {
            set_last_error("B row-padding copy failed: %s", cudaGetErrorString(ce));
            return (int)ce;
        }
    }
    // Schedule of the last, partial wave: stream-K when the plan asks for it and the
    // workspace has room for the partials (never with the fused all-gather); else
    // split the last wave's tiles in two when they would fill at most half of it.
    uint32_t* zero_words = nullptr;
    int n_zero = 0;
    int min_clusters = 0;
    const SkPlan plan = gather ? SkPlan{0, 0} : gemm_sk_plan(M, N, K);
    const size_t sk_off = round_up(operand_bytes(M, N, K, copy_b), kWsAlign);
    if (plan.tiles > 0 && workspace_bytes >= sk_off + sk_region_bytes(plan.clusters)) {
        uint8_t* region = static_cast<uint8_t*>(workspace) + sk_off;
        p.sk_tiles = plan.tiles;
        p.sk_clusters = plan.clusters;
        p.sk_iters = (int64_t)plan.tiles * p.num_kb;
        p.sk_partial = reinterpret_cast<float*>(region);
        p.sk_sync = reinterpret_cast<uint32_t*>(region + (size_t)plan.clusters * 2u * kSkSlotFloats * 4u);
        zero_words = p.sk_sync;
        n_zero = 1 + 2 * plan.clusters;
        min_clusters = plan.clusters;
    } else {
        const int tiles = p.num_m_tiles * p.num_n_tiles;
        const int clusters = std::min(tiles, device_sm_count() / 2);
        const int rem = tiles % clusters;
        if (tiles > clusters && rem > 0 && 2 * rem <= clusters) {
            p.split_from = tiles - rem;
            p.num_items = tiles + rem;
        }
    }
    using TileLay = PLayout<P_TILE_STAGES, 0>;
    using SkLay = PLayout<P_SK_STAGES, P_SK_SLOTS>;
    const auto k_tiles = gemm_bf16a_mxfp8_kernel<false, P_TILE_STAGES, 0>;
    const auto k_sk = gemm_bf16a_mxfp8_kernel<false, P_SK_STAGES, P_SK_SLOTS>;
    const auto k_gather = gemm_bf16a_mxfp8_kernel<true, P_TILE_STAGES, 0>;
    if (gather) {
        if ((rc = ensure_smem_attr((const void*)k_gather, TileLay::SMEM_BYTES, &g_smem_attr_gather[dev]))) return rc;
    } else if (p.sk_tiles > 0) {
        if ((rc = ensure_smem_attr((const void*)k_sk, SkLay::SMEM_BYTES, &g_smem_attr_sk[dev]))) return rc;
    } else if ((rc = ensure_smem_attr((const void*)k_tiles, TileLay::SMEM_BYTES, &g_smem_attr_bf16a[dev]))) {
        return rc;
    }
    cudaError_t e = launch_mxfp8_dequantize_bf16(A_data, A_scales, workspace, M, K, lda, stream, zero_words,
                                                 n_zero);
    if (e != cudaSuccess) {
        set_last_error("A pre-pass launch failed: %s", cudaGetErrorString(e));
        return (int)e;
    }
    if (gather)
        return launch_pair_kernel(k_gather, TileLay::SMEM_BYTES, P_THREADS, tmap_a16, tmap_b, p, stream, true);
    if (p.sk_tiles > 0)
        return launch_pair_kernel(k_sk, SkLay::SMEM_BYTES, P_THREADS, tmap_a16, tmap_b, p, stream, true,
                                  min_clusters);
    return launch_pair_kernel(k_tiles, TileLay::SMEM_BYTES, P_THREADS, tmap_a16, tmap_b, p, stream, true);
}

int launch_peer_barrier(uint32_t* const* flags, int rank, int world, uint32_t epoch, cudaStream_t stream)
{
    int dev = 0, rc = get_device(dev);
    if (rc) return rc;
    int* status = nullptr;
    if ((rc = status_ptr(dev, &status))) return rc;
    gemm::PeerFlags pf = {};
    for (int i = 0; i < world; ++i) pf.f[i] = flags[i];
    gemm::peer_barrier_kernel<<<1, 32, 0, stream>>>(pf, rank, world, epoch, status, wait_timeout_ns());
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_error("peer barrier launch failed: %s", cudaGetErrorString(e));
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
