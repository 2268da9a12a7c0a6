// ZipGEMM for B200: C = W * X^T with W stored in TCA-TBE form.
// Replaces csrc/L_Kernel.cuh:295/575 BF16TripleBitmap_MM_Kernel_Fast/_Safe,
// csrc/Reduction_Kernel.cuh:15 SplitK_Reduction_BF16 and the launcher
// csrc/L_API.cu:119 BF16TripleBitmap_MM_API.
//
// Shapes (reference contract, test_mm.cu:410-428): W is M x K (compressed),
// X is N x K row-major (token-major, K contiguous), C is column-major M x N:
// C[n*M + m] = sum_k W[m][k] * X[n][k], fp32 accumulate, bf16 output.
//
// Work decomposition. An output tile is 128 rows of W (two global-tile (GT)
// rows) x BN columns (BN = N rounded up to 16, <= 256). A "unit" is one K
// block of 64 columns of a tile: two GTs of W and the 64 x BN block of X. The
// K blocks of a tile are split into S contiguous ranges, one per CTA of a
// thread-block cluster of S CTAs (S in {1, 2, 4, 8}, chosen on the host so
// the grid fills the SMs in as few waves as possible). At the end the S fp32
// partial tiles are summed through distributed shared memory: every CTA
// parks its partial in its own shared memory, and after a cluster barrier
// CTA r sums rows [128 r / S, 128 (r+1) / S) over the S partials in rank order
// (deterministic) and writes bf16. There is no global workspace, no second
// kernel and no wait on CTAs outside the cluster.
//
// Inside a CTA (kDecWarps + 4 warps):
//   warps D, D+3 compressed producers. Per chunk of cu units (cu = 2 at the
//               shapes measured), warp D loads bitmaps 1-3 and the median
//               offsets of both GT rows with one 2-D tensor copy each, and warp
//               D+3 the sign/mantissa and fallback streams of both GT rows with
//               one 1-D bulk copy each, into a ring of nc slots. Every stream is
//               contiguous in HBM because a CTA's units are consecutive K blocks
//               of one tile, and the CTA's GT offsets are staged in shared
//               memory once, at the start. (Issuing a copy costs the issuing
//               warp about 50 cycles per copy in the instruction, whatever its
//               size, and separate warps issue in parallel: hence few, large
//               copies split over two warps.)
//   warp D+1    X producer: 2-D TMA (128-byte swizzle) of the 64 x BN X block
//   warp D+2    MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16 x 4 per
//               unit, operands from shared memory, fp32 accumulator in TMEM
//   warps 0..D-1 decoders. A unit is four tasks, one per pair of median tiles
//               (32 rows x 64 columns); warp w decodes pair w % 4 of units
//               w / 4 + (D / 4) j into the A ring, in the UMMA canonical
//               K-major 128-byte-swizzle layout, then drain the accumulator.
//               Decoding is bound by the SM's integer/logic pipe (byte permutes
//               and bit logic), so more decoder warps do not help.
// All waits use the hardware-suspended mbarrier test, so waiting warps take no
// issue slots from the decoders. Every wait is bounded (about 2 s); on a
// timeout the kernel records an error bit, every role stops, and the CTA still
// reaches its cluster barriers.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

// Decoder warps (a multiple of 4: a unit is four tasks); kDecWarps / 4 units
// are decoded at once.
#ifndef ZS_DEC_WARPS
#define ZS_DEC_WARPS 16
#endif
constexpr int kDecWarps = ZS_DEC_WARPS;
static_assert(kDecWarps % 4 == 0 && kDecWarps <= 28, "decoder warps: a multiple of 4, at most 28");
constexpr int kTasksPerUnit = 4;
constexpr int kUG = kDecWarps / kTasksPerUnit;   // units decoded at once
constexpr int kBmWarp = kDecWarps;          // producer of the bitmaps
constexpr int kXWarp = kDecWarps + 1;       // producer of X
constexpr int kMmaWarp = kDecWarps + 2;     // MMA issuer
constexpr int kStreamWarp = kDecWarps + 3;  // producer of the median offsets and both streams
constexpr int kGemmThreads = (kDecWarps + 4) * 32;
constexpr int kMaxRing = 16;
constexpr uint32_t kATileBytes = 128 * 128;   // 128 rows x 64 bf16
constexpr uint32_t kHeaderBytes = 2048;

struct GemmParams {
    const uint8_t* sm;
    const uint16_t* full;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* mt_off;
    const int* gt_off;
    int start_exp;
    uint16_t* C;
    int M, N, K;
    int gtk, mgt;                   // K blocks per GT row, GT rows
    int BN, xrows;                  // accumulator columns; rows of the X box = min(BN, N)
    int S;                          // CTAs per cluster (K split)
    int tiles;                      // output tiles (128 rows) of the launch
    int cu, nc, na, nb;             // units per compressed chunk; ring depths
    uint32_t off_offs;              // staged GT offsets: [2 GT rows][nmax + 1] int2 (hf, fallback) unit boundaries
    int nmax;                       // most units of any CTA
    uint32_t off_a, off_b, off_c;   // ring bases in shared memory (A ring, X ring, compressed ring)
    uint32_t off_part;              // epilogue partial tile (S > 1): [BN][128] fp32, over the idle rings
    uint32_t b_slot, c_slot;
    uint32_t c_mt;                  // chunk slot: bitmaps [3 planes][2 GT rows][cu][512 B] | mt [2][cu][32 B] |
    uint32_t c_hf[2], c_full[2];    //             hf stream of each GT row | fallback stream of each GT row
    uint32_t hf_area, full_area;    // bytes (hf) / elements (fallback) one GT row of a chunk may hold
    uint32_t tmem_cols;
    unsigned* err;
    // Row-parallel all-reduce fused into the epilogue (world > 1): recv[j] is
    // rank j's exchange buffer [2][world][Ntot][M / 2] words of (bf16 x 2,
    // flag) (this rank's own at [rank]); epoch (local) counts the exchanges
    // each tile has completed. Column chunk n0 of Ntot; flag_base offsets the
    // chunk's counters.
    int world, rank, Ntot, n0, flag_base;
    int ar_owned;   // 1: reduce-scatter + all-gather by tile owner, 0: all-to-all
    uint16_t* recv[8];
    unsigned* epoch;
    int debug;   // diagnostic builds only (-DZS_TRACE): experiment bits
};

// TMA descriptors: X (64 x BN boxes, 128-byte swizzle), and bitmaps 1-3 and the
// median offsets viewed as [GT rows][K blocks x 64 u64] and [GT rows][K blocks x
// 8 int32], boxes of {cu K blocks, 2 GT rows}.
struct GemmMaps {
    CUtensorMap x, b1, b2, b3, mt;
};

struct GemmHeader {
    uint64_t comp_full[kMaxRing], comp_empty[kMaxRing];
    uint64_t a_full[kMaxRing], a_empty[kMaxRing];
    uint64_t b_full[kMaxRing], b_empty[kMaxRing];
    uint64_t acc_full;
    uint64_t acc_full_p[2], acc_empty_p[2];   // persistent mode: the two TMEM accumulators
    uint32_t tmem_base;
    int abort_flag;
    int ctag[kMaxRing];   // newest chunk issued into each compressed slot (-1: none)
};
static_assert(sizeof(GemmHeader) <= kHeaderBytes, "CTA header overlaps the rings");

#ifdef ZS_TRACE
// Diagnostic build only (-DZS_TRACE): per-CTA %globaltimer stamps of the
// pipeline's phases, [cta][128] u64 (16 + i: MMA issue of unit i < 32; 48 + c:
// chunk c < 16 issued; 64 + u / 96 + u: decode of unit u < 32 starts / ends,
// seen by its first task), set with zs_trace_set.
__device__ unsigned long long* g_zs_trace = nullptr;
#define ZS_STAMP(slot)                                                                      \
    do {                                                                                    \
        if (g_zs_trace && (slot) < 256) g_zs_trace[(size_t)blockIdx.x * 256 + (slot)] = globaltimer_ns(); \
    } while (0)
// cycle-counter stamps (slots 128..255): durations inside one CTA
#define ZS_CLK(slot)                                                                        \
    do {                                                                                    \
        if (g_zs_trace && (slot) < 256) g_zs_trace[(size_t)blockIdx.x * 256 + (slot)] = clock64(); \
    } while (0)
#else
#define ZS_STAMP(slot) \
    do {               \
    } while (0)
#define ZS_CLK(slot) \
    do {             \
    } while (0)
#endif

// Sum of the S partial tiles of a cluster, each parked as [BN][128] fp32 at
// shared offset `part` of its CTA: CTA r owns rows [R r, R (r+1)), R = 128 / S,
// adds the partials in rank order (deterministic) and writes bf16. Each thread
// keeps the S remote loads of one or two items in flight before it sums.
template <int S>
__device__ __forceinline__ void cluster_reduce(const GemmParams& p, uint32_t part, int T, int r, int tid) {
    constexpr int R = 128 / S, R4 = R / 4;
    constexpr int NI = S >= 8 ? 1 : 2;   // items in flight per thread
    const int items = p.BN * R4;
    for (int e0 = tid; e0 < items; e0 += NI * kGemmThreads) {
        float4 v[NI][S];
#pragma unroll
        for (int t = 0; t < NI; ++t) {
            const int e = min(e0 + t * kGemmThreads, items - 1);
            const int col = e / R4, m4 = R * r + 4 * (e - col * R4);
            const uint32_t a = part + 4u * (uint32_t)(col * 128 + m4);
#pragma unroll
            for (int j = 0; j < S; ++j) {
#ifdef ZS_TRACE
                if (p.debug & 1) { v[t][j] = ld_dsmem_f4(mapa_shared(a, (uint32_t)r)); continue; }
#endif
                v[t][j] = ld_dsmem_f4(mapa_shared(a, (uint32_t)j));
            }
        }
#pragma unroll
        for (int t = 0; t < NI; ++t) {
            const int e = e0 + t * kGemmThreads;
            if (e >= items) break;
            float4 acc = v[t][0];
#pragma unroll
            for (int j = 1; j < S; ++j) {
                acc.x += v[t][j].x; acc.y += v[t][j].y; acc.z += v[t][j].z; acc.w += v[t][j].w;
            }
            const int col = e / R4, m4 = R * r + 4 * (e - col * R4);
            const int m = 128 * T + m4;
            if (col < p.N && m < p.M) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t*>(&lo);
                pk.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(p.C + (size_t)col * p.M + m) = pk;
            }
        }
    }
}

// The split-tile sum fused with the row-parallel all-reduce over `world` GPUs.
// CTA r of the cluster sums its rows of the S partial tiles (as cluster_reduce)
// and rounds this rank's result to bf16 (what an all-reduce of the bf16
// partial Ys would receive). Each 8-byte word sent over NVLink holds two bf16
// values and the tile's exchange number (flag = exchanges completed + 1), so a
// word is complete the moment it is visible; a thread stores two words (four
// rows of one column) with one 16-byte store, so a warp writes whole 128-byte
// lines. The `world` partials are added in rank order in fp32, so every rank
// ends with bit-identical Y. No fence, counter or barrier crosses the GPUs.
//   all-to-all (the default for world == 2). Each rank stores its partial into slot `rank` of
//     the peer's exchange buffer, waits for the peer's words in its own, and
//     sums (2 MiB of words per MiB of Y leave each GPU).
//   by tile owner (the default for world >= 3): reduce-scatter + all-gather. Tile T belongs
//     to rank T % world. The other ranks store their partial rows of T into
//     the owner's buffer (slot = their rank); the owner sums them, writes C and
//     stores the final bf16 rows into slot `owner` of every other rank's
//     buffer, where the other ranks wait for them. Each GPU sends
//     2 (world - 1) / world words per value instead of world - 1.
// The buffer has two halves, chosen by the parity of the exchange number: a
// rank can be one exchange ahead of a peer that is still reading, never two
// (its next exchange of a tile needs that peer's words of this one, which the
// peer stores only after it has read this exchange's).
__device__ __forceinline__ void st_volatile_v2u64(unsigned long long* p, unsigned long long a, unsigned long long b) {
    asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}
__device__ __forceinline__ void ld_volatile_v2u64(const unsigned long long* p, unsigned long long& a,
                                                  unsigned long long& b) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
// Wait (bounded) until both words at src carry `flag`; returns their payloads.
__device__ __forceinline__ uint2 wait_words(const unsigned long long* src, unsigned long long flag, bool& ok,
                                            long long t0, unsigned* err) {
    unsigned long long w0 = 0, w1 = 0;
    for (uint32_t it = 0;; ++it) {
        ld_volatile_v2u64(src, w0, w1);
        if ((w0 & 0xFFFFFFFF00000000ull) == flag && (w1 & 0xFFFFFFFF00000000ull) == flag) break;
        if (!ok || ((it & 255) == 255 && clock64() - t0 > kWaitLimitCycles)) {
            if (ok && err) atomicOr(err, kErrWaitTimeout);
            ok = false;
            break;
        }
    }
    return make_uint2((uint32_t)w0, (uint32_t)w1);
}
constexpr int kArMaxItems = 8;   // items (4 rows x 1 column) per thread: BN * 32 / S / kGemmThreads <= 7
template <int S>
__device__ __forceinline__ void cluster_reduce_allreduce(const GemmParams& p, uint32_t part, int T, int r, int tid) {
    constexpr int R = 128 / S, R4 = R / 4;
    const int items = p.BN * R4;
    const int fidx = p.flag_base + T * S + r;
    const unsigned cnt = p.epoch[fidx];
    const unsigned long long flag = (unsigned long long)(cnt + 1u) << 32;
    const size_t slot = (size_t)p.Ntot * (size_t)p.M / 2;   // 8-byte words of one rank's partial
    const size_t half = (size_t)(cnt & 1u) * (size_t)p.world * slot;
    const bool owned = p.ar_owned != 0;
    const int owner = owned ? T % p.world : p.rank;   // the rank that sums this tile
    uint2 own[kArMaxItems];
#pragma unroll
    for (int t = 0; t < kArMaxItems; ++t) {
        const int e = tid + t * kGemmThreads;
        if (e >= items) break;
        const int col = e / R4, m4 = R * r + 4 * (e - col * R4);
        const uint32_t a = part + 4u * (uint32_t)(col * 128 + m4);
        float4 v[S];
#pragma unroll
        for (int j = 0; j < S; ++j) v[j] = ld_dsmem_f4(mapa_shared(a, (uint32_t)j));
        float4 acc = v[0];
#pragma unroll
        for (int j = 1; j < S; ++j) {
            acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
        own[t].x = *reinterpret_cast<uint32_t*>(&lo);
        own[t].y = *reinterpret_cast<uint32_t*>(&hi);
        const int m = 128 * T + m4;
        if (col < p.N && m < p.M) {
            const size_t off = half + (size_t)p.rank * slot + ((size_t)(p.n0 + col) * p.M + m) / 2;
            for (int j = 0; j < p.world; ++j) {
                if (j == p.rank || (owned && j != owner)) continue;
                st_volatile_v2u64(reinterpret_cast<unsigned long long*>(p.recv[j]) + off, flag | own[t].x,
                                  flag | own[t].y);
            }
        }
    }
    bool ok = true;
    const long long t0 = clock64();
#pragma unroll
    for (int t = 0; t < kArMaxItems; ++t) {
        const int e = tid + t * kGemmThreads;
        if (e >= items) break;
        const int col = e / R4, m4 = R * r + 4 * (e - col * R4);
        const int m = 128 * T + m4;
        if (col >= p.N || m >= p.M) continue;
        const size_t word = ((size_t)(p.n0 + col) * p.M + m) / 2;
        const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.recv[p.rank]) + half + word;
        uint2 pk;
        if (p.rank == owner) {
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int j = 0; j < p.world; ++j) {
                const uint2 q = j == p.rank ? own[t] : wait_words(src + (size_t)j * slot, flag, ok, t0, p.err);
                const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.x));
                const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&q.y));
                if (j == 0) {
                    acc = make_float4(lo.x, lo.y, hi.x, hi.y);
                } else {
                    acc.x += lo.x; acc.y += lo.y; acc.z += hi.x; acc.w += hi.y;
                }
            }
            __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
            pk.x = *reinterpret_cast<uint32_t*>(&lo);
            pk.y = *reinterpret_cast<uint32_t*>(&hi);
            if (owned) {   // all-gather: the final rows to every other rank (slot `owner`)
                const size_t off = half + (size_t)p.rank * slot + word;
                for (int j = 0; j < p.world; ++j)
                    if (j != p.rank)
                        st_volatile_v2u64(reinterpret_cast<unsigned long long*>(p.recv[j]) + off, flag | pk.x,
                                          flag | pk.y);
            }
        } else {
            pk = wait_words(src + (size_t)owner * slot, flag, ok, t0, p.err);
        }
        *reinterpret_cast<uint2*>(p.C + (size_t)col * p.M + m) = pk;
    }
    if (tid == 0) p.epoch[fidx] = cnt + 1u;
}

// PERSIST = false: one CTA per (tile, K range), the K ranges of a tile in one
// thread-block cluster (above). PERSIST = true (no K split, shapes with more
// tiles than SMs): one CTA per SM loops over tiles blockIdx.x, + gridDim.x, ...;
// its units are the K blocks of those tiles in order, so the producers and
// decoders run on across tile boundaries; the MMA alternates between two TMEM
// accumulators, and four more warps (one per TMEM lane quarter) drain each
// finished tile to C while the next tile is decoded.
constexpr int kEpiWarp0 = kDecWarps + 4;   // persistent mode: epilogue warps kEpiWarp0 .. + 3
template <bool PERSIST>
__global__ void __launch_bounds__(kGemmThreads + (PERSIST ? 128 : 0), 1)
    zipgemm_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    GemmHeader* hd = reinterpret_cast<GemmHeader*>(smem);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // this CTA: first output tile T, cluster rank r, K blocks [kb0, kb0 + per)
    // of each of its ntile tiles; n units in all
    const int r = PERSIST ? 0 : (int)(blockIdx.x % (unsigned)p.S);
    const int T = PERSIST ? (int)blockIdx.x : (int)(blockIdx.x / (unsigned)p.S);
    const int kb0 = PERSIST ? 0 : (int)((long long)p.gtk * r / p.S);
    const int per = PERSIST ? p.gtk : (int)((long long)p.gtk * (r + 1) / p.S) - kb0;
    const int ntile = PERSIST ? (p.tiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x : 1;
    const int n = per * ntile;
    auto tile_of = [&](int jt) { return PERSIST ? T + jt * (int)gridDim.x : T; };
    auto nsub_of = [&](int t) { return (2 * t + 1 < p.mgt) ? 2 : 1; };
    const int rowlen = p.nmax + 1;   // staged offsets: [ntile][2 GT rows][nmax + 1]

    if (tid == 0) ZS_STAMP(0);
    int2* offs = reinterpret_cast<int2*>(smem + p.off_offs);
    if (warp == kStreamWarp) {
        // Stage the GT offsets of the CTA's unit boundaries 0..per of both GT rows
        // of each of its tiles (asynchronous copies, in flight during the set-up below).
        for (int idx = lane; idx < ntile * 2 * (per + 1); idx += 32) {
            const int jt = idx / (2 * (per + 1)), rem = idx - jt * 2 * (per + 1);
            const int row = rem / (per + 1), b = rem - row * (per + 1);
            const int t = tile_of(jt);
            int2* dst = offs + (jt * 2 + row) * rowlen + b;
            if (row < nsub_of(t))
                cp_async8(dst, p.gt_off + 2 * ((long long)(2 * t + row) * p.gtk + kb0 + b));
            else
                *dst = make_int2(0, 0);
        }
    }
    if (warp == kBmWarp) {
        if (lane < p.nc) {
            mbar_init(&hd->comp_full[lane], 2);   // one arrival per producer warp
            mbar_init(&hd->comp_empty[lane], kTasksPerUnit * p.cu);
        }
        if (lane == 0) hd->abort_flag = 0;
        if (lane < kMaxRing) hd->ctag[lane] = -1;
        fence_mbar_init();
    } else if (warp == kXWarp) {
        if (lane < p.na) { mbar_init(&hd->a_full[lane], kTasksPerUnit); mbar_init(&hd->a_empty[lane], 1); }
        if (lane < p.nb) { mbar_init(&hd->b_full[lane], 1); mbar_init(&hd->b_empty[lane], 1); }
        if (lane == 0) {
            mbar_init(&hd->acc_full, 1);
            if (PERSIST) {
                mbar_init(&hd->acc_full_p[0], 1);
                mbar_init(&hd->acc_full_p[1], 1);
                mbar_init(&hd->acc_empty_p[0], 4);
                mbar_init(&hd->acc_empty_p[1], 4);
            }
            prefetch_tmap(&maps.x);
            if ((smem_u32(smem) & 1023u) && p.err) atomicOr(p.err, kErrStreamOverflow);
        }
        fence_mbar_init();
    } else if (warp == kMmaWarp) {
        tmem_alloc(&hd->tmem_base, p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // The next grid on the stream may start as soon as every CTA of this one is
    // running; it waits (griddepcontrol.wait) before it reads X or writes C.
    if (tid == 0) grid_dep_launch();
    const uint32_t tmem_d = hd->tmem_base;
    volatile int* abort_flag = &hd->abort_flag;
    const uint32_t smem0 = smem_u32(smem);

    if (warp == kBmWarp || warp == kStreamWarp) {
        // Two producer warps fill each chunk slot; each arrives once on the slot's
        // full barrier with its own byte count. The bitmap warp loads bitmaps 1-3
        // and the median offsets of both GT rows with one 2-D tensor copy each
        // (lanes 0-3); the stream warp loads the sign/mantissa (lanes 0-1) and
        // fallback (lanes 2-3) streams of GT row lane & 1. A chunk shorter than cu
        // units, or a tile with one GT row, takes 1-D copies for the bitmaps and
        // median offsets instead (lanes 0-7), so no tensor box ever leaves its
        // tensor. Issue cost grows with the copies per warp instruction and not
        // with their size, hence few large copies and two warps.
        const bool bmw = warp == kBmWarp;
        if (!bmw) cp_async_wait_all();
        __syncwarp();   // staged offsets visible to the whole warp (and, via the arrives below, to the decoders)
        const int crow = lane & 1;
        const CUtensorMap* tmap = lane == 0 ? &maps.b1 : lane == 1 ? &maps.b2 : lane == 2 ? &maps.b3 : &maps.mt;
        const uint64_t* plane = lane < 2 ? p.b1 : lane < 4 ? p.b2 : p.b3;
        int s = 0;
        uint32_t ph = 0;
        for (int c = 0, i0 = 0; i0 < n; ++c, i0 += p.cu) {
            // the chunk's tile (index jt of this CTA's tiles) and its first unit il in it;
            // chunks never cross a tile (per is a multiple of cu in persistent mode)
            const int jt = PERSIST ? i0 / per : 0, il = i0 - jt * per;
            const int tt = tile_of(jt), ns = nsub_of(tt);
            const int len = min(p.cu, per - il);
            const int2* orow0 = offs + (jt * 2) * rowlen;
            const int2* orow1 = orow0 + rowlen;
            if (bmw && c < 8 && lane == 0) ZS_CLK(128 + 4 * c);
            if (c >= p.nc) {
                bool ok = true;
                if (lane == 0) ok = mbar_wait(&hd->comp_empty[s], ph ^ 1u, p.err, abort_flag);
                if (!__shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0)) break;
            }
            uint8_t* slot = smem + p.off_c + (size_t)s * p.c_slot;
            uint64_t* full_bar = &hd->comp_full[s];
#ifdef ZS_TRACE
            if (p.debug & 16) {   // diagnostic: no weight traffic
                if (lane == 0) { if (!bmw) st_release_cta(&hd->ctag[s], c); mbar_arrive(full_bar); }
                __syncwarp();
                if (++s == p.nc) { s = 0; ph ^= 1u; }
                continue;
            }
#endif
            if (bmw) {
                const bool tiled = len == p.cu && ns == 2;
                if (lane == 0) mbar_arrive_expect_tx(full_bar, (3u * 512u + 32u) * (uint32_t)(len * ns));
                __syncwarp();
                if (bmw && c < 8 && lane == 0) ZS_CLK(129 + 4 * c);
                if (tiled) {
                    if (lane < 4)
                        tma_load_2d(slot + (lane < 3 ? 1024u * (uint32_t)(lane * p.cu) : p.c_mt), tmap,
                                    (kb0 + il) * (lane < 3 ? 64 : 8), 2 * tt, full_bar);
                } else if (lane < 8 && crow < ns) {
                    const long long g = (long long)(2 * tt + crow) * p.gtk + kb0 + il;   // first GT of the chunk
                    if (lane < 6)
                        bulk_g2s(slot + 512u * (uint32_t)(((lane >> 1) * 2 + crow) * p.cu), plane + 64 * g,
                                 512u * (uint32_t)len, full_bar);
                    else
                        bulk_g2s(slot + p.c_mt + 32u * (uint32_t)(crow * p.cu), p.mt_off + 8 * g, 32u * (uint32_t)len,
                                 full_bar);
                }
            } else {
                // stream ranges of the chunk, validated against the slot: lane 0 sums all four
                auto range = [&](int row, bool hf, uint32_t& bytes, int& b0) {
                    const int2* o = row ? orow1 : orow0;
                    const int2 f = o[il], e = o[il + len];
                    const int beg = hf ? f.x : f.y, end = hf ? e.x : e.y;
                    const uint32_t cap = hf ? p.hf_area : 2u * p.full_area;
                    const int al = hf ? 16 : 8;
                    bytes = end > beg ? (uint32_t)(end - beg) * (hf ? 1u : 2u) : 0u;
                    b0 = beg;
                    if (bytes > cap || (bytes & 15u) || (b0 & (al - 1)) || b0 < 0) {   // corrupt offsets: clamp, report
                        if (p.err && lane < 4) atomicOr(p.err, kErrStreamOverflow);
                        bytes = min(bytes, cap) & ~15u;
                        b0 = max(b0, 0) & ~(al - 1);
                    }
                    if (row >= ns) bytes = 0;
                };
                uint32_t bytes = 0;
                int b0 = 0;
                if (lane < 4) range(crow, lane < 2, bytes, b0);
                if (lane == 0) {
                    uint32_t t = bytes, x;
                    int y;
                    range(1, true, x, y); t += x;
                    range(0, false, x, y); t += x;
                    range(1, false, x, y); t += x;
                    st_release_cta(&hd->ctag[s], c);   // the slot's previous fill has landed and been consumed
                    mbar_arrive_expect_tx(full_bar, t);
                }
                __syncwarp();
                if (lane < 4 && bytes) {
                    const bool hf = lane < 2;
                    bulk_g2s(slot + (hf ? p.c_hf[crow] : p.c_full[crow]),
                             hf ? (const void*)(p.sm + b0) : (const void*)(p.full + b0), bytes, full_bar);
                }
            }
            if (bmw && c < 8) { __syncwarp(); if (lane == 0) ZS_CLK(130 + 4 * c); }
            if (bmw && c == 0 && lane == 0) ZS_STAMP(1);
            if (bmw && c < 16 && lane == 0) ZS_STAMP(48 + c);
            if (++s == p.nc) { s = 0; ph ^= 1u; }
        }
    } else if (warp == kXWarp) {
        if (lane == 0) {
            grid_dep_wait();   // X may be the previous grid's output
            int s = 0;
            uint32_t ph = 0;
            for (int i = 0; i < n; ++i) {
                if (i >= p.nb && !mbar_wait(&hd->b_empty[s], ph ^ 1u, p.err, abort_flag)) break;
#ifdef ZS_TRACE
                if (p.debug & 8) {   // diagnostic: no X traffic
                    mbar_arrive(&hd->b_full[s]);
                    if (++s == p.nb) { s = 0; ph ^= 1u; }
                    continue;
                }
#endif
                mbar_arrive_expect_tx(&hd->b_full[s], (uint32_t)p.xrows * 128u);
                tma_load_2d(smem + p.off_b + (size_t)s * p.b_slot, &maps.x, (kb0 + (PERSIST ? i % per : i)) * kGT, 0,
                            &hd->b_full[s]);
                if (++s == p.nb) { s = 0; ph ^= 1u; }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(128, p.BN);
            const uint64_t da0 = umma_desc_sw128(smem0 + p.off_a), db0 = umma_desc_sw128(smem0 + p.off_b);
            const uint32_t bstep = p.b_slot >> 4;
            uint64_t da = da0, db = db0;
            int sa = 0, sb = 0;
            uint32_t pa = 0, pb = 0;
            for (int i = 0; i < n; ++i) {
                // persistent mode: tile jt accumulates in TMEM half jt & 1, which the
                // epilogue warps must have drained (tile jt - 2) before its first MMA
                const int jt = PERSIST ? i / per : 0, il = i - jt * per;
                if (PERSIST && il == 0 && jt >= 2 &&
                    !mbar_wait(&hd->acc_empty_p[jt & 1], (uint32_t)(((jt >> 1) - 1) & 1), p.err, abort_flag))
                    break;
                const uint32_t acc = tmem_d + (PERSIST ? (uint32_t)(jt & 1) * (p.tmem_cols / 2) : 0u);
                if (!mbar_wait2(&hd->a_full[sa], pa, &hd->b_full[sb], pb, p.err, abort_flag)) break;
                tc_fence_after();
                if (i < 32) ZS_CLK(160 + i);
                umma_bf16_ss(acc, da, db, idesc, il > 0 ? 1u : 0u);
                umma_bf16_ss(acc, da + 2, db + 2, idesc, 1u);
                umma_bf16_ss(acc, da + 4, db + 4, idesc, 1u);
                umma_bf16_ss(acc, da + 6, db + 6, idesc, 1u);
                umma_commit(&hd->a_empty[sa]);
                umma_commit(&hd->b_empty[sb]);
                if (PERSIST && il == per - 1) umma_commit(&hd->acc_full_p[jt & 1]);
                if (++sa == p.na) { sa = 0; pa ^= 1u; da = da0; } else { da += kATileBytes >> 4; }
                if (++sb == p.nb) { sb = 0; pb ^= 1u; db = db0; } else { db += bstep; }
            }
            if (!PERSIST) umma_commit(&hd->acc_full);
            ZS_STAMP(2);
        }
    } else if (PERSIST && warp >= kEpiWarp0) {
        // ------------------- epilogue warps (persistent mode) -------------------
        // warp kEpiWarp0 + q reads TMEM lane quarter q (rows 32 q .. 32 q + 31) of
        // each finished tile, writes bf16 C and frees the accumulator half
        const int q = warp & 3;
        for (int jt = 0; jt < ntile; ++jt) {
            if (!mbar_wait_sleep(&hd->acc_full_p[jt & 1], (uint32_t)((jt >> 1) & 1), p.err, abort_flag)) break;
            tc_fence_after();
            if (jt == 0) grid_dep_wait();   // C may still be in use by the previous grid
            const int m = 128 * tile_of(jt) + 32 * q + lane;
            const uint32_t acc = tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)(jt & 1) * (p.tmem_cols / 2);
            for (int c16 = 0; c16 < p.BN; c16 += 16) {
                uint32_t v[16];
                tmem_ld16(acc + (uint32_t)c16, v);
                tmem_wait_ld();
                if (m < p.M) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) {
                        const int nn = c16 + j;
                        if (nn < p.N) {
                            const __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(v[j]));
                            p.C[(size_t)nn * p.M + m] = *reinterpret_cast<const uint16_t*>(&b);
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&hd->acc_empty_p[jt & 1]);
        }
    } else {
        // ------------------------------ decoders ------------------------------
        const DecodeTables tabs = make_decode_tables(p.start_exp);
        const int k = warp & 3, sub = k >> 1, w0 = 2 * (k & 1);   // GT row, first median tile of the pair
        int u = warp >> 2;
        int c = u / p.cu, pos = u - c * p.cu;       // chunk of unit u and position inside it
        int cs = c % p.nc, cround = c / p.nc;       // its ring slot and fill round
        int sa = u % p.na, around = u / p.na;       // A slot of unit u and its use round
        for (; u < n; u += kUG) {
            // The unit's compressed chunk, and its A slot free again (the first na
            // units have one). A decoder can run up to two fills of a compressed
            // slot ahead of the chunks it last saw, so it first waits until its
            // chunk has been issued (the slot's previous fill has then landed), after
            // which the slot barrier's parity names the chunk exactly. For the A
            // ring na >= kUG: the warp saw the MMA of unit u - kUG - na finish, and
            // MMAs complete in order, so the phase before the awaited one is done.
            if (!wait_tag_at_least(&hd->ctag[cs], c, p.err, abort_flag)) break;
            const bool ok = u >= p.na ? mbar_wait2(&hd->comp_full[cs], (uint32_t)(cround & 1), &hd->a_empty[sa],
                                                   (uint32_t)((around - 1) & 1), p.err, abort_flag, true)
                                      : mbar_wait_sleep(&hd->comp_full[cs], (uint32_t)(cround & 1), p.err,
                                                        abort_flag);
            if (!ok) break;
            if (warp == 0 && u == 0 && lane == 0) ZS_STAMP(3);
            if ((warp & 3) == 0 && u < 32 && lane == 0) ZS_CLK(192 + u);
            const int jt = PERSIST ? u / per : 0, ul = u - jt * per;   // the unit's tile, K block in it
            if (sub < nsub_of(tile_of(jt))) {
                const uint32_t base = launder(smem0 + p.off_c + (uint32_t)cs * p.c_slot);
                // the unit's stream starts inside its chunk, from the staged GT offsets
                const int2* orow = offs + (jt * 2 + sub) * rowlen;
                const int2 ou = orow[ul], oc = orow[ul - pos];
                const uint32_t h0 = min((uint32_t)max(ou.x - oc.x, 0), p.hf_area);
                const uint32_t f0 = min((uint32_t)max(ou.y - oc.y, 0), p.full_area);
                const uint32_t su = (uint32_t)(sub * p.cu + pos);
                GtView gv;
                gv.bm = base + 512u * su;
                gv.bstride = 1024u * (uint32_t)p.cu;
                gv.mt = base + p.c_mt + 32u * su;
                gv.sm = base + p.c_hf[sub] + h0;
                gv.full = base + p.c_full[sub] + 2u * f0;
                gv.hf_cap = p.hf_area - h0;
                gv.full_cap = p.full_area - f0;
                const uint32_t rows = smem0 + p.off_a + (uint32_t)sa * kATileBytes + 128u * (uint32_t)(64 * sub + 16 * w0);
#ifdef ZS_TRACE
                if (!(p.debug & 2))
#endif
                decode_mt2_to_tile(gv, tabs, w0, rows);
            }
            fence_proxy_async_smem();   // the tensor core reads the tile through the async proxy
            __syncwarp();
            if ((warp & 3) == 0 && u < 32 && lane == 0) ZS_CLK(224 + u);
            if (lane == 0) {
                mbar_arrive(&hd->a_full[sa]);
                mbar_arrive(&hd->comp_empty[cs]);
            }
            pos += kUG;
            while (pos >= p.cu) {
                pos -= p.cu;
                ++c;
                if (++cs == p.nc) { cs = 0; ++cround; }
            }
            sa += kUG;
            while (sa >= p.na) { sa -= p.na; ++around; }
        }
        // drain: warp w reads TMEM lane quarter w % 4 (rows 32 q .. 32 q + 31), columns 16 j + 16 (w / 4) ..
        if (!PERSIST && !*abort_flag && mbar_wait_sleep(&hd->acc_full, 0u, p.err, abort_flag)) {
            if (warp == 0 && lane == 0) ZS_STAMP(4);
            tc_fence_after();
            if (p.S == 1) grid_dep_wait();   // C may still be in use by the previous grid
            const int q = warp & 3;
            const int m = 128 * T + 32 * q + lane;
            float* part = reinterpret_cast<float*>(smem + p.off_part);   // [BN][128] fp32 (rings are idle now)
            for (int c16 = 16 * (warp >> 2); c16 < p.BN; c16 += 16 * kUG) {
                uint32_t v[16];
                tmem_ld16(tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)c16, v);
                tmem_wait_ld();
                if (p.S == 1) {
                    if (m < p.M) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int nn = c16 + j;
                            if (nn < p.N) {
                                const __nv_bfloat16 b = __float2bfloat16_rn(__uint_as_float(v[j]));
                                p.C[(size_t)nn * p.M + m] = *reinterpret_cast<const uint16_t*>(&b);
                            }
                        }
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) part[(c16 + j) * 128 + 32 * q + lane] = __uint_as_float(v[j]);
                }
            }
        }
    }
    __syncwarp();
    tc_fence_before();
    if (p.S > 1) {
        cluster_sync();   // every partial of the cluster is parked
        if (tid == 0) ZS_STAMP(5);
        grid_dep_wait();  // C may still be in use by the previous grid
        if (p.world > 1) {
            switch (p.S) {
                case 2: cluster_reduce_allreduce<2>(p, smem0 + p.off_part, T, r, tid); break;
                case 4: cluster_reduce_allreduce<4>(p, smem0 + p.off_part, T, r, tid); break;
                default: cluster_reduce_allreduce<8>(p, smem0 + p.off_part, T, r, tid); break;
            }
        } else {
            switch (p.S) {
                case 2: cluster_reduce<2>(p, smem0 + p.off_part, T, r, tid); break;
                case 4: cluster_reduce<4>(p, smem0 + p.off_part, T, r, tid); break;
                default: cluster_reduce<8>(p, smem0 + p.off_part, T, r, tid); break;
            }
        }
        if (tid == 0) ZS_STAMP(7);
        cluster_sync();   // peers may still be reading this CTA's partial
    } else {
        __syncthreads();
    }
    if (tid == 0) ZS_STAMP(6);
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_d, p.tmem_cols);
    }
}

#ifdef ZS_TRACE
extern "C" int zs_trace_set(unsigned long long* d_buf) {
    return (int)cudaMemcpyToSymbol(g_zs_trace, &d_buf, sizeof(d_buf));
}
#endif

// ------------------------------- host side ---------------------------------
static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
    });
    return fn;
}

struct DevInfo {
    int sms = 148;
    int max_smem = 232448;
    int clusters[4] = {0, 0, 0, 0};   // co-resident clusters of 1, 2, 4, 8 CTAs at full shared memory
    bool ready = false;
};

// Per-device properties, kernel attributes and cluster occupancy, queried once
// per device, so launches made during CUDA-graph capture issue no attribute calls.
static cudaError_t dev_setup(int dev, DevInfo* out) {
    static DevInfo info[64];
    static std::mutex mu;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = info[dev];
    if (!d.ready) {
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        ZS_RETURN_IF_ERR(
            cudaFuncSetAttribute(zipgemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem));
        ZS_RETURN_IF_ERR(cudaFuncSetAttribute(zipgemm_kernel<false>, cudaFuncAttributeNonPortableClusterSizeAllowed, 0));
        ZS_RETURN_IF_ERR(
            cudaFuncSetAttribute(zipgemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem));
        for (int i = 0; i < 4; ++i) {
            const int S = 1 << i;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3((unsigned)(S * d.sms), 1, 1);
            cfg.blockDim = dim3(kGemmThreads, 1, 1);
            cfg.dynamicSmemBytes = (size_t)d.max_smem;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeClusterDimension;
            attr[0].val.clusterDim.x = (unsigned)S;
            attr[0].val.clusterDim.y = 1;
            attr[0].val.clusterDim.z = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            int nclusters = 0;
            if (cudaOccupancyMaxActiveClusters(&nclusters, zipgemm_kernel<false>, &cfg) != cudaSuccess) {
                (void)cudaGetLastError();
                nclusters = 0;
            }
            d.clusters[i] = nclusters;
        }
        if (d.clusters[0] <= 0) d.clusters[0] = d.sms;
        d.ready = true;
    }
    *out = d;
    return cudaSuccess;
}

// K split: the cluster size S in {1, 2, 4, 8} that minimises waves x units per
// CTA (plus one unit's worth for the partial-tile exchange when S > 1).
static int choose_split(const DevInfo& di, long long tiles, int gtk, int min_s = 1) {
    int best = 0;
    double best_cost = 1e30;
    for (int i = 0; i < 4; ++i) {
        const int S = 1 << i;
        if (S < min_s || S > gtk || di.clusters[i] <= 0) continue;
        if (min_s > 1 && tiles > di.clusters[i]) continue;   // fused all-reduce: one wave only
        const long long waves = (tiles + di.clusters[i] - 1) / di.clusters[i];
        const double cost = (double)waves * (double)((gtk + S - 1) / S) + (S > 1 ? 1.0 : 0.0);
        if (cost < best_cost - 1e-9) { best_cost = cost; best = S; }
    }
    return best;
}

// Persistent mode (one CTA per SM looping over its tiles, no K split) for
// shapes with more tiles than SMs: chosen when its critical path, the units of
// its busiest CTA plus one set-up and epilogue (about 8 units' time), is
// shorter than the clustered launch's, which pays the set-up and epilogue once
// per wave. ZS_ZIPGEMM_PERSIST=0 / 1 in the environment forces either mode
// where both apply (for tests and comparisons).
static bool choose_persistent(const DevInfo& di, long long tiles, int gtk, int S, int BN) {
    constexpr double kWaveOverheadUnits = 8.0;
    const int G = di.sms;
    const long long ntm = (tiles + G - 1) / G;
    int half = 32;
    while (half < BN) half <<= 1;
    if (tiles < 2 || 2 * half > 512 || ntm * 2 * (gtk + 1) * 8 > 16384) return false;
    if (const char* e = getenv("ZS_ZIPGEMM_PERSIST")) {
        if (e[0] == '0') return false;
        if (e[0] == '1') return true;
    }
    int li = 0;
    while ((1 << li) < S) ++li;
    if (di.clusters[li] <= 0) return true;
    const double np_cost = (double)((tiles + di.clusters[li] - 1) / di.clusters[li]) *
                           ((double)((gtk + S - 1) / S) + kWaveOverheadUnits);
    const double p_cost = (double)ntm * (double)gtk + kWaveOverheadUnits;
    return p_cost < np_cost;
}

static cudaError_t launch_chunk(cudaStream_t stream, const DevInfo& di, GemmParams p, const uint16_t* X,
                                int max_hf, int max_full) {
    auto encode = get_encode_fn();
    if (!encode) return cudaErrorNotSupported;
    const int N = p.N;
    p.BN = (N + 15) / 16 * 16;
    p.xrows = std::min(p.BN, N);
    p.gtk = p.K / kGT;
    p.mgt = p.M / kGT;
    const long long tiles = (p.M + 127) / 128;
    // The fused all-reduce sums the split tiles in the cluster epilogue (S >= 2)
    // and waits there for the other GPUs' CTAs of the same tile, so the whole
    // grid must be resident at once (one wave).
    p.S = choose_split(di, tiles, p.gtk, p.world > 1 ? 2 : 1);
    if (p.S == 0) return cudaErrorInvalidValue;
    if (p.world > 1) {
        int li = 0;
        while ((1 << li) < p.S) ++li;
        if (tiles > di.clusters[li]) return cudaErrorInvalidValue;
    }
    p.tmem_cols = 32;
    while (p.tmem_cols < (uint32_t)p.BN) p.tmem_cols <<= 1;
    p.tiles = (int)tiles;
    const bool persist = p.world == 1 && choose_persistent(di, tiles, p.gtk, p.S, p.BN);
    long long ntm = 1;   // most tiles of any CTA
    if (persist) {
        p.S = 1;
        p.tmem_cols *= 2;   // two accumulators
        ntm = (tiles + di.sms - 1) / di.sms;
    }

    // Shared memory: header | staged GT offsets | A ring | X ring | compressed ring. The compressed ring takes chunks of cu units (the
    // decoders check each slot's chunk tag before its parity, so any depth is
    // safe); the A ring holds at least kUG slots (see the decoders' wait).
    const uint32_t hfc = round_up_u32((uint32_t)std::max(max_hf, 16), 16);
    const uint32_t ffc = round_up_u32((uint32_t)std::max(max_full, 8), 8);
    p.b_slot = (uint32_t)p.BN * 128u;
    const uint32_t budget = (uint32_t)di.max_smem;
    auto layout = [&](int cu) {
        p.cu = cu;
        p.c_mt = 3u * 1024u * (uint32_t)cu;
        p.hf_area = hfc * (uint32_t)cu;
        p.full_area = ffc * (uint32_t)cu;
        p.c_hf[0] = p.c_mt + 64u * (uint32_t)cu;
        p.c_hf[1] = p.c_hf[0] + p.hf_area + 16;   // 16 bytes of read slack after each hf stream
        p.c_full[0] = p.c_hf[1] + p.hf_area + 16;
        p.c_full[1] = p.c_full[0] + 2u * p.full_area + 16;
        p.c_slot = round_up_u32(p.c_full[1] + 2u * p.full_area + 16, 128);
    };
    p.nmax = (p.gtk + p.S - 1) / p.S;
    p.off_offs = kHeaderBytes;
    const uint32_t ring0 = round_up_u32(kHeaderBytes + 16u * (uint32_t)ntm * (uint32_t)(p.nmax + 1), 1024);
    auto fits = [&](int na, int nb, int nc) {
        return ring0 + (uint32_t)na * kATileBytes + (uint32_t)nb * p.b_slot + (uint32_t)nc * p.c_slot <= budget;
    };
    // preference order: a compressed ring deep enough to hide HBM latency, A
    // slots beyond kUG (the MMA may lag the decoders), then the X ring
    struct Cfg { int cu, nc, na, nb; };
    constexpr int U = kUG;
    const Cfg prefs[] = {{2, 4, U + 2, 2}, {2, 4, U + 1, 2}, {2, 4, U, 2}, {2, 3, U + 2, 2}, {2, 3, U + 1, 2},
                         {2, 3, U, 2},     {1, 6, U, 2},     {1, 4, U, 2}, {1, 3, U, 2},     {1, 2, U, 2}};
    bool placed = false;
    for (const Cfg& q : prefs) {
        if (q.cu > p.gtk) continue;   // a tensor box spans cu K blocks of one GT row
        if (persist && p.gtk % q.cu) continue;   // chunks must not cross a tile
        layout(q.cu);
        if (q.na <= kMaxRing && fits(q.na, q.nb, q.nc)) { p.nc = q.nc; p.na = q.na; p.nb = q.nb; placed = true; break; }
    }
    if (!placed) return cudaErrorInvalidValue;
#ifdef ZS_TRACE
    if (const char* e = getenv("ZS_DEBUG")) p.debug = atoi(e);
    if (const char* e = getenv("ZS_RINGS")) {   // "cu,nc,na,nb" for experiments
        int a = 0, b = 0, c = 0, d = 0;
        if (sscanf(e, "%d,%d,%d,%d", &a, &b, &c, &d) == 4) { layout(a); p.nc = b; p.na = c; p.nb = d; }
    }
#endif
    p.off_a = ring0;
    p.off_b = p.off_a + (uint32_t)p.na * kATileBytes;
    p.off_c = p.off_b + (uint32_t)p.nb * p.b_slot;
    p.off_part = ring0;
    uint32_t smem_bytes = p.off_c + (uint32_t)p.nc * p.c_slot;
    if (p.S > 1) smem_bytes = std::max(smem_bytes, ring0 + 128u * (uint32_t)p.BN * 4u);
    if (smem_bytes > budget) return cudaErrorInvalidValue;

    GemmMaps maps;
    {
        cuuint64_t gdim[2] = {(cuuint64_t)p.K, (cuuint64_t)N};
        cuuint64_t gstride[1] = {(cuuint64_t)p.K * 2};
        cuuint32_t box[2] = {64, (cuuint32_t)p.xrows};
        cuuint32_t estr[2] = {1, 1};
        if (encode(&maps.x, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(X), gdim, gstride, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
            return cudaErrorInvalidValue;
    }
    // [GT rows][K blocks x per_gt elements], boxes {cu x per_gt, 2 rows}; only
    // used for full chunks of two-row tiles, so every box lies inside the tensor
    auto encode_rows = [&](CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint32_t per_gt, uint32_t esz) {
        cuuint64_t gdim[2] = {(cuuint64_t)p.gtk * per_gt, (cuuint64_t)p.mgt};
        cuuint64_t gstride[1] = {(cuuint64_t)p.gtk * per_gt * esz};
        cuuint32_t box[2] = {(cuuint32_t)(per_gt * p.cu), p.mgt >= 2 ? 2u : 1u};
        cuuint32_t estr[2] = {1, 1};
        return encode(m, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    if (!encode_rows(&maps.b1, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b1, 64, 8) ||
        !encode_rows(&maps.b2, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b2, 64, 8) ||
        !encode_rows(&maps.b3, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b3, 64, 8) ||
        !encode_rows(&maps.mt, CU_TENSOR_MAP_DATA_TYPE_INT32, p.mt_off, 8, 4))
        return cudaErrorInvalidValue;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(persist ? std::min<long long>(tiles, di.sms) : tiles * p.S), 1, 1);
    cfg.blockDim = dim3(kGemmThreads + (persist ? 128 : 0), 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)p.S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // Programmatic dependent launch: this grid's CTAs may start (set-up,
    // weight loads, decoding) while the previous grid on the stream finishes;
    // the kernel waits for it before reading X and before writing C.
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return persist ? cudaLaunchKernelEx(&cfg, zipgemm_kernel<true>, maps, p)
                   : cudaLaunchKernelEx(&cfg, zipgemm_kernel<false>, maps, p);
}

static cudaError_t zipgemm_impl(cudaStream_t stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                                const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                                int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M,
                                int N, int K, int split_k, unsigned* err, const PeerExchange* px) {
    // split_k is accepted for the reference signature; the K split is chosen
    // from the shape and the SM count.
    if (M <= 0 || N <= 0 || K <= 0 || (M % 64) || (K % 64)) return cudaErrorInvalidValue;
    if (split_k < 1) return cudaErrorInvalidValue;
    if (max_hf < 0 || max_full < 0 || max_hf > 4096 + 15 || max_full > 4096 + 7) return cudaErrorInvalidValue;
    if (!b1 || !b2 || !b3 || !mt_off || !gt_off || !X || !C) return cudaErrorInvalidValue;
    if ((max_hf > 0 && !sm) || (max_full > 0 && !full)) return cudaErrorInvalidValue;
    if (!aligned16(sm) || !aligned16(full) || !aligned16(b1) || !aligned16(b2) || !aligned16(b3) ||
        !aligned16(mt_off) || !aligned16(X) || (reinterpret_cast<uintptr_t>(C) & 7u) ||
        (reinterpret_cast<uintptr_t>(gt_off) & 7u))
        return cudaErrorInvalidValue;
    int dev = 0;
    ZS_RETURN_IF_ERR(cudaGetDevice(&dev));
    DevInfo di;
    ZS_RETURN_IF_ERR(dev_setup(dev, &di));

    GemmParams p{};
    p.sm = sm; p.full = full; p.b1 = b1; p.b2 = b2; p.b3 = b3; p.mt_off = mt_off; p.gt_off = gt_off;
    p.start_exp = start_exp & 0xFF;
    p.M = M; p.K = K; p.err = err;
    p.world = 1;
    if (px) {
        p.world = px->world;
        p.rank = px->rank;
        p.Ntot = N;
        p.epoch = px->epoch;
        // ZS_ALLREDUCE_SCHEME=owner|all2all overrides the default, to compare the two
        static const int forced = [] {
            const char* e = getenv("ZS_ALLREDUCE_SCHEME");
            return !e ? -1 : (std::string(e) == "owner" ? 1 : (std::string(e) == "all2all" ? 0 : -1));
        }();
        p.ar_owned = forced >= 0 ? forced : (px->world >= 3 ? 1 : 0);
        for (int j = 0; j < px->world; ++j) p.recv[j] = px->recv[j];
    }
    // N > 256 runs as column chunks of 256 (each re-decodes W; such N are
    // tensor-bound, so the repeated decode is a small share of the time)
    const int tiles = (M + 127) / 128;
    for (int n0 = 0, chunk = 0; n0 < N; n0 += 256, ++chunk) {
        GemmParams q = p;
        q.N = std::min(256, N - n0);
        q.C = C + (size_t)n0 * M;
        q.n0 = n0;
        q.flag_base = chunk * tiles * 8;
        ZS_RETURN_IF_ERR(launch_chunk(stream, di, q, X + (size_t)n0 * K, max_hf, max_full));
    }
    return cudaSuccess;
}

cudaError_t launch_zipgemm(cudaStream_t stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                           const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                           int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M, int N,
                           int K, int split_k, unsigned* err) {
    return zipgemm_impl(stream, sm, full, b1, b2, b3, mt_off, gt_off, max_hf, max_full, start_exp, X, C, M, N, K,
                        split_k, err, nullptr);
}

size_t zipgemm_allreduce_counters(int M, int N) {
    if (M <= 0 || N <= 0) return 0;
    return (size_t)((N + 255) / 256) * (size_t)((M + 127) / 128) * 8;
}

size_t zipgemm_allreduce_buffer_bytes(int M, int N, int world) {
    if (M <= 0 || N <= 0 || world < 2 || world > 8) return 0;
    return 2ull * (size_t)world * (size_t)N * (size_t)M * 4ull;   // 2 halves x world slots x M N / 2 words
}

cudaError_t launch_zipgemm_allreduce(cudaStream_t stream, const uint8_t* sm, const uint16_t* full,
                                     const uint64_t* b1, const uint64_t* b2, const uint64_t* b3, const int* mt_off,
                                     const int* gt_off, int max_hf, int max_full, int start_exp, const uint16_t* X,
                                     uint16_t* C, int M, int N, int K, int world, int rank, void* const* peer_bufs,
                                     unsigned* epoch, unsigned* err) {
    if (world < 2 || world > 8 || rank < 0 || rank >= world || !peer_bufs || !epoch) return cudaErrorInvalidValue;
    if (M <= 0 || N <= 0) return cudaErrorInvalidValue;
    PeerExchange px;
    px.world = world;
    px.rank = rank;
    px.epoch = epoch;
    for (int j = 0; j < world; ++j) {
        if (!peer_bufs[j] || (reinterpret_cast<uintptr_t>(peer_bufs[j]) & 255u)) return cudaErrorInvalidValue;
        px.recv[j] = reinterpret_cast<uint16_t*>(peer_bufs[j]);
    }
    return zipgemm_impl(stream, sm, full, b1, b2, b3, mt_off, gt_off, max_hf, max_full, start_exp, X, C, M, N, K, 1,
                        err, &px);
}

}  // namespace zs
