// ZipGEMM for B200: C = W * X^T with W stored in TCA-TBE form.
// Replaces csrc/L_Kernel.cuh:295/575 BF16TripleBitmap_MM_Kernel_Fast/_Safe,
// csrc/Reduction_Kernel.cuh:15 SplitK_Reduction_BF16 and the launcher
// csrc/L_API.cu:119 BF16TripleBitmap_MM_API.
//
// Shapes (reference contract, test_mm.cu:410-428): W is M x K (compressed),
// X is N x K row-major (token-major, K contiguous), C is column-major M x N:
// C[n*M + m] = sum_k W[m][k] * X[n][k], fp32 accumulate, bf16 output.
//
// Work decomposition (stream-K). A "unit" is one 128-row x 64-column block of
// W (two vertically adjacent global tiles, GT) times the matching 64 x BN block
// of X. Units are ordered tile-major (all K blocks of output tile 0, then tile
// 1, ...). The grid has one CTA per SM and CTA c takes the contiguous unit range
// [c U / G, (c+1) U / G), so every SM decodes the same number of weight
// elements whatever the shape. A CTA's range splits into segments, one per
// output tile it touches; a segment that covers a whole tile is written as
// bf16 directly, partial segments are written as fp32 partial tiles to a
// workspace and reduced at the end by the tile's contributing CTAs, each
// summing a slice of the columns over the contributors in CTA order (a fixed
// order, so results are deterministic). The grid never exceeds one CTA per SM,
// so the CTAs of a grid are co-resident and the end-of-kernel wait on the other
// contributors is safe. Consecutive GEMMs overlap through programmatic
// dependent launch: every CTA allows the next grid to launch right after its
// set-up, and only X, C and the workspace wait for the previous grid.
//
// Inside a CTA (kDecWarps + 4 warps; 640 threads with the default 16 decoders):
//   warps D, D+3 compressed producers (D = kDecWarps; alternate chunks of 1, 2
//                or 4 units): 2-D TMA loads of the bitmaps and median offsets
//                of both GT rows, 1-D bulk copies of their sign/mantissa and
//                fallback streams, into a ring of shared-memory slots
//   warp D+1     X producer: 2-D TMA (128-byte swizzle) of the 64 x BN tile
//   warp D+2     MMA issuer: tcgen05.mma kind::f16, M=128, N=BN, K=16 x 4 per
//                unit, operands from shared memory, fp32 accumulators in TMEM
//                (up to four, one per segment in flight)
//   warps 0..D-1 decoders. A unit is four tasks, one per pair of median tiles
//                (32 rows x 64 columns); warp w decodes pair w % 4 of units
//                w / 4 + (D / 4) j. The decoded tile lands in the A ring in the
//                UMMA canonical K-major 128-byte-swizzle layout. "Drain" tasks
//                (16 columns of one TMEM lane quarter each) move a finished
//                accumulator to C or to the workspace.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

// Decoder warps: each task is a pair of median tiles (32 rows x 64 columns), so
// a unit (128 rows x 64 columns) is 4 tasks and the 16 decoders work on 4 units
// at a time (one per A-ring slot).
#ifndef ZS_DEC_WARPS
#define ZS_DEC_WARPS 16
#endif
constexpr int kDecWarps = ZS_DEC_WARPS;
static_assert(kDecWarps % 4 == 0, "decoder warps come in groups of four (one unit each)");
constexpr int kTasksPerUnit = 4;
constexpr int kUnitsInFlight = kDecWarps / kTasksPerUnit;
constexpr int kCompWarp = kDecWarps;   // compressed producers: warps kDecWarps and kDecWarps + 3 (even / odd chunks)
constexpr int kCompWarp1 = kDecWarps + 3;
constexpr int kBWarp = kDecWarps + 1;
constexpr int kMmaWarp = kDecWarps + 2;
constexpr int kGemmThreads = (kDecWarps + 4) * 32;
constexpr int kMaxRing = 16;
constexpr int kMaxAcc = 4;
constexpr uint32_t kHeaderBytes = 1024;
constexpr uint32_t kOffsStage = kHeaderBytes;                    // staged GT offsets: 64 units x 2 GT rows x int4
constexpr uint32_t kChunkInfo = kOffsStage + 2u * 2048u;         // [slot][unit][GT row] int2 offsets in a chunk
constexpr int kMaxChunk = 4;
constexpr uint32_t kStageEnd = kChunkInfo + (uint32_t)kMaxRing * kMaxChunk * 2 * 8;
constexpr uint32_t kATileBytes = 128 * 128;   // 128 rows x 64 bf16
constexpr uint32_t kTmemCols = 512;

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
    int BN;        // output columns (multiple of 16, <= 256)
    int xrows;     // rows of the X box: min(BN, N)
    int n_acc;     // TMEM accumulators (BN columns each)
    int gtk;       // K blocks per output tile = K / 64
    int mgt;       // GT rows = M / 64
    long long units;
    int nb, na, nc;
    int cu;                         // units per compressed chunk (1, 2 or 4)
    int lcu, lnc, lacc;             // log2 of cu, nc, n_acc (powers of two)
    uint32_t off_b, off_a, off_c;   // ring bases (shared-memory offsets)
    uint32_t b_slot, c_slot;
    uint32_t c_mt;                  // chunk slot: [b1 | b2 | b3] x [2 GT rows][cu][512 B], mt [2][cu][32 B],
    uint32_t c_hf[2], c_full[2];    // then the hf and fallback streams of each GT row
    uint32_t hf_area, full_area;    // bytes (hf) and elements (fallback) one GT row of a chunk holds
    float* ws;                      // [grid][2][BN][128] fp32 partial tiles
    int* cnt;                       // [mtiles][2] arrival / done counters (zero between launches)
    unsigned* err;
    int debug;
    uint32_t smem_bytes;            // dynamic shared memory of the launch (bounds checks)
    size_t ws_floats;               // workspace size (bounds checks)
};

#ifdef ZS_CHECK
// Diagnostic build only: validate an access, record `code` and skip it when invalid.
#define ZS_GUARD(cond, code) if (!(cond)) { if (p.err) atomicOr(p.err, (unsigned)(code)); } else
#else
#define ZS_GUARD(cond, code)
#endif

// TMA descriptors: X (64 x BN tiles, 128-byte swizzle) and the bitmap / median
// offset arrays viewed as [GT rows][K blocks x 512 B] and [GT rows][K blocks x 32 B],
// so one box of {cu K blocks, 2 GT rows} fetches a chunk's part of each array.
// Every box lies inside its tensor: chunks never cross the end of a GT row (cu
// divides K / 64), the last GT row of an odd number of rows uses the one-row
// maps (b1h .. mth), and the X box is at most N rows high.
struct GemmMaps {
    CUtensorMap x, b1, b2, b3, mt;
    CUtensorMap b1h, b2h, b3h, mth;
};

struct GemmHeader {
    uint64_t comp_full[kMaxRing], comp_empty[kMaxRing];
    uint64_t a_full[kMaxRing], a_empty[kMaxRing];
    uint64_t b_full[kMaxRing], b_empty[kMaxRing];
    uint64_t acc_full[kMaxAcc], acc_empty[kMaxAcc];
    uint32_t tmem_base;
    int abort_flag;
    int ctag[kMaxRing];   // newest chunk issued into each compressed slot (-1: none)
    int go[2];
    uint32_t drained[2];   // drain tasks finished, per partial-segment slot
    unsigned trace_gen;   // diagnostic builds only
};
static_assert(sizeof(GemmHeader) <= kHeaderBytes, "CTA header overlaps the offset staging area");

#ifdef ZS_TRACE
// Diagnostic build only (-DZS_TRACE): per-launch, per-CTA %globaltimer stamps.
// Layout: [4096 generation counters][gen][cta][256 slots].
__device__ unsigned long long* g_zs_trace = nullptr;
#define ZS_STAMP(slot)                                                                               \
    do {                                                                                             \
        if (zs_trace_ptr && (slot) < 256 && blockIdx.x < 4096 && zs_gen < 4)                         \
            zs_trace_ptr[4096 + ((size_t)zs_gen * 4096 + blockIdx.x) * 256 + (slot)] = clock64(); \
    } while (0)
#define ZS_STAMP0(slot)                                                                                      \
    do {                                                                                                     \
        if (zs_trace_ptr && hd->trace_gen < 4)                                                               \
            zs_trace_ptr[4096 + ((size_t)hd->trace_gen * 4096 + blockIdx.x) * 256 + (slot)] = clock64();    \
    } while (0)
#else
#define ZS_STAMP0(slot) \
    do {                \
    } while (0)
#define ZS_STAMP(slot) \
    do {               \
    } while (0)
#endif

__host__ __device__ __forceinline__ long long unit_begin(long long c, long long U, int G) { return div_nonneg(c * U, G); }
// CTA whose range holds unit g
__host__ __device__ __forceinline__ long long unit_owner(long long g, long long U, int G) {
    return div_nonneg((g + 1) * G - 1, U);
}

// Slot and phase of a ring of n mbarrier-guarded slots, advanced one use at a
// time (no divisions on the issue paths).
struct Ring {
    int slot = 0, n = 1;
    uint32_t phase = 0;
    bool wrapped = false;   // every slot has been used at least once
    __device__ void init(int nslots) { slot = 0; n = nslots; phase = 0; wrapped = false; }
    __device__ void step() {
        if (++slot == n) { slot = 0; phase ^= 1u; wrapped = true; }
    }
};

// This CTA's units and segments.
struct CtaRange {
    long long u0;   // first global unit
    int n;          // units
    long long T0;   // first output tile
    int nseg;       // segments (output tiles touched)
    int gtk;
    int off0;       // u0 - T0 * gtk: position of the first unit inside its tile
    int len0;       // units of the first segment
    __device__ bool seg_full(int s) const { return (T0 + s) * gtk >= u0 && (T0 + s + 1) * gtk <= u0 + n; }
    // workspace slot of a partial segment: 0 = the CTA's first segment, 1 = its last
    __device__ int seg_slot(int s) const { return s == 0 ? 0 : 1; }
};

// Per-unit pipeline position, advanced one unit at a time: output tile, K block,
// A-ring slot and the compressed chunk holding the unit. Chunks are up to cu
// consecutive units of one output tile starting at K blocks that are multiples
// of cu (and at the ends of the CTA's range); their streams are contiguous in
// every array, so each is fetched with a handful of TMA requests.
struct UnitCursor {
    int i = 0;      // unit
    int t = 0;      // output tile - T0
    int kb = 0;     // K block inside the tile
    int cpos = 0;   // kb % cu
    int u = 0;      // position inside the chunk
    int clen = 0;   // units in the chunk
    Ring ra, rc;    // A ring slot of unit i, compressed ring slot of its chunk
    __device__ int chunk_len(const CtaRange& R, const GemmParams& p) const {
        return min(min(p.cu - cpos, R.gtk - kb), R.n - i);
    }
    __device__ void init(const CtaRange& R, const GemmParams& p) {
        i = 0; t = 0; kb = R.off0; cpos = R.off0 % p.cu; u = 0;
        ra.init(p.na);
        rc.init(p.nc);
        clen = R.n > 0 ? chunk_len(R, p) : 0;
    }
    __device__ void step(const CtaRange& R, const GemmParams& p) {
        ra.step();
        ++i; ++u; ++kb;
        if (++cpos == p.cu) cpos = 0;
        if (kb == R.gtk) { kb = 0; cpos = 0; ++t; }
        if (u == clen) {
            u = 0;
            rc.step();
            if (i < R.n) clen = chunk_len(R, p);
        }
    }
};

// GT offsets (hf, fallback) at the start and end of the unit's two GTs.
__device__ __forceinline__ void fetch_gt_offsets(const GemmParams& p, const CtaRange& R, int i, int4& e0, int4& e1) {
    e0 = e1 = make_int4(0, 0, 0, 0);
    if (i < R.n) {
        const int t = (R.off0 + i) / R.gtk, kb = R.off0 + i - t * R.gtk;   // tile offset and K block
        const long long T = R.T0 + t;
        const long long gi = (2 * T) * p.gtk + kb;
        const int2* o = reinterpret_cast<const int2*>(p.gt_off);
        const int2 a0 = o[gi], a1 = o[gi + 1];
        e0 = make_int4(a0.x, a0.y, a1.x, a1.y);
        if (2 * T + 1 < p.mgt) {
            const int2 c0 = o[gi + p.gtk], c1 = o[gi + p.gtk + 1];
            e1 = make_int4(c0.x, c0.y, c1.x, c1.y);
        }
    }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    zipgemm_kernel(const __grid_constant__ GemmMaps maps, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    GemmHeader* hd = reinterpret_cast<GemmHeader*>(smem);
#ifdef ZS_TRACE
    unsigned long long* const zs_trace_ptr = g_zs_trace;
    if (threadIdx.x == 0 && zs_trace_ptr) {
        hd->trace_gen = (unsigned)atomicAdd(zs_trace_ptr + (blockIdx.x & 4095), 1ull);
        if (hd->trace_gen < 4) {
            zs_trace_ptr[4096 + ((size_t)hd->trace_gen * 4096 + blockIdx.x) * 256 + 255] = clock64();
            zs_trace_ptr[4096 + ((size_t)hd->trace_gen * 4096 + blockIdx.x) * 256 + 254] = globaltimer_ns();
        }
    }
#endif
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x;

    CtaRange R;
    R.gtk = p.gtk;
    R.u0 = unit_begin(blockIdx.x, p.units, G);
    R.n = (int)(unit_begin(blockIdx.x + 1, p.units, G) - R.u0);
    R.T0 = div_nonneg(R.u0, p.gtk);
    R.nseg = R.n > 0 ? (int)(div_nonneg(R.u0 + R.n - 1, p.gtk) - R.T0 + 1) : 0;
    R.off0 = (int)(R.u0 - R.T0 * p.gtk);
    R.len0 = min(p.gtk - R.off0, R.n);

    // The producers start fetching as soon as their own barriers exist: they
    // initialise the compressed ring (one lane per slot), meet each other on
    // named barrier 2 and only signal (bar.arrive) the CTA-wide start barrier 1,
    // on which every other warp waits after its own set-up.
    int4 e0, e1;
    const bool producer = (warp == kCompWarp || warp == kCompWarp1);
    if (producer) fetch_gt_offsets(p, R, lane, e0, e1);
    if (warp == kCompWarp) {
        if (lane < p.nc) {
            mbar_init(&hd->comp_full[lane], 1);
            mbar_init(&hd->comp_empty[lane], kTasksPerUnit * p.cu);
        }
        if (lane < kMaxRing) hd->ctag[lane] = -1;
        if (lane == 0) hd->abort_flag = 0;
        fence_mbar_init();
    } else if (warp == 0) {
        if (lane < p.na) { mbar_init(&hd->a_full[lane], kTasksPerUnit); mbar_init(&hd->a_empty[lane], 1); }
        if (lane < p.nb) { mbar_init(&hd->b_full[lane], 1); mbar_init(&hd->b_empty[lane], 1); }
        if (lane < kMaxAcc) {
            mbar_init(&hd->acc_full[lane], 1);
            mbar_init(&hd->acc_empty[lane], 4 * (p.BN / 16));
        }
        if (lane < 2) hd->drained[lane] = 0;
        if (lane == 0 && (smem_u32(smem) & 1023u) && p.err) atomicOr(p.err, kErrStreamOverflow);
        fence_mbar_init();
    } else if (warp == kMmaWarp) {
        tmem_alloc(&hd->tmem_base, kTmemCols);
        tmem_relinquish();
    }
    if (warp == kBWarp && lane == 0) prefetch_tmap(&maps.x);
    if (producer && lane < 4)
        prefetch_tmap(lane == 0 ? &maps.b1 : lane == 1 ? &maps.b2 : lane == 2 ? &maps.b3 : &maps.mt);
    if (producer) {
        named_bar_sync(2, 64);
        named_bar_arrive(1, kGemmThreads);
    } else {
        tc_fence_before();
        named_bar_sync(1, kGemmThreads);
        tc_fence_after();
    }
#ifdef ZS_TRACE
    const unsigned zs_gen = zs_trace_ptr ? hd->trace_gen : 0u;
#endif
    if (tid == 0) ZS_STAMP(0);
    // The next grid on the stream may launch as soon as every CTA of this one
    // is running: its CTAs then take SMs the moment this grid's CTAs exit,
    // instead of idling until the slowest CTA of this grid reaches its
    // epilogue. It waits for this grid (griddepcontrol.wait) before it reads
    // X or touches C and the workspace.
    if (tid == 0) grid_dep_launch();
    const uint32_t tmem_d = hd->tmem_base;
    volatile int* abort_flag = &hd->abort_flag;
    const uint32_t smem0 = smem_u32(smem);

    if (producer) {
        // Two producer warps take alternate chunks (their issue latency, not the
        // TMA, bounds how fast one warp can refill slots). Per chunk: lanes 0-3 issue the 2-D tensor loads
        // of bitmaps 1-3 and the median offsets (both GT rows, cu K blocks each),
        // lanes 4-7 the 1-D bulk copies of the hf and fallback streams of the two
        // GT rows, all in one warp instruction; lanes 0..2*len-1 publish the
        // units' stream offsets inside the chunk for the decoders. GT offsets are
        // fetched 32 units ahead (lane = unit) into a 64-unit staging ring.
        const int pw = warp == kCompWarp ? 0 : 1;
        int4* uoffs = reinterpret_cast<int4*>(smem + kOffsStage + 2048u * (uint32_t)pw);   // [64 units][2 GT rows]
        int2* cinfo = reinterpret_cast<int2*>(smem + kChunkInfo);   // [slot][kMaxChunk][2 GT rows]
        const CUtensorMap* lmap = lane == 0 ? &maps.b1 : lane == 1 ? &maps.b2 : lane == 2 ? &maps.b3 : &maps.mt;
        const CUtensorMap* lmap1 = lane == 0 ? &maps.b1h : lane == 1 ? &maps.b2h : lane == 2 ? &maps.b3h : &maps.mth;
        const uint32_t ldst = lane < 3 ? 1024u * (uint32_t)(lane * p.cu) : p.c_mt;
        const int ssub = lane & 1;   // lanes 4-7: GT row of the stream copy
        const bool is_hf = lane < 6;
        const uint32_t fixed_bytes = 3136u * (uint32_t)p.cu;   // 3 x 2 x cu x 512 + 2 x cu x 32
        int staged = 0;
        UnitCursor uc;
        uc.init(R, p);
        bool ok = true;
        for (int cidx = 0; uc.i < R.n; ++cidx) {
            const int len = uc.clen, i0 = uc.i;
            if ((cidx & 1) != pw) {   // the other producer's chunk
                for (int j = 0; j < len; ++j) uc.step(R, p);
                continue;
            }
            while (staged < i0 + len) {
                __syncwarp();
                uoffs[((staged + lane) & 63) * 2] = e0;
                uoffs[((staged + lane) & 63) * 2 + 1] = e1;
                staged += 32;
                fetch_gt_offsets(p, R, staged + lane, e0, e1);   // in flight while these units are issued
                __syncwarp();
            }
            const int s = uc.rc.slot;
            if (lane == 0 && uc.rc.wrapped)
                ok = mbar_wait(&hd->comp_empty[s], uc.rc.phase ^ 1u, p.err, abort_flag);
            ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            if (lane == 0 && uc.rc.wrapped == false && i0 < 60) ZS_STAMP(150 + i0 / 2);
            const long long T = R.T0 + uc.t;
            const int nsub = (2 * T + 1 < p.mgt) ? 2 : 1;
            uint32_t size = 0;
            const uint8_t* src = nullptr;
            if (lane >= 4 && lane < 8 && ssub < nsub) {
                // hf or fallback stream of GT row ssub, validated against the slot
                const int4 f = uoffs[(i0 & 63) * 2 + ssub], l = uoffs[((i0 + len - 1) & 63) * 2 + ssub];
                const int beg = is_hf ? f.x : f.y, end = is_hf ? l.z : l.w;
                const uint32_t esz = is_hf ? 1u : 2u;
                const uint32_t cap = is_hf ? p.hf_area : 2u * p.full_area;
                const int al = is_hf ? 16 : 8;
                uint32_t bytes = end > beg ? (uint32_t)(end - beg) * esz : 0u;
                int b = beg;
                if (bytes > cap || (bytes & 15u) || (b & (al - 1)) || b < 0) {
                    if (p.err) atomicOr(p.err, kErrStreamOverflow);
                    bytes = min(bytes, cap) & ~15u;
                    b = max(b, 0) & ~(al - 1);
                }
                size = bytes;
                src = is_hf ? p.sm + b : reinterpret_cast<const uint8_t*>(p.full + b);
            }
            if (lane < 2 * len) {
                const int u = lane >> 1, sb = lane & 1;
                const int4 f = uoffs[(i0 & 63) * 2 + sb], e = uoffs[((i0 + u) & 63) * 2 + sb];
                cinfo[(s * kMaxChunk + u) * 2 + sb] = make_int2(max(e.x - f.x, 0), max(e.y - f.y, 0));
            }
            uint32_t total = __reduce_add_sync(0xFFFFFFFFu, size) + (nsub == 2 ? fixed_bytes : fixed_bytes / 2);
#ifdef ZS_TRACE
            if (p.debug & 4) { total = 0; size = 0; }   // diagnostic: no weight traffic
#endif
            __syncwarp();   // the chunk offsets above are released by lane 0's arrive
            uint64_t* bar = &hd->comp_full[s];
            if (lane == 0) {
                if (i0 < 100) ZS_STAMP(110 + i0);
                st_release_cta(&hd->ctag[s], cidx);   // slot s's previous fill has been consumed (and landed)
                mbar_arrive_expect_tx(bar, total);
            }
            __syncwarp();
            uint8_t* slot = smem + p.off_c + (size_t)s * p.c_slot;
            if (lane < 4 && total) {
                ZS_GUARD(p.off_c + (uint32_t)s * p.c_slot + ldst + (lane < 3 ? 1024u : 64u) * (uint32_t)p.cu <= p.smem_bytes, 0x100)
                tma_load_2d(slot + ldst, nsub == 2 ? lmap : lmap1, uc.kb * (lane < 3 ? 64 : 8), (int)(2 * T), bar);
            } else if (size) {
                ZS_GUARD(p.off_c + (uint32_t)s * p.c_slot + (is_hf ? p.c_hf[ssub] : p.c_full[ssub]) + size <= p.smem_bytes, 0x200)
                bulk_g2s(slot + (is_hf ? p.c_hf[ssub] : p.c_full[ssub]), src, size, bar);
            }
            __syncwarp();
            if (lane == 0 && i0 < 60) ZS_STAMP(180 + i0 / 2);
            for (int j = 0; j < len; ++j) uc.step(R, p);
        }
    } else if (warp == kBWarp) {
        if (lane == 0) {
            // X is the previous kernel's output in a layer pipeline: wait for it
            // (weights, decoding and the MMA ring setup do not depend on it)
            grid_dep_wait();
            Ring rb;
            rb.init(p.nb);
            int kb = R.off0;
            for (int i = 0; i < R.n; ++i) {
                if (rb.wrapped && !mbar_wait(&hd->b_empty[rb.slot], rb.phase ^ 1u, p.err, abort_flag)) break;
                if (i < 14) ZS_STAMP(94 + i);
                uint64_t* bar = &hd->b_full[rb.slot];
                if (p.debug & 2) {
                    mbar_arrive(bar);
                } else {
                    mbar_arrive_expect_tx(bar, (uint32_t)p.xrows * 128u);
                    ZS_GUARD(p.off_b + (uint32_t)(rb.slot + 1) * p.b_slot <= p.off_a, 0x40000)
                    tma_load_2d(smem + p.off_b + (size_t)rb.slot * p.b_slot, &maps.x, kb * kGT, 0, bar);
                }
                rb.step();
                if (++kb == p.gtk) kb = 0;
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            // The issuing thread shares its scheduler with four decoder warps, so the
            // per-unit path is kept short: shared-memory descriptors advance by
            // constants (A slot: 16 KB = 1024 descriptor units; K step of 16
            // elements: 32 bytes = 2 units) and the rings are plain counters.
            const uint32_t idesc = umma_idesc_bf16(128, p.BN);
            const uint64_t da0 = umma_desc_sw128(smem0 + p.off_a), db0 = umma_desc_sw128(smem0 + p.off_b);
            const uint32_t bstep = p.b_slot >> 4;
            uint64_t da = da0, db = db0;
            int sa = 0, sb = 0;
            uint32_t pa = 0, pb = 0;
            Ring racc;
            racc.init(p.n_acc);
            uint32_t d = tmem_d;
            int seg_left = R.len0;
            bool first = true;
            for (int i = 0; i < R.n; ++i) {
                if (i < 6) ZS_STAMP(42 + i);
                if (first && racc.wrapped &&
                    !mbar_wait(&hd->acc_empty[racc.slot], racc.phase ^ 1u, p.err, abort_flag))
                    break;
                if (!mbar_wait2(&hd->a_full[sa], pa, &hd->b_full[sb], pb, p.err, abort_flag)) break;
                if (i < 14) ZS_STAMP(50 + i);
                tc_fence_after();
#ifdef ZS_TRACE
                if (!(p.debug & 8))   // diagnostic: bit 8 skips the MMAs (commits still signal)
#endif
                ZS_GUARD(sa < p.na && sb < p.nb && racc.slot * p.BN + p.BN <= (int)kTmemCols, 0x10000) {
                    umma_bf16_ss(d, da, db, idesc, first ? 0u : 1u);
                    umma_bf16_ss(d, da + 2, db + 2, idesc, 1u);
                    umma_bf16_ss(d, da + 4, db + 4, idesc, 1u);
                    umma_bf16_ss(d, da + 6, db + 6, idesc, 1u);
                }
                if (i < 6) ZS_STAMP(30 + i);
                umma_commit(&hd->a_empty[sa]);
                umma_commit(&hd->b_empty[sb]);
                if (i < 6) ZS_STAMP(36 + i);
                if (++sa == p.na) { sa = 0; pa ^= 1u; da = da0; } else { da += 1024; }
                if (++sb == p.nb) { sb = 0; pb ^= 1u; db = db0; } else { db += bstep; }
                first = false;
                if (--seg_left == 0) {
                    umma_commit(&hd->acc_full[racc.slot]);
                    racc.step();
                    d = tmem_d + (uint32_t)(racc.slot * p.BN);
                    seg_left = min(p.gtk, R.n - i - 1);
                    first = true;
                }
                if (i < 40) ZS_STAMP(210 + i);
            }
            ZS_STAMP(1);
        }
    } else if (warp < kDecWarps) {
        // Decoder warps. The task list is a sequence of rows of 16 tasks: a unit
        // row holds the 4 median-tile-pair tasks of 4 consecutive units, a drain
        // row 16 drain tasks of one segment (a segment needs ceil(4 * BN/16 / 16)
        // rows). Warp w therefore always decodes median-tile pair w % 4 of units
        // w / 4 + 4j, and takes drain task 16 r + w of each drain row: no search
        // per task.
        // Drains of all segments follow the last unit row, except when the CTA
        // has more segments than accumulators: then segment s is drained in the
        // unit row that starts after the first unit of segment s + 1.
        const DecodeTables tabs = make_decode_tables(p.start_exp);
        const int2* cinfo = reinterpret_cast<const int2*>(smem + kChunkInfo);
        const int k = warp & 3, sub = k >> 1, w = 2 * (k & 1);   // GT row, first median tile
        const int dsize = 4 * (p.BN / 16), drows = (dsize + kDecWarps - 1) / kDecWarps;
        const int cmask = p.cu - 1;
        // mid-run drains: segment s before unit G * ceil((len0 + s * gtk + 1) / G), G = units in flight
        constexpr int UG = kUnitsInFlight;
        int mid_end = 0;
        if (R.nseg > p.n_acc)
            while (mid_end < R.nseg - 1 && UG * ((R.len0 + mid_end * R.gtk + UG) / UG) < R.n) ++mid_end;
        int sd = 0;
        int dpos = UG * ((R.len0 + UG) / UG);
        auto drain = [&](int s) {
            grid_dep_wait();   // C and the split-tile workspace may still be in use by the previous grid
            const int acc = s & (p.n_acc - 1);
            const long long T = R.T0 + s;
            const bool full = R.seg_full(s);
            for (int rr = 0; rr < drows; ++rr) {
                const int kk = kDecWarps * rr + warp;
                if (kk >= dsize) break;
                // 16 columns (kk / 4) of the accumulator, TMEM lane quarter kk % 4 (== warp % 4)
                const int q = kk & 3, c = 16 * (kk >> 2);
                if (!mbar_wait_sleep(&hd->acc_full[acc], (uint32_t)((s >> p.lacc) & 1), p.err, abort_flag)) return;
                tc_fence_after();
                const int m = (int)(T * 128) + 32 * q + lane;
                uint32_t r[16] = {0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0};
                ZS_GUARD(acc * p.BN + c + 16 <= (int)kTmemCols, 0x800)
                tmem_ld16(tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)(acc * p.BN + c), r);
                tmem_wait_ld();
                if (full) {
                    if (m < p.M) {
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int n = c + j;
                            if (n < p.N) {
                                const __nv_bfloat16 v = __float2bfloat16_rn(__uint_as_float(r[j]));
                                p.C[(size_t)n * p.M + m] = *reinterpret_cast<const uint16_t*>(&v);
                            }
                        }
                    }
                } else {
                    float* part = p.ws + ((size_t)blockIdx.x * 2 + R.seg_slot(s)) * (size_t)p.BN * 128;
                    ZS_GUARD(((size_t)blockIdx.x * 2 + R.seg_slot(s)) * (size_t)p.BN * 128 + (size_t)(c + 16) * 128 <=
                                 p.ws_floats,
                             0x1000)
#pragma unroll
                    for (int j = 0; j < 16; ++j) part[(size_t)(c + j) * 128 + 32 * q + lane] = __uint_as_float(r[j]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&hd->acc_empty[acc]);
                if (!full) {
                    // The last of the segment's drain tasks publishes the partial tile:
                    // the CTA-scope acq_rel counter orders every task's stores before
                    // one gpu-scope release increment of the tile's arrival counter.
                    __syncwarp();
                    if (lane == 0) {
                        uint32_t old;
                        asm volatile("atom.acq_rel.cta.shared::cta.add.u32 %0, [%1], 1;"
                                     : "=r"(old)
                                     : "r"(smem_u32(&hd->drained[R.seg_slot(s)]))
                                     : "memory");
                        if (old == (uint32_t)dsize - 1)
                            asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(p.cnt + 2 * T) : "memory");
                    }
                }
            }
        };
        // unit i = UG g + warp / 4: its tile row T and K block kb advance by UG units per row
        int i = warp >> 2;
        long long T = R.T0;
        int kb = R.off0 + i;
        while (kb >= R.gtk) { kb -= R.gtk; ++T; }
        // A-ring slot and use count of unit i, advanced by UG units per row (na is any size >= 2)
        int sa = i % p.na, around = i / p.na;
        for (int g = 0; UG * g < R.n; ++g, i += UG) {
#ifdef ZS_TRACE
            if (lane == 0 && warp == 0 && g < 6) ZS_STAMP(131 + 4 * g);
#endif
            while (sd < mid_end && dpos == UG * g) {
                drain(sd);
                ++sd;
                dpos = UG * ((R.len0 + sd * R.gtk + UG) / UG);
            }
            if (*abort_flag) break;
            if (i < R.n) {
                // chunk of unit i: chunks start at global units that are multiples of cu
                // (and at the CTA's first unit)
                const long long gu = R.u0 + i;
                const int c = (int)((gu >> p.lcu) - (R.u0 >> p.lcu));
                const int u = (int)(gu & cmask) - (c == 0 ? (int)(R.u0 & cmask) : 0);
                const int start = i - u;
                const int clen = min(p.cu - (int)((R.u0 + start) & cmask), R.n - start);
                const int cs = c & (p.nc - 1);
#ifdef ZS_TRACE
                const int tq = g;
                if (lane == 0 && warp == 0 && tq < 6) ZS_STAMP(70 + 4 * tq );
#endif
                // A parity wait only separates neighbouring phases. A decoder can run up to
                // ceil((UG - 1) / cu) + 1 chunks ahead of the oldest chunk in use, which may be
                // two fills of one slot ahead; so it first waits until its chunk has been issued
                // (the slot's previous fill has then landed and been consumed), after which the
                // parity of the slot's barrier identifies the chunk exactly.
                if (!wait_tag_at_least(&hd->ctag[cs], c, p.err, abort_flag)) break;
                // the unit's compressed chunk and a free A slot (the first na units have one)
                if (i >= p.na) {
                    if (!mbar_wait2(&hd->comp_full[cs], (uint32_t)((c >> p.lnc) & 1), &hd->a_empty[sa],
                                    (uint32_t)((around + 1) & 1), p.err, abort_flag, true))
                        break;
                } else if (!mbar_wait_sleep(&hd->comp_full[cs], (uint32_t)((c >> p.lnc) & 1), p.err, abort_flag)) {
                    break;
                }
#ifdef ZS_TRACE
                if (lane == 0 && warp == 0 && tq < 6) ZS_STAMP(72 + 4 * tq );
#endif
                if (2 * T + sub < p.mgt && !(p.debug & 1)) {
                    const uint32_t base = launder(smem0 + p.off_c + (uint32_t)cs * p.c_slot);
                    const int2 info = cinfo[(cs * kMaxChunk + u) * 2 + sub];
                    const uint32_t h0 = min((uint32_t)info.x, p.hf_area), f0 = min((uint32_t)info.y, p.full_area);
                    const uint32_t su = (uint32_t)(sub * p.cu + u);
                    GtView gv;
                    gv.bm = base + 512u * su;
                    gv.bstride = 1024u * (uint32_t)p.cu;
                    gv.mt = base + p.c_mt + 32u * su;
                    gv.sm = base + p.c_hf[sub] + h0;
                    gv.full = base + p.c_full[sub] + 2u * f0;
                    gv.hf_cap = p.hf_area - h0;
                    gv.full_cap = p.full_area - f0;
                    const uint32_t rows =
                        smem0 + p.off_a + (uint32_t)sa * kATileBytes + 128u * (uint32_t)(64 * sub + 16 * w);
                    ZS_GUARD(rows + 4096u <= smem0 + p.off_c && gv.sm + gv.hf_cap + 12u <= smem0 + p.smem_bytes &&
                                 gv.full + 2u * gv.full_cap + 2u <= smem0 + p.smem_bytes &&
                                 gv.bm + 2u * gv.bstride + 8u * 64u <= smem0 + p.smem_bytes &&
                                 gv.mt + 32u <= smem0 + p.smem_bytes,
                             0x400)
                    decode_mt2_to_tile(gv, tabs, w, rows);
                }
#ifdef ZS_TRACE
                __syncwarp();
                if (lane == 0 && warp == 0 && tq < 6) ZS_STAMP(73 + 4 * tq );
#endif
                fence_proxy_async_smem();   // the tensor core reads the tile through the async proxy
#ifdef ZS_TRACE
                if (lane == 0 && warp == 0 && tq < 6) ZS_STAMP(130 + 4 * tq);
#endif
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(&hd->a_full[sa]);
                    // a short chunk's missing units are accounted for by its first task
                    const uint32_t extra = (k == 0 && u == 0) ? (uint32_t)(kTasksPerUnit * (p.cu - clen)) : 0u;
                    mbar_arrive_cnt(&hd->comp_empty[cs], 1u + extra);
                    if (k == 0 && i < 20) ZS_STAMP(10 + i);
                }
            }
            kb += UG;
            while (kb >= R.gtk) { kb -= R.gtk; ++T; }
            sa += UG;
            while (sa >= p.na) { sa -= p.na; ++around; }
        }
        if (!*abort_flag)
            for (; sd < R.nseg; ++sd) drain(sd);
    }
    __syncwarp();
    __syncthreads();
    if (tid == 0) ZS_STAMP(2);

#ifndef ZS_NO_EPI
    // ---------------- split-tile fixup (stream-K reduction) ----------------
    // The CTA's first and last segments may be partial. Threads 0 and 32 wait
    // (concurrently) until every contributor of the respective tile has
    // published its partial tile; then the CTA sums its slice of the columns of
    // each such tile over the contributors in CTA order and writes bf16.
    grid_dep_wait();   // C and the workspace may still be in use by the previous grid
    const long long U = p.units;
    long long fT[2] = {-1, -1}, fcf[2] = {0, 0};
    int fn[2] = {0, 0}, fidx[2] = {0, 0}, fslot0[2] = {0, 0};
    for (int which = 0; which < 2; ++which) {
        if (R.nseg == 0 || (which == 1 && R.nseg == 1)) continue;
        const int s = which == 0 ? 0 : R.nseg - 1;
        if (R.seg_full(s)) continue;
        const long long T = R.T0 + s;
        const long long cf = unit_owner(T * p.gtk, U, G), cl = unit_owner((T + 1) * p.gtk - 1, U, G);
        fT[which] = T;
        fcf[which] = cf;
        fn[which] = (int)(cl - cf + 1);
        fidx[which] = (int)(blockIdx.x - cf);
        // contributor cf holds T as its last segment (slot 1) unless its range starts at
        // T's first unit; every later contributor's range starts inside T (slot 0)
        fslot0[which] = unit_begin(cf, U, G) < T * p.gtk ? 1 : 0;
    }
    if ((tid == 0 || tid == 32) && fT[tid >> 5] >= 0) {
        const int which = tid >> 5;
        int ready = 0;
        const long long t0 = clock64();
        for (uint32_t it = 0;; ++it) {
            int v;
            asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p.cnt + 2 * fT[which]) : "memory");
            if (v >= fn[which]) { ready = 1; break; }
            if (*abort_flag) break;
            if ((it & 15) == 15 && clock64() - t0 > kWaitLimitCycles) {
                if (p.err) atomicOr(p.err, kErrWaitTimeout);
                *abort_flag = 1;
                break;
            }
            __nanosleep(20);
        }
        hd->go[which] = ready;
        ZS_STAMP(4 + 2 * which);
    }
    __syncthreads();
    {
        // This CTA's column slices of both split tiles form one list of float4
        // items (32 per column), so every thread has at most a few items and all
        // contributors' loads of an item (eight at a time) are in flight at once.
        // Contributors are summed in CTA order, so the result is deterministic.
        int sn0[2], slen[2];
#pragma unroll
        for (int which = 0; which < 2; ++which) {
            const bool on = fT[which] >= 0 && hd->go[which];
            const int ncon = on ? fn[which] : 1, idx = on ? fidx[which] : 0;
            sn0[which] = idx * p.BN / ncon;
            slen[which] = on ? ((idx + 1) * p.BN / ncon - sn0[which]) * 32 : 0;
        }
        const size_t cstride = 2 * (size_t)p.BN * 128;
        for (int e = tid; e < slen[0] + slen[1]; e += kGemmThreads) {
            const bool w1 = e >= slen[0];   // second split tile (selects keep the arrays in registers)
            const int el = w1 ? e - slen[0] : e;
            const int ncon = w1 ? fn[1] : fn[0];
            const long long cf = w1 ? fcf[1] : fcf[0], Tw = w1 ? fT[1] : fT[0];
            const int nl = (w1 ? sn0[1] : sn0[0]) + (el >> 5), m4 = (el & 31) * 4;
            const float* base = p.ws + (size_t)nl * 128 + m4 + (size_t)cf * cstride;
            const size_t first = (size_t)(w1 ? fslot0[1] : fslot0[0]) * p.BN * 128;
            float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int c0 = 0; c0 < ncon; c0 += 8) {
                float4 v[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                    const int cc = c0 + j;
                    if (cc < ncon) {
                        const size_t off = (size_t)cc * cstride + (cc == 0 ? first : 0);
                        ZS_GUARD((size_t)cf * cstride + off + (size_t)nl * 128 + m4 + 4 <= p.ws_floats, 0x4000)
                        v[j] = __ldcg(reinterpret_cast<const float4*>(base + off));
                    }
                }
#pragma unroll
                for (int j = 0; j < 8; ++j) { a.x += v[j].x; a.y += v[j].y; a.z += v[j].z; a.w += v[j].w; }
            }
            const int m = (int)(Tw * 128) + m4;
            if (nl < p.N && m < p.M) {
                __nv_bfloat162 lo = __floats2bfloat162_rn(a.x, a.y), hi = __floats2bfloat162_rn(a.z, a.w);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t*>(&lo);
                pk.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(p.C + (size_t)nl * p.M + m) = pk;
            }
        }
    }
    __syncthreads();
    if (tid == 0) ZS_STAMP(5);
    if ((tid == 0 || tid == 32) && fT[tid >> 5] >= 0 && hd->go[tid >> 5]) {
        // the last contributor to finish resets the tile's counters for the next launch
        const long long T = fT[tid >> 5];
        if (atomicAdd(p.cnt + 2 * T + 1, 1) == fn[tid >> 5] - 1) {
            p.cnt[2 * T] = 0;
            p.cnt[2 * T + 1] = 0;
        }
    }
#endif
    if (tid == 0) ZS_STAMP(3);
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_d, kTmemCols);
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
    bool attr_set = false;
};

// Per-device properties, and (once per device) the kernel attributes, so
// launches made during CUDA-graph capture issue no attribute calls.
static cudaError_t dev_setup(int dev, DevInfo* out) {
    static DevInfo info[64];
    static std::mutex mu;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = info[dev];
    if (!d.attr_set) {
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        ZS_RETURN_IF_ERR(
            cudaFuncSetAttribute(zipgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem));
        d.attr_set = true;
    }
    *out = d;
    return cudaSuccess;
}

// Split-tile workspace, one per (device, stream) so launches on different
// streams never share counters. Allocated (and zeroed) on first use and grown
// when a larger problem arrives; growth synchronizes the stream, so warm a
// stream up with the largest shape before capturing it into a CUDA graph.
struct Workspace {
    float* ws = nullptr;
    size_t ws_floats = 0;
    int* cnt = nullptr;
    size_t cnt_ints = 0;
};

static cudaError_t get_workspace(int dev, cudaStream_t stream, size_t ws_floats, size_t cnt_ints, Workspace* out) {
    static std::map<std::pair<int, cudaStream_t>, Workspace> cache;
    static std::mutex mu;
    std::lock_guard<std::mutex> g(mu);
    Workspace& w = cache[{dev, stream}];
    if (w.ws_floats < ws_floats || w.cnt_ints < cnt_ints) {
        cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
        ZS_RETURN_IF_ERR(cudaStreamIsCapturing(stream, &st));
        if (st != cudaStreamCaptureStatusNone) return cudaErrorStreamCaptureUnsupported;
        ZS_RETURN_IF_ERR(cudaStreamSynchronize(stream));
        if (w.ws) cudaFree(w.ws);
        if (w.cnt) cudaFree(w.cnt);
        w = Workspace{};
        const size_t nf = std::max(ws_floats, (size_t)1 << 20), nc = std::max(cnt_ints, (size_t)4096);
        ZS_RETURN_IF_ERR(cudaMalloc(&w.ws, nf * sizeof(float)));
        ZS_RETURN_IF_ERR(cudaMalloc(&w.cnt, nc * sizeof(int)));
        ZS_RETURN_IF_ERR(cudaMemset(w.cnt, 0, nc * sizeof(int)));
        w.ws_floats = nf;
        w.cnt_ints = nc;
    }
    *out = w;
    return cudaSuccess;
}

static cudaError_t launch_chunk(cudaStream_t stream, const DevInfo& di, int dev, GemmParams p, const uint16_t* X,
                                int max_hf, int max_full) {
    auto encode = get_encode_fn();
    if (!encode) return cudaErrorNotSupported;
    const int N = p.N;
    p.BN = (N + 15) / 16 * 16;
    // accumulators of BN columns: the largest power of two <= 4 that fits in TMEM
    p.n_acc = 4;
    while (p.n_acc > 1 && (uint32_t)(p.n_acc * p.BN) > kTmemCols) p.n_acc >>= 1;
    p.gtk = p.K / kGT;
    p.mgt = p.M / kGT;
    const long long mtiles = (p.M + 127) / 128;
    p.units = mtiles * p.gtk;
    const int G = (int)std::min<long long>(di.sms, p.units);

    // Shared memory: header | offset staging | B ring | A ring | compressed ring
    const uint32_t hfc = round_up_u32((uint32_t)max_hf, 16), ffc = round_up_u32((uint32_t)max_full, 8);
    p.b_slot = (uint32_t)p.BN * 128u;
    const uint32_t base = round_up_u32(kStageEnd, 1024);
    const uint32_t budget = (uint32_t)di.max_smem - base;
    auto layout = [&](int cu) {
        p.cu = cu;
        p.c_mt = 3u * 1024u * (uint32_t)cu;
        p.hf_area = hfc * (uint32_t)cu;
        p.full_area = ffc * (uint32_t)cu;
        p.c_hf[0] = round_up_u32(p.c_mt + 64u * (uint32_t)cu, 16);
        p.c_hf[1] = p.c_hf[0] + p.hf_area + 16;   // 16 bytes of read slack after each hf stream
        p.c_full[0] = p.c_hf[1] + p.hf_area + 16;
        p.c_full[1] = p.c_full[0] + 2u * p.full_area + 16;
        p.c_slot = round_up_u32(p.c_full[1] + 2u * p.full_area + 16, 128);
    };
    // Compressed ring first: the largest chunk of 4, 2 units that divides the K
    // blocks of a GT row (no TMA box crosses a row end) with four slots, else
    // two slots, else single-unit chunks, next to the minimum A ring (one slot
    // per unit the decoders work on) and a two-slot X ring. (Measured at config
    // 2: rings that force smaller chunks are slower -- the producers' TMA
    // request rate binds.) The rest deepens the A ring (the MMA may lag the
    // decoders by a unit without stalling them) and the X ring (X tiles are
    // L2 reads issued only when a slot frees).
    int cu = 1;
    bool placed = false;
    const uint32_t min_fixed = 2u * p.b_slot + (uint32_t)kUnitsInFlight * kATileBytes;
    for (int want = 4; want >= 2 && !placed; want -= 2) {
        for (int c = kMaxChunk; c >= 1 && !placed; c >>= 1) {
            if (c > p.gtk || p.gtk % c) continue;
            if (c == 1 && want == 4 && p.gtk % 2 == 0) continue;   // prefer 2 slots of 2 units
            layout(c);
            if (min_fixed + (uint32_t)want * p.c_slot <= budget) { cu = c; p.nc = want; placed = true; }
        }
    }
    if (!placed) return cudaErrorInvalidValue;
    layout(cu);
    p.na = kUnitsInFlight;
    p.nb = 2;
    {
        constexpr int U = kUnitsInFlight;
        const int pref[][2] = {{U + 2, 3}, {U + 1, 3}, {U + 2, 2}, {U + 1, 2}, {U, 3}};
        for (const auto& q : pref) {
            if ((uint32_t)q[1] * p.b_slot + (uint32_t)q[0] * kATileBytes + (uint32_t)p.nc * p.c_slot <= budget) {
                p.na = q[0];
                p.nb = q[1];
                break;
            }
        }
    }
#ifdef ZS_TRACE
    if (const char* e = getenv("ZS_RINGS")) {   // "na,nb,nc,cu" for experiments
        int a = 0, b = 0, c = 0, d = 0;
        if (sscanf(e, "%d,%d,%d,%d", &a, &b, &c, &d) == 4) { p.na = a; p.nb = b; p.nc = c; cu = d; layout(cu); }
    }
#endif
    auto ilog2 = [](int v) { int l = 0; while ((1 << l) < v) ++l; return l; };
    p.lcu = ilog2(p.cu);
    p.lnc = ilog2(p.nc);
    p.lacc = ilog2(p.n_acc);
    p.off_b = base;
    p.off_a = p.off_b + (uint32_t)p.nb * p.b_slot;
    p.off_c = p.off_a + (uint32_t)p.na * kATileBytes;
    const uint32_t smem_bytes = p.off_c + (uint32_t)p.nc * p.c_slot;

    Workspace w;
    ZS_RETURN_IF_ERR(get_workspace(dev, stream, (size_t)G * 2 * (size_t)p.BN * 128, (size_t)(2 * mtiles), &w));
    p.ws = w.ws;
    p.cnt = w.cnt;
    p.ws_floats = w.ws_floats;

    GemmMaps maps;
    p.xrows = std::min(p.BN, N);
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
    // bitmaps: [GT rows][K/64 x 64 u64]; median offsets: [GT rows][K/64 x 8 int32]
    auto encode_rows = [&](CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint32_t per_gt, uint32_t esz,
                           uint32_t rows) {
        cuuint64_t gdim[2] = {(cuuint64_t)p.gtk * per_gt, (cuuint64_t)p.mgt};
        cuuint64_t gstride[1] = {(cuuint64_t)p.gtk * per_gt * esz};
        cuuint32_t box[2] = {(cuuint32_t)(per_gt * p.cu), rows};
        cuuint32_t estr[2] = {1, 1};
        return encode(m, dt, 2, const_cast<void*>(base), gdim, gstride, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    const uint32_t rows2 = p.mgt >= 2 ? 2u : 1u;
    if (!encode_rows(&maps.b1, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b1, 64, 8, rows2) ||
        !encode_rows(&maps.b2, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b2, 64, 8, rows2) ||
        !encode_rows(&maps.b3, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b3, 64, 8, rows2) ||
        !encode_rows(&maps.mt, CU_TENSOR_MAP_DATA_TYPE_INT32, p.mt_off, 8, 4, rows2) ||
        !encode_rows(&maps.b1h, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b1, 64, 8, 1) ||
        !encode_rows(&maps.b2h, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b2, 64, 8, 1) ||
        !encode_rows(&maps.b3h, CU_TENSOR_MAP_DATA_TYPE_UINT64, p.b3, 64, 8, 1) ||
        !encode_rows(&maps.mth, CU_TENSOR_MAP_DATA_TYPE_INT32, p.mt_off, 8, 4, 1))
        return cudaErrorInvalidValue;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)G, 1, 1);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    p.smem_bytes = smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    // Programmatic dependent launch: this grid's CTAs may start (prologue,
    // weight loads, decoding) while the previous grid on the stream finishes;
    // the kernel waits on it (griddepcontrol.wait) before reading X and before
    // touching C and the workspace. All CTAs of a grid are resident at once
    // (G <= #SMs, one CTA per SM) and a grid never waits on a later one, so the
    // split-tile wait cannot deadlock.
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, zipgemm_kernel, maps, p);
}

cudaError_t launch_zipgemm(cudaStream_t stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                           const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                           int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M, int N,
                           int K, int split_k, unsigned* err) {
    // split_k is accepted for the reference signature; the stream-K split is
    // chosen from the shape and the SM count.
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
#ifdef ZS_TRACE
    // diagnostic builds: ZS_DEBUG bits switch off parts of the pipeline for timing experiments
    if (const char* d = getenv("ZS_DEBUG")) p.debug = atoi(d);
#endif
    // N > 256 runs as column chunks of 256 (each re-decodes W; such N are
    // tensor-bound, so the repeated decode is a small share of the time)
    for (int n0 = 0; n0 < N; n0 += 256) {
        GemmParams q = p;
        q.N = std::min(256, N - n0);
        q.C = C + (size_t)n0 * M;
        ZS_RETURN_IF_ERR(launch_chunk(stream, di, dev, q, X + (size_t)n0 * K, max_hf, max_full));
    }
    return cudaSuccess;
}

}  // namespace zs
