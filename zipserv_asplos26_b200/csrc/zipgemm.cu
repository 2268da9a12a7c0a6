// ZipGEMM for B200: C = W * X^T with W stored in TCA-TBE form.
// Replaces csrc/L_Kernel.cuh:295/575 BF16TripleBitmap_MM_Kernel_Fast/_Safe,
// csrc/Reduction_Kernel.cuh:15 SplitK_Reduction_BF16 and the launcher
// csrc/L_API.cu:119 BF16TripleBitmap_MM_API.
//
// Shapes (reference contract, test_mm.cu:410-428): W is M x K (compressed),
// X is N x K row-major (token-major, K contiguous), C is column-major M x N:
// C[n*M + m] = sum_k W[m][k] * X[n][k], fp32 accumulate, bf16 output.
//
// One CTA computes a 128-row x BN-column output tile over a range of K blocks
// (64 columns each = one global-tile (GT) column; a block holds two GTs).
// Three shared-memory rings decouple the stages of the pipeline:
//   compressed ring  per K block: both GTs' bitmaps, median offsets and hf /
//                    fallback streams, pulled by 1-D bulk copies (warp kCompWarp)
//   B ring           the 64 x BN activation tile, 2-D TMA with 128-byte swizzle
//                    (warp kBWarp)
//   A ring           the decoded 128 x 64 bf16 weight tile in the UMMA canonical
//                    K-major 128-byte-swizzled layout (written by the decoders)
// Decoders: kDecodeGroups groups of 8 warps, each group decoding every
// kDecodeGroups-th K block. In a group, warp (kh, q) owns rows 32q..32q+31 and
// column blocks 4kh..4kh+3; lane = weight row. The decoder is latency bound per
// warp, so many warps are kept resident (one CTA per SM, 27 warps).
// MMA: warp kMmaWarp owns TMEM and issues tcgen05.mma kind::f16 (M=128, N=BN,
// K=16) x4 per K block, fp32 accumulator in TMEM; tcgen05.commit frees the A
// and B slots.
// Split-K: the K blocks are split over the CTAs of a thread-block cluster
// (1 x S x 1). Each CTA drains its accumulator into its own shared memory, and
// after a cluster barrier every CTA reduces a slice of the output columns by
// reading all S partial tiles over distributed shared memory, then writes bf16
// with coalesced 8-byte stores. No global workspace and no second kernel.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

constexpr int kKSplit = 1;                          // warps per GT-half row block (column split)
constexpr int kDecodeGroups = 6 / kKSplit;          // groups of 4 * kKSplit warps, one K block each
constexpr int kGroupWarps = 4 * kKSplit;
constexpr int kDecodeWarps = kGroupWarps * kDecodeGroups;
constexpr int kCompWarp = kDecodeWarps;
constexpr int kBWarp = kDecodeWarps + 1;
constexpr int kMmaWarp = kDecodeWarps + 2;
constexpr int kGemmThreads = 32 * (kDecodeWarps + 3);
constexpr int kMaxRing = 12;
constexpr uint32_t kLutOffset = 1024;
constexpr uint32_t kOffsOffset = kLutOffset + 4u * kLutWords;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kASlotCols = 32;      // one decoded 128 x 64 bf16 A tile in TMEM

struct GemmParams {
    const uint8_t* sm;
    const uint16_t* full;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* mt_off;
    const int* gt_off;
    int max_hf, max_full, start_exp;
    uint16_t* C;
    int M, N, K;
    int BN;            // output columns per CTA (multiple of 16, <= 256)
    int kb_per_split;  // K blocks per cluster rank
    int nc, na, nb;    // ring depths
    int chunk;         // K blocks per compressed-ring slot (one bulk copy per stream per GT row)
    uint32_t tmem_cols;
    uint32_t off_b, off_c;          // smem ring bases (contiguous: B, compressed)
    uint32_t a_col;                 // TMEM column of A slot 0 (slots are kASlotCols apart)
    uint32_t b_slot, c_slot;        // smem slot sizes
    // compressed slot = 2 GT rows x [b1 | b2 | b3 (512*chunk each) | mt (32*chunk) | hf | fallback]
    uint32_t c_row, c_mt, c_hf, c_full;
    uint32_t hf_cap, full_cap;      // bytes available for one row's hf / fallback streams of a chunk
    unsigned* err;
};

struct GemmHeader {
    uint64_t comp_full[kMaxRing], comp_empty[kMaxRing];
    uint64_t a_full[kMaxRing], a_empty[kMaxRing];
    uint64_t b_full[kMaxRing], b_empty[kMaxRing];
    uint64_t accum;
    uint64_t red_bar;   // peers' partial slices landed in this CTA's receive slots
    uint32_t tmem_base;
    int abort_flag;
};

#ifdef ZS_TRACE
// Diagnostic build only (-DZS_TRACE): per-CTA %globaltimer stamps.
__device__ unsigned long long* g_zs_trace = nullptr;
#define ZS_STAMP(slot)                                                                                    \
    do {                                                                                                  \
        if (zs_trace_ptr && (slot) < 256) {                                                               \
            const size_t cta_ = blockIdx.x + (size_t)gridDim.x * (blockIdx.y + (size_t)gridDim.y * blockIdx.z); \
            zs_trace_ptr[cta_ * 256 + (slot)] = (unsigned long long)clock64();                                  \
        }                                                                                                 \
    } while (0)
#else
#define ZS_STAMP(slot) \
    do {               \
    } while (0)
#endif

__device__ __forceinline__ uint32_t ring_parity(int i, int n) { return (uint32_t)((i / n) & 1); }
// parity of the previous use of slot i % n (i >= n)
__device__ __forceinline__ uint32_t ring_prev_parity(int i, int n) { return (uint32_t)(((i / n) + 1) & 1); }

__global__ void __launch_bounds__(kGemmThreads, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
#ifdef ZS_TRACE
    unsigned long long* const zs_trace_ptr = g_zs_trace;
#endif
    GemmHeader* hd = reinterpret_cast<GemmHeader*>(smem);
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem + kLutOffset);
    int2* offs = reinterpret_cast<int2*>(smem + kOffsOffset);   // [2][kb_per_split + 1]

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mtile = blockIdx.x, ntile = blockIdx.z;
    const uint32_t rank = cluster_ctarank();
    const int S = gridDim.y;
    const int gtk = p.K / kGT;
    const int kb0 = (int)rank * p.kb_per_split;
    const int nk = max(0, min(gtk, kb0 + p.kb_per_split) - kb0);
    const int gm0 = 2 * mtile;                      // first GT row of this tile
    const bool has_g1 = (gm0 + 1) < (p.M / kGT);    // second GT row present
    const int ostride = p.kb_per_split + 1;

    // The producer warp stages the GT offsets first; the global-load latency
    // overlaps the table fill and the TMEM allocation.
    if (warp == kCompWarp) {
        for (int sub = 0; sub < (has_g1 ? 2 : 1); ++sub) {
            const int2* src = reinterpret_cast<const int2*>(p.gt_off) + (long long)(gm0 + sub) * gtk + kb0;
            for (int i = lane; i <= nk; i += 32) offs[sub * ostride + i] = src[i];
        }
    }
    fill_spread_table(lut, tid, kGemmThreads);
    if (tid == 0) {
        // the 128-byte-swizzled operand tiles need a 1024-byte aligned window
        if ((smem_u32(smem) & 1023u) && p.err) atomicOr(p.err, kErrStreamOverflow);
        for (int s = 0; s < p.nc; ++s) {
            mbar_init(&hd->comp_full[s], 1);
            mbar_init(&hd->comp_empty[s], kGroupWarps * p.chunk);   // every K block of the chunk, each group warp
        }
        for (int s = 0; s < p.na; ++s) { mbar_init(&hd->a_full[s], kGroupWarps); mbar_init(&hd->a_empty[s], 1); }
        for (int s = 0; s < p.nb; ++s) { mbar_init(&hd->b_full[s], 1); mbar_init(&hd->b_empty[s], 1); }
        mbar_init(&hd->accum, 1);
        mbar_init(&hd->red_bar, 1);
        hd->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&hd->tmem_base, p.tmem_cols);
        tmem_relinquish();
    }
    if (warp == kBWarp && lane == 0) prefetch_tmap(&tmap_x);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = hd->tmem_base;
    volatile int* abort_flag = &hd->abort_flag;
    if (tid == 0) ZS_STAMP(0);

    if (warp == kCompWarp) {
        if (lane == 0) {
            const int nchunks = (nk + p.chunk - 1) / p.chunk;
            for (int j = 0; j < nchunks; ++j) {
                const int s = j % p.nc;
                if (j >= p.nc && !mbar_wait(&hd->comp_empty[s], ring_prev_parity(j, p.nc), p.err, abort_flag))
                    break;
                const int i0 = j * p.chunk, i1 = min(nk, i0 + p.chunk), cn = i1 - i0;
                uint8_t* slot = smem + p.off_c + (size_t)s * p.c_slot;
                uint32_t hb[2] = {0, 0}, fb[2] = {0, 0}, bytes = 0;
                int h0[2] = {0, 0}, f0[2] = {0, 0};
                for (int sub = 0; sub < (has_g1 ? 2 : 1); ++sub) {
                    const int2 a0 = offs[sub * ostride + i0], a1 = offs[sub * ostride + i1];
                    h0[sub] = a0.x;
                    f0[sub] = a0.y;
                    hb[sub] = a1.x > a0.x ? (uint32_t)(a1.x - a0.x) : 0u;
                    fb[sub] = a1.y > a0.y ? (uint32_t)(a1.y - a0.y) * 2u : 0u;
                    if (hb[sub] > p.hf_cap || fb[sub] > p.full_cap || (hb[sub] & 15u) || (fb[sub] & 15u) ||
                        (a0.x & 15) || (a0.y & 7) || a0.x < 0 || a0.y < 0) {
                        if (p.err) atomicOr(p.err, kErrStreamOverflow);
                        hb[sub] = min(hb[sub], p.hf_cap) & ~15u;
                        fb[sub] = min(fb[sub], p.full_cap) & ~15u;
                        h0[sub] = max(h0[sub], 0) & ~15;
                        f0[sub] = max(f0[sub], 0) & ~7;
                    }
                    bytes += (3 * 512 + 32) * (uint32_t)cn + hb[sub] + fb[sub];
                }
                uint64_t* bar = &hd->comp_full[s];
                ZS_STAMP(1 + j);
                mbar_arrive_expect_tx(bar, bytes);
                for (int sub = 0; sub < (has_g1 ? 2 : 1); ++sub) {
                    const long long g = (long long)(gm0 + sub) * gtk + kb0 + i0;
                    uint8_t* row = slot + sub * p.c_row;
                    const uint32_t bmb = 512u * (uint32_t)cn;
                    bulk_g2s(row, p.b1 + g * 64, bmb, bar);
                    bulk_g2s(row + 512u * p.chunk, p.b2 + g * 64, bmb, bar);
                    bulk_g2s(row + 1024u * p.chunk, p.b3 + g * 64, bmb, bar);
                    bulk_g2s(row + p.c_mt, p.mt_off + g * 8, 32u * (uint32_t)cn, bar);
                    if (hb[sub]) bulk_g2s(row + p.c_hf, p.sm + h0[sub], hb[sub], bar);
                    if (fb[sub]) bulk_g2s(row + p.c_full, p.full + f0[sub], fb[sub], bar);
                }
            }
        }
    } else if (warp == kBWarp) {
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % p.nb;
                if (i >= p.nb && !mbar_wait(&hd->b_empty[s], ring_prev_parity(i, p.nb), p.err, abort_flag)) break;
                uint64_t* bar = &hd->b_full[s];
                ZS_STAMP(20 + i);
                mbar_arrive_expect_tx(bar, (uint32_t)p.BN * 128u);
                tma_load_2d(smem + p.off_b + (size_t)s * p.b_slot, &tmap_x, (kb0 + i) * kGT, ntile * p.BN, bar);
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(128, p.BN);
            for (int i = 0; i < nk; ++i) {
                const int sa = i % p.na, sb = i % p.nb;
                if (!mbar_wait(&hd->a_full[sa], ring_parity(i, p.na), p.err, abort_flag) ||
                    !mbar_wait(&hd->b_full[sb], ring_parity(i, p.nb), p.err, abort_flag))
                    break;
                ZS_STAMP(100 + i);
                tc_fence_after();
                const uint32_t a_tm = tmem_d + p.a_col + (uint32_t)sa * kASlotCols;
                const uint32_t b_addr = smem_u32(smem + p.off_b + (size_t)sb * p.b_slot);
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_bf16_ts(tmem_d, a_tm + 8u * k, umma_desc_sw128(b_addr + 32 * k), idesc,
                                 (i > 0 || k > 0) ? 1u : 0u);
                umma_commit(&hd->a_empty[sa]);
                umma_commit(&hd->b_empty[sb]);
            }
            umma_commit(&hd->accum);
        }
    } else {
        // decoders: warp = kGroupWarps*group + 4*ks + q; q = TMEM lane quarter =
        // rows 32q..32q+31; ks selects column blocks [ks*8/kKSplit, (ks+1)*8/kKSplit)
        const int group = warp / kGroupWarps, ks = (warp % kGroupWarps) >> 2, q = warp & 3;
        const int sub = q >> 1, half = q & 1;
        const DecodeTables tabs = make_decode_tables(p.start_exp);
        const bool active = (sub == 0) || has_g1;
        const uint32_t lut_lane = launder(smem_u32(lut)) + 4u * (uint32_t)lane;
        const uint32_t smem0 = smem_u32(smem);
        const uint32_t tlane = tmem_d + ((uint32_t)(32 * q) << 16) + p.a_col;
        for (int i = group; i < nk; i += kDecodeGroups) {
            const int jc = i / p.chunk, u = i - jc * p.chunk;
            const int sc = jc % p.nc, sa = i % p.na;
            if (!mbar_wait(&hd->comp_full[sc], ring_parity(jc, p.nc), p.err, abort_flag)) break;
            if (i >= p.na && !mbar_wait(&hd->a_empty[sa], ring_prev_parity(i, p.na), p.err, abort_flag)) break;
            tc_fence_after();
            if (active) {
                const uint32_t row = launder(smem0 + p.off_c + (uint32_t)sc * p.c_slot + (uint32_t)sub * p.c_row);
                const int2 base = offs[sub * ostride + jc * p.chunk], cur = offs[sub * ostride + i];
                const uint32_t hl = min((uint32_t)max(cur.x - base.x, 0), p.hf_cap);
                const uint32_t fl = min((uint32_t)max(cur.y - base.y, 0) * 2u, p.full_cap);
                GtView g;
                g.bm = row + 512u * (uint32_t)u;
                g.bstride = 512u * (uint32_t)p.chunk;
                g.mt = row + p.c_mt + 32u * (uint32_t)u;
                g.sm = row + p.c_hf + hl;
                g.full = row + p.c_full + fl;
                g.hf_cap = p.hf_cap - hl;
                g.full_cap = (p.full_cap - fl) / 2;
                const uint32_t ta = tlane + (uint32_t)sa * kASlotCols;
                decode_gt_half_regs<8 / kKSplit>(g, lut_lane, tabs, half, ks * (8 / kKSplit),
                                    [&](int kc, uint32_t o0, uint32_t o1, uint32_t o2, uint32_t o3) {
                                        tmem_st4(ta + 4u * (uint32_t)kc, o0, o1, o2, o3);
                                    });
                tmem_wait_st();
            }
            tc_fence_before();
            __syncwarp();
            if (warp % kGroupWarps == 0 && lane == 0) ZS_STAMP(60 + i);
            if (lane == 0) {
                mbar_arrive(&hd->a_full[sa]);
                mbar_arrive(&hd->comp_empty[sc]);
            }
        }
    }

    // Single-thread roles (producers, MMA) must reconverge before the warp-wide
    // .aligned cluster barriers below; otherwise the idle lanes sit in the
    // barrier while lane 0 still runs its loop.
    __syncwarp();

    // ---------------- epilogue: split-K reduction over the cluster -----------
    // Columns of the BN-wide tile are split over the S cluster ranks. Each CTA
    // drains its fp32 accumulator into its own shared memory ([BN][128], the
    // drained ring area), then after one cluster barrier sends every other
    // rank the slice that rank owns with one bulk copy (TMA engine, shared ->
    // peer shared) into the receive slot reserved for this source rank. Each
    // rank waits on its own mbarrier for the S-1 slices, sums the S partials of
    // its columns in a fixed order (deterministic) and writes bf16.
    // BN > 128 runs in passes of 128 columns so the buffers fit.
    const int EB = min(p.BN, 128);
    const int cols_per = (EB + S - 1) / S;
    const int own_nb = (int)rank * cols_per;
    const int own_cols = max(0, min(EB, own_nb + cols_per) - own_nb);
    float* part = reinterpret_cast<float*>(smem + p.off_b);             // [EB][128] local partial
    float* recv = part + (size_t)EB * 128;                               // [S][cols_per][128]
    bool acc_ok = false;
    if (warp < 4) acc_ok = (nk > 0) && mbar_wait(&hd->accum, 0, p.err, abort_flag);
    for (int pass = 0; pass * EB < p.BN; ++pass) {
        if (pass > 0) cluster_sync();   // every rank is done with the previous pass's buffers
        if (warp < 4) {
            const int q = warp;
            if (acc_ok) {
                tc_fence_after();
                for (int c = 0; c < EB; c += 16) {
                    uint32_t r[16];
                    tmem_ld16(tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)(pass * EB + c), r);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 16; ++j) part[(c + j) * 128 + 32 * q + lane] = __uint_as_float(r[j]);
                }
            } else {
                for (int c = 0; c < EB; ++c) part[c * 128 + 32 * q + lane] = 0.f;
            }
            fence_proxy_async_smem();   // the bulk copies below read these values through the async proxy
        }
        if (tid == 0 && S > 1) mbar_arrive_expect_tx(&hd->red_bar, (uint32_t)(S - 1) * (uint32_t)own_cols * 512u);
        tc_fence_before();
        if (tid == 0 && pass == 0) ZS_STAMP(220);
        cluster_sync();
        if (tid == 0 && pass == 0) ZS_STAMP(221);
        if (tid == 0) {
            for (int r2 = 0; r2 < S; ++r2) {
                if (r2 == (int)rank) continue;
                const int nb2 = r2 * cols_per, nc2 = max(0, min(EB, nb2 + cols_per) - nb2);
                if (nc2 == 0) continue;
                const uint32_t dst = smem_u32(recv + ((size_t)rank * cols_per) * 128);
                bulk_s2peer(mapa_shared(dst, (uint32_t)r2), smem_u32(part + (size_t)nb2 * 128),
                            (uint32_t)nc2 * 512u, mapa_shared(smem_u32(&hd->red_bar), (uint32_t)r2));
            }
            bulk_commit();
        }
        const bool got = (S == 1) || own_cols == 0 || mbar_wait(&hd->red_bar, (uint32_t)(pass & 1), p.err, abort_flag);
        if (tid == 0 && pass == 0) ZS_STAMP(222);
        if (got) {
            for (int idx = tid; idx < own_cols * 32; idx += kGemmThreads) {
                const int nl = idx >> 5, m4 = (idx & 31) * 4;
                const int n = ntile * p.BN + pass * EB + own_nb + nl;
                const int m = mtile * 128 + m4;
                if (n >= p.N || m >= p.M) continue;
                float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int sr = 0; sr < S; ++sr) {
                    const float* src = (sr == (int)rank) ? part + (size_t)(own_nb + nl) * 128
                                                         : recv + ((size_t)sr * cols_per + nl) * 128;
                    const float4 v = *reinterpret_cast<const float4*>(src + m4);
                    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
                }
                __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
                __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
                uint2 pk;
                pk.x = *reinterpret_cast<uint32_t*>(&lo);
                pk.y = *reinterpret_cast<uint32_t*>(&hi);
                *reinterpret_cast<uint2*>(p.C + (size_t)n * p.M + m) = pk;
            }
        }
        // our outgoing copies must finish reading `part` before it is reused or the CTA exits
        if (tid == 0) bulk_wait_read0();
        __syncthreads();
    }
    if (tid == 0) ZS_STAMP(223);
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

static uint32_t pow2_cols(int n) {
    uint32_t c = 32;
    while ((int)c < n) c <<= 1;
    return c;
}

struct DevInfo {
    int sms = 148;
    int max_smem = 232448;
    bool attr_set = false;
};

// Per-device properties, and (once per device) the kernel attributes, so
// launches made during CUDA-graph capture issue no attribute calls.
static cudaError_t dev_setup(DevInfo* out) {
    static DevInfo info[64];
    static std::mutex mu;
    int dev = 0;
    ZS_RETURN_IF_ERR(cudaGetDevice(&dev));
    if (dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    DevInfo& d = info[dev];
    if (!d.attr_set) {
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev));
        ZS_RETURN_IF_ERR(cudaDeviceGetAttribute(&d.max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        ZS_RETURN_IF_ERR(
            cudaFuncSetAttribute(zipgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, d.max_smem));
        ZS_RETURN_IF_ERR(cudaFuncSetAttribute(zipgemm_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
        d.attr_set = true;
    }
    *out = d;
    return cudaSuccess;
}

cudaError_t launch_zipgemm(cudaStream_t stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                           const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                           int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M, int N,
                           int K, int split_k, unsigned* err) {
    if (M <= 0 || N <= 0 || K <= 0 || (M % 64) || (K % 64)) return cudaErrorInvalidValue;
    if (split_k < 1) return cudaErrorInvalidValue;
    if (max_hf < 0 || max_full < 0 || max_hf > 4096 + 15 || max_full > 4096 + 7) return cudaErrorInvalidValue;
    if (!b1 || !b2 || !b3 || !mt_off || !gt_off || !X || !C) return cudaErrorInvalidValue;
    if ((max_hf > 0 && !sm) || (max_full > 0 && !full)) return cudaErrorInvalidValue;
    if (!aligned16(sm) || !aligned16(full) || !aligned16(b1) || !aligned16(b2) || !aligned16(b3) ||
        !aligned16(mt_off) || !aligned16(X) || (reinterpret_cast<uintptr_t>(C) & 7u) ||
        (reinterpret_cast<uintptr_t>(gt_off) & 7u))
        return cudaErrorInvalidValue;
    auto encode = get_encode_fn();
    if (!encode) return cudaErrorNotSupported;
    DevInfo di;
    ZS_RETURN_IF_ERR(dev_setup(&di));

    GemmParams p{};
    p.sm = sm; p.full = full; p.b1 = b1; p.b2 = b2; p.b3 = b3; p.mt_off = mt_off; p.gt_off = gt_off;
    p.max_hf = max_hf; p.max_full = max_full; p.start_exp = start_exp & 0xFF;
    p.C = C; p.M = M; p.N = N; p.K = K; p.err = err;
    p.BN = std::min(256, (N + 15) / 16 * 16);
    p.tmem_cols = kTmemCols;
    p.a_col = round_up_u32((uint32_t)p.BN, kASlotCols);
    p.b_slot = (uint32_t)p.BN * 128u;

    const int mtiles = (M + 127) / 128;
    const int ntiles = (N + p.BN - 1) / p.BN;
    const int nkb = K / 64;
    int S = std::max(1, di.sms / std::max(1, mtiles * ntiles));
    S = std::max(S, split_k);
    S = std::min(S, std::min(8, nkb));
    p.kb_per_split = (nkb + S - 1) / S;
    S = (nkb + p.kb_per_split - 1) / p.kb_per_split;  // drop empty ranks

    // Shared memory: header | spread table | staged offsets | B ring | A ring | compressed ring
    const uint32_t offs_bytes = round_up_u32(2u * (uint32_t)(p.kb_per_split + 1) * 8u, 1024);
    const uint32_t base = round_up_u32(kOffsOffset + offs_bytes, 1024);
    const uint32_t budget = (uint32_t)di.max_smem - base;
    p.na = (int)std::min<uint32_t>(kMaxRing, (kTmemCols - p.a_col) / kASlotCols);
    p.nb = p.BN <= 128 ? 6 : 3;
    const uint32_t hfc = round_up_u32((uint32_t)max_hf, 16), ffc = round_up_u32((uint32_t)max_full * 2u, 16);
    auto slot_bytes = [&](int ch) {
        const uint32_t row = round_up_u32((1536u + 32u) * ch + (hfc * ch + 16) + (ffc * ch + 16), 128);
        return 2u * row;
    };
    uint32_t ab = (uint32_t)p.nb * p.b_slot;
    while (p.nb > 2 && ab + 3 * slot_bytes(2) > budget) ab = (uint32_t)(--p.nb) * p.b_slot;
    if (ab + 2 * slot_bytes(1) > budget) return cudaErrorInvalidValue;
    // Largest chunk (<= 8 K blocks) that still leaves a double-buffered ring.
    p.chunk = 1;
    for (int ch = 8; ch > 1; --ch)
        if (ab + 3 * slot_bytes(ch) <= budget) { p.chunk = ch; break; }
    p.chunk = std::min(p.chunk, p.kb_per_split);
    p.c_slot = slot_bytes(p.chunk);
    p.c_row = p.c_slot / 2;
    p.c_mt = 1536u * p.chunk;
    p.c_hf = p.c_mt + 32u * p.chunk;
    p.hf_cap = hfc * p.chunk;
    p.c_full = p.c_hf + p.hf_cap + 16;
    p.full_cap = ffc * p.chunk;
    p.nc = (int)std::min<uint32_t>(kMaxRing, (budget - ab) / p.c_slot);
    p.off_b = base;
    p.off_c = p.off_b + (uint32_t)p.nb * p.b_slot;
    const uint32_t smem_bytes = p.off_c + (uint32_t)p.nc * p.c_slot;
    const uint32_t eb = (uint32_t)std::min(p.BN, 128);
    const uint32_t cols_per = (eb + (uint32_t)S - 1) / (uint32_t)S;
    if (smem_bytes - p.off_b < (eb + (uint32_t)S * cols_per) * 512u) return cudaErrorInvalidValue;

    CUtensorMap tmap;
    cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t gstride[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)p.BN};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(X), gdim, gstride, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)mtiles, (unsigned)S, (unsigned)ntiles);
    cfg.blockDim = dim3(kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 1;
    attr[0].val.clusterDim.y = (unsigned)S;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, zipgemm_kernel, tmap, p);
}

}  // namespace zs
