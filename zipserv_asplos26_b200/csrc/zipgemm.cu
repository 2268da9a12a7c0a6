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
// (64 columns each = one global tile column). Warp roles (320 threads):
//   warp 8      producer: per K block, 1-D bulk copies of the two GTs' bitmaps,
//               median offsets and hf / fallback streams, plus a 2-D TMA load
//               of the 64 x BN activation tile (128-byte swizzle), all on one
//               mbarrier with expect_tx.
//   warps 0..7  decoders, two groups of four alternating K blocks. Lane = W row:
//               each thread decodes its row's 8 column blocks with the
//               branch-free row decoder and stores 16-byte chunks straight into
//               the UMMA canonical K-major 128-byte-swizzled A tile.
//   warp 9      TMEM allocator + MMA issuer: tcgen05.mma kind::f16
//               (M=128, N=BN, K=16) x4 per K block, accumulator in TMEM;
//               tcgen05.commit releases the stage.
// Split-K: the K blocks are split over the CTAs of a thread-block cluster
// (1 x S x 1). Each CTA drains its TMEM accumulator into its own shared memory,
// and after a cluster barrier every CTA reduces a slice of the output columns
// by reading all S partial tiles over distributed shared memory, then writes
// bf16 with coalesced 8-byte stores. No global workspace, no second kernel.
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

constexpr int kGemmThreads = 320;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr uint32_t kHeaderBytes = 2048;
constexpr int kMaxStages = 8;

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
    int nstages;
    uint32_t tmem_cols;
    // stage layout (bytes)
    uint32_t stage_bytes, off_b, off_bm, off_mt, off_hf, off_full, hf_slot, full_slot;
    unsigned* err;
};

struct GemmHeader {
    uint64_t full[kMaxStages];
    uint64_t decoded[kMaxStages];
    uint64_t empty[kMaxStages];
    uint64_t accum;
    uint32_t tmem_base;
    int abort_flag;
};

__global__ void __launch_bounds__(kGemmThreads, 1)
    zipgemm_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem);
    GemmHeader* hd = reinterpret_cast<GemmHeader*>(smem + 1024);
    uint8_t* stages = smem + kHeaderBytes;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mtile = blockIdx.x, ntile = blockIdx.z;
    const uint32_t rank = cluster_ctarank();
    const int S = gridDim.y;
    const int nkb = p.K / kGT, gtk = nkb;
    const int kb0 = (int)rank * p.kb_per_split;
    const int nk = max(0, min(nkb, kb0 + p.kb_per_split) - kb0);
    const int gm0 = 2 * mtile;                      // first GT row of this tile
    const bool has_g1 = (gm0 + 1) < (p.M / kGT);    // second GT row present
    const int NS = p.nstages;

    for (int i = tid; i < 256; i += kGemmThreads) lut[i] = spread8_value(i);
    if (tid == 0) {
        // the 128-byte-swizzled operand tiles need a 1024-byte aligned window
        if ((smem_u32(smem) & 1023u) && p.err) atomicOr(p.err, kErrStreamOverflow);
        for (int s = 0; s < NS; ++s) {
            mbar_init(&hd->full[s], 1);
            mbar_init(&hd->decoded[s], 4);
            mbar_init(&hd->empty[s], 1);
        }
        mbar_init(&hd->accum, 1);
        hd->abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == kMmaWarp) {
        tmem_alloc(&hd->tmem_base, p.tmem_cols);
        tmem_relinquish();
    }
    if (warp == kProducerWarp && lane == 0) prefetch_tmap(&tmap_x);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = hd->tmem_base;
    volatile int* abort_flag = &hd->abort_flag;

    if (warp == kProducerWarp) {
        if (lane == 0) {
            for (int i = 0; i < nk; ++i) {
                const int s = i % NS;
                if (i >= NS && !mbar_wait(&hd->empty[s], ((i / NS) + 1) & 1, p.err, abort_flag)) break;
                uint8_t* st = stages + (size_t)s * p.stage_bytes;
                const int kb = kb0 + i;
                const long long g0 = (long long)gm0 * gtk + kb;
                GtCopy c0 = gt_copy_range(p.gt_off, g0, p.max_hf, p.max_full, p.err);
                GtCopy c1{0, 0, 0u, 0u};
                if (has_g1) c1 = gt_copy_range(p.gt_off, g0 + gtk, p.max_hf, p.max_full, p.err);
                const uint32_t fixed = 3 * 512 + 32;
                uint32_t bytes = (uint32_t)p.BN * 128u + fixed + c0.hb + c0.fb;
                if (has_g1) bytes += fixed + c1.hb + c1.fb;
                uint64_t* bar = &hd->full[s];
                mbar_arrive_expect_tx(bar, bytes);
                tma_load_2d(st + p.off_b, &tmap_x, kb * kGT, ntile * p.BN, bar);
                for (int sub = 0; sub < (has_g1 ? 2 : 1); ++sub) {
                    const long long g = g0 + sub * gtk;
                    const GtCopy& c = sub ? c1 : c0;
                    uint8_t* bm = st + p.off_bm + sub * 1536;
                    bulk_g2s(bm, p.b1 + g * 64, 512, bar);
                    bulk_g2s(bm + 512, p.b2 + g * 64, 512, bar);
                    bulk_g2s(bm + 1024, p.b3 + g * 64, 512, bar);
                    bulk_g2s(st + p.off_mt + sub * 32, p.mt_off + g * 8, 32, bar);
                    if (c.hb) bulk_g2s(st + p.off_hf + sub * p.hf_slot, p.sm + c.h0, c.hb, bar);
                    if (c.fb) bulk_g2s(st + p.off_full + sub * p.full_slot, p.full + c.f0, c.fb, bar);
                }
            }
        }
    } else if (warp == kMmaWarp) {
        if (lane == 0) {
            const uint32_t idesc = umma_idesc_bf16(128, p.BN);
            bool ok = true;
            for (int i = 0; i < nk && ok; ++i) {
                const int s = i % NS;
                const uint32_t par = (i / NS) & 1;
                ok = mbar_wait(&hd->full[s], par, p.err, abort_flag) &&
                     mbar_wait(&hd->decoded[s], par, p.err, abort_flag);
                if (!ok) break;
                tc_fence_after();
                const uint32_t a_addr = smem_u32(stages + (size_t)s * p.stage_bytes);
                const uint32_t b_addr = a_addr + p.off_b;
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    umma_bf16_ss(tmem_d, umma_desc_sw128(a_addr + 32 * k), umma_desc_sw128(b_addr + 32 * k), idesc,
                                 (i > 0 || k > 0) ? 1u : 0u);
                umma_commit(&hd->empty[s]);
            }
            umma_commit(&hd->accum);
        }
    } else {
        // decoders: warp = 4*group + q; q selects rows 32q..32q+31 of the tile
        const int group = warp >> 2, q = warp & 3, sub = q >> 1, half = q & 1;
        const DecodeTables tabs = make_decode_tables(p.start_exp);
        const bool active = (sub == 0) || has_g1;
        for (int i = group; i < nk; i += 2) {
            const int s = i % NS;
            if (!mbar_wait(&hd->full[s], (i / NS) & 1, p.err, abort_flag)) break;
            uint8_t* st = stages + (size_t)s * p.stage_bytes;
            if (active) {
                GtSmem g;
                g.bm1 = reinterpret_cast<const uint64_t*>(st + p.off_bm + sub * 1536);
                g.bm2 = g.bm1 + 64;
                g.bm3 = g.bm1 + 128;
                g.mt = reinterpret_cast<const int*>(st + p.off_mt + sub * 32);
                g.sm = st + p.off_hf + sub * p.hf_slot;
                g.full = reinterpret_cast<const uint16_t*>(st + p.off_full + sub * p.full_slot);
                g.hf_cap = p.hf_slot - 16;
                g.full_cap = p.full_slot / 2 - 8;
                uint8_t* a_tile = st + sub * 64 * 128;
                decode_gt_half(g, lut, tabs, half, [&](int m, int kc, const uint32_t(&o)[4]) {
                    *reinterpret_cast<uint4*>(a_tile + m * 128 + ((kc ^ (m & 7)) << 4)) =
                        make_uint4(o[0], o[1], o[2], o[3]);
                });
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&hd->decoded[s]);
        }
    }

    // ---------------- epilogue: TMEM -> smem partial tile -> cluster reduce --
    float* red = reinterpret_cast<float*>(stages);  // [BN][128] fp32, reuses the drained stages
    if (warp < 4) {
        const int q = warp;
        bool ok = (nk > 0) && mbar_wait(&hd->accum, 0, p.err, abort_flag);
        if (ok) {
            tc_fence_after();
            for (int c = 0; c < p.BN; c += 16) {
                uint32_t r[16];
                tmem_ld16(tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)c, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) red[(c + j) * 128 + 32 * q + lane] = __uint_as_float(r[j]);
            }
        } else {
            for (int c = 0; c < p.BN; ++c) red[c * 128 + 32 * q + lane] = 0.f;
        }
    }
    tc_fence_before();
    cluster_sync();
    {
        const int cols_per = (p.BN + S - 1) / S;
        const int nb = (int)rank * cols_per;
        const int ncols = max(0, min(p.BN, nb + cols_per) - nb);
        const uint32_t red_addr = smem_u32(red);
        for (int idx = tid; idx < ncols * 32; idx += kGemmThreads) {
            const int nl = nb + (idx >> 5), m4 = (idx & 31) * 4;
            const int n = ntile * p.BN + nl;
            const int m = mtile * 128 + m4;
            if (n >= p.N || m >= p.M) continue;
            const uint32_t off = (uint32_t)(nl * 128 + m4) * 4u;
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int rr = 0; rr < S; ++rr) {
                const float4 v = ld_dsmem_f4(mapa_shared(red_addr + off, (uint32_t)rr));
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
    cluster_sync();
    if (warp == kMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem_d, p.tmem_cols);
    }
}

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
};

static DevInfo dev_info() {
    static DevInfo info[64];
    static bool have[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> g(mu);
    if (dev < 64 && !have[dev]) {
        cudaDeviceGetAttribute(&info[dev].sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&info[dev].max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        have[dev] = true;
    }
    return dev < 64 ? info[dev] : DevInfo{};
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
        !aligned16(mt_off) || !aligned16(X) || (reinterpret_cast<uintptr_t>(C) & 7u))
        return cudaErrorInvalidValue;
    auto encode = get_encode_fn();
    if (!encode) return cudaErrorNotSupported;
    const DevInfo di = dev_info();

    GemmParams p{};
    p.sm = sm; p.full = full; p.b1 = b1; p.b2 = b2; p.b3 = b3; p.mt_off = mt_off; p.gt_off = gt_off;
    p.max_hf = max_hf; p.max_full = max_full; p.start_exp = start_exp & 0xFF;
    p.C = C; p.M = M; p.N = N; p.K = K; p.err = err;
    p.BN = std::min(256, (N + 15) / 16 * 16);
    p.tmem_cols = pow2_cols(p.BN);
    p.hf_slot = hf_slot_bytes(max_hf);
    p.full_slot = full_slot_bytes(max_full);
    p.off_b = 128 * 128;
    p.off_bm = p.off_b + (uint32_t)p.BN * 128u;
    p.off_mt = p.off_bm + 2 * 1536;
    p.off_hf = p.off_mt + 64;
    p.off_full = p.off_hf + 2 * p.hf_slot;
    p.stage_bytes = round_up_u32(p.off_full + 2 * p.full_slot, 1024);
    const uint32_t red_bytes = (uint32_t)p.BN * 128u * 4u;
    int ns = (int)((di.max_smem - (int)kHeaderBytes) / (int)p.stage_bytes);
    ns = std::min(ns, kMaxStages);
    if (ns < 2) return cudaErrorInvalidValue;
    p.nstages = ns;
    if ((uint32_t)ns * p.stage_bytes < red_bytes) return cudaErrorInvalidValue;
    const uint32_t smem_bytes = kHeaderBytes + (uint32_t)ns * p.stage_bytes;

    const int mtiles = (M + 127) / 128;
    const int ntiles = (N + p.BN - 1) / p.BN;
    const int nkb = K / 64;
    int S = std::max(1, di.sms / std::max(1, mtiles * ntiles));
    S = std::max(S, split_k);
    S = std::min(S, std::min(8, nkb));
    p.kb_per_split = (nkb + S - 1) / S;
    S = (nkb + p.kb_per_split - 1) / p.kb_per_split;  // drop empty ranks

    CUtensorMap tmap;
    cuuint64_t gdim[2] = {(cuuint64_t)K, (cuuint64_t)N};
    cuuint64_t gstride[1] = {(cuuint64_t)K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)p.BN};
    cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(&tmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(X), gdim, gstride, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return cudaErrorInvalidValue;

    ZS_RETURN_IF_ERR(cudaFuncSetAttribute(zipgemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem_bytes));
    ZS_RETURN_IF_ERR(cudaFuncSetAttribute(zipgemm_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
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
