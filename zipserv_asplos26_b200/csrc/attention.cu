// Compressed-KV split-KV decode attention (one new query token per sequence).
// Replaces the ZipServ-patched FlashAttention decode path
// (FA csrc/flash_attn/src/flash_fwd_kernel.h:432-601 zipserv_begin/finish_block_load,
// FA csrc/flash_attn/flash_api.cpp:1346-1520 mha_fwd_kvcache ZipServ arguments) and
// the standalone FA csrc/flash_attn_ck/zipserv_fwd_kvcache.cu:181 kernel.
//
// K and V are TCA-TBE compressed 2-D matrices in the head-major layout of
// kernel_benchmark/bench_zipserv_decode_attention.py:347 (pad_batched_kv_prefix_by_kv_head):
// row (b * Hkv + h) * T_pad + t, columns = head dim (D = 128 -> two 64-wide GTs),
// so one 64-token page of one (b, kv head) is one GT row (two GTs).
//
// Grid: (B * Hkv) x S splits; each CTA owns a contiguous range of pages of one
// (b, kv head) and the G = Hq / Hkv query heads that share it. Warp roles are
// listed at attn_decode_kernel: one producer warp bulk-copies the compressed
// pages, 16 decoder warps expand K and V pages into 128-byte-swizzled bf16
// tiles with the small-tile decoder shared with ZipGEMM, and two math warps
// take alternate pages (S = Q K^T, online base-2 softmax, O += P V).
// With S > 1 every CTA writes (m, l, unnormalised O) to a caller-provided fp32
// workspace and combine_kernel merges the splits; with S = 1 the CTA writes
// the normalised bf16 output itself.
#include <algorithm>
#include <mutex>
#include <cmath>
#include <cstddef>
#include <cstdlib>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

#ifndef ZS_ATTN_P_SPLIT
#define ZS_ATTN_P_SPLIT 1   // P.V with P as bf16 high part + bf16 residual (0: high part only, as FlashAttention)
#endif
constexpr int kAttnMaxG = 8;        // query heads per KV head
constexpr int kAttnD = 128;         // head dim (two 64-wide GTs)
constexpr int kAttnDecWarps = 16;   // one median-tile task of K or V per page each
constexpr int kAttnProducer = 16;
constexpr int kAttnMath0 = 17;      // math warps 17 and 18 take alternate pages
constexpr int kAttnWarps = 19;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnSlots = 4;       // compressed pages (K + V) in flight (ring depth up to 4)
constexpr int kAttnTiles = 3;       // decoded pages: K 16 KB + V 16 KB each (ring depth up to 3)
constexpr uint32_t kAttnTileBytes = 32768;

struct AttnStream {
    const uint8_t* sm;
    const uint16_t* full;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* mt_off;
    const int* gt_off;
    const int* page_off;   // paged layout: [pages][6] stream offsets (GT 0 start, GT 1 start, end)
    int max_hf, max_full, start_exp;
};

struct AttnParams {
    AttnStream k, v;
    const uint16_t* q;        // [B][Hq][D] bf16
    const int* seqlens;       // [B]
    uint16_t* out;            // [B][Hq][D] bf16
    float* ws;                // [B*Hkv][S][G][D + 2] fp32 when S > 1
    int B, Hq, Hkv, G, T_pad, S, pages_per_split;
    float scale_log2;         // softmax_scale * log2(e)
    // compressed page slot: per matrix (K at 0, V at c_mat):
    //   [b1 | b2 | b3: 2 GTs x 512 B each] [mt: 2 x 32 B] [hf: 2 GTs] [fallback: 2 GTs]
    uint32_t c_mat, c_hf, c_full, hf_cap, full_cap, c_slot;
    uint32_t off_tiles, off_slots;
    int nslots;               // depth of the compressed page ring (attn_rings)
    int ntiles;               // depth of the decoded tile ring (attn_rings)
    unsigned* err;
    // Paged layout (block_table != nullptr): logical page g of sequence b is
    // physical page block_table[b * max_blocks + g] * Hkv + kv head; when the
    // dense tails are given, a sequence whose length is not a multiple of 64
    // ends with a dense page read from tail_k / tail_v ([B][64][Hkv][D] bf16).
    const int* block_table;
    int max_blocks, num_blocks;
    const uint16_t* tail_k;
    const uint16_t* tail_v;
    // Dense mode (dense_all != 0): every page is read from tail_k / tail_v, laid
    // out [B][dense_rows][Hkv][D] bf16 (token-major, uncompressed); the paged
    // tails use dense_rows = 64.
    int dense_all, dense_rows;
    // Paged pools' running maxima of a GT's padded {hf bytes, fallback elements}
    // (nullable): when given, every CTA sizes its page slots from them and
    // fits as many (2 or 3) as the launch's shared memory allows.
    const unsigned long long* k_max;
    const unsigned long long* v_max;
    uint32_t smem_bytes;
    int ring_pref;            // first candidate of attn_rings to try
};

// Shared-memory carve-up of the page rings (from the host, or from the pools'
// device-side maxima in the paged layout).
struct AttnLayout {
    uint32_t c_hf, hf_cap, c_full, full_cap, c_mat, c_slot, off_slots;
    int nslots, ntiles;
};

// Depths of the compressed-page ring and the decoded-tile ring: the first
// candidate (from `pref` on) whose rings fit in `smem` bytes after the
// `off_tiles` header; (2, 2) always fits the largest streams.
__host__ __device__ inline void attn_rings(uint32_t off_tiles, uint32_t c_slot, uint32_t smem, int pref, int& nc,
                                           int& nt) {
    const int cand[3][2] = {{4, 3}, {3, 3}, {2, 2}};
    for (int i = pref < 0 ? 0 : (pref > 2 ? 2 : pref); i < 3; ++i) {
        nc = cand[i][0];
        nt = cand[i][1];
        if (off_tiles + (uint32_t)nt * kAttnTileBytes + (uint32_t)nc * c_slot <= smem) return;
    }
}

__device__ __forceinline__ AttnLayout attn_layout(const AttnParams& p) {
    AttnLayout L{p.c_hf, p.hf_cap, p.c_full, p.full_cap, p.c_mat, p.c_slot, p.off_slots, p.nslots, p.ntiles};
    if (p.k_max) {
        const unsigned long long mh = max(p.k_max[0], p.v_max[0]), mf = max(p.k_max[1], p.v_max[1]);
        const uint32_t hfc = (uint32_t)min(mh, 4096ull + 16), ffc = (uint32_t)min(mf, 4096ull + 8) * 2u;
        L.hf_cap = 2u * ((hfc + 15u) & ~15u);
        L.c_full = L.c_hf + L.hf_cap + 16u;
        L.full_cap = 2u * ((ffc + 15u) & ~15u);
        L.c_mat = (L.c_full + L.full_cap + 16u + 127u) & ~127u;
        L.c_slot = 2u * L.c_mat;
        attn_rings(p.off_tiles, L.c_slot, p.smem_bytes, p.ring_pref, L.nslots, L.ntiles);
        L.off_slots = p.off_tiles + (uint32_t)L.ntiles * kAttnTileBytes;
    }
    return L;
}

struct AttnSmem {
    uint64_t cfull[kAttnSlots], cempty[kAttnSlots];
    uint64_t tfull[kAttnTiles], tempty[kAttnTiles];
    int abort_flag;
    int2 info[kAttnSlots][2];          // per slot and matrix: stream offsets of the page's second GT
    float mo[kAttnMaxG][kAttnD];       // second math warp's partial output (final merge)
    __align__(16) uint16_t qs[kAttnMaxG][kAttnD + 8];   // query heads (bf16), rows padded against bank conflicts
    float mm[kAttnMaxG], ml[kAttnMaxG];
};

// ---------------- warp-level tensor-core helpers for the small attention math ----------------
// (G <= 8 query heads per page: far too small for tcgen05 tiles; mma.sync m16n8k16 with the
// heads in the 8 columns and ldmatrix from the decoded, 128-byte-swizzled page tiles.)
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// d[0..3] += A (16x16, row) * B (16x8, col), bf16 in, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                          uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Transpose an 8x8 b16 matrix held in the m8n8 fragment layout across the warp.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
}

// Kernel: one CTA per (b, kv head, split) works through its pages:
//   warp 16      producer: per page, lanes 0-11 bulk-copy the six streams of the
//                two GTs of K and of V (one warp instruction); GT offsets are
//                fetched one page ahead
//   warps 0-15   decoders: warp w always decodes median tile w % 4 of GT (w / 4) % 2
//                of K (w < 8) or V into the page's 128-byte-swizzled bf16 tiles
//   warps 17-18  math on alternate pages with mma.sync m16n8k16: S^T = K Q^T
//                (tokens in the tile rows, query heads in its 8 columns, K by
//                ldmatrix), online base-2 softmax per head column, then
//                O^T += V^T P^T (head dims in the rows, V by ldmatrix.trans,
//                P^T from the S^T accumulators by movmatrix.trans)
// The two math warps merge (m, l, O) at the end; with S > 1 splits the CTA writes
// (m, l, unnormalised O) to the workspace for attn_combine_kernel.
__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    AttnSmem& A = *reinterpret_cast<AttnSmem*>(smem);
    const uint32_t smem0 = smem_u32(smem);
    const AttnLayout L = attn_layout(p);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x, split = blockIdx.y;
    const int b = bh / p.Hkv, hk = bh % p.Hkv;
    const int len = p.block_table ? max(0, min(p.seqlens[b], 64 * p.max_blocks)) : max(0, min(p.seqlens[b], p.T_pad));
    const int npages = (len + 63) >> 6;
    const bool has_tail = p.tail_k != nullptr && (len & 63) != 0;
    // the last page of a paged sequence with a dense tail is read from tail_k / tail_v
    auto is_dense_page = [&](int g) { return p.dense_all || (has_tail && g == npages - 1); };
    const int pg0 = split * p.pages_per_split;
    const int np = max(0, min(npages, pg0 + p.pages_per_split) - pg0);
    const int G = p.G;
    const long long rb = ((long long)bh * p.T_pad) >> 6;   // first GT row of this (b, kv head)

    for (int i = tid; i < kAttnMaxG * kAttnD; i += kAttnThreads) {
        const int h = i / kAttnD, d = i % kAttnD;
        A.qs[h][d] = h < G ? p.q[((size_t)b * p.Hq + hk * G + h) * kAttnD + d] : (uint16_t)0;
    }
    if (tid == 0) {
        for (int s = 0; s < L.nslots; ++s) {
            mbar_init(&A.cfull[s], 1);
            mbar_init(&A.cempty[s], kAttnDecWarps);
        }
        for (int s = 0; s < L.ntiles; ++s) {
            mbar_init(&A.tfull[s], kAttnDecWarps);
            mbar_init(&A.tempty[s], 1);
        }
        A.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    volatile int* abort_flag = &A.abort_flag;

    if (warp == kAttnProducer) {
        // lanes 0-5: K streams (b1, b2, b3, mt, hf, fallback), lanes 6-11: V streams;
        // lanes 0-2 / 3-5 hold the K / V GT offsets of GTs 2r, 2r+1, 2r+2 of the page
        const int mat = lane / 6, kind = lane % 6;
        const AttnStream& S = mat ? p.v : p.k;
        const AttnStream& So = lane < 3 ? p.k : p.v;
        // page record: the lane's GT offset entry and the page's first GT index
        struct PageRec { int2 e; long long gt0; };
        auto fetch = [&](int pi) {
            PageRec r{make_int2(0, 0), (rb + pg0 + pi) * 2};
            if (pi >= np) return r;
            if (p.block_table) {
                const int g = pg0 + pi;
                if (is_dense_page(g)) return r;
                int blk = p.block_table[(size_t)b * p.max_blocks + g];
                if (blk < 0 || blk >= p.num_blocks) {
                    if (lane == 0 && p.err) atomicOr(p.err, kErrStreamOverflow);
                    blk = 0;
                }
                const long long P = (long long)blk * p.Hkv + hk;
                r.gt0 = 2 * P;
                if (lane < 6) r.e = reinterpret_cast<const int2*>(So.page_off)[P * 3 + (lane % 3)];
            } else if (lane < 6 && !p.dense_all) {
                r.e = reinterpret_cast<const int2*>(So.gt_off)[(rb + pg0 + pi) * 2 + (lane % 3)];
            }
            return r;
        };
        PageRec cur = fetch(0);
        int s = 0;
        uint32_t ph = 0;
        bool ok = true;
        for (int pi = 0; pi < np && ok; ++pi) {
            const PageRec nxt = fetch(pi + 1);   // in flight while this page is issued
            if (lane == 0 && pi >= L.nslots) ok = mbar_wait(&A.cempty[s], ph ^ 1u, p.err, abort_flag);
            ok = __shfl_sync(0xFFFFFFFFu, ok ? 1 : 0, 0) != 0;
            if (!ok) break;
            const int mb = 3 * mat;
            const int h0 = __shfl_sync(0xFFFFFFFFu, cur.e.x, mb), f0 = __shfl_sync(0xFFFFFFFFu, cur.e.y, mb);
            const int h1 = __shfl_sync(0xFFFFFFFFu, cur.e.x, mb + 1), f1 = __shfl_sync(0xFFFFFFFFu, cur.e.y, mb + 1);
            const int h2 = __shfl_sync(0xFFFFFFFFu, cur.e.x, mb + 2), f2 = __shfl_sync(0xFFFFFFFFu, cur.e.y, mb + 2);
            uint8_t* slot = smem + L.off_slots + (size_t)s * L.c_slot + (size_t)mat * L.c_mat;
            const long long gt0 = cur.gt0;
            uint32_t size = 0, dst = 0;
            const void* src = nullptr;
            if (lane < 12 && !is_dense_page(pg0 + pi)) {   // a dense tail page is read by the decoders
                if (kind < 3) {
                    size = 1024u;
                    dst = 1024u * (uint32_t)kind;
                    src = (kind == 0 ? S.b1 : (kind == 1 ? S.b2 : S.b3)) + gt0 * 64;
                } else if (kind == 3) {
                    size = 64u;
                    dst = 3072u;
                    src = S.mt_off + gt0 * 8;
                } else {
                    const bool hf = kind == 4;
                    const int beg = hf ? h0 : f0, end = hf ? h2 : f2;
                    const uint32_t esz = hf ? 1u : 2u, cap = hf ? L.hf_cap : L.full_cap;
                    const int al = hf ? 16 : 8;
                    uint32_t bytes = end > beg ? (uint32_t)(end - beg) * esz : 0u;
                    int bg = beg;
                    if (bytes > cap || (bytes & 15u) || (bg & (al - 1)) || bg < 0) {
                        if (p.err) atomicOr(p.err, kErrStreamOverflow);
                        bytes = min(bytes, cap) & ~15u;
                        bg = max(bg, 0) & ~(al - 1);
                    }
                    size = bytes;
                    dst = hf ? L.c_hf : L.c_full;
                    src = hf ? (const void*)(S.sm + bg) : (const void*)(S.full + bg);
                }
            }
            if (lane == 0 || lane == 6)
                A.info[s][mat] = make_int2(max(h1 - h0, 0), max(f1 - f0, 0));
            const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, size);
            __syncwarp();   // the page's offsets above are released by lane 0's arrive
            if (lane == 0) mbar_arrive_expect_tx(&A.cfull[s], total);
            __syncwarp();
            if (size) bulk_g2s(slot + dst, src, size, &A.cfull[s]);
            cur = nxt;
            if (++s == L.nslots) { s = 0; ph ^= 1u; }
        }
    } else if (warp < kAttnDecWarps) {
        const int mat = warp >> 3, gc = (warp >> 2) & 1, mtile = warp & 3;
        const DecodeTables tabs = make_decode_tables(mat ? p.v.start_exp : p.k.start_exp);
        int s = 0, t = 0;   // compressed slot, tile slot
        uint32_t ph = 0, tph = 0;
        for (int pi = 0; pi < np; ++pi) {
            if (*abort_flag) break;
            if (!mbar_wait_sleep(&A.cfull[s], ph, p.err, abort_flag)) break;
            if (pi >= L.ntiles && !mbar_wait_sleep(&A.tempty[t], tph ^ 1u, p.err, abort_flag)) break;
            const uint32_t base = launder(smem0 + L.off_slots + (uint32_t)s * L.c_slot + (uint32_t)mat * L.c_mat);
            const int2 inf = gc ? A.info[s][mat] : make_int2(0, 0);
            const uint32_t h0 = min((uint32_t)inf.x, L.hf_cap), f0 = min((uint32_t)inf.y, L.full_cap / 2);
            GtView g;
            g.bm = base + 512u * (uint32_t)gc;
            g.bstride = 1024u;
            g.mt = base + 3072u + 32u * (uint32_t)gc;
            g.sm = base + L.c_hf + h0;
            g.full = base + L.c_full + 2u * f0;
            g.hf_cap = L.hf_cap - h0;
            g.full_cap = L.full_cap / 2 - f0;
            const uint32_t rows = smem0 + p.off_tiles + (uint32_t)t * kAttnTileBytes + 16384u * (uint32_t)mat +
                                  8192u * (uint32_t)gc + 2048u * (uint32_t)mtile;
            if (is_dense_page(pg0 + pi)) {
                // dense page (a paged sequence's tail, or every page in dense mode):
                // rows 16 mtile .. +15 (tokens), columns 64 gc .. +63 of K or V, zero
                // past the sequence end, in the swizzled tile layout
                const int g = pg0 + pi;
                const uint16_t* tb = (mat ? p.tail_v : p.tail_k) + ((size_t)b * p.dense_rows * p.Hkv + hk) * kAttnD +
                                     (p.dense_all ? (size_t)64 * g * p.Hkv * kAttnD : 0) + 64 * gc;
                const int tl = p.dense_all ? min(64, len - 64 * g) : (len & 63);
#pragma unroll
                for (int c = lane; c < 128; c += 32) {
                    const int rr = c >> 3, ch = c & 7, m = 16 * mtile + rr;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (m < tl) v = *reinterpret_cast<const uint4*>(tb + (size_t)m * p.Hkv * kAttnD + 8 * ch);
                    sts128(rows + 128u * (uint32_t)rr + (((uint32_t)ch ^ ((uint32_t)rr & 7u)) << 4), v.x, v.y, v.z,
                           v.w);
                }
            } else {
                decode_mt_to_tile(g, tabs, mtile, rows);
            }
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&A.tfull[t]);
                mbar_arrive(&A.cempty[s]);
            }
            if (++s == L.nslots) { s = 0; ph ^= 1u; }
            if (++t == L.ntiles) { t = 0; tph ^= 1u; }
        }
    } else {
        // Math warps, one page each in turn. The m16n8k16 tiles put the page's
        // tokens (S^T = K Q^T) or head dims (O^T = V^T P^T) in the 16 rows and
        // the G <= 8 query heads in the 8 columns, so no MMA row is padding.
        // Lane (g = lane / 4, t4 = lane % 4) holds heads 2 t4 and 2 t4 + 1;
        // movmatrix turns the S^T accumulator layout into the P^T operand.
        const int mw = warp - kAttnMath0;
        const int g8 = lane >> 2, t4 = lane & 3;
        // Q^T B fragments for the 8 k-steps of 16 dims (rows of heads >= G are zero)
        uint32_t qb[8][2];
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
            qb[ks][0] = *reinterpret_cast<const uint32_t*>(&A.qs[g8][16 * ks + 2 * t4]);
            qb[ks][1] = *reinterpret_cast<const uint32_t*>(&A.qs[g8][16 * ks + 8 + 2 * t4]);
        }
        float o[8][4];   // O^T: dim tile dt, rows g8 / g8 + 8, heads 2 t4 / 2 t4 + 1
#pragma unroll
        for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
        float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
        const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lc = lane >> 4;   // ldmatrix row / 8-column half (K)
        const int vr = (lane & 7) + 8 * (lane >> 4), vc = (lane >> 3) & 1;    // ldmatrix.trans token / dim half (V)
        int s = mw % L.ntiles, kround = mw / L.ntiles;   // page pi = mw + 2j: tile slot pi % n, round pi / n
        for (int pi = mw; pi < np; pi += 2) {
            if (!mbar_wait(&A.tfull[s], (uint32_t)(kround & 1), p.err, abort_flag)) break;
            const uint32_t kt = smem0 + p.off_tiles + (uint32_t)s * kAttnTileBytes, vt = kt + 16384u;
            // S^T = K Q^T: 4 token tiles x 8 dim steps
            float sc[4][4];
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
                sc[mt][0] = sc[mt][1] = sc[mt][2] = sc[mt][3] = 0.f;
                const uint32_t tok = 16u * (uint32_t)mt + (uint32_t)lr;
#pragma unroll
                for (int ks = 0; ks < 8; ++ks) {
                    const uint32_t chunk = 2u * (uint32_t)(ks & 3) + (uint32_t)lc;
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(kt + 8192u * (uint32_t)(ks >> 2) + tok * 128u + ((chunk ^ (tok & 7u)) << 4), a0, a1, a2, a3);
                    mma_16816(sc[mt], a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
                }
            }
            // online softmax per head column over the page's 64 tokens
            const int tok0 = (pg0 + pi) * 64;
            float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int t = tok0 + 16 * mt + g8 + 8 * (e >> 1);
                    const float x = t < len ? sc[mt][e] * p.scale_log2 : -INFINITY;
                    sc[mt][e] = x;
                    mx[e & 1] = fmaxf(mx[e & 1], x);
                }
            float alpha[2], mref[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 4));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 8));
                mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xFFFFFFFFu, mx[h], 16));
                const float m_new = fmaxf(m_run[h], mx[h]);
                mref[h] = m_new == -INFINITY ? 0.f : m_new;
                alpha[h] = exp2f(m_run[h] - mref[h]);
                m_run[h] = m_new;
            }
            // P as a bf16 pair hi + lo (lo = the rounding residual) so that P.V keeps
            // about 16 bits of P; movmatrix.trans makes each 8x8 block a P^T fragment
            uint32_t ph[4][2], pl[4][2];
            float sum[2] = {0.f, 0.f};
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const float e0 = exp2f(sc[mt][2 * r] - mref[0]), e1 = exp2f(sc[mt][2 * r + 1] - mref[1]);
                    sum[0] += e0;
                    sum[1] += e1;
                    const __nv_bfloat162 hi = __floats2bfloat162_rn(e0, e1);
                    const float2 hf = __bfloat1622float2(hi);
                    ph[mt][r] = movmatrix_trans(*reinterpret_cast<const uint32_t*>(&hi));
                    pl[mt][r] = movmatrix_trans(pack_bf16(e0 - hf.x, e1 - hf.y));
                }
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                sum[h] += __shfl_xor_sync(0xFFFFFFFFu, sum[h], 4);
                sum[h] += __shfl_xor_sync(0xFFFFFFFFu, sum[h], 8);
                sum[h] += __shfl_xor_sync(0xFFFFFFFFu, sum[h], 16);
                l_run[h] = l_run[h] * alpha[h] + sum[h];
            }
#pragma unroll
            for (int dt = 0; dt < 8; ++dt) {
                o[dt][0] *= alpha[0];
                o[dt][1] *= alpha[1];
                o[dt][2] *= alpha[0];
                o[dt][3] *= alpha[1];
            }
            // O^T += V^T P^T: 8 dim tiles x 4 token steps (hi and lo parts of P)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                const uint32_t tok = 16u * (uint32_t)ks + (uint32_t)vr;
#pragma unroll
                for (int dt = 0; dt < 8; ++dt) {
                    const uint32_t chunk = 2u * (uint32_t)(dt & 3) + (uint32_t)vc;
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(vt + 8192u * (uint32_t)(dt >> 2) + tok * 128u + ((chunk ^ (tok & 7u)) << 4), a0, a1, a2,
                              a3);
                    mma_16816(o[dt], a0, a1, a2, a3, ph[ks][0], ph[ks][1]);
#if ZS_ATTN_P_SPLIT
                    mma_16816(o[dt], a0, a1, a2, a3, pl[ks][0], pl[ks][1]);
#endif
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&A.tempty[s]);
            s += 2;
            while (s >= L.ntiles) { s -= L.ntiles; ++kround; }
        }
        // merge the two math warps: warp kAttnMath0 + 1 publishes, kAttnMath0 combines and writes
        if (mw == 1) {
#pragma unroll
            for (int dt = 0; dt < 8; ++dt)
#pragma unroll
                for (int e = 0; e < 4; ++e) A.mo[2 * t4 + (e & 1)][16 * dt + g8 + 8 * (e >> 1)] = o[dt][e];
            if (g8 == 0) {
                A.mm[2 * t4] = m_run[0]; A.mm[2 * t4 + 1] = m_run[1];
                A.ml[2 * t4] = l_run[0]; A.ml[2 * t4 + 1] = l_run[1];
            }
        }
        asm volatile("bar.sync 1, 64;" ::: "memory");
        if (mw == 0) {
            float s0[2], s1[2], Mh[2], Lh[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int hh = 2 * t4 + h;
                const float m1 = A.mm[hh], l1 = A.ml[hh];
                Mh[h] = fmaxf(m_run[h], m1);
                const float Mref = Mh[h] == -INFINITY ? 0.f : Mh[h];
                s0[h] = exp2f(m_run[h] - Mref);
                s1[h] = exp2f(m1 - Mref);
                Lh[h] = l_run[h] * s0[h] + l1 * s1[h];
            }
#pragma unroll
            for (int dt = 0; dt < 8; ++dt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int h = e & 1, hh = 2 * t4 + h, d = 16 * dt + g8 + 8 * (e >> 1);
                    if (hh >= G) continue;
                    const float v = o[dt][e] * s0[h] + A.mo[hh][d] * s1[h];
                    if (p.S == 1) {
                        const float inv = Lh[h] > 0.f ? 1.f / Lh[h] : 0.f;
                        p.out[((size_t)b * p.Hq + hk * G + hh) * kAttnD + d] =
                            __bfloat16_as_ushort(__float2bfloat16_rn(v * inv));
                    } else {
                        p.ws[(((size_t)bh * p.S + split) * G + hh) * (kAttnD + 2) + d] = v;
                    }
                }
            if (p.S > 1 && g8 == 0) {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int hh = 2 * t4 + h;
                    if (hh >= G) continue;
                    float* w = p.ws + (((size_t)bh * p.S + split) * G + hh) * (kAttnD + 2);
                    w[kAttnD] = Mh[h];
                    w[kAttnD + 1] = Lh[h];
                }
            }
        }
    }
}

// Merge the S split partials of each (b, query head): O = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.
__global__ void attn_combine_kernel(const float* __restrict__ ws, uint16_t* __restrict__ out, int Hq, int Hkv,
                                    int G, int S) {
    const int bq = blockIdx.x;   // b * Hq + hq
    const int b = bq / Hq, hq = bq % Hq, hk = hq / G, h = hq % G;
    const size_t base = (size_t)(b * Hkv + hk) * S;
    float M = -INFINITY;
    for (int s = 0; s < S; ++s) M = fmaxf(M, ws[((base + s) * G + h) * (kAttnD + 2) + kAttnD]);
    float L = 0.f;
    for (int s = 0; s < S; ++s) {
        const float* w = ws + ((base + s) * G + h) * (kAttnD + 2);
        if (w[kAttnD + 1] > 0.f) L += exp2f(w[kAttnD] - M) * w[kAttnD + 1];
    }
    const float inv = L > 0.f ? 1.f / L : 0.f;
    for (int d = threadIdx.x; d < kAttnD; d += blockDim.x) {
        float o = 0.f;
        for (int s = 0; s < S; ++s) {
            const float* w = ws + ((base + s) * G + h) * (kAttnD + 2);
            if (w[kAttnD + 1] > 0.f) o += exp2f(w[kAttnD] - M) * w[d];
        }
        out[(size_t)bq * kAttnD + d] = __bfloat16_as_ushort(__float2bfloat16_rn(o * inv));
    }
}

size_t attn_workspace_bytes(int B, int Hq, int Hkv, int num_splits) {
    if (num_splits <= 1) return 0;
    return (size_t)B * Hq * num_splits * (kAttnD + 2) * sizeof(float);
}

// Split-KV factor for (B, Hkv) sequences of up to max_pages pages. One CTA per
// (sequence, KV head, split) fills an SM (its page rings take most of the
// shared memory), so the grid runs in ceil(B Hkv S / #SMs) waves of
// ceil(max_pages / S) pages each; S minimises waves x (pages per CTA + 2), the
// 2 standing for a CTA's set-up and its share of the combine. (A count that
// only targeted about two CTAs per SM left 320 CTAs = 2.2 waves at B = 8,
// T = 32768: a last wave 16% full.)
// First ring candidate to try (attn_rings): 0 unless ZS_ATTN_RING in the
// environment names another, to compare ring depths on the same build.
static int attn_ring_pref() {
    static const int v = [] {
        const char* e = std::getenv("ZS_ATTN_RING");
        return e ? std::atoi(e) : 0;
    }();
    return v;
}

int attn_default_splits(int B, int Hkv, int max_pages) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const long long pairs = (long long)std::max(1, B) * std::max(1, Hkv);
    const int P = std::max(1, max_pages);
    int best = 1;
    long long best_cost = -1;
    for (int S = 1; S <= P; ++S) {
        const long long waves = (pairs * S + sms - 1) / sms;
        const long long cost = waves * ((P + S - 1) / S + 2);
        if (best_cost < 0 || cost < best_cost) { best_cost = cost; best = S; }
    }
    return best;
}

static cudaError_t attention_core(cudaStream_t stream, const AttnCompressed& kc, const AttnCompressed& vc,
                                  const uint16_t* q, const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D,
                                  int T_pad, int max_seqlen, float softmax_scale, int num_splits, float* ws,
                                  size_t ws_bytes, unsigned* err, int* splits_used, const AttnPaged* pg,
                                  const AttnDense* dn = nullptr) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D != kAttnD) return cudaErrorInvalidValue;
    if (dn && (pg || !dn->k || !dn->v || !aligned16(dn->k) || !aligned16(dn->v))) return cudaErrorInvalidValue;
    if (!pg && (T_pad <= 0 || T_pad % 64)) return cudaErrorInvalidValue;
    const int G = Hq / Hkv;
    if (G > kAttnMaxG) return cudaErrorInvalidValue;
    if (!q || !seqlens || !out || max_seqlen < 0) return cudaErrorInvalidValue;
    if (!pg && max_seqlen > T_pad) return cudaErrorInvalidValue;
    if (pg) {
        if (!pg->block_table || pg->max_blocks <= 0 || pg->num_blocks <= 0 || !pg->k_page_off || !pg->v_page_off ||
            max_seqlen > 64 * pg->max_blocks || (reinterpret_cast<uintptr_t>(pg->k_page_off) & 7u) ||
            (reinterpret_cast<uintptr_t>(pg->v_page_off) & 7u))
            return cudaErrorInvalidValue;
        if ((pg->tail_k == nullptr) != (pg->tail_v == nullptr) || !aligned16(pg->tail_k) || !aligned16(pg->tail_v))
            return cudaErrorInvalidValue;
    }
    const AttnCompressed* cs[2] = {&kc, &vc};
    for (const AttnCompressed* c : cs) {
        if (dn) break;   // dense mode reads no compressed stream
        if (!c->b1 || !c->b2 || !c->b3 || !c->mt_off || (!pg && !c->gt_off)) return cudaErrorInvalidValue;
        if (!pg && (c->rows != B * Hkv * T_pad || c->cols != D)) return cudaErrorInvalidValue;
        if (c->max_hf < 0 || c->max_full < 0 || c->max_hf > 4096 + 15 || c->max_full > 4096 + 7)
            return cudaErrorInvalidValue;
        if (!aligned16(c->sm) || !aligned16(c->full) || !aligned16(c->b1) || !aligned16(c->b2) ||
            !aligned16(c->b3) || !aligned16(c->mt_off) || (reinterpret_cast<uintptr_t>(c->gt_off) & 7u))
            return cudaErrorInvalidValue;
    }
    if (reinterpret_cast<uintptr_t>(out) & 3u) return cudaErrorInvalidValue;
    const int max_pages = (max_seqlen + 63) / 64;
    const int S = num_splits > 0 ? std::min(num_splits, std::max(1, max_pages))
                                 : attn_default_splits(B, Hkv, max_pages);
    if (S > 1 && (!ws || ws_bytes < attn_workspace_bytes(B, Hq, Hkv, S))) return cudaErrorInvalidValue;
    if (splits_used) *splits_used = S;

    AttnParams p{};
    auto fill = [&](AttnStream& d, const AttnCompressed& c) {
        d.sm = c.sm; d.full = c.full; d.b1 = c.b1; d.b2 = c.b2; d.b3 = c.b3; d.mt_off = c.mt_off;
        d.gt_off = c.gt_off; d.max_hf = c.max_hf; d.max_full = c.max_full; d.start_exp = c.start_exp & 0xFF;
    };
    fill(p.k, kc);
    fill(p.v, vc);
    if (pg) {
        p.k.page_off = pg->k_page_off;
        p.v.page_off = pg->v_page_off;
        p.block_table = pg->block_table;
        p.max_blocks = pg->max_blocks;
        p.num_blocks = pg->num_blocks;
        p.tail_k = pg->tail_k;
        p.tail_v = pg->tail_v;
        p.dense_rows = 64;
        p.k_max = pg->k_max;
        p.v_max = pg->v_max;
    }
    if (dn) {
        p.tail_k = dn->k;
        p.tail_v = dn->v;
        p.dense_all = 1;
        p.dense_rows = T_pad;
    }
    p.q = q; p.seqlens = seqlens; p.out = out; p.ws = ws; p.err = err;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = G; p.T_pad = T_pad; p.S = S;
    p.pages_per_split = (max_pages + S - 1) / S;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;
    const uint32_t hfc = dn ? 16u : round_up_u32((uint32_t)std::max(kc.max_hf, vc.max_hf), 16);
    const uint32_t ffc = dn ? 16u : round_up_u32((uint32_t)std::max(kc.max_full, vc.max_full) * 2u, 16);
    // compressed page slot per matrix: 3 x 1 KB bitmaps, 64 B median offsets, the
    // two GTs' hf stream (+16 B read slack) and fallback stream
    p.c_hf = 3072u + 64u;
    p.hf_cap = 2u * hfc;
    p.c_full = p.c_hf + p.hf_cap + 16u;
    p.full_cap = 2u * ffc;
    p.c_mat = round_up_u32(p.c_full + p.full_cap + 16u, 128);
    p.c_slot = 2u * p.c_mat;
    p.off_tiles = round_up_u32(sizeof(AttnSmem), 1024);
    int dev = 0, max_smem = 232448;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    // four compressed pages and three decoded tiles when the streams allow (the
    // compressed ring hides the HBM latency of a page's copies; a fourth slot
    // measured 3% faster at B=8, T=32768, a fourth tile nothing); large fallback
    // streams (e.g. zero-padded pages) leave room for two of each
    p.ring_pref = attn_ring_pref();
    attn_rings(p.off_tiles, p.c_slot, (uint32_t)max_smem, p.ring_pref, p.nslots, p.ntiles);
    p.off_slots = p.off_tiles + (uint32_t)p.ntiles * kAttnTileBytes;
    uint32_t smem_bytes = p.off_slots + (uint32_t)p.nslots * p.c_slot;
    if (smem_bytes > (uint32_t)max_smem) return cudaErrorInvalidValue;
    // with the pools' device-side maxima the kernel sizes its own page slots
    // (the worst case above fits two), so it gets all the shared memory there is
    if (p.k_max) smem_bytes = (uint32_t)max_smem;
    p.smem_bytes = smem_bytes;
    ZS_RETURN_IF_ERR(cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)smem_bytes));
    attn_decode_kernel<<<dim3((unsigned)(B * Hkv), (unsigned)S), kAttnThreads, smem_bytes, stream>>>(p);
    ZS_RETURN_IF_ERR(cudaGetLastError());
    if (S > 1) {
        attn_combine_kernel<<<(unsigned)(B * Hq), 128, 0, stream>>>(ws, out, Hq, Hkv, G, S);
        ZS_RETURN_IF_ERR(cudaGetLastError());
    }
    return cudaSuccess;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of launch_attention.
//
// Some callers cannot allocate device memory at the point where they run
// attention: code that executes while an allocator is not available (for
// example inside a custom memory pool's own callbacks, or in an embedding that
// forbids cudaMalloc after start-up so its memory budget stays fixed). For them
// the split-KV workspace lives in this file-scope device array instead of a
// caller buffer. It is created when the library is loaded on a GPU and kept
// until the process exits (kNoAllocWsFloats * 4 bytes = 2 MiB per GPU).
//
// Every call on a device shares the same array and leaves the last call's
// partial results in it. Nothing in it has to start at zero: each split writes
// all of its slots before the combine kernel reads them. Two calls whose
// kernels overlap on the GPU (different streams, no ordering between them)
// race on the array and may return wrong results; order them on one stream.
constexpr size_t kNoAllocWsFloats = 512 * 1024;
static __device__ __align__(256) float g_attn_noalloc_ws[kNoAllocWsFloats];

// The array's device address for the current device, looked up with that
// device current (cudaGetSymbolAddress) the first time a context of the device
// calls, and again whenever the device's current context has changed since
// (after cudaDeviceReset the module is loaded anew and the array may move).
// The first call on a device does this look-up; make that first call outside
// any stream capture.
static cudaError_t noalloc_ws_ptr(float** out) {
    using CtxGetCurrent = CUresult (*)(CUcontext*);
    static CtxGetCurrent get_ctx = nullptr;
    static float* ptrs[64] = {};
    static CUcontext ctxs[64] = {};
    static std::mutex mu;
    int dev = 0;
    ZS_RETURN_IF_ERR(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (!get_ctx) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        ZS_RETURN_IF_ERR(cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q));
        if (q != cudaDriverEntryPointSuccess || !fn) return cudaErrorNotSupported;
        get_ctx = reinterpret_cast<CtxGetCurrent>(fn);
    }
    CUcontext ctx = nullptr;
    // the caller's device pointers were made in the current context, so one is current
    if (get_ctx(&ctx) != CUDA_SUCCESS || !ctx) return cudaErrorDeviceUninitialized;
    if (!ptrs[dev] || ctxs[dev] != ctx) {
        void* ptr = nullptr;
        ZS_RETURN_IF_ERR(cudaGetSymbolAddress(&ptr, g_attn_noalloc_ws));
        ptrs[dev] = static_cast<float*>(ptr);
        ctxs[dev] = ctx;
    }
    *out = ptrs[dev];
    return cudaSuccess;
}

cudaError_t launch_attention(cudaStream_t stream, const AttnCompressed& kc, const AttnCompressed& vc,
                             const uint16_t* q, const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D,
                             int T_pad, int max_seqlen, float softmax_scale, int num_splits, float* ws,
                             size_t ws_bytes, unsigned* err, int* splits_used) {
    return attention_core(stream, kc, vc, q, seqlens, out, B, Hq, Hkv, D, T_pad, max_seqlen, softmax_scale,
                          num_splits, ws, ws_bytes, err, splits_used, nullptr);
}

cudaError_t launch_attention_paged(cudaStream_t stream, const AttnCompressed& kc, const AttnCompressed& vc,
                                   const AttnPaged& pg, const uint16_t* q, const int* seqlens, uint16_t* out, int B,
                                   int Hq, int Hkv, int D, int max_seqlen, float softmax_scale, int num_splits,
                                   float* ws, size_t ws_bytes, unsigned* err, int* splits_used) {
    return attention_core(stream, kc, vc, q, seqlens, out, B, Hq, Hkv, D, 64, max_seqlen, softmax_scale,
                          num_splits, ws, ws_bytes, err, splits_used, &pg);
}

cudaError_t launch_attention_dense(cudaStream_t stream, const uint16_t* k, const uint16_t* v, const uint16_t* q,
                                   const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int T_rows,
                                   int max_seqlen, float softmax_scale, int num_splits, float* ws, size_t ws_bytes,
                                   unsigned* err, int* splits_used) {
    const AttnCompressed none{};
    const AttnDense dn{k, v};
    return attention_core(stream, none, none, q, seqlens, out, B, Hq, Hkv, D, T_rows, max_seqlen, softmax_scale,
                          num_splits, ws, ws_bytes, err, splits_used, nullptr, &dn);
}

size_t attn_noalloc_ws_bytes() { return kNoAllocWsFloats * sizeof(float); }

cudaError_t launch_attention_noalloc(cudaStream_t stream, const AttnCompressed& k, const AttnCompressed& v,
                                     const uint16_t* q, const int* seqlens, uint16_t* out, int B, int Hq, int Hkv,
                                     int D, int T_pad, int max_seqlen, float softmax_scale, int num_splits,
                                     unsigned* err, int* splits_used) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || max_seqlen < 0) return cudaErrorInvalidValue;
    const int max_pages = std::max(1, (max_seqlen + 63) / 64);
    const int S = num_splits > 0 ? std::min(num_splits, max_pages) : attn_default_splits(B, Hkv, max_pages);
    // Sizes whose split workspace does not fit the fixed array are rejected.
    if (attn_workspace_bytes(B, Hq, Hkv, S) > attn_noalloc_ws_bytes()) return cudaErrorInvalidValue;
    float* ws = nullptr;
    ZS_RETURN_IF_ERR(noalloc_ws_ptr(&ws));
    return launch_attention(stream, k, v, q, seqlens, out, B, Hq, Hkv, D, T_pad, max_seqlen, softmax_scale, S, ws,
                            attn_noalloc_ws_bytes(), err, splits_used);
}

}  // namespace zs
