// Warp-level decode of a 64x64 TCA-TBE global tile (GT) that has been staged in
// shared memory. A warp decodes 32 rows (one half of the GT); lane L owns row
// 32*half + L and walks the 8 column blocks (kc = 0..7) of that row.
//
// Row/stream bookkeeping (format of csrc/L_API.cu:559-771):
//   row m -> median tile w = m/16, row block mr = (m/8)%2, row r = m%8;
//   small tile (ST) of column block kc = w*16 + 2*kc + mr;
//   high-frequency (hf) bytes of the MT are stored ST by ST, row by row.
// The hf offset of (ST, row r) is the MT base (from TileOffsets_Median) plus
// the hf counts of all earlier STs of the MT plus popc(indicator bits of rows
// < r). The two STs of one column block are held by lanes L and L^8, so one
// shuffle exchanges their totals.
#pragma once
#include "common.cuh"

namespace zs {

// Shared-memory view of one staged GT (32-bit shared addresses).
struct GtView {
    uint32_t bm;         // bitmap 1 of the GT: 64 x u64; bitmap 2 at bm + bstride, bitmap 3 at bm + 2 bstride
    uint32_t bstride;
    uint32_t mt;         // 8 ints: median-tile (hf, fallback) offsets within the GT
    uint32_t sm;         // GT's sign/mantissa stream (16-byte aligned, GT-local offset 0)
    uint32_t full;       // GT's fallback stream (GT-local offset 0)
    uint32_t hf_cap;     // largest hf offset a row may start at
    uint32_t full_cap;   // largest fallback offset (elements) a row may start at
};

// Decode 32 rows of a GT for column blocks kc0 .. kc0+NKC-1 into a
// 128-byte-row, 16-byte-chunk-swizzled tile (chunk c of row m at
// (c ^ (m & 7)) * 16). HI selects the rows: lane L owns row block rb = L/4
// (median tile w = rb/2, row block mr = rb%2) and row r = L%4 + 4*HI of it, so
// the half of each 64-bit bitmap a warp reads is fixed at compile time.
// The two small tiles of one column block (mr = 0, 1) sit in lanes L and L^4,
// so one shuffle exchanges their high-frequency counts. When kc0 > 0 the warp
// first sums the counts of the skipped column blocks.
template <bool HI, int NKC>
__device__ __forceinline__ void decode_gt_rows(const GtView& g, uint32_t lut_lane, const DecodeTables& t,
                                               uint32_t tile, int kc0) {
    const int lane = threadIdx.x & 31;
    const int rb = lane >> 2, w = rb >> 1, mr = rb & 1, r = (lane & 3) + (HI ? 4 : 0);
    const int m = 16 * w + 8 * mr + r;
    const uint32_t mj = (1u << (8 * (lane & 3))) - 1u;
    const uint32_t bsel = (uint32_t)(lane & 3) | 0x4440u;
    const uint32_t bm = g.bm + 8u * (uint32_t)(w * 16 + mr);
    const uint32_t row = tile + 128u * (uint32_t)m;
    const uint32_t rx = (uint32_t)(m & 7) << 4;
    uint32_t skipped = 0;
    for (int kc = 0; kc < kc0; ++kc) {
        const uint2 v1 = lds64(bm + 16u * kc), v2 = lds64(bm + g.bstride + 16u * kc),
                    v3 = lds64(bm + 2u * g.bstride + 16u * kc);
        const uint32_t tot = __popc(v1.x | v2.x | v3.x) + __popc(v1.y | v2.y | v3.y);
        skipped += tot + __shfl_xor_sync(0xFFFFFFFFu, tot, 4);
    }
    uint32_t acc_h = lds32(g.mt + 8u * w) + skipped;
    uint32_t acc_f = lds32(g.mt + 8u * w + 4u) + 128u * (uint32_t)kc0 - skipped;
    // Phase 1: all bitmap words of this lane's NKC small tiles.
    uint2 v1[NKC], v2[NKC], v3[NKC];
#pragma unroll
    for (int u = 0; u < NKC; ++u) {
        const uint32_t bo = bm + 16u * (uint32_t)(kc0 + u);
        v1[u] = lds64(bo);
        v2[u] = lds64(bo + g.bstride);
        v3[u] = lds64(bo + 2u * g.bstride);
    }
    // Phase 2: stream offsets (popcounts, partner shuffle, running sums).
    uint32_t hf[NKC], fo[NKC], c1[NKC], c2[NKC], c3[NKC];
#pragma unroll
    for (int u = 0; u < NKC; ++u) {
        const uint32_t ilo = v1[u].x | v2[u].x | v3[u].x;
        const uint32_t ihi = v1[u].y | v2[u].y | v3[u].y;
        const uint32_t plo = __popc(ilo);
        const uint32_t tot = plo + __popc(ihi);
        const uint32_t pre = HI ? plo + __popc(ihi & mj) : __popc(ilo & mj);
        const uint32_t ptot = __shfl_xor_sync(0xFFFFFFFFu, tot, 4);
        // Clamp keeps a corrupt offset array inside the staged slots.
        hf[u] = min(acc_h + (mr ? ptot : 0u) + pre, g.hf_cap);
        fo[u] = min(acc_f + (mr ? 64u - ptot : 0u) + 8u * (uint32_t)r - pre, g.full_cap);
        // clean bitmap bytes of this row
        c1[u] = prmt(HI ? v1[u].y : v1[u].x, 0, bsel);
        c2[u] = prmt(HI ? v2[u].y : v2[u].x, 0, bsel);
        c3[u] = prmt(HI ? v3[u].y : v3[u].x, 0, bsel);
        acc_h += tot + ptot;
        acc_f += 128u - tot - ptot;
    }
    // Phase 3: table lookups and stream windows for all NKC rows.
    uint32_t sp1[NKC], sp2[NKC], sp3[NKC], q0[NKC], q1[NKC], q2[NKC];
#pragma unroll
    for (int u = 0; u < NKC; ++u) {
        sp1[u] = lds32(lut_lane + (c1[u] << 7));
        sp2[u] = lds32(lut_lane + (c2[u] << 7));
        sp3[u] = lds32(lut_lane + (c3[u] << 7));
        const uint32_t wa = (g.sm + hf[u]) & ~3u;
        q0[u] = lds32(wa);
        q1[u] = lds32(wa + 4);
        q2[u] = lds32(wa + 8);
    }
    // Phase 4: assemble and store; then patch fallbacks.
#pragma unroll
    for (int u = 0; u < NKC; ++u) {
        const uint32_t X = sp1[u] + (sp2[u] << 1) + (sp3[u] << 2);
        const uint32_t sel = (sp1[u] | sp2[u] | sp3[u]) * 0x11111110u;
        const uint32_t sh = ((g.sm + hf[u]) & 3u) * 8u;
        const uint32_t lo = __funnelshift_r(q0[u], q1[u], sh);
        const uint32_t hi = __funnelshift_r(q1[u], q2[u], sh);
        const uint32_t s_lo = prmt(lo, hi, sel);
        const uint32_t s_hi = prmt(lo, hi, sel >> 16);
        const uint32_t hb_lo = lop_or_and(s_lo, 0x80808080u, prmt(t.thb0, t.thb1, X));
        const uint32_t hb_hi = lop_or_and(s_hi, 0x80808080u, prmt(t.thb0, t.thb1, X >> 16));
        const uint32_t lb_lo = lop_or_and(s_lo, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X));
        const uint32_t lb_hi = lop_or_and(s_hi, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X >> 16));
        const uint32_t dst = row + (((uint32_t)(kc0 + u) << 4) ^ rx);
        sts128(dst, prmt(lb_lo, hb_lo, 0x5140), prmt(lb_lo, hb_lo, 0x7362), prmt(lb_hi, hb_hi, 0x5140),
               prmt(lb_hi, hb_hi, 0x7362));
    }
#pragma unroll
    for (int u = 0; u < NKC; ++u) {
        uint32_t fm = ~(c1[u] | c2[u] | c3[u]) & 0xFFu;
        if (fm) {
            const uint32_t dst = row + (((uint32_t)(kc0 + u) << 4) ^ rx);
            uint32_t f = fo[u];
            do {
                const int j = __ffs(fm) - 1;
                fm &= fm - 1;
                sts16(dst + 2u * (uint32_t)j, lds16(g.full + 2u * f));
                ++f;
            } while (fm);
        }
    }
}

// Decode rows 32*half .. 32*half+31 of a GT (lane L owns row 32*half + L, all
// 8 column blocks) into registers and hand each 8-element row segment to
// emit(kc, o0, o1, o2, o3), fallbacks already patched in. This is the layout
// tcgen05.st 32x32b wants: lane = row, 4 consecutive 32-bit columns per block.
// The 8 blocks are processed in two phases of four so the shared-memory loads
// of a phase are all issued before any of its values is consumed.
template <int NKC, class Emit>
__device__ __forceinline__ void decode_gt_half_regs(const GtView& g, uint32_t lut_lane, const DecodeTables& t,
                                                    int half, int kc0, Emit&& emit) {
    const int lane = threadIdx.x & 31;
    const int m = half * 32 + lane;
    const int w = m >> 4, mr = (m >> 3) & 1, r = m & 7;
    const bool use_hi = r >= 4;
    const uint32_t mlo = r < 4 ? ((1u << (8 * r)) - 1u) : 0xFFFFFFFFu;
    const uint32_t mhi = r < 4 ? 0u : ((1u << (8 * (r - 4))) - 1u);
    const uint32_t bsel = (uint32_t)(r & 3) | 0x4440u;
    const uint32_t bm = g.bm + 8u * (uint32_t)(w * 16 + mr);
    // high-frequency elements in the column blocks before kc0 (both row blocks)
    uint32_t skipped = 0;
    for (int kc = 0; kc < kc0; ++kc) {
        const uint32_t bo = bm + 16u * (uint32_t)kc;
        const uint2 v1 = lds64(bo), v2 = lds64(bo + g.bstride), v3 = lds64(bo + 2u * g.bstride);
        const uint32_t tot = __popc(v1.x | v2.x | v3.x) + __popc(v1.y | v2.y | v3.y);
        skipped += tot + __shfl_xor_sync(0xFFFFFFFFu, tot, 8);
    }
    uint32_t acc_h = lds32(g.mt + 8u * w) + skipped;
    uint32_t acc_f = lds32(g.mt + 8u * w + 4u) + 128u * (uint32_t)kc0 - skipped;
    constexpr int PH = NKC < 4 ? NKC : 4;
#pragma unroll
    for (int ph = 0; ph < NKC / PH; ++ph) {
        uint32_t c1[PH], c2[PH], c3[PH], hf[PH], fo[PH];
#pragma unroll
        for (int u = 0; u < PH; ++u) {
            const uint32_t bo = bm + 16u * (uint32_t)(kc0 + PH * ph + u);
            const uint2 v1 = lds64(bo), v2 = lds64(bo + g.bstride), v3 = lds64(bo + 2u * g.bstride);
            const uint32_t ilo = v1.x | v2.x | v3.x;
            const uint32_t ihi = v1.y | v2.y | v3.y;
            const uint32_t tot = __popc(ilo) + __popc(ihi);
            const uint32_t pre = __popc(ilo & mlo) + __popc(ihi & mhi);
            const uint32_t ptot = __shfl_xor_sync(0xFFFFFFFFu, tot, 8);
            // Clamp keeps a corrupt offset array inside the staged slots.
            hf[u] = min(acc_h + (mr ? ptot : 0u) + pre, g.hf_cap);
            fo[u] = min(acc_f + (mr ? 64u - ptot : 0u) + 8u * (uint32_t)r - pre, g.full_cap);
            c1[u] = prmt(use_hi ? v1.y : v1.x, 0, bsel);
            c2[u] = prmt(use_hi ? v2.y : v2.x, 0, bsel);
            c3[u] = prmt(use_hi ? v3.y : v3.x, 0, bsel);
            acc_h += tot + ptot;
            acc_f += 128u - tot - ptot;
        }
        uint32_t s1[PH], s2[PH], s3[PH], q0[PH], q1[PH], q2[PH];
#pragma unroll
        for (int u = 0; u < PH; ++u) {
            s1[u] = lds32(lut_lane + (c1[u] << 7));
            s2[u] = lds32(lut_lane + (c2[u] << 7));
            s3[u] = lds32(lut_lane + (c3[u] << 7));
            const uint32_t wa = (g.sm + hf[u]) & ~3u;
            q0[u] = lds32(wa);
            q1[u] = lds32(wa + 4);
            q2[u] = lds32(wa + 8);
        }
#pragma unroll
        for (int u = 0; u < PH; ++u) {
            const uint32_t X = s1[u] + (s2[u] << 1) + (s3[u] << 2);
            const uint32_t sel = (s1[u] | s2[u] | s3[u]) * 0x11111110u;
            const uint32_t sh = ((g.sm + hf[u]) & 3u) * 8u;
            const uint32_t lo = __funnelshift_r(q0[u], q1[u], sh);
            const uint32_t hi = __funnelshift_r(q1[u], q2[u], sh);
            const uint32_t s_lo = prmt(lo, hi, sel);
            const uint32_t s_hi = prmt(lo, hi, sel >> 16);
            const uint32_t hb_lo = lop_or_and(s_lo, 0x80808080u, prmt(t.thb0, t.thb1, X));
            const uint32_t hb_hi = lop_or_and(s_hi, 0x80808080u, prmt(t.thb0, t.thb1, X >> 16));
            const uint32_t lb_lo = lop_or_and(s_lo, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X));
            const uint32_t lb_hi = lop_or_and(s_hi, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X >> 16));
            uint32_t o0 = prmt(lb_lo, hb_lo, 0x5140), o1 = prmt(lb_lo, hb_lo, 0x7362);
            uint32_t o2 = prmt(lb_hi, hb_hi, 0x5140), o3 = prmt(lb_hi, hb_hi, 0x7362);
            uint32_t fm = ~(c1[u] | c2[u] | c3[u]) & 0xFFu;
            if (fm) {
                uint32_t f = fo[u];
                do {
                    const uint32_t j = __ffs(fm) - 1;
                    fm &= fm - 1;
                    const uint32_t v = lds16(g.full + 2u * f);
                    ++f;
                    const uint32_t hsh = (j & 1u) * 16u;
                    const uint32_t keep = ~(0xFFFFu << hsh), ins = v << hsh;
                    const uint32_t pj = j >> 1;
                    o0 = pj == 0 ? (o0 & keep) | ins : o0;
                    o1 = pj == 1 ? (o1 & keep) | ins : o1;
                    o2 = pj == 2 ? (o2 & keep) | ins : o2;
                    o3 = pj == 3 ? (o3 & keep) | ins : o3;
                } while (fm);
            }
            emit(kc0 + PH * ph + u, o0, o1, o2, o3);
        }
    }
}

// Inclusive scan of per-small-tile values over the 16 small tiles of a median
// tile in ST order (s = 2 kc + mr), for the lane order of decode_mt_to_tile
// (lane = 16 rh + 8 mr + kc; both row halves hold the same values). Values
// may pack two 16-bit counts.
__device__ __forceinline__ uint32_t st_order_inclusive_scan(uint32_t v, int lane) {
    const int p = lane & 15;   // scan position = small tile p, held by lane 8 (p & 1) + (p >> 1)
    uint32_t x = __shfl_sync(0xFFFFFFFFu, v, (lane & 16) | (8 * (p & 1) + (p >> 1)));
#pragma unroll
    for (int d = 1; d < 16; d <<= 1) {
        const uint32_t y = __shfl_up_sync(0xFFFFFFFFu, x, d, 16);
        if (p >= d) x += y;
    }
    const int s = 2 * (lane & 7) + ((lane >> 3) & 1);   // this lane's small tile
    return __shfl_sync(0xFFFFFFFFu, x, (lane & 16) | s);
}

// Decode median tile w (16 rows x 64 columns = 16 small tiles) of a staged GT
// into 16 consecutive rows of a 128-byte-row bf16 tile in the UMMA canonical
// 128-byte-swizzle layout (16-byte chunk c of tile row m at (c ^ (m & 7)) * 16).
// `rows` is the tile address of the median tile's first row (a multiple of 8
// rows into the tile).
//
// Lane L owns column block kc = L & 7 of row block mr = (L >> 3) & 1, i.e.
// small tile s = 2 kc + mr, and rows 4 * (L >> 4) .. +3 of it. Lanes are
// ordered (mr, kc) so that the 8 lanes of a quarter-warp store 8 different
// 16-byte chunk positions of the swizzled tile (no bank conflicts). The hf
// offset of each small tile is the median-tile base plus an exclusive scan of
// the small-tile hf counts in ST order (s = 2 kc + mr, csrc/L_API.cu:623-644),
// done by shuffling the counts into ST order, scanning and shuffling back; the
// offset of a row adds the popcount of the indicator bits of the rows above
// it. Each lane then decodes its rows with decode_row_hf and finally
// overwrites its own fallback elements (code 0) in place, reading the fallback
// stream in ST order.
__device__ __forceinline__ void decode_mt_to_tile(const GtView& g, const DecodeTables& t, int w, uint32_t rows) {
    const int lane = threadIdx.x & 31;
    const int rh = lane >> 4, kc = lane & 7, mr = (lane >> 3) & 1, s = 2 * kc + mr;
    const uint32_t st = 16u * (uint32_t)w + (uint32_t)s;
    const uint2 v1 = lds64(g.bm + 8u * st), v2 = lds64(g.bm + g.bstride + 8u * st),
                v3 = lds64(g.bm + 2u * g.bstride + 8u * st);
    const uint32_t ilo = v1.x | v2.x | v3.x, ihi = v1.y | v2.y | v3.y;
    const uint32_t plo = __popc(ilo);
    const uint32_t hc = plo + __popc(ihi);
    const uint32_t excl = st_order_inclusive_scan(hc, lane) - hc;
    const uint32_t hs = lds32(g.mt + 8u * (uint32_t)w) + excl + (rh ? plo : 0u);
    const uint32_t fs = lds32(g.mt + 8u * (uint32_t)w + 4u) + 64u * (uint32_t)s - excl + (rh ? 32u - plo : 0u);
    const uint32_t ind = rh ? ihi : ilo;   // indicator bits of this lane's 4 rows
    const uint32_t w1 = rh ? v1.y : v1.x, w2 = rh ? v2.y : v2.x, w3 = rh ? v3.y : v3.x;
    const uint32_t base = rows + 128u * (8u * (uint32_t)mr + 4u * (uint32_t)rh);
    const uint32_t sw = (uint32_t)kc ^ (4u * (uint32_t)rh);   // swizzled chunk of row r is sw ^ r
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint32_t pre = r ? (uint32_t)__popc(ind & ((1u << (8 * r)) - 1u)) : 0u;
        const uint32_t hf = min(hs + pre, g.hf_cap);
        uint32_t o[4];
        decode_row_words(w1, w2, w3, (uint32_t)r, g.sm + hf, t, o);
        sts128(base + 128u * (uint32_t)r + ((sw ^ (uint32_t)r) << 4), o[0], o[1], o[2], o[3]);
    }
    uint32_t fm = ~ind;
    uint32_t f = fs;
    while (fm) {
        const uint32_t j = __ffs(fm) - 1;
        fm &= fm - 1;
        const uint32_t r = j >> 3, c = j & 7;
        sts16(base + 128u * r + ((sw ^ r) << 4) + 2u * c, lds16(g.full + 2u * min(f, g.full_cap)));
        ++f;
    }
}

// Decode median tiles w0 and w0 + 1 of a staged GT (32 consecutive rows) into
// the 128-byte-swizzled tile rows starting at `rows`, with the lane mapping of
// decode_mt_to_tile. Both tiles' small-tile hf counts ride in one 16-bit-packed
// scan (a median tile holds at most 1024 hf elements), so the per-tile prologue
// (bitmap loads, scan, offsets) is shared and each lane has 8 independent rows
// to interleave. Fallbacks of both tiles are patched in one loop.
__device__ __forceinline__ void decode_mt2_to_tile(const GtView& g, const DecodeTables& t, int w0, uint32_t rows) {
    const int lane = threadIdx.x & 31;
    const int rh = lane >> 4, kc = lane & 7, mr = (lane >> 3) & 1, s = 2 * kc + mr;
    uint32_t W1[2], W2[2], W3[2], IND[2], PLO[2], HC[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        const uint32_t st = 16u * (uint32_t)(w0 + q) + (uint32_t)s;
        const uint2 v1 = lds64(g.bm + 8u * st), v2 = lds64(g.bm + g.bstride + 8u * st),
                    v3 = lds64(g.bm + 2u * g.bstride + 8u * st);
        const uint32_t ilo = v1.x | v2.x | v3.x, ihi = v1.y | v2.y | v3.y;
        PLO[q] = __popc(ilo);
        HC[q] = PLO[q] + __popc(ihi);
        IND[q] = rh ? ihi : ilo;
        W1[q] = rh ? v1.y : v1.x;
        W2[q] = rh ? v2.y : v2.x;
        W3[q] = rh ? v3.y : v3.x;
    }
    const uint32_t hcp = HC[0] | (HC[1] << 16);
    const uint32_t ex = st_order_inclusive_scan(hcp, lane) - hcp;
    const uint2 mo0 = lds64(g.mt + 8u * (uint32_t)w0), mo1 = lds64(g.mt + 8u * (uint32_t)w0 + 8u);
    uint32_t HS[2], FS[2];
    HS[0] = mo0.x + (ex & 0xFFFFu) + (rh ? PLO[0] : 0u);
    FS[0] = mo0.y + 64u * (uint32_t)s - (ex & 0xFFFFu) + (rh ? 32u - PLO[0] : 0u);
    HS[1] = mo1.x + (ex >> 16) + (rh ? PLO[1] : 0u);
    FS[1] = mo1.y + 64u * (uint32_t)s - (ex >> 16) + (rh ? 32u - PLO[1] : 0u);
    const uint32_t sw = (uint32_t)kc ^ (4u * (uint32_t)rh);   // swizzled chunk of row r is sw ^ r
    const uint32_t b0 = rows + 128u * (8u * (uint32_t)mr + 4u * (uint32_t)rh);
#pragma unroll
    for (int q = 0; q < 2; ++q) {
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t pre = r ? (uint32_t)__popc(IND[q] & ((1u << (8 * r)) - 1u)) : 0u;
            const uint32_t hf = min(HS[q] + pre, g.hf_cap);
            uint32_t o[4];
            decode_row_words(W1[q], W2[q], W3[q], (uint32_t)r, g.sm + hf, t, o);
            sts128(b0 + 2048u * (uint32_t)q + 128u * (uint32_t)r + ((sw ^ (uint32_t)r) << 4), o[0], o[1], o[2], o[3]);
        }
    }
    uint32_t fm0 = ~IND[0], fm1 = ~IND[1];
    uint32_t f0 = FS[0], f1 = FS[1];
    while (fm0 | fm1) {
        const bool a = fm0 != 0;
        const uint32_t fm = a ? fm0 : fm1;
        const uint32_t j = __ffs(fm) - 1;
        const uint32_t r = j >> 3, c = j & 7;
        const uint32_t f = a ? f0 : f1;
        sts16(b0 + (a ? 0u : 2048u) + 128u * r + ((sw ^ r) << 4) + 2u * c, lds16(g.full + 2u * min(f, g.full_cap)));
        if (a) { fm0 &= fm0 - 1; ++f0; } else { fm1 &= fm1 - 1; ++f1; }
    }
}

// Shared-memory footprint helpers for one staged GT.
__host__ __device__ inline uint32_t round_up_u32(uint32_t x, uint32_t a) { return (x + a - 1) / a * a; }
// Bytes reserved for a GT's hf stream: capacity plus 16 bytes of read slack
// (decode_row reads up to 11 bytes past the row's first hf byte).
__host__ __device__ inline uint32_t hf_slot_bytes(int max_hf) { return round_up_u32((uint32_t)max_hf, 16) + 16; }
__host__ __device__ inline uint32_t full_slot_bytes(int max_full) {
    return round_up_u32((uint32_t)max_full * 2u, 16) + 16;
}

// Byte ranges of one GT's hf and fallback streams, validated against the
// staging slot capacity. A corrupt offset array is clamped (and reported via
// kErrStreamOverflow) so a copy can never run past its shared-memory slot.
struct GtCopy {
    int h0, f0;        // stream start (hf byte index, fallback element index)
    uint32_t hb, fb;   // bytes to copy (multiples of 16)
};

__device__ __forceinline__ GtCopy gt_copy_range(const int* gt_off, long long gt, int max_hf, int max_full,
                                                unsigned* err) {
    GtCopy c;
    c.h0 = gt_off[2 * gt];
    c.f0 = gt_off[2 * gt + 1];
    const int h1 = gt_off[2 * gt + 2], f1 = gt_off[2 * gt + 3];
    c.hb = (h1 > c.h0) ? (uint32_t)(h1 - c.h0) : 0u;
    c.fb = (f1 > c.f0) ? (uint32_t)(f1 - c.f0) * 2u : 0u;
    const uint32_t hcap = round_up_u32((uint32_t)max_hf, 16), fcap = round_up_u32((uint32_t)max_full, 8) * 2u;
    if (c.hb > hcap || c.fb > fcap || (c.hb & 15u) || (c.fb & 15u) || (c.h0 & 15) || (c.f0 & 7) || c.h0 < 0 ||
        c.f0 < 0) {
        if (err) atomicOr(err, kErrStreamOverflow);
        c.hb = min(c.hb, hcap) & ~15u;
        c.fb = min(c.fb, fcap) & ~15u;
        c.h0 = max(c.h0, 0) & ~15;
        c.f0 = max(c.f0, 0) & ~7;
    }
    return c;
}

}  // namespace zs
