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

// Overwrite one lane's fallback elements (code 0) in place. Bit j of fm
// (j = 8 * row + column, rows relative to row0) marks a fallback; its value is
// the next element of the fallback stream from element f on (clamped to
// full_cap). Values are fetched kFbBatch at a time with independent loads, so
// their shared-memory latencies overlap, and then stored; the loop runs until
// the lane with the most fallbacks is done.
#ifndef ZS_FB_BATCH
#define ZS_FB_BATCH 2
#endif
constexpr int kFbBatch = ZS_FB_BATCH;
__device__ __forceinline__ void patch_fallbacks(uint32_t fm, uint32_t f, uint32_t full, uint32_t full_cap,
                                                uint32_t row0, uint32_t sw) {
    while (fm) {
        uint32_t pos[kFbBatch], val[kFbBatch];
#pragma unroll
        for (int k = 0; k < kFbBatch; ++k) {
            pos[k] = (uint32_t)__ffs(fm) - 1u;   // all ones once fm is empty
            fm &= fm - 1u;
            val[k] = lds16(full + 2u * min(f + (uint32_t)k, full_cap));
        }
#pragma unroll
        for (int k = 0; k < kFbBatch; ++k) {
            if (pos[k] < 32u) {
                const uint32_t r = pos[k] >> 3, c = pos[k] & 7u;
                sts16(row0 + 128u * r + ((sw ^ r) << 4) + 2u * c, val[k]);
            }
        }
        f += kFbBatch;
    }
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
// it. Each lane then decodes its rows with decode_row_words and finally
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
    const RowGroups rg = row_groups(w1, w2, w3);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        const uint32_t pre = r ? (uint32_t)__popc(ind & ((1u << (8 * r)) - 1u)) : 0u;
        const uint32_t hf = min(hs + pre, g.hf_cap);
        uint32_t o[4];
        decode_row_words(rg, (uint32_t)r, g.sm + hf, t, o);
        sts128(base + 128u * (uint32_t)r + ((sw ^ (uint32_t)r) << 4), o[0], o[1], o[2], o[3]);
    }
    patch_fallbacks(~ind, fs, g.full, g.full_cap, base, sw);
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
        const RowGroups rg = row_groups(W1[q], W2[q], W3[q]);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const uint32_t pre = r ? (uint32_t)__popc(IND[q] & ((1u << (8 * r)) - 1u)) : 0u;
            const uint32_t hf = min(HS[q] + pre, g.hf_cap);
            uint32_t o[4];
            decode_row_words(rg, (uint32_t)r, g.sm + hf, t, o);
            sts128(b0 + 2048u * (uint32_t)q + 128u * (uint32_t)r + ((sw ^ (uint32_t)r) << 4), o[0], o[1], o[2], o[3]);
        }
    }
    patch_fallbacks(~IND[0], FS[0], g.full, g.full_cap, b0, sw);
    patch_fallbacks(~IND[1], FS[1], g.full, g.full_cap, b0 + 2048u, sw);
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
