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

struct GtSmem {
    const uint64_t* bm1;   // [64] bitmaps of this GT
    const uint64_t* bm2;
    const uint64_t* bm3;
    const int* mt;         // [8] median-tile (hf, fallback) offsets within the GT
    const uint8_t* sm;     // GT's sign/mantissa stream (GT-local offset 0)
    const uint16_t* full;  // GT's fallback stream (GT-local offset 0)
    uint32_t hf_cap;       // largest hf offset a row may start at (slot bytes - 16)
    uint32_t full_cap;     // largest fallback offset a row may start at (slot elems - 8)
};

// Store functor signature: store(row_in_gt, kc, const uint32_t (&o)[4]).
template <class Store>
__device__ __forceinline__ void decode_gt_half(const GtSmem& g, const uint32_t* spread, const DecodeTables& t,
                                               int half, Store&& store) {
    const int lane = threadIdx.x & 31;
    const int m = half * 32 + lane;
    const int w = m >> 4, mr = (m >> 3) & 1, r = m & 7;
    uint32_t acc_h = (uint32_t)g.mt[2 * w];
    uint32_t acc_f = (uint32_t)g.mt[2 * w + 1];
    const uint32_t mlo = r < 4 ? ((1u << (8 * r)) - 1u) : 0xFFFFFFFFu;
    const uint32_t mhi = r < 4 ? 0u : ((1u << (8 * (r - 4))) - 1u);
    const bool use_hi = r >= 4;
    const uint32_t bsh = 8u * (uint32_t)(r & 3);
#pragma unroll 2
    for (int kc = 0; kc < 8; ++kc) {
        const int st = w * 16 + 2 * kc + mr;
        const uint2 v1 = reinterpret_cast<const uint2*>(g.bm1)[st];
        const uint2 v2 = reinterpret_cast<const uint2*>(g.bm2)[st];
        const uint2 v3 = reinterpret_cast<const uint2*>(g.bm3)[st];
        const uint32_t ilo = v1.x | v2.x | v3.x;
        const uint32_t ihi = v1.y | v2.y | v3.y;
        const uint32_t tot = __popc(ilo) + __popc(ihi);
        const uint32_t pre = __popc(ilo & mlo) + __popc(ihi & mhi);
        const uint32_t ptot = __shfl_xor_sync(0xFFFFFFFFu, tot, 8);
        // Clamp keeps a corrupt offset array inside the staged slots.
        const uint32_t hf = min(acc_h + (mr ? ptot : 0u) + pre, g.hf_cap);
        const uint32_t fo = min(acc_f + (mr ? 64u - ptot : 0u) + 8u * (uint32_t)r - pre, g.full_cap);
        const uint32_t c1 = ((use_hi ? v1.y : v1.x) >> bsh) & 0xFFu;
        const uint32_t c2 = ((use_hi ? v2.y : v2.x) >> bsh) & 0xFFu;
        const uint32_t c3 = ((use_hi ? v3.y : v3.x) >> bsh) & 0xFFu;
        uint32_t o[4];
        decode_row(c1, c2, c3, spread, g.sm, hf, g.full, fo, t, o);
        store(m, kc, o);
        acc_h += tot + ptot;
        acc_f += 128u - tot - ptot;
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
