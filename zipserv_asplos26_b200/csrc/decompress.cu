// Standalone TCA-TBE decompressor: compressed streams -> dense row-major bf16.
// Replaces csrc/L_Kernel.cuh:1110 BF16TripleBitmap_Decompress_Kernel and
// csrc/L_API.cu:234 BF16TripleBitmap_Decompress_API.
//
// One CTA (8 warps) per group of four 64x64 global tiles. Thread 0 pulls each
// GT's five streams into shared memory with 1-D bulk copies (the GT's hf and
// fallback streams are contiguous and 16-byte aligned thanks to the format's
// per-GT padding); two warps per GT then decode 32 rows each with the
// branch-free row decoder into a bank-swizzled 64x64 tile, and the CTA writes
// the tiles out with 16-byte coalesced stores (8 threads per 128-byte row).
// The decoder is latency bound per warp, so the CTA is kept small enough for
// several to share an SM.
#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

constexpr int kDecompGTs = 4;                     // global tiles per CTA
constexpr int kDecompThreads = 64 * kDecompGTs;   // two warps per GT

struct DecompSmemLayout {
    uint32_t lut, bar, gt_base, gt_stride, bm, mt, hfs, fulls, tile, total;
    __host__ __device__ DecompSmemLayout(int max_hf, int max_full) {
        lut = 0;                          // replicated spread table
        bar = 4 * kLutWords;              // mbarrier
        gt_base = bar + 16;
        bm = 0;                           // 3 x 512 B
        mt = 1536;                        // 32 B
        hfs = 1568;                       // hf slot
        fulls = hfs + hf_slot_bytes(max_hf);
        tile = round_up_u32(fulls + full_slot_bytes(max_full), 16);
        gt_stride = round_up_u32(tile + 8192, 16);
        total = gt_base + kDecompGTs * gt_stride;
    }
};

__device__ __forceinline__ void issue_gt_copies(uint8_t* base, const DecompSmemLayout& L, long long gt,
                                                const GtCopy& c, const uint8_t* sm, const uint16_t* full,
                                                const uint64_t* b1, const uint64_t* b2, const uint64_t* b3,
                                                const int* mt_off, uint64_t* bar) {
    bulk_g2s(base + L.bm, b1 + gt * 64, 512, bar);
    bulk_g2s(base + L.bm + 512, b2 + gt * 64, 512, bar);
    bulk_g2s(base + L.bm + 1024, b3 + gt * 64, 512, bar);
    bulk_g2s(base + L.mt, mt_off + gt * 8, 32, bar);
    if (c.hb) bulk_g2s(base + L.hfs, sm + c.h0, c.hb, bar);
    if (c.fb) bulk_g2s(base + L.fulls, full + c.f0, c.fb, bar);
}

__global__ void __launch_bounds__(kDecompThreads) decompress_kernel(const uint8_t* __restrict__ sm,
                                                         const uint16_t* __restrict__ full,
                                                         const uint64_t* __restrict__ b1,
                                                         const uint64_t* __restrict__ b2,
                                                         const uint64_t* __restrict__ b3,
                                                         const int* __restrict__ mt_off,
                                                         const int* __restrict__ gt_off, int max_hf, int max_full,
                                                         int start_exp, uint16_t* __restrict__ out, int M, int K,
                                                         unsigned* err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const DecompSmemLayout L(max_hf, max_full);
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem + L.lut);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    __shared__ int abort_flag;
    const int tid = threadIdx.x;
    const int gtk = K / kGT;
    const long long ngt = (long long)(M / kGT) * gtk;
    const long long gt0 = (long long)kDecompGTs * blockIdx.x;
    const int nsub = (int)min((long long)kDecompGTs, ngt - gt0);

    fill_spread_table(lut, tid, kDecompThreads);
    if (tid == 0) {
        abort_flag = 0;
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {
        GtCopy c[kDecompGTs];
        uint32_t total = 0;
        for (int s = 0; s < nsub; ++s) {
            c[s] = gt_copy_range(gt_off, gt0 + s, max_hf, max_full, err);
            total += 3 * 512 + 32 + c[s].hb + c[s].fb;
        }
        // expect_tx is posted before any copy so the phase cannot complete early.
        mbar_arrive_expect_tx(bar, total);
        for (int s = 0; s < nsub; ++s)
            issue_gt_copies(smem + L.gt_base + s * L.gt_stride, L, gt0 + s, c[s], sm, full, b1, b2, b3, mt_off,
                            bar);
    }
    const bool ok = mbar_wait(bar, 0, err, &abort_flag);
    const int warp = tid >> 5;
    const int sub = warp >> 1;
    const DecodeTables tabs = make_decode_tables(start_exp);
    if (ok && sub < nsub) {
        const uint32_t base = launder(smem_u32(smem + L.gt_base + sub * L.gt_stride));
        GtView g;
        g.bm = base + L.bm;
        g.bstride = 512;
        g.mt = base + L.mt;
        g.sm = base + L.hfs;
        g.full = base + L.fulls;
        g.hf_cap = hf_slot_bytes(max_hf) - 16;
        g.full_cap = full_slot_bytes(max_full) / 2 - 8;
        const uint32_t lut_lane = launder(smem_u32(lut)) + 4u * (uint32_t)(tid & 31);
        if (warp & 1)
            decode_gt_rows<true, 8>(g, lut_lane, tabs, base + L.tile, 0);
        else
            decode_gt_rows<false, 8>(g, lut_lane, tabs, base + L.tile, 0);
    }
    __syncthreads();
    if (!ok) return;
    for (int idx = tid; idx < nsub * 512; idx += kDecompThreads) {
        const int s = idx >> 9, row = (idx >> 3) & 63, c = idx & 7;
        const long long gt = gt0 + s;
        const uint8_t* tile = smem + L.gt_base + s * L.gt_stride + L.tile;
        const uint4 v = *reinterpret_cast<const uint4*>(tile + row * 128 + ((c ^ (row & 7)) << 4));
        const size_t grow = (size_t)(gt / gtk) * kGT + row;
        const size_t gcol = (size_t)(gt % gtk) * kGT + c * 8;
        *reinterpret_cast<uint4*>(out + grow * K + gcol) = v;
    }
}

cudaError_t launch_decompress(cudaStream_t stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                              const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                              int max_hf, int max_full, int start_exp, uint16_t* out, int M, int K,
                              unsigned* err) {
    if (M <= 0 || K <= 0 || (M % 64) || (K % 64)) return cudaErrorInvalidValue;
    if (max_hf < 0 || max_full < 0 || max_hf > 4096 + 15 || max_full > 4096 + 7) return cudaErrorInvalidValue;
    if (!b1 || !b2 || !b3 || !mt_off || !gt_off || !out) return cudaErrorInvalidValue;
    if ((max_hf > 0 && !sm) || (max_full > 0 && !full)) return cudaErrorInvalidValue;
    if (!aligned16(sm) || !aligned16(full) || !aligned16(b1) || !aligned16(b2) || !aligned16(b3) ||
        !aligned16(mt_off) || !aligned16(out))
        return cudaErrorInvalidValue;
    const long long ngt = (long long)(M / 64) * (K / 64);
    const DecompSmemLayout L(max_hf, max_full);
    ZS_RETURN_IF_ERR(cudaFuncSetAttribute(decompress_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          (int)L.total));
    const long long grid = (ngt + kDecompGTs - 1) / kDecompGTs;
    decompress_kernel<<<(unsigned)grid, kDecompThreads, L.total, stream>>>(sm, full, b1, b2, b3, mt_off, gt_off, max_hf,
                                                                max_full, start_exp & 0xFF, out, M, K, err);
    return cudaGetLastError();
}

}  // namespace zs
