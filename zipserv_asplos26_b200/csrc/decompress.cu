// Standalone TCA-TBE decompressor: compressed streams -> dense row-major bf16.
// Replaces csrc/L_Kernel.cuh:1110 BF16TripleBitmap_Decompress_Kernel and
// csrc/L_API.cu:234 BF16TripleBitmap_Decompress_API.
//
// One CTA (8 warps) per run of four consecutive 64x64 global tiles (GTs).
// Consecutive GTs are contiguous in every array of the format (bitmaps and
// median offsets are indexed by GT, the streams by the global prefix), so six
// lanes of warp 0 pull the whole run with six 1-D bulk copies (bitmaps 1-3,
// median offsets, sign/mantissa and fallback streams; the issue cost of a bulk
// copy grows with the copies per instruction, not with their size). Two warps
// per GT then decode a pair of median tiles each with the table-free row
// decoder into a swizzled 64x64 tile, and the CTA writes the tiles out with
// 16-byte coalesced stores (8 threads per 128-byte row). About 55 KB of shared
// memory per CTA lets four CTAs share an SM, so copies, decoding and stores of
// different CTAs overlap.
#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

constexpr int kDecompGTs = 4;                     // global tiles per CTA
constexpr int kDecompThreads = 64 * kDecompGTs;   // two warps per GT

struct DecompSmemLayout {
    uint32_t bar, bm, mt, hfs, fulls, tiles, total;
    uint32_t hf_cap, full_cap;   // bytes / elements the run's streams may hold
    __host__ __device__ DecompSmemLayout(int max_hf, int max_full) {
        hf_cap = round_up_u32((uint32_t)max_hf, 16) * kDecompGTs;
        full_cap = round_up_u32((uint32_t)max_full, 8) * kDecompGTs;
        bar = 0;                                   // mbarrier
        bm = 128;                                  // [3 planes][4 GTs][512 B]
        mt = bm + 3 * 512 * kDecompGTs;            // [4 GTs][32 B]
        hfs = mt + 32 * kDecompGTs;                // hf streams of the run (+16 B read slack)
        fulls = hfs + hf_cap + 16;                 // fallback streams of the run (+16 B)
        tiles = round_up_u32(fulls + 2 * full_cap + 16, 1024);   // [4 GTs][64 rows][128 B], swizzled
        total = tiles + 8192 * kDecompGTs;
    }
};

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
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gtk = K / kGT;
    const long long ngt = (long long)(M / kGT) * gtk;
    const long long gt0 = (long long)kDecompGTs * blockIdx.x;
    const int nsub = (int)min((long long)kDecompGTs, ngt - gt0);
    const int2* go = reinterpret_cast<const int2*>(gt_off);

    if (tid == 0) {
        abort_flag = 0;
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == 0) {
        // lanes 0-2: bitmap planes, 3: median offsets, 4: hf streams, 5: fallback streams of the run
        const int2 f = go[gt0], e = go[gt0 + nsub];
        uint32_t bytes = 0, dst = 0;
        const void* src = nullptr;
        if (lane < 3) {
            bytes = 512u * (uint32_t)nsub;
            src = (lane == 0 ? b1 : lane == 1 ? b2 : b3) + gt0 * 64;
            dst = L.bm + 512u * kDecompGTs * (uint32_t)lane;
        } else if (lane == 3) {
            bytes = 32u * (uint32_t)nsub;
            src = mt_off + gt0 * 8;
            dst = L.mt;
        } else if (lane < 6) {
            const bool hf = lane == 4;
            const int beg = hf ? f.x : f.y, end = hf ? e.x : e.y;
            const uint32_t cap = hf ? L.hf_cap : 2u * L.full_cap;
            const int al = hf ? 16 : 8;
            uint32_t b = end > beg ? (uint32_t)(end - beg) * (hf ? 1u : 2u) : 0u;
            int b0 = beg;
            if (b > cap || (b & 15u) || (b0 & (al - 1)) || b0 < 0) {   // corrupt offsets: clamp, report
                if (err) atomicOr(err, kErrStreamOverflow);
                b = min(b, cap) & ~15u;
                b0 = max(b0, 0) & ~(al - 1);
            }
            bytes = b;
            src = hf ? (const void*)(sm + b0) : (const void*)(full + b0);
            dst = hf ? L.hfs : L.fulls;
        }
        const uint32_t total = __reduce_add_sync(0xFFFFFFFFu, bytes);
        if (lane == 0) mbar_arrive_expect_tx(bar, total);   // posted before any copy lands
        __syncwarp();
        if (bytes) bulk_g2s(smem + dst, src, bytes, bar);
    }
    const bool ok = mbar_wait(bar, 0, err, &abort_flag);
    const int sub = warp >> 1;
    if (ok && sub < nsub) {
        const DecodeTables tabs = make_decode_tables(start_exp);
        const int2 f0 = go[gt0], fs = go[gt0 + sub];   // stream starts of the run and of this GT
        const uint32_t h0 = min((uint32_t)max(fs.x - f0.x, 0), L.hf_cap);
        const uint32_t q0 = min((uint32_t)max(fs.y - f0.y, 0), L.full_cap);
        const uint32_t base = launder(smem_u32(smem));
        GtView g;
        g.bm = base + L.bm + 512u * (uint32_t)sub;
        g.bstride = 512u * kDecompGTs;
        g.mt = base + L.mt + 32u * (uint32_t)sub;
        g.sm = base + L.hfs + h0;
        g.full = base + L.fulls + 2u * q0;
        g.hf_cap = L.hf_cap - h0;
        g.full_cap = L.full_cap - q0;
        const int w0 = 2 * (warp & 1);   // median tiles w0, w0 + 1 (rows 16 w0 .. 16 w0 + 31)
        decode_mt2_to_tile(g, tabs, w0, base + L.tiles + 8192u * (uint32_t)sub + 128u * (uint32_t)(16 * w0));
    }
    __syncthreads();
    if (!ok) return;
    for (int idx = tid; idx < nsub * 512; idx += kDecompThreads) {
        const int s = idx >> 9, row = (idx >> 3) & 63, c = idx & 7;
        const long long gt = gt0 + s;
        const uint8_t* tile = smem + L.tiles + s * 8192;
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
        !aligned16(mt_off) || !aligned16(out) || (reinterpret_cast<uintptr_t>(gt_off) & 7u))
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
