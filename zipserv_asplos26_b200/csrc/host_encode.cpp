// Host (CPU) TCA-TBE encoders behind the reference's host ABI
// (build/L_API.cuh:54-144: InitBF16MatrixTripleBitmap, _Reuse, _Reuse_SIMD)
// and the host exponent-window analysis (kernel_benchmark/utils.h:189).
//
// These are the reference's offline "compress once" entry points; they produce
// exactly the reference's bytes. One core does the work for all three:
//   pass 1  (parallel over 64x64 global tiles, OpenMP) classify each 8-element
//           row of every small tile with a 256-entry exponent->code table,
//           write bitmaps / per-ST counts / median offsets, and compact the
//           tile's hf bytes and fallbacks into its private temp slot;
//   pass 2  exclusive prefix of the padded per-GT counts (TileOffsets_global);
//   pass 3  (parallel) copy each temp slot to its final stream position.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <omp.h>
#include <stdint.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "zs_host.h"
#include "L_API.cuh"

namespace zs {

static constexpr int kSlotHf = 4096 + 15;    // per-GT temp capacity (csrc/L_API.cu:596)
static constexpr int kSlotFull = 4096 + 7;

void analyze_host(const uint16_t* a, long long n, int rule, int* top) {
    std::vector<unsigned long long> cnt(256, 0);
#pragma omp parallel
    {
        unsigned long long loc[256] = {0};
#pragma omp for schedule(static)
        for (long long i = 0; i < n; ++i) loc[(a[i] >> 7) & 0xFF]++;
#pragma omp critical
        for (int e = 0; e < 256; ++e) cnt[e] += loc[e];
    }
    int picks[7], np = 0;
    if (rule == 0) {
        bool used[256] = {false};
        for (int t = 0; t < 7; ++t) {
            int best = -1;
            unsigned long long bc = 0;
            for (int e = 0; e < 256; ++e)
                if (!used[e] && cnt[e] > bc) { bc = cnt[e]; best = e; }
            if (best >= 0) { picks[np++] = best; used[best] = true; }
        }
    } else {
        int te[7];
        long long tc[7];
        for (int i = 0; i < 7; ++i) { te[i] = -1; tc[i] = -1; }
        for (int e = 0; e < 256; ++e) {
            int mi = 0;
            for (int i = 1; i < 7; ++i) if (tc[i] < tc[mi]) mi = i;
            if ((long long)cnt[e] > tc[mi]) { tc[mi] = (long long)cnt[e]; te[mi] = e; }
        }
        for (int i = 0; i < 7; ++i) if (te[i] >= 0) picks[np++] = te[i];
    }
    while (np < 7) { picks[np] = 127 - np; ++np; }
    std::sort(picks, picks + 7);
    for (int c = 0; c < 7; ++c) {
        const int s = picks[c];
        if (s < 0 || s + 6 > 255) continue;
        bool ok = true;
        for (int i = 0; i < 7; ++i) if (cnt[s + i] == 0) { ok = false; break; }
        if (!ok) continue;
        for (int i = 0; i < 7; ++i) top[i] = s + i;
        return;
    }
    int best_start = picks[0], best_len = 1, cur = 1;
    for (int i = 1; i < 7; ++i) {
        if (picks[i] == picks[i - 1] + 1) {
            if (++cur > best_len) { best_len = cur; best_start = picks[i] - cur + 1; }
        } else {
            cur = 1;
        }
    }
    if (rule != 0) best_start = std::min(std::max(best_start, 0), 248);
    for (int i = 0; i < 7; ++i) top[i] = best_start + i;
}

// Pass 1 for one GT. Returns padded (hf, fallback) counts through *nh, *nf.
static void encode_gt(const uint16_t* a, int K, long long gt, int gtk, const uint8_t* code_of, uint8_t* tsm,
                      uint16_t* tfull, uint64_t* b1, uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off,
                      int* nh, int* nf) {
    const long long r0 = (gt / gtk) * 64, c0 = (gt % gtk) * 64;
    int hp = 0, fp = 0;
    for (int w = 0; w < 4; ++w) {
        mt_off[2 * (gt * 4 + w)] = hp;
        mt_off[2 * (gt * 4 + w) + 1] = fp;
        for (int s = 0; s < 16; ++s) {
            const int kc = s >> 1, mr = s & 1;
            const uint16_t* base = a + (r0 + w * 16 + mr * 8) * K + c0 + kc * 8;
            uint64_t p1 = 0, p2 = 0, p3 = 0;
            const int hp0 = hp, fp0 = fp;
            for (int r = 0; r < 8; ++r) {
                const uint16_t* row = base + (long long)r * K;
                for (int j = 0; j < 8; ++j) {
                    const uint16_t v = row[j];
                    const uint32_t c = code_of[(v >> 7) & 0xFF];
                    const int pos = r * 8 + j;
                    if (c) {
                        p1 |= (uint64_t)(c & 1u) << pos;
                        p2 |= (uint64_t)((c >> 1) & 1u) << pos;
                        p3 |= (uint64_t)((c >> 2) & 1u) << pos;
                        tsm[hp++] = (uint8_t)(((v >> 8) & 0x80) | (v & 0x7F));
                    } else {
                        tfull[fp++] = v;
                    }
                }
            }
            const long long st = gt * 64 + w * 16 + s;
            b1[st] = p1; b2[st] = p2; b3[st] = p3;
            st_counts[2 * st] = hp - hp0;
            st_counts[2 * st + 1] = fp - fp0;
        }
    }
    while (hp & 15) tsm[hp++] = 0;
    while (fp & 7) tfull[fp++] = 0;
    *nh = hp;
    *nf = fp;
}

int encode_host(const uint16_t* a, int M, int K, const int* top, uint8_t* sm, uint16_t* full, uint64_t* b1,
                uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off, uint8_t* temp_sm,
                uint16_t* temp_full, int* gt_hf, int* gt_full, int* hf_pre, int* full_pre, int* max_hf,
                int* max_full, int* total_hf, int* total_full) {
    if (M <= 0 || K <= 0 || (M % 64) || (K % 64)) return -1;
    uint8_t code_of[256];
    memset(code_of, 0, sizeof(code_of));
    for (int i = 0; i < 7; ++i)
        if (top[i] >= 0 && top[i] <= 255) code_of[top[i]] = (uint8_t)(i + 1);
    const int gtk = K / 64;
    const long long ngt = (long long)(M / 64) * gtk;
#pragma omp parallel for schedule(dynamic, 16)
    for (long long g = 0; g < ngt; ++g)
        encode_gt(a, K, g, gtk, code_of, temp_sm + g * kSlotHf, temp_full + g * kSlotFull, b1, b2, b3, st_counts,
                  mt_off, &gt_hf[g], &gt_full[g]);
    int mh = 0, mf = 0;
    hf_pre[0] = 0;
    full_pre[0] = 0;
    gt_off[0] = 0;
    gt_off[1] = 0;
    for (long long g = 0; g < ngt; ++g) {
        hf_pre[g + 1] = hf_pre[g] + gt_hf[g];
        full_pre[g + 1] = full_pre[g] + gt_full[g];
        gt_off[2 * (g + 1)] = hf_pre[g + 1];
        gt_off[2 * (g + 1) + 1] = full_pre[g + 1];
        mh = std::max(mh, gt_hf[g]);
        mf = std::max(mf, gt_full[g]);
    }
#pragma omp parallel for schedule(static)
    for (long long g = 0; g < ngt; ++g) {
        if (gt_hf[g]) memcpy(sm + hf_pre[g], temp_sm + g * kSlotHf, gt_hf[g]);
        if (gt_full[g]) memcpy(full + full_pre[g], temp_full + g * kSlotFull, (size_t)gt_full[g] * 2);
    }
    *max_hf = mh;
    *max_full = mf;
    *total_hf = hf_pre[ngt];
    *total_full = full_pre[ngt];
    return (int)ngt;
}

}  // namespace zs

// ----------------------- reference host ABI (C++ names) ---------------------
static bool standard_tiles(int tm, int tmm, int tmg, int tk, int tkm, int tkg) {
    return tm == 8 && tmm == 16 && tmg == 64 && tk == 8 && tkm == 64 && tkg == 64;
}

// build/L_API.cuh:54-74 (csrc/L_API.cu:314). Allocates outputs with malloc;
// the caller frees them with free(). Returns #GT, or -1 on failure.
__host__ int InitBF16MatrixTripleBitmap(__nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median,
                                        int tile_M_global, int tile_K, int tile_K_median, int tile_K_global,
                                        const int* top_exponents, uint8_t** sign_mantissa,
                                        __nv_bfloat16** compressed_full, uint64_t** bitmap1, uint64_t** bitmap2,
                                        uint64_t** bitmap3, int** TileOffsets, int** TileOffsets_median,
                                        int** TileOffsets_global, int& max_high_freq_count, int& max_full_count) {
    if (!standard_tiles(tile_M, tile_M_median, tile_M_global, tile_K, tile_K_median, tile_K_global)) return -1;
    if (M <= 0 || K <= 0 || (M % 64) || (K % 64)) return -1;
    const long long ngt = (long long)(M / 64) * (K / 64), nst = (long long)M * K / 64, nmt = nst / 16;
    uint8_t* tsm = (uint8_t*)malloc((size_t)ngt * zs::kSlotHf);
    uint16_t* tfu = (uint16_t*)malloc((size_t)ngt * zs::kSlotFull * 2);
    std::vector<int> c1(ngt + 1), c2(ngt + 1), o1(ngt + 1), o2(ngt + 1);
    uint8_t* sm = (uint8_t*)malloc((size_t)M * K + 16 * ngt);
    uint16_t* fu = (uint16_t*)malloc(((size_t)M * K + 8 * ngt) * 2);
    uint64_t* b1 = (uint64_t*)malloc(nst * 8);
    uint64_t* b2 = (uint64_t*)malloc(nst * 8);
    uint64_t* b3 = (uint64_t*)malloc(nst * 8);
    int* st = (int*)malloc(nst * 8);
    int* mt = (int*)malloc(nmt * 8);
    int* gt = (int*)malloc((ngt + 1) * 8);
    if (!tsm || !tfu || !sm || !fu || !b1 || !b2 || !b3 || !st || !mt || !gt) {
        free(tsm); free(tfu); free(sm); free(fu); free(b1); free(b2); free(b3); free(st); free(mt); free(gt);
        return -1;
    }
    int th = 0, tf = 0;
    zs::encode_host(reinterpret_cast<const uint16_t*>(A_bf16), M, K, top_exponents, sm, fu, b1, b2, b3, st, mt, gt,
                    tsm, tfu, c1.data(), c2.data(), o1.data(), o2.data(), &max_high_freq_count, &max_full_count,
                    &th, &tf);
    free(tsm);
    free(tfu);
    // shrink the streams to their used size (csrc/L_API.cu:553-554)
    uint8_t* sm2 = (uint8_t*)realloc(sm, th > 0 ? th : 1);
    uint16_t* fu2 = (uint16_t*)realloc(fu, tf > 0 ? (size_t)tf * 2 : 2);
    *sign_mantissa = sm2 ? sm2 : sm;
    *compressed_full = reinterpret_cast<__nv_bfloat16*>(fu2 ? fu2 : fu);
    *bitmap1 = b1; *bitmap2 = b2; *bitmap3 = b3;
    *TileOffsets = st; *TileOffsets_median = mt; *TileOffsets_global = gt;
    return (int)ngt;
}

static int reuse_common(__nv_bfloat16* A_bf16, int M, int K, int tm, int tmm, int tmg, int tk, int tkm, int tkg,
                        const int* top, uint8_t* sm, __nv_bfloat16* full, uint64_t* b1, uint64_t* b2, uint64_t* b3,
                        int* st, int* mt, int* gt, uint8_t* temp_sm, __nv_bfloat16* temp_full, int* c1, int* c2,
                        int* o1, int* o2, int& mh, int& mf, int& th, int& tf) {
    if (!standard_tiles(tm, tmm, tmg, tk, tkm, tkg)) return -1;
    return zs::encode_host(reinterpret_cast<const uint16_t*>(A_bf16), M, K, top, sm,
                           reinterpret_cast<uint16_t*>(full), b1, b2, b3, st, mt, gt, temp_sm,
                           reinterpret_cast<uint16_t*>(temp_full), c1, c2, o1, o2, &mh, &mf, &th, &tf);
}

// build/L_API.cuh:77-110 (csrc/L_API.cu:559). Caller-provided buffers;
// temp_sm holds #GT*(4096+15) bytes, temp_full #GT*(4096+7) bf16.
__host__ int InitBF16MatrixTripleBitmap_Reuse(__nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median,
                                              int tile_M_global, int tile_K, int tile_K_median, int tile_K_global,
                                              const int* top_exponents, uint8_t* sign_mantissa,
                                              __nv_bfloat16* compressed_full, uint64_t* bitmap1, uint64_t* bitmap2,
                                              uint64_t* bitmap3, int* TileOffsets, int* TileOffsets_median,
                                              int* TileOffsets_global, uint8_t* temp_sm, __nv_bfloat16* temp_full,
                                              int* gt_hf_count, int* gt_full_count, int* hf_offsets,
                                              int* full_offsets, int& max_high_freq_count, int& max_full_count,
                                              int& out_total_hf, int& out_total_full) {
    return reuse_common(A_bf16, M, K, tile_M, tile_M_median, tile_M_global, tile_K, tile_K_median, tile_K_global,
                        top_exponents, sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3, TileOffsets,
                        TileOffsets_median, TileOffsets_global, temp_sm, temp_full, gt_hf_count, gt_full_count,
                        hf_offsets, full_offsets, max_high_freq_count, max_full_count, out_total_hf,
                        out_total_full);
}

// build/L_API.cuh:113-144 (csrc/L_API.cu:804). Same contract and bytes as
// _Reuse (this build's core is already table-driven and multi-threaded, so
// both names share it).
__host__ int InitBF16MatrixTripleBitmap_Reuse_SIMD(
    __nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median, int tile_M_global, int tile_K,
    int tile_K_median, int tile_K_global, const int* top_exponents, uint8_t* sign_mantissa,
    __nv_bfloat16* compressed_full, uint64_t* bitmap1, uint64_t* bitmap2, uint64_t* bitmap3, int* TileOffsets,
    int* TileOffsets_median, int* TileOffsets_global, uint8_t* temp_sm, __nv_bfloat16* temp_full, int* gt_hf_count,
    int* gt_full_count, int* hf_offsets, int* full_offsets, int& max_high_freq_count, int& max_full_count,
    int& out_total_hf, int& out_total_full) {
    return reuse_common(A_bf16, M, K, tile_M, tile_M_median, tile_M_global, tile_K, tile_K_median, tile_K_global,
                        top_exponents, sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3, TileOffsets,
                        TileOffsets_median, TileOffsets_global, temp_sm, temp_full, gt_hf_count, gt_full_count,
                        hf_offsets, full_offsets, max_high_freq_count, max_full_count, out_total_hf,
                        out_total_full);
}
