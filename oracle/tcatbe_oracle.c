/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the TCA-TBE hot path.
 *
 * This file is a plain-C restatement of the reference ZipServ algorithms. It is
 * the checker that the CUDA product path is compared against. Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU-baseline leg may load it. The
 * product library (zipserv_asplos26_b200/lib/libzipserv_b200.so) never links,
 * loads or calls anything in this directory.
 *
 * Parity is pinned: tests/golden/ holds fixtures produced by the reference's own
 * host encoder (csrc/L_API.cu, compiled from source by oracle/Makefile into
 * oracle/_ref/) and tests/test_oracle_golden.py checks this oracle against them
 * byte for byte.
 *
 * Reference functions restated here (paths inside the reference project):
 *   oracle_analyze_host   kernel_benchmark/utils.h:189-272 analyzeExponentDistribution_BF16
 *   oracle_analyze_ext    kernel_benchmark/zipserv_decode_attention_ext.cu:35-133
 *                         AnalyzeTopExponentsFusedKernel (top-7 selection rule)
 *   oracle_encode         csrc/L_API.cu:559-771 InitBF16MatrixTripleBitmap_Reuse
 *   oracle_decode         kernel_benchmark/bench_kv_cache_zipserv_decompress_token_scaling.cu:2106-2218
 *                         DecompressZipServChunkCPU
 *   oracle_gemm           test_mm.cu:410-428 (cuBLAS C = W * X^T, col-major M x N)
 *                         computed exactly in double after decoding
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define GT_ROWS 64
#define GT_COLS 64
#define ST_PER_GT 64
#define MT_PER_GT 4
#define ST_PER_MT 16

/* Row/column offset of small tile `s` (0..63) inside a 64x64 global tile.
 * Median tile w = s/16 covers rows 16w..16w+15. Inside it the 16 small tiles
 * go column pair by column pair, and each 2x2 group is column-major:
 * index j = s%16, kc = j/2 (8-column block), mr = j%2 (8-row block).
 * (csrc/L_API.cu:623-644 builds the same order with a 7-deep loop nest.) */
static void st_origin(int s, int* row_off, int* col_off) {
    int w = s / ST_PER_MT, j = s % ST_PER_MT;
    *row_off = w * 16 + (j % 2) * 8;
    *col_off = (j / 2) * 8;
}

/* kernel_benchmark/utils.h:189-272. Histogram of the 8-bit exponent field;
 * seven passes pick the largest count with a strict '>' (ties -> the lower
 * exponent, zero counts never picked); missing picks default to 127-n; sort;
 * the first pick p whose run p..p+6 has all counts > 0 (and p+6 <= 255) wins;
 * otherwise the start of the longest run of consecutive picks. */
void oracle_analyze_host(const uint16_t* a, int64_t n, int* top) {
    int64_t cnt[256];
    memset(cnt, 0, sizeof(cnt));
    for (int64_t i = 0; i < n; ++i) cnt[(a[i] >> 7) & 0xFF]++;
    int picks[7], npick = 0;
    unsigned char used[256];
    memset(used, 0, sizeof(used));
    for (int t = 0; t < 7; ++t) {
        int best = -1;
        int64_t bestc = 0;
        for (int e = 0; e < 256; ++e)
            if (!used[e] && cnt[e] > bestc) { bestc = cnt[e]; best = e; }
        if (best >= 0) { picks[npick++] = best; used[best] = 1; }
    }
    while (npick < 7) { picks[npick] = 127 - npick; npick++; }
    /* insertion sort of 7 values */
    for (int i = 1; i < 7; ++i) {
        int v = picks[i], j = i - 1;
        while (j >= 0 && picks[j] > v) { picks[j + 1] = picks[j]; --j; }
        picks[j + 1] = v;
    }
    for (int c = 0; c < 7; ++c) {
        int s = picks[c];
        if (s < 0 || s + 6 > 255) continue;
        int ok = 1;
        for (int i = 0; i < 7; ++i) if (cnt[s + i] <= 0) { ok = 0; break; }
        if (!ok) continue;
        for (int i = 0; i < 7; ++i) top[i] = s + i;
        return;
    }
    int best_start = picks[0], best_len = 1, cur = 1;
    for (int i = 1; i < 7; ++i) {
        if (picks[i] == picks[i - 1] + 1) {
            cur++;
            if (cur > best_len) { best_len = cur; best_start = picks[i] - cur + 1; }
        } else {
            cur = 1;
        }
    }
    for (int i = 0; i < 7; ++i) top[i] = best_start + i;
}

/* kernel_benchmark/zipserv_decode_attention_ext.cu:65-133 (the torch
 * extension's GPU rule). Differences from the host rule: a replace-the-minimum
 * top-7 scan initialised with count -1 (so zero-count exponents can be picked,
 * and on ties the earlier slot is replaced first), and the fallback start is
 * clamped to [0, 248]. */
void oracle_analyze_ext(const uint16_t* a, int64_t n, int* top) {
    int64_t cnt[256];
    memset(cnt, 0, sizeof(cnt));
    for (int64_t i = 0; i < n; ++i) cnt[(a[i] >> 7) & 0xFF]++;
    int te[7];
    int64_t tc[7];
    for (int i = 0; i < 7; ++i) { te[i] = -1; tc[i] = -1; }
    for (int e = 0; e < 256; ++e) {
        int mi = 0;
        for (int i = 1; i < 7; ++i) if (tc[i] < tc[mi]) mi = i;
        if (cnt[e] > tc[mi]) { tc[mi] = cnt[e]; te[mi] = e; }
    }
    int picks[7], np = 0;
    for (int i = 0; i < 7; ++i) if (te[i] >= 0) picks[np++] = te[i];
    while (np < 7) { picks[np] = 127 - np; np++; }
    for (int i = 1; i < 7; ++i) {
        int v = picks[i], j = i - 1;
        while (j >= 0 && picks[j] > v) { picks[j + 1] = picks[j]; --j; }
        picks[j + 1] = v;
    }
    for (int c = 0; c < 7; ++c) {
        int s = picks[c];
        if (s < 0 || s + 6 > 255) continue;
        int ok = 1;
        for (int i = 0; i < 7; ++i) if (cnt[s + i] <= 0) { ok = 0; break; }
        if (!ok) continue;
        for (int i = 0; i < 7; ++i) top[i] = s + i;
        return;
    }
    int best_start = picks[0], best_len = 1, cur = 1;
    for (int i = 1; i < 7; ++i) {
        if (picks[i] == picks[i - 1] + 1) {
            cur++;
            if (cur > best_len) { best_len = cur; best_start = picks[i] - cur + 1; }
        } else {
            cur = 1;
        }
    }
    if (best_start < 0) best_start = 0;
    if (best_start > 248) best_start = 248;
    for (int i = 0; i < 7; ++i) top[i] = best_start + i;
}

/* csrc/L_API.cu:559-771. Encode a row-major M x K bf16 matrix (M, K multiples
 * of 64) with the exponent list `top` (code = index in `top` + 1; exponents not
 * in the list are fallbacks). Output arrays must be sized by the caller:
 *   sign_mantissa  >= total padded hf bytes   (M*K + 16*#GT is always enough)
 *   full           >= total padded fallbacks  (M*K + 8*#GT)
 *   bitmap1..3     #ST = M*K/64 u64 each
 *   st_counts      2*#ST ints  (per small tile: hf, fallback; "TileOffsets")
 *   mt_offsets     2*#MT ints  (per median tile: cumulative hf, fallback in GT)
 *   gt_offsets     2*(#GT+1) ints (exclusive prefix of padded per-GT counts)
 * Returns #GT. */
int oracle_encode(const uint16_t* a, int M, int K, const int* top,
                  uint8_t* sign_mantissa, uint16_t* full,
                  uint64_t* bitmap1, uint64_t* bitmap2, uint64_t* bitmap3,
                  int* st_counts, int* mt_offsets, int* gt_offsets,
                  int* max_hf, int* max_full, int* total_hf, int* total_full) {
    unsigned char code_of[256];
    memset(code_of, 0, sizeof(code_of));
    for (int e = 0; e < 7; ++e)
        if (top[e] >= 0 && top[e] <= 255) code_of[top[e]] = (unsigned char)(e + 1);
    const int gtk = K / GT_COLS, gtm = M / GT_ROWS, ngt = gtm * gtk;
    int64_t hf_pos = 0, full_pos = 0;
    *max_hf = 0; *max_full = 0;
    gt_offsets[0] = 0; gt_offsets[1] = 0;
    for (int g = 0; g < ngt; ++g) {
        const int r0 = (g / gtk) * GT_ROWS, c0 = (g % gtk) * GT_COLS;
        int64_t hf_start = hf_pos, full_start = full_pos;
        int mt_hf = 0, mt_full = 0;
        for (int s = 0; s < ST_PER_GT; ++s) {
            if (s % ST_PER_MT == 0) {
                int mt = g * MT_PER_GT + s / ST_PER_MT;
                mt_offsets[2 * mt] = mt_hf;
                mt_offsets[2 * mt + 1] = mt_full;
            }
            int ro, co;
            st_origin(s, &ro, &co);
            uint64_t b1 = 0, b2 = 0, b3 = 0;
            int nh = 0, nf = 0;
            for (int p = 0; p < 64; ++p) {
                uint16_t v = a[(int64_t)(r0 + ro + p / 8) * K + c0 + co + p % 8];
                int c = code_of[(v >> 7) & 0xFF];
                if (c) {
                    if (c & 1) b1 |= 1ull << p;
                    if (c & 2) b2 |= 1ull << p;
                    if (c & 4) b3 |= 1ull << p;
                    sign_mantissa[hf_pos++] = (uint8_t)(((v >> 8) & 0x80) | (v & 0x7F));
                    nh++;
                } else {
                    full[full_pos++] = v;
                    nf++;
                }
            }
            int st = g * ST_PER_GT + s;
            bitmap1[st] = b1; bitmap2[st] = b2; bitmap3[st] = b3;
            st_counts[2 * st] = nh;
            st_counts[2 * st + 1] = nf;
            mt_hf += nh;
            mt_full += nf;
        }
        while ((hf_pos - hf_start) % 16) sign_mantissa[hf_pos++] = 0;
        while ((full_pos - full_start) % 8) full[full_pos++] = 0;
        int ghf = (int)(hf_pos - hf_start), gfl = (int)(full_pos - full_start);
        if (ghf > *max_hf) *max_hf = ghf;
        if (gfl > *max_full) *max_full = gfl;
        gt_offsets[2 * (g + 1)] = (int)hf_pos;
        gt_offsets[2 * (g + 1) + 1] = (int)full_pos;
    }
    *total_hf = (int)hf_pos;
    *total_full = (int)full_pos;
    return ngt;
}

/* bench_kv_cache_zipserv_decompress_token_scaling.cu:2106-2218. Decode using
 * only the per-GT offsets (each GT's streams are contiguous). The exponent of a
 * high-frequency element is (start_exp + code) mod 256, as in that CPU decoder.
 * Returns 0 on success, -1 if a stream index would leave the given arrays. */
int oracle_decode(const uint8_t* sign_mantissa, int64_t n_sm,
                  const uint16_t* full, int64_t n_full,
                  const uint64_t* bitmap1, const uint64_t* bitmap2, const uint64_t* bitmap3,
                  const int* gt_offsets, int start_exp, int M, int K, uint16_t* out) {
    const int gtk = K / GT_COLS, ngt = (M / GT_ROWS) * gtk;
    for (int g = 0; g < ngt; ++g) {
        const int r0 = (g / gtk) * GT_ROWS, c0 = (g % gtk) * GT_COLS;
        int64_t h = gt_offsets[2 * g], f = gt_offsets[2 * g + 1];
        for (int s = 0; s < ST_PER_GT; ++s) {
            int ro, co;
            st_origin(s, &ro, &co);
            int st = g * ST_PER_GT + s;
            uint64_t b1 = bitmap1[st], b2 = bitmap2[st], b3 = bitmap3[st];
            uint64_t ind = b1 | b2 | b3;
            for (int p = 0; p < 64; ++p) {
                uint16_t v;
                if ((ind >> p) & 1) {
                    if (h < 0 || h >= n_sm) return -1;
                    uint8_t sm = sign_mantissa[h++];
                    int c = (int)(((b3 >> p) & 1) << 2 | ((b2 >> p) & 1) << 1 | ((b1 >> p) & 1));
                    uint8_t e = (uint8_t)(start_exp + c);
                    v = (uint16_t)(((sm & 0x80) << 8) | ((uint16_t)e << 7) | (sm & 0x7F));
                } else {
                    if (f < 0 || f >= n_full) return -1;
                    v = full[f++];
                }
                out[(int64_t)(r0 + ro + p / 8) * K + c0 + co + p % 8] = v;
            }
        }
    }
    return 0;
}

static double bf16_to_double(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return (double)f;
}

/* Reference GEMM contract (csrc/L_API.cu:119 BF16TripleBitmap_MM_API as used
 * by test_mm.cu:410-428): W is M x K row-major (dense, already decoded), X is
 * N x K row-major (token-major), C is written column-major M x N, i.e.
 * C[n*M + m] = sum_k W[m][k] * X[n][k], accumulated in double. */
void oracle_gemm(const uint16_t* w, const uint16_t* x, int M, int N, int K, double* c) {
    double* xr = (double*)malloc(sizeof(double) * (size_t)K);
    double* wr = (double*)malloc(sizeof(double) * (size_t)K * 64);
    for (int m0 = 0; m0 < M; m0 += 64) {
        int mb = M - m0 < 64 ? M - m0 : 64;
        for (int i = 0; i < mb; ++i)
            for (int k = 0; k < K; ++k) wr[(size_t)i * K + k] = bf16_to_double(w[(size_t)(m0 + i) * K + k]);
        for (int n = 0; n < N; ++n) {
            for (int k = 0; k < K; ++k) xr[k] = bf16_to_double(x[(size_t)n * K + k]);
            for (int i = 0; i < mb; ++i) {
                double acc = 0.0;
                const double* wp = wr + (size_t)i * K;
                for (int k = 0; k < K; ++k) acc += wp[k] * xr[k];
                c[(size_t)n * M + m0 + i] = acc;
            }
        }
    }
    free(xr);
    free(wr);
}
