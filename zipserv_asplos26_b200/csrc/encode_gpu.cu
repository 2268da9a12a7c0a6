// GPU TCA-TBE encoder, byte-identical to the reference host encoder
// (csrc/L_API.cu:559 InitBF16MatrixTripleBitmap_Reuse), and the exponent-window
// analysis (kernel_benchmark/utils.h:189 host rule; kernel_benchmark/
// zipserv_decode_attention_ext.cu:35 extension rule).
//
// Pipeline (all stream-ordered, no host synchronisation, no spin-waits):
//   analyze_kernel  exponent histogram (warp-private shared bins, 16-byte
//                   loads); the last CTA to finish (atomic ticket) picks the
//                   7-exponent window, its 256 threads ranking one exponent each.
//   count_kernel    one CTA per 64x64 GT: padded hf / fallback counts.
//   scan_kernel     one CTA: exclusive prefix of the per-GT counts
//                   (TileOffsets_Global), maxima and totals.
//   encode_kernel   one CTA per GT: bitmaps, per-ST counts, median offsets,
//                   and both streams compacted in shared memory and written to
//                   their final position with aligned 16-byte stores.
// Unlike the reference GPU path (L_API.cu:1114-1348) there is no per-GT
// temporary stream copy and no serial <<<1,1>>> prefix.
#include "common.cuh"
#include "zs_internal.h"

namespace zs {

// ------------------------------ window selection ---------------------------
// Window rule from the 7 picked exponents (sorted here): the first start in the
// picks whose 7 consecutive exponents all occur, else the longest run of
// consecutive picks (kernel_benchmark/utils.h:240-272; the extension rule of
// zipserv_decode_attention_ext.cu:100-133 also clamps the start to [0, 248]).
// cnt: the 256-bin histogram. The host rule pads missing picks with 127 - np.
__device__ void window_from_picks(const unsigned long long* cnt, int* picks, int np, int rule, int* top) {
    while (np < 7) { picks[np] = 127 - np; ++np; }
    for (int i = 1; i < 7; ++i) {
        int v = picks[i], j = i - 1;
        while (j >= 0 && picks[j] > v) { picks[j + 1] = picks[j]; --j; }
        picks[j + 1] = v;
    }
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
            ++cur;
            if (cur > best_len) { best_len = cur; best_start = picks[i] - cur + 1; }
        } else {
            cur = 1;
        }
    }
    if (rule == kRuleExt) best_start = min(max(best_start, 0), 248);
    for (int i = 0; i < 7; ++i) top[i] = best_start + i;
}

// The 7 picks of both rules. Host rule (utils.h:189-239): 7 arg-max passes
// with a strict '>' from zero, i.e. the first 7 exponents in the order (count
// descending, exponent ascending) among those that occur; every one of the 256
// threads ranks its own exponent in that order at once. Extension rule
// (zipserv_decode_attention_ext.cu:65-99): a replace-the-minimum top 7 seeded
// with -1 that replaces the lowest-index slot holding the minimum on a strictly
// larger count. Which tied minimum it drops depends on the slot history, so it
// is run as written, by one thread, with the seven slots in registers.
// cnt: the histogram in shared memory; all kAnalyzeThreads (= 256) threads call.
__device__ void select_window_parallel(const unsigned long long* cnt, int rule, int* top, unsigned* masks) {
    const int e = threadIdx.x;
    if (rule == kRuleHost) {
        const unsigned long long c = cnt[e];
        int rank = 0;
        for (int f = 0; f < 256; ++f) {
            const unsigned long long d = cnt[f];
            rank += (d > c || (d == c && f < e)) ? 1 : 0;
        }
        const unsigned m = __ballot_sync(0xFFFFFFFFu, rank < 7 && c > 0);
        if ((e & 31) == 0) masks[e >> 5] = m;
    }
    __syncthreads();
    if (e == 0) {
        int picks[7], np = 0;
        if (rule == kRuleHost) {
            for (int w = 0; w < 8; ++w)
                for (unsigned mm = masks[w]; mm && np < 7; mm &= mm - 1) picks[np++] = 32 * w + __ffs(mm) - 1;
        } else {
            int te[7];
            long long tc[7];
#pragma unroll
            for (int i = 0; i < 7; ++i) { te[i] = -1; tc[i] = -1; }
            for (int f = 0; f < 256; ++f) {
                const long long c = (long long)cnt[f];
                int mi = 0;
                long long mv = tc[0];
#pragma unroll
                for (int i = 1; i < 7; ++i)
                    if (tc[i] < mv) { mv = tc[i]; mi = i; }
                if (c > mv) {
#pragma unroll
                    for (int i = 0; i < 7; ++i)
                        if (i == mi) { tc[i] = c; te[i] = f; }
                }
            }
#pragma unroll
            for (int i = 0; i < 7; ++i)
                if (te[i] >= 0) picks[np++] = te[i];
        }
        window_from_picks(cnt, picks, np, rule, top);
    }
}

constexpr int kAnalyzeThreads = 256;

__global__ void __launch_bounds__(kAnalyzeThreads) analyze_kernel(const uint16_t* __restrict__ in, long long numel,
                                                                  int rule, unsigned long long* counts,
                                                                  unsigned* ticket, int* top) {
    __shared__ unsigned bins[kAnalyzeThreads / 32][256];
    __shared__ bool last;
    const int tid = threadIdx.x, warp = tid >> 5;
    for (int i = tid; i < (kAnalyzeThreads / 32) * 256; i += kAnalyzeThreads) (&bins[0][0])[i] = 0;
    __syncthreads();
    const long long nvec = numel >> 3;
    const uint4* v4 = reinterpret_cast<const uint4*>(in);
    for (long long i = (long long)blockIdx.x * kAnalyzeThreads + tid; i < nvec;
         i += (long long)gridDim.x * kAnalyzeThreads) {
        const uint4 v = __ldcs(v4 + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            atomicAdd(&bins[warp][(w[k] >> 7) & 0xFF], 1u);
            atomicAdd(&bins[warp][(w[k] >> 23) & 0xFF], 1u);
        }
    }
    if (blockIdx.x == 0)
        for (long long i = (nvec << 3) + tid; i < numel; i += kAnalyzeThreads)
            atomicAdd(&bins[warp][(in[i] >> 7) & 0xFF], 1u);
    __syncthreads();
    for (int e = tid; e < 256; e += kAnalyzeThreads) {
        unsigned long long s = 0;
        for (int w = 0; w < kAnalyzeThreads / 32; ++w) s += bins[w][e];
        if (s) atomicAdd(counts + e, s);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last = (atomicAdd(ticket, 1u) == gridDim.x - 1);
    __syncthreads();
    if (last) {   // CTA-uniform: the last CTA to finish picks the window from the full histogram
        __shared__ unsigned long long hist[256];
        __shared__ unsigned masks[8];
        __threadfence();
        hist[tid] = *((volatile unsigned long long*)counts + tid);
        __syncthreads();
        select_window_parallel(hist, rule, top, masks);
    }
}

cudaError_t launch_analyze(cudaStream_t s, const uint16_t* in, long long numel, int rule, void* scratch,
                           int* d_top) {
    if (!in || !scratch || !d_top || numel <= 0 || (rule != kRuleHost && rule != kRuleExt))
        return cudaErrorInvalidValue;
    if (!aligned16(in) || !aligned16(scratch)) return cudaErrorInvalidValue;
    ZS_RETURN_IF_ERR(cudaMemsetAsync(scratch, 0, kAnalyzeScratchBytes, s));
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    long long want = ((numel >> 3) + kAnalyzeThreads - 1) / kAnalyzeThreads;
    int grid = (int)std::max(1ll, std::min(want, (long long)sms * 4));
    unsigned long long* counts = reinterpret_cast<unsigned long long*>(scratch);
    unsigned* ticket = reinterpret_cast<unsigned*>(counts + 256);
    analyze_kernel<<<grid, kAnalyzeThreads, 0, s>>>(in, numel, rule, counts, ticket, d_top);
    return cudaGetLastError();
}

// --------------------------------- encoder ---------------------------------
// code_of[e] = index of exponent e in the top list + 1 (0 = fallback). A later
// duplicate wins, as in the reference's exp_to_idx table (L_API.cu:618-621).
__device__ __forceinline__ void build_code_lut(uint8_t* lut, const int* top) {
    for (int e = threadIdx.x; e < 256; e += blockDim.x) lut[e] = 0;
    __syncthreads();
    if (threadIdx.x == 0)
        for (int i = 0; i < 7; ++i) {
            const int e = top[i];
            if (e >= 0 && e <= 255) lut[e] = (uint8_t)(i + 1);
        }
    __syncthreads();
}

// Row-task mapping inside a GT (128 threads): thread t owns row m = t & 63 and
// column blocks kc = 4*(t>>6) .. +3; each row-task is 8 elements (16 bytes).
__global__ void __launch_bounds__(128) count_kernel(const uint16_t* __restrict__ in, int K, const int* top,
                                                     int* gt_hf_cnt, int* gt_full_cnt) {
    __shared__ uint8_t lut[256];
    __shared__ int part[4];
    build_code_lut(lut, top);
    const int gtk = K >> 6;
    const long long gt = blockIdx.x;
    const long long r0 = (gt / gtk) * 64, c0 = (gt % gtk) * 64;
    const int t = threadIdx.x, m = t & 63, kc0 = 4 * (t >> 6);
    int hf = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint4 v = *reinterpret_cast<const uint4*>(in + (r0 + m) * K + c0 + (kc0 + i) * 8);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int k = 0; k < 4; ++k)
            hf += (lut[(w[k] >> 7) & 0xFF] != 0) + (lut[(w[k] >> 23) & 0xFF] != 0);
    }
    for (int o = 16; o; o >>= 1) hf += __shfl_xor_sync(0xFFFFFFFFu, hf, o);
    if ((t & 31) == 0) part[t >> 5] = hf;
    __syncthreads();
    if (t == 0) {
        const int h = part[0] + part[1] + part[2] + part[3];
        const int f = 4096 - h;
        gt_hf_cnt[gt] = (h + 15) & ~15;
        gt_full_cnt[gt] = (f + 7) & ~7;
    }
}

// Single-CTA exclusive scan of per-GT (hf, fallback) counts.
constexpr int kScanThreads = 1024;
constexpr int kScanItems = 4;

__global__ void __launch_bounds__(kScanThreads) scan_kernel(const int* gt_hf_cnt, const int* gt_full_cnt,
                                                             long long ngt, int* gt_off, int* hf_prefix,
                                                             int* full_prefix, int* d_max_hf, int* d_max_full,
                                                             int* d_total_hf, int* d_total_full) {
    __shared__ long long wsum_h[32], wsum_f[32];
    __shared__ long long carry_h, carry_f;
    __shared__ int mx_h[32], mx_f[32];
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    if (t == 0) { carry_h = 0; carry_f = 0; }
    int my_mh = 0, my_mf = 0;
    __syncthreads();
    for (long long base = 0; base < ngt; base += (long long)kScanThreads * kScanItems) {
        int vh[kScanItems], vf[kScanItems];
        long long sh = 0, sf = 0;
#pragma unroll
        for (int i = 0; i < kScanItems; ++i) {
            const long long idx = base + (long long)t * kScanItems + i;
            vh[i] = idx < ngt ? gt_hf_cnt[idx] : 0;
            vf[i] = idx < ngt ? gt_full_cnt[idx] : 0;
            my_mh = max(my_mh, vh[i]);
            my_mf = max(my_mf, vf[i]);
            sh += vh[i];
            sf += vf[i];
        }
        long long ih = sh, iff = sf;  // inclusive warp scan
        for (int o = 1; o < 32; o <<= 1) {
            const long long a = __shfl_up_sync(0xFFFFFFFFu, ih, o), b = __shfl_up_sync(0xFFFFFFFFu, iff, o);
            if (lane >= o) { ih += a; iff += b; }
        }
        if (lane == 31) { wsum_h[warp] = ih; wsum_f[warp] = iff; }
        __syncthreads();
        if (warp == 0) {
            long long a = wsum_h[lane], b = wsum_f[lane];
            for (int o = 1; o < 32; o <<= 1) {
                const long long x = __shfl_up_sync(0xFFFFFFFFu, a, o), y = __shfl_up_sync(0xFFFFFFFFu, b, o);
                if (lane >= o) { a += x; b += y; }
            }
            wsum_h[lane] = a;
            wsum_f[lane] = b;
        }
        __syncthreads();
        long long eh = carry_h + (warp ? wsum_h[warp - 1] : 0) + ih - sh;
        long long ef = carry_f + (warp ? wsum_f[warp - 1] : 0) + iff - sf;
#pragma unroll
        for (int i = 0; i < kScanItems; ++i) {
            const long long idx = base + (long long)t * kScanItems + i;
            if (idx < ngt) {
                if (idx == 0) {
                    gt_off[0] = 0; gt_off[1] = 0;
                    if (hf_prefix) hf_prefix[0] = 0;
                    if (full_prefix) full_prefix[0] = 0;
                }
                eh += vh[i];
                ef += vf[i];
                gt_off[2 * (idx + 1)] = (int)eh;
                gt_off[2 * (idx + 1) + 1] = (int)ef;
                if (hf_prefix) hf_prefix[idx + 1] = (int)eh;
                if (full_prefix) full_prefix[idx + 1] = (int)ef;
            }
        }
        __syncthreads();
        if (t == kScanThreads - 1) { carry_h += wsum_h[31]; carry_f += wsum_f[31]; }
        __syncthreads();
    }
    for (int o = 16; o; o >>= 1) {
        my_mh = max(my_mh, __shfl_xor_sync(0xFFFFFFFFu, my_mh, o));
        my_mf = max(my_mf, __shfl_xor_sync(0xFFFFFFFFu, my_mf, o));
    }
    if (lane == 0) { mx_h[warp] = my_mh; mx_f[warp] = my_mf; }
    __syncthreads();
    if (t == 0) {
        int a = 0, b = 0;
        for (int w = 0; w < 32; ++w) { a = max(a, mx_h[w]); b = max(b, mx_f[w]); }
        if (d_max_hf) *d_max_hf = a;
        if (d_max_full) *d_max_full = b;
        if (d_total_hf) *d_total_hf = (int)carry_h;
        if (d_total_full) *d_total_full = (int)carry_f;
    }
}

// Shared-memory state of one GT being encoded by a group of 128 threads.
struct GtEncodeSmem {
    __align__(16) uint8_t bmp[3][512];   // bitmap bytes: [plane][st*8 + r]
    int cnt[513];                        // per row-task exclusive hf prefix, stream order; [512] = total
    int wsum[4];
    __align__(16) uint8_t sbuf[4096 + 16];    // compacted hf bytes (zero padded to 16)
    __align__(16) uint16_t fbuf[4096 + 8];    // compacted fallbacks (zero padded to 8)
};

// Encode one 64x64 GT whose element (m, c) is at src[m * ld + c] into `S`
// (bitmaps, prefix counts, compacted streams), with the 128 threads t of one
// group synchronising on named barrier `bar` (a 128-thread CTA passes 0).
// Row-task mapping: thread t owns row m = t & 63 and column blocks
// kc = 4*(t>>6) .. +3; each row-task is 8 elements (16 bytes). Returns the
// unpadded hf count (the fallback count is 4096 minus it).
__device__ int encode_gt_core(const uint16_t* __restrict__ src, long long ld, const uint8_t* lut, GtEncodeSmem& S,
                              int t, int bar) {
    const int m = t & 63, kc0 = 4 * (t >> 6);
    const int w = m >> 4, mr = (m >> 3) & 1, r = m & 7;
    uint4 rows[4];
    uint32_t codes[4];  // per row-task: 8 codes as nibbles
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int kc = kc0 + i;
        rows[i] = *reinterpret_cast<const uint4*>(src + (long long)m * ld + kc * 8);
        const uint32_t wv[4] = {rows[i].x, rows[i].y, rows[i].z, rows[i].w};
        uint32_t p1 = 0, p2 = 0, p3 = 0, nib = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t v = (wv[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
            const uint32_t c = lut[(v >> 7) & 0xFF];
            p1 |= (c & 1u) << j;
            p2 |= ((c >> 1) & 1u) << j;
            p3 |= ((c >> 2) & 1u) << j;
            nib |= c << (4 * j);
        }
        codes[i] = nib;
        const int st = w * 16 + 2 * kc + mr;
        S.bmp[0][st * 8 + r] = (uint8_t)p1;
        S.bmp[1][st * 8 + r] = (uint8_t)p2;
        S.bmp[2][st * 8 + r] = (uint8_t)p3;
        S.cnt[st * 8 + r] = __popc(p1 | p2 | p3);
    }
    named_bar_sync(bar, 128);
    // exclusive scan of cnt[0..511] (thread t owns entries 4t..4t+3)
    int v0 = S.cnt[4 * t], v1 = S.cnt[4 * t + 1], v2 = S.cnt[4 * t + 2], v3 = S.cnt[4 * t + 3];
    int s = v0 + v1 + v2 + v3, inc = s;
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xFFFFFFFFu, inc, o);
        if ((t & 31) >= o) inc += a;
    }
    if ((t & 31) == 31) S.wsum[t >> 5] = inc;
    named_bar_sync(bar, 128);
    int wbase = 0;
    for (int i = 0; i < (t >> 5); ++i) wbase += S.wsum[i];
    const int total_hf = S.wsum[0] + S.wsum[1] + S.wsum[2] + S.wsum[3];
    named_bar_sync(bar, 128);
    int e = wbase + inc - s;
    S.cnt[4 * t] = e; e += v0;
    S.cnt[4 * t + 1] = e; e += v1;
    S.cnt[4 * t + 2] = e; e += v2;
    S.cnt[4 * t + 3] = e;
    if (t == 0) S.cnt[512] = total_hf;
    named_bar_sync(bar, 128);
    // scatter into the compaction buffers
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int kc = kc0 + i;
        const int idx = (w * 16 + 2 * kc + mr) * 8 + r;
        int hp = S.cnt[idx];
        int fp = idx * 8 - hp;
        const uint32_t wv[4] = {rows[i].x, rows[i].y, rows[i].z, rows[i].w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t v = (wv[j >> 1] >> (16 * (j & 1))) & 0xFFFFu;
            if ((codes[i] >> (4 * j)) & 7u) {
                S.sbuf[hp++] = (uint8_t)(((v >> 8) & 0x80u) | (v & 0x7Fu));
            } else {
                S.fbuf[fp++] = (uint16_t)v;
            }
        }
    }
    const int total_full = 4096 - total_hf;
    const int pad_hf = (total_hf + 15) & ~15, pad_full = (total_full + 7) & ~7;
    if (t < pad_hf - total_hf) S.sbuf[total_hf + t] = 0;
    if (t < pad_full - total_full) S.fbuf[total_full + t] = 0;
    named_bar_sync(bar, 128);
    return total_hf;
}

// Write the encoded GT's bitmaps (GT slot g of the bitmap arrays), median
// offsets, optional small-tile counts, and both padded streams at (h0, f0).
__device__ void write_gt(const GtEncodeSmem& S, int t, long long g, int total_hf, uint8_t* __restrict__ sm,
                         uint16_t* __restrict__ full, long long h0, long long f0, uint64_t* __restrict__ b1,
                         uint64_t* __restrict__ b2, uint64_t* __restrict__ b3, int* __restrict__ st_counts,
                         int* __restrict__ mt_off) {
    if (t < 64) {
        if (st_counts) {
            const int a = S.cnt[t * 8], b = S.cnt[t * 8 + 8];
            st_counts[2 * (g * 64 + t)] = b - a;
            st_counts[2 * (g * 64 + t) + 1] = 64 - (b - a);
        }
    } else if (t < 68) {
        const int q = t - 64;
        mt_off[2 * (g * 4 + q)] = S.cnt[q * 128];
        mt_off[2 * (g * 4 + q) + 1] = q * 1024 - S.cnt[q * 128];
    }
    {
        const int plane = t >> 6, st = t & 63;  // threads 0..127 cover planes 0, 1; plane 2 below
        const uint64_t* bsrc = reinterpret_cast<const uint64_t*>(&S.bmp[0][0]);
        uint64_t* dst = plane == 0 ? b1 : b2;
        dst[g * 64 + st] = bsrc[plane * 64 + st];
        if (t < 64) b3[g * 64 + t] = bsrc[128 + t];
    }
    const int pad_hf = (total_hf + 15) & ~15, pad_full = (4096 - total_hf + 7) & ~7;
    for (int i = t; i < pad_hf / 16; i += 128)
        *reinterpret_cast<uint4*>(sm + h0 + 16 * i) = reinterpret_cast<const uint4*>(S.sbuf)[i];
    for (int i = t; i < pad_full / 8; i += 128)
        *reinterpret_cast<uint4*>(full + f0 + 8 * i) = reinterpret_cast<const uint4*>(S.fbuf)[i];
}

__global__ void __launch_bounds__(128) encode_kernel(const uint16_t* __restrict__ in, int K, const int* top,
                                                      const int* __restrict__ gt_off, uint8_t* __restrict__ sm,
                                                      uint16_t* __restrict__ full, uint64_t* __restrict__ b1,
                                                      uint64_t* __restrict__ b2, uint64_t* __restrict__ b3,
                                                      int* __restrict__ st_counts, int* __restrict__ mt_off) {
    __shared__ uint8_t lut[256];
    __shared__ GtEncodeSmem S;
    build_code_lut(lut, top);
    const int gtk = K >> 6;
    const long long gt = blockIdx.x;
    const long long r0 = (gt / gtk) * 64, c0 = (gt % gtk) * 64;
    const int t = threadIdx.x;
    const int total_hf = encode_gt_core(in + r0 * K + c0, K, lut, S, t, 0);
    write_gt(S, t, gt, total_hf, sm, full, gt_off[2 * gt], gt_off[2 * gt + 1], b1, b2, b3, st_counts, mt_off);
}

// Online KV page append (no counterpart kernel in the reference, whose KV
// benchmarks compress a whole cache at once with the matrix encoder,
// kernel_benchmark/bench_kv_cache_zipserv_compress_token_scaling.cu:1606-1647).
// One CTA per page of 64 tokens x 128 dims of one KV head: x holds B sequences
// of npg pages each, token-major [B][64 npg][Hkv][128]; page (b, j, h) is
// encoded with the pool's fixed exponent window into physical page
// P = dst_pages[(b * npg + j) * Hkv + h] (negative: skipped). Its two GTs go to
// bitmap / median-offset slots 2P and 2P+1; its streams are appended to the
// pools at positions taken from the pool cursors (one atomic per stream and
// page, so the two GTs' streams are contiguous) and recorded in
// page_off[6P .. 6P+5] = {hf, fallback} starts of GT 0 and GT 1, and the end;
// cursor[2], cursor[3] keep the largest padded hf and fallback length of a GT.
// A page that does not fit in the pools sets kErrStreamOverflow and records
// an empty page.
__global__ void __launch_bounds__(256) kv_append_kernel(const uint16_t* __restrict__ x, int Hkv,
                                                         const int* __restrict__ dst_pages, int num_pages,
                                                         const int* top, uint8_t* __restrict__ sm,
                                                         uint16_t* __restrict__ full, uint64_t* __restrict__ b1,
                                                         uint64_t* __restrict__ b2, uint64_t* __restrict__ b3,
                                                         int* __restrict__ mt_off, int* __restrict__ page_off,
                                                         unsigned long long* cursor, long long hf_cap,
                                                         long long full_cap, unsigned* err) {
    __shared__ uint8_t lut[256];
    __shared__ GtEncodeSmem S[2];
    __shared__ long long base[2];
    const long long i = blockIdx.x;
    const int P = dst_pages[i];
    if (P < 0) return;
    if (P >= num_pages) {
        if (threadIdx.x == 0 && err) atomicOr(err, kErrStreamOverflow);
        return;
    }
    build_code_lut(lut, top);
    constexpr long long D = 128;
    const long long h = i % Hkv, bj = i / Hkv;   // bj = b * npg + j
    const uint16_t* src = x + (bj * 64 * Hkv + h) * D;
    const int t = threadIdx.x & 127, g = threadIdx.x >> 7;
    const int hf = encode_gt_core(src + 64 * g, (long long)Hkv * D, lut, S[g], t, 1 + g);
    __syncthreads();
    const int hf0 = S[0].cnt[512], hf1 = S[1].cnt[512];
    const long long ph0 = (hf0 + 15) & ~15, ph1 = (hf1 + 15) & ~15;
    const long long pf0 = (4096 - hf0 + 7) & ~7, pf1 = (4096 - hf1 + 7) & ~7;
    if (threadIdx.x == 0) {
        const long long hb = (long long)atomicAdd(&cursor[0], (unsigned long long)(ph0 + ph1));
        const long long fb = (long long)atomicAdd(&cursor[1], (unsigned long long)(pf0 + pf1));
        const bool ok = hb + ph0 + ph1 <= hf_cap && fb + pf0 + pf1 <= full_cap && hb + ph0 + ph1 <= 0x7FFFFFFFll &&
                        fb + pf0 + pf1 <= 0x7FFFFFFFll;
        int* po = page_off + 6LL * P;
        // running maxima of a GT's padded stream lengths (decode attention sizes its slots from them)
        atomicMax(&cursor[2], (unsigned long long)max(ph0, ph1));
        atomicMax(&cursor[3], (unsigned long long)max(pf0, pf1));
        if (ok) {
            base[0] = hb;
            base[1] = fb;
            po[0] = (int)hb; po[1] = (int)fb;
            po[2] = (int)(hb + ph0); po[3] = (int)(fb + pf0);
            po[4] = (int)(hb + ph0 + ph1); po[5] = (int)(fb + pf0 + pf1);
        } else {
            base[0] = -1;
            for (int k = 0; k < 6; ++k) po[k] = 0;
            if (err) atomicOr(err, kErrStreamOverflow);
        }
    }
    __syncthreads();
    if (base[0] < 0) return;
    write_gt(S[g], t, 2LL * P + g, hf, sm, full, base[0] + (g ? ph0 : 0), base[1] + (g ? pf0 : 0), b1, b2, b3,
             nullptr, mt_off);
}

cudaError_t launch_kv_append(cudaStream_t s, const uint16_t* x, int B, int npg, int Hkv, int D,
                             const int* dst_pages, int num_pages, const int* d_top, uint8_t* sm, uint16_t* full,
                             uint64_t* b1, uint64_t* b2, uint64_t* b3, int* mt_off, int* page_off,
                             unsigned long long* cursor, long long hf_cap, long long full_cap, unsigned* err) {
    if (B < 0 || npg < 0 || Hkv <= 0 || D != 128 || num_pages <= 0) return cudaErrorInvalidValue;
    const long long n = (long long)B * npg * Hkv;
    if (n == 0) return cudaSuccess;
    if (n > 0x7FFFFFFFll) return cudaErrorInvalidValue;
    if (!x || !dst_pages || !d_top || !sm || !full || !b1 || !b2 || !b3 || !mt_off || !page_off || !cursor)
        return cudaErrorInvalidValue;
    if (!aligned16(x) || !aligned16(sm) || !aligned16(full) || hf_cap < 0 || full_cap < 0)
        return cudaErrorInvalidValue;
    kv_append_kernel<<<(unsigned)n, 256, 0, s>>>(x, Hkv, dst_pages, num_pages, d_top, sm, full, b1, b2, b3, mt_off,
                                                 page_off, cursor, hf_cap, full_cap, err);
    return cudaGetLastError();
}

cudaError_t launch_encode(cudaStream_t s, const uint16_t* in, int M, int K, const int* d_top, uint8_t* sm,
                          uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3, int* st_counts,
                          int* mt_off, int* gt_off, int* gt_hf_cnt, int* gt_full_cnt, int* hf_prefix,
                          int* full_prefix, int* d_max_hf, int* d_max_full, int* d_total_hf, int* d_total_full) {
    if (M <= 0 || K <= 0 || (M % 64) || (K % 64)) return cudaErrorInvalidValue;
    if (!in || !d_top || !sm || !full || !b1 || !b2 || !b3 || !st_counts || !mt_off || !gt_off || !gt_hf_cnt ||
        !gt_full_cnt)
        return cudaErrorInvalidValue;
    if (!aligned16(in) || !aligned16(sm) || !aligned16(full)) return cudaErrorInvalidValue;
    const long long ngt = (long long)(M / 64) * (K / 64);
    if (ngt > 0x7FFFFFFFll) return cudaErrorInvalidValue;
    count_kernel<<<(unsigned)ngt, 128, 0, s>>>(in, K, d_top, gt_hf_cnt, gt_full_cnt);
    ZS_RETURN_IF_ERR(cudaGetLastError());
    scan_kernel<<<1, kScanThreads, 0, s>>>(gt_hf_cnt, gt_full_cnt, ngt, gt_off, hf_prefix, full_prefix, d_max_hf,
                                           d_max_full, d_total_hf, d_total_full);
    ZS_RETURN_IF_ERR(cudaGetLastError());
    encode_kernel<<<(unsigned)ngt, 128, 0, s>>>(in, K, d_top, gt_off, sm, full, b1, b2, b3, st_counts, mt_off);
    return cudaGetLastError();
}

}  // namespace zs
