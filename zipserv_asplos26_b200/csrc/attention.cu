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
// (b, kv head) and the G = Hq / Hkv query heads that share it:
//   warp 8      producer: bulk-copies chunks of consecutive pages (K and V
//               streams are contiguous in GT order, one copy per stream)
//   warps 0..3  decode K (lane = token, 64 dims each) and form the fp32 dot
//               products with the G query heads
//   warps 4..7  decode V into a shared bf16 tile
//   then an online base-2 softmax (warp h = query head h) and an fp32 P.V
//   accumulation (thread = pair of dims x token quarter).
// With S > 1 every CTA writes (m, l, unnormalised O) to a caller-provided fp32
// workspace and combine_kernel merges the splits; with S = 1 the CTA writes
// the normalised bf16 output itself.
#include <algorithm>
#include <mutex>
#include <cmath>
#include <cstddef>

#include "common.cuh"
#include "tile_decode.cuh"
#include "zs_internal.h"

namespace zs {

constexpr int kAttnMaxG = 8;        // query heads per KV head
constexpr int kAttnD = 128;         // head dim (two 64-wide GTs)
constexpr int kAttnWarps = 9;
constexpr int kAttnThreads = 32 * kAttnWarps;
constexpr int kAttnProducer = 8;
constexpr int kAttnMaxChunk = 4;    // pages per compressed slot
constexpr int kAttnSlots = 3;

struct AttnStream {
    const uint8_t* sm;
    const uint16_t* full;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* mt_off;
    const int* gt_off;
    int max_hf, max_full, start_exp;
};

struct AttnParams {
    AttnStream k, v;
    const uint16_t* q;        // [B][Hq][D] bf16
    const int* seqlens;       // [B]
    uint16_t* out;            // [B][Hq][D] bf16
    float* ws;                // [B*Hkv][S][G][D + 2] fp32 when S > 1
    int B, Hq, Hkv, G, T_pad, S, pages_per_split, chunk;
    float scale_log2;         // softmax_scale * log2(e)
    // compressed slot layout (bytes), per stream (K at 0, V at c_stream)
    uint32_t c_stream, c_mt, c_hf, c_full, hf_cap, full_cap, c_slot;
    unsigned* err;
};

struct AttnSmem {
    uint64_t full[kAttnSlots], empty[kAttnSlots];
    int abort_flag;
    // per slot and stream: GT-local stream offsets of each GT of the chunk
    int hoff[kAttnSlots][2][2 * kAttnMaxChunk + 1];
    int foff[kAttnSlots][2][2 * kAttnMaxChunk + 1];
    __align__(16) float q[kAttnMaxG][kAttnD];   // query heads of this KV head, fp32 (read as float2)
    float sc[2][kAttnMaxG][64];            // partial scores from the two 64-dim halves
    float p[64][kAttnMaxG];                // softmax weights of the current page
    float alpha[kAttnMaxG];                // rescale of the running output
    __align__(16) uint16_t v[64][kAttnD + 8];   // decoded V page (+16 B row pad)
};

static_assert(offsetof(AttnSmem, q) % 16 == 0 && offsetof(AttnSmem, v) % 16 == 0, "vector-accessed members");

// Barrier over the 8 compute warps only (the producer warp never joins).
__device__ __forceinline__ void compute_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

// One producer step: copy `np` pages starting at page `pg` of row block `rb`
// (= (b * Hkv + h) * T_pad / 64) of one stream into the slot.
__device__ __forceinline__ uint32_t attn_issue_stream(const AttnStream& s, uint8_t* dst, long long gt0, int ngt,
                                                      int* hoff, int* foff, const AttnParams& p, uint64_t* bar,
                                                      bool issue) {
    const int2* go = reinterpret_cast<const int2*>(s.gt_off) + gt0;
    const int2 a0 = go[0];
    for (int i = 0; i <= ngt; ++i) {
        const int2 a = go[i];
        hoff[i] = a.x - a0.x;
        foff[i] = a.y - a0.y;
    }
    const int2 a1 = go[ngt];
    uint32_t hb = a1.x > a0.x ? (uint32_t)(a1.x - a0.x) : 0u;
    uint32_t fb = a1.y > a0.y ? (uint32_t)(a1.y - a0.y) * 2u : 0u;
    int h0 = a0.x, f0 = a0.y;
    if (hb > p.hf_cap || fb > p.full_cap || (hb & 15u) || (fb & 15u) || (h0 & 15) || (f0 & 7) || h0 < 0 || f0 < 0) {
        if (p.err) atomicOr(p.err, kErrStreamOverflow);
        hb = min(hb, p.hf_cap) & ~15u;
        fb = min(fb, p.full_cap) & ~15u;
        h0 = max(h0, 0) & ~15;
        f0 = max(f0, 0) & ~7;
    }
    const uint32_t bytes = (uint32_t)ngt * (3 * 512 + 32) + hb + fb;
    if (issue) {
        const uint32_t bmb = 512u * (uint32_t)ngt;
        bulk_g2s(dst, s.b1 + gt0 * 64, bmb, bar);
        bulk_g2s(dst + 512u * 2 * p.chunk, s.b2 + gt0 * 64, bmb, bar);
        bulk_g2s(dst + 1024u * 2 * p.chunk, s.b3 + gt0 * 64, bmb, bar);
        bulk_g2s(dst + p.c_mt, s.mt_off + gt0 * 8, 32u * (uint32_t)ngt, bar);
        if (hb) bulk_g2s(dst + p.c_hf, s.sm + h0, hb, bar);
        if (fb) bulk_g2s(dst + p.c_full, s.full + f0, fb, bar);
    }
    return bytes;
}

__global__ void __launch_bounds__(kAttnThreads, 1) attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    AttnSmem& A = *reinterpret_cast<AttnSmem*>(smem);
    uint32_t* lut = reinterpret_cast<uint32_t*>(smem + round_up_u32(sizeof(AttnSmem), 1024));
    uint8_t* slots = reinterpret_cast<uint8_t*>(lut + kLutWords);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int bh = blockIdx.x, split = blockIdx.y;
    const int b = bh / p.Hkv, hk = bh % p.Hkv;
    const int len = max(0, min(p.seqlens[b], p.T_pad));
    const int npages = (len + 63) >> 6;
    const int pg0 = split * p.pages_per_split;
    const int np = max(0, min(npages, pg0 + p.pages_per_split) - pg0);
    const int G = p.G;
    const long long rb = ((long long)bh * p.T_pad) >> 6;   // first GT row of this (b, kv head)

    fill_spread_table(lut, tid, kAttnThreads);
    for (int i = tid; i < G * kAttnD; i += kAttnThreads) {
        const int h = i / kAttnD, d = i % kAttnD;
        A.q[h][d] = __uint_as_float((uint32_t)p.q[((size_t)b * p.Hq + hk * G + h) * kAttnD + d] << 16);
    }
    if (tid == 0) {
        for (int s = 0; s < kAttnSlots; ++s) { mbar_init(&A.full[s], 1); mbar_init(&A.empty[s], 8); }
        A.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    volatile int* abort_flag = &A.abort_flag;
    const int nchunks = (np + p.chunk - 1) / p.chunk;

    // per-lane online-softmax state (warp h < G owns head h) and P.V accumulators
    float m_run = -INFINITY, l_run = 0.f;
    const int dp = tid & 63, tq = (tid >> 6) & 3;   // P.V: dims 2dp, 2dp+1; tokens 16tq..16tq+15
    float acc[kAttnMaxG][2];
#pragma unroll
    for (int h = 0; h < kAttnMaxG; ++h) acc[h][0] = acc[h][1] = 0.f;

    if (warp == kAttnProducer) {
        if (lane == 0) {
            for (int j = 0; j < nchunks; ++j) {
                const int s = j % kAttnSlots;
                if (j >= kAttnSlots && !mbar_wait(&A.empty[s], ((j / kAttnSlots) + 1) & 1, p.err, abort_flag)) break;
                const int pj = pg0 + j * p.chunk, cn = min(p.chunk, np - j * p.chunk);
                const long long gt0 = (rb + pj) * 2;
                uint8_t* slot = slots + (size_t)s * p.c_slot;
                uint32_t bytes = attn_issue_stream(p.k, slot, gt0, 2 * cn, A.hoff[s][0], A.foff[s][0], p, nullptr, false) +
                                 attn_issue_stream(p.v, slot + p.c_stream, gt0, 2 * cn, A.hoff[s][1], A.foff[s][1], p,
                                                   nullptr, false);
                mbar_arrive_expect_tx(&A.full[s], bytes);
                attn_issue_stream(p.k, slot, gt0, 2 * cn, A.hoff[s][0], A.foff[s][0], p, &A.full[s], true);
                attn_issue_stream(p.v, slot + p.c_stream, gt0, 2 * cn, A.hoff[s][1], A.foff[s][1], p, &A.full[s],
                                  true);
            }
        }
        // The producer takes no part in the compute-warp barriers below; its
        // copies complete on the slot barriers the compute warps wait on.
        return;
    }

    const DecodeTables tk = make_decode_tables(p.k.start_exp), tv = make_decode_tables(p.v.start_exp);
    const uint32_t lut_lane = launder(smem_u32(lut)) + 4u * (uint32_t)lane;
    for (int pi = 0; pi < np; ++pi) {
        const int j = pi / p.chunk, u = pi - j * p.chunk, s = j % kAttnSlots;
        const int tok0 = (pg0 + pi) * 64;
        const bool ok = mbar_wait(&A.full[s], (j / kAttnSlots) & 1, p.err, abort_flag);
        if (ok) {
            const int isv = warp >> 2, sub = (warp >> 1) & 1, half = warp & 1;
            const uint32_t base = launder(smem_u32(slots + (size_t)s * p.c_slot + isv * p.c_stream));
            const int gi = 2 * u + sub;
            GtView g;
            g.bm = base + 512u * (uint32_t)gi;
            g.bstride = 512u * 2u * (uint32_t)p.chunk;
            g.mt = base + p.c_mt + 32u * (uint32_t)gi;
            const uint32_t hl = (uint32_t)min(max(A.hoff[s][isv][gi], 0), (int)p.hf_cap);
            const uint32_t fl = (uint32_t)min(max(A.foff[s][isv][gi], 0) * 2, (int)p.full_cap);
            g.sm = base + p.c_hf + hl;
            g.full = base + p.c_full + fl;
            g.hf_cap = p.hf_cap - hl;
            g.full_cap = (p.full_cap - fl) / 2;
            const int t = 32 * half + lane;   // token within the page
            if (isv == 0) {
                float dot[kAttnMaxG];
#pragma unroll
                for (int h = 0; h < kAttnMaxG; ++h) dot[h] = 0.f;
                decode_gt_half_regs<8>(g, lut_lane, tk, half, 0,
                                       [&](int kc, uint32_t o0, uint32_t o1, uint32_t o2, uint32_t o3) {
                                           const uint32_t ow[4] = {o0, o1, o2, o3};
                                           const int d0 = sub * 64 + kc * 8;
#pragma unroll
                                           for (int e = 0; e < 4; ++e) {
                                               const float k0 = __uint_as_float(ow[e] << 16);
                                               const float k1 = __uint_as_float(ow[e] & 0xFFFF0000u);
#pragma unroll
                                               for (int h = 0; h < kAttnMaxG; ++h)
                                                   if (h < G) {
                                                       const float2 qq = *reinterpret_cast<const float2*>(
                                                           &A.q[h][d0 + 2 * e]);
                                                       dot[h] = fmaf(k0, qq.x, fmaf(k1, qq.y, dot[h]));
                                                   }
                                           }
                                       });
#pragma unroll
                for (int h = 0; h < kAttnMaxG; ++h)
                    if (h < G) A.sc[sub][h][t] = dot[h];
            } else {
                decode_gt_half_regs<8>(g, lut_lane, tv, half, 0,
                                       [&](int kc, uint32_t o0, uint32_t o1, uint32_t o2, uint32_t o3) {
                                           *reinterpret_cast<uint4*>(&A.v[t][sub * 64 + kc * 8]) =
                                               make_uint4(o0, o1, o2, o3);
                                       });
            }
        }
        compute_sync();
        // the slot holds a chunk of pages: release it after the chunk's last page
        if (lane == 0 && (u == p.chunk - 1 || pi == np - 1)) mbar_arrive(&A.empty[s]);
        // online softmax: warp h owns query head h, lanes own tokens lane, lane + 32
        if (warp < G) {
            const int h = warp;
            float s0 = (A.sc[0][h][lane] + A.sc[1][h][lane]) * p.scale_log2;
            float s1 = (A.sc[0][h][lane + 32] + A.sc[1][h][lane + 32]) * p.scale_log2;
            if (tok0 + lane >= len) s0 = -INFINITY;
            if (tok0 + lane + 32 >= len) s1 = -INFINITY;
            float mx = fmaxf(s0, s1);
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
            const float m_new = fmaxf(m_run, mx);
            const float e0 = exp2f(s0 - m_new), e1 = exp2f(s1 - m_new);
            float sum = e0 + e1;
            for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xFFFFFFFFu, sum, o);
            const float al = exp2f(m_run - m_new);   // 0 on the first page (m_run = -inf)
            l_run = l_run * al + sum;
            m_run = m_new;
            A.p[lane][h] = e0;
            A.p[lane + 32][h] = e1;
            if (lane == 0) A.alpha[h] = al;
        }
        compute_sync();
        {
#pragma unroll
            for (int h = 0; h < kAttnMaxG; ++h)
                if (h < G) {
                    const float al = A.alpha[h];
                    acc[h][0] *= al;
                    acc[h][1] *= al;
                }
#pragma unroll 4
            for (int tt = 0; tt < 16; ++tt) {
                const int t = tq * 16 + tt;
                const uint32_t vv = *reinterpret_cast<const uint32_t*>(&A.v[t][2 * dp]);
                const float v0 = __uint_as_float(vv << 16), v1 = __uint_as_float(vv & 0xFFFF0000u);
#pragma unroll
                for (int h = 0; h < kAttnMaxG; ++h)
                    if (h < G) {
                        const float pp = A.p[t][h];
                        acc[h][0] = fmaf(pp, v0, acc[h][0]);
                        acc[h][1] = fmaf(pp, v1, acc[h][1]);
                    }
            }
        }
        compute_sync();
    }

    // reduce the four token quarters; reuse the V tile as fp32 scratch [4][G][D]
    float* red = reinterpret_cast<float*>(&A.v[0][0]);
    if (tq > 0) {
#pragma unroll
        for (int h = 0; h < kAttnMaxG; ++h)
            if (h < G) {
                red[((tq - 1) * G + h) * kAttnD + 2 * dp] = acc[h][0];
                red[((tq - 1) * G + h) * kAttnD + 2 * dp + 1] = acc[h][1];
            }
    }
    if (warp < G && lane == 0) {
        A.alpha[warp] = m_run;      // reuse: running max and sum of head h
        A.sc[0][warp][0] = l_run;
    }
    compute_sync();
    if (tq == 0) {
        for (int h = 0; h < G; ++h) {
            float a0 = acc[h][0], a1 = acc[h][1];
            for (int k = 0; k < 3; ++k) {
                a0 += red[(k * G + h) * kAttnD + 2 * dp];
                a1 += red[(k * G + h) * kAttnD + 2 * dp + 1];
            }
            const float m = A.alpha[h], l = A.sc[0][h][0];
            const int hq = hk * G + h;
            if (p.S == 1) {
                const float inv = l > 0.f ? 1.f / l : 0.f;
                __nv_bfloat162 o = __floats2bfloat162_rn(a0 * inv, a1 * inv);
                *reinterpret_cast<__nv_bfloat162*>(&p.out[((size_t)b * p.Hq + hq) * kAttnD + 2 * dp]) = o;
            } else {
                float* w = p.ws + (((size_t)bh * p.S + split) * G + h) * (kAttnD + 2);
                w[2 * dp] = a0;
                w[2 * dp + 1] = a1;
                if (dp == 0) {
                    w[kAttnD] = m;
                    w[kAttnD + 1] = l;
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

static int attn_default_splits(int B, int Hkv, int max_pages) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int s = std::max(1, (2 * sms + B * Hkv - 1) / (B * Hkv));
    return std::min(s, std::max(1, max_pages));
}

cudaError_t launch_attention(cudaStream_t stream, const AttnCompressed& kc, const AttnCompressed& vc,
                             const uint16_t* q, const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D,
                             int T_pad, int max_seqlen, float softmax_scale, int num_splits, float* ws,
                             size_t ws_bytes, unsigned* err, int* splits_used) {
    if (B <= 0 || Hq <= 0 || Hkv <= 0 || Hq % Hkv || D != kAttnD || T_pad <= 0 || T_pad % 64)
        return cudaErrorInvalidValue;
    const int G = Hq / Hkv;
    if (G > kAttnMaxG) return cudaErrorInvalidValue;
    if (!q || !seqlens || !out || max_seqlen < 0 || max_seqlen > T_pad) return cudaErrorInvalidValue;
    const AttnCompressed* cs[2] = {&kc, &vc};
    for (const AttnCompressed* c : cs) {
        if (!c->b1 || !c->b2 || !c->b3 || !c->mt_off || !c->gt_off) return cudaErrorInvalidValue;
        if (c->rows != B * Hkv * T_pad || c->cols != D) return cudaErrorInvalidValue;
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
    p.q = q; p.seqlens = seqlens; p.out = out; p.ws = ws; p.err = err;
    p.B = B; p.Hq = Hq; p.Hkv = Hkv; p.G = G; p.T_pad = T_pad; p.S = S;
    p.pages_per_split = (max_pages + S - 1) / S;
    p.scale_log2 = softmax_scale * 1.4426950408889634f;
    const uint32_t hfc = round_up_u32((uint32_t)std::max(kc.max_hf, vc.max_hf), 16);
    const uint32_t ffc = round_up_u32((uint32_t)std::max(kc.max_full, vc.max_full) * 2u, 16);
    const uint32_t head = round_up_u32(sizeof(AttnSmem), 1024) + 4u * kLutWords;
    int dev = 0, max_smem = 232448;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    p.chunk = 1;
    for (int ch = kAttnMaxChunk; ch >= 1; --ch) {
        const uint32_t ngt = 2u * ch;
        const uint32_t stream = round_up_u32(ngt * (1536u + 32u) + ngt * hfc + 16 + ngt * ffc + 16, 128);
        if (head + kAttnSlots * 2 * stream <= (uint32_t)max_smem) { p.chunk = ch; break; }
    }
    {
        const uint32_t ngt = 2u * p.chunk;
        p.c_mt = 1536u * ngt;
        p.c_hf = p.c_mt + 32u * ngt;
        p.hf_cap = hfc * ngt;
        p.c_full = p.c_hf + p.hf_cap + 16;
        p.full_cap = ffc * ngt;
        p.c_stream = round_up_u32(p.c_full + p.full_cap + 16, 128);
        p.c_slot = 2 * p.c_stream;
    }
    const uint32_t smem_bytes = head + kAttnSlots * p.c_slot;
    if (smem_bytes > (uint32_t)max_smem) return cudaErrorInvalidValue;
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

// The array's device address for the current device, looked up once per
// device (cudaGetSymbolAddress with that device current). The first call on a
// device does this look-up; make that first call outside any stream capture.
static cudaError_t noalloc_ws_ptr(float** out) {
    static float* ptrs[64] = {};
    static std::mutex mu;
    int dev = 0;
    ZS_RETURN_IF_ERR(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> g(mu);
    if (!ptrs[dev]) {
        void* ptr = nullptr;
        ZS_RETURN_IF_ERR(cudaGetSymbolAddress(&ptr, g_attn_noalloc_ws));
        ptrs[dev] = static_cast<float*>(ptr);
    }
    *out = ptrs[dev];
    return cudaSuccess;
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
