// Shared device/host helpers for the B200 (sm_100a) ZipServ kernels:
// TCA-TBE format constants, mbarrier / bulk-copy / TMA / tcgen05 PTX wrappers
// with bounded waits, and the branch-free small-tile row decoder.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace zs {

// ---------------------------------------------------------------------------
// Format constants (csrc/L_API.cu:559-771 tiling: 8x8 small tile (ST),
// 16x64 median tile (MT), 64x64 global tile (GT)).
// ---------------------------------------------------------------------------
constexpr int kGT = 64;            // global tile edge
constexpr int kSTPerGT = 64;       // small tiles per global tile
constexpr int kMTPerGT = 4;        // median tiles per global tile
constexpr int kSTPerMT = 16;       // small tiles per median tile
constexpr int kHfPad = 16;         // per-GT sign/mantissa stream padding (bytes)
constexpr int kFullPad = 8;        // per-GT fallback stream padding (elements)

// Error codes written to the optional device error word by bounded waits.
constexpr unsigned kErrWaitTimeout = 1u;
constexpr unsigned kErrStreamOverflow = 2u;

// Upper bound on any single mbarrier wait: 2 s of wall time measured with
// %globaltimer. Real waits in these kernels last microseconds.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
constexpr long long kWaitLimitCycles = 4000000000ll;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------- mbarrier -----------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

// Arrive `count` times at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

// One potentially blocking test of an mbarrier phase. The suspend-time hint
// lets the hardware park the waiting thread until the phase completes (or
// about 0.1 ms pass), so waiting warps take no issue slots from the warps
// that share their scheduler.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records kErrWaitTimeout
// in *err when err != nullptr) if the phase did not complete within the limit.
// `abort_flag` (shared memory) lets one thread's timeout stop the others early.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned* err,
                                          volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    // Deadline on the SM cycle counter (cheap to read, unlike %globaltimer):
    // kWaitLimitCycles is ~2 s at B200 clocks.
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
#ifdef ZS_SPIN_SLEEP
        __nanosleep(ZS_SPIN_SLEEP);
#endif
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63) == 63) {
            if (abort_flag && *abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                if (err) atomicOr(err, kErrWaitTimeout);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// Bounded wait for warps that wait often and long (decoders waiting for data):
// between polls the warp sleeps, so it does not take issue slots from the
// producer and MMA warps that share its scheduler.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, unsigned* err,
                                                volatile int* abort_flag, uint32_t sleep_ns = 128) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        __nanosleep(sleep_ns);
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15) == 15) {
            if (abort_flag && *abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                if (err) atomicOr(err, kErrWaitTimeout);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// Non-blocking test of an mbarrier phase.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for two mbarrier phases. Both are tested back to back first, so when
// both are already complete (the common case in a full pipeline) the two
// round trips to the barrier unit overlap; otherwise each is waited for in turn.
__device__ __forceinline__ bool mbar_wait2(uint64_t* b1, uint32_t p1, uint64_t* b2, uint32_t p2, unsigned* err,
                                           volatile int* abort_flag, bool sleep = false) {
    const bool r1 = mbar_test(b1, p1);
    const bool r2 = mbar_test(b2, p2);
    if (r1 && r2) return true;
    if (sleep)
        return (r1 || mbar_wait_sleep(b1, p1, err, abort_flag)) && (r2 || mbar_wait_sleep(b2, p2, err, abort_flag));
    return (r1 || mbar_wait(b1, p1, err, abort_flag)) && (r2 || mbar_wait(b2, p2, err, abort_flag));
}

// ------------------- programmatic dependent launch -------------------------
// Wait until the preceding grid on the stream (launched before this one) has
// completed and its memory operations are visible. A no-op without PDL.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Allow the next grid on the stream to start launching its CTAs.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------- bulk copies (TMA engine) ------------------------
// 1-D bulk copy global -> shared (this CTA), completion counted on `bar`.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst_smem, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled TMA load (no multicast), coordinates {c0 (innermost), c1}.
__device__ __forceinline__ void tma_load_2d(void* dst_smem, const CUtensorMap* map, int c0, int c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst_smem)),
        "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// 8-byte asynchronous global -> shared copy (no register staging); complete with
// cp_async_wait_all() in the issuing thread.
__device__ __forceinline__ void cp_async8(void* dst_smem, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// CTA-scope release store / acquire load of a shared int.
__device__ __forceinline__ void st_release_cta(int* a, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(a)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta(const int* a) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(a)) : "memory");
    return v;
}
// Bounded wait until a shared counter reaches `want` (same error / abort contract as mbar_wait).
__device__ __forceinline__ bool wait_tag_at_least(const int* tag, int want, unsigned* err, volatile int* abort_flag) {
    if (ld_acquire_cta(tag) >= want) return true;
    const long long t0 = clock64();
    for (uint32_t it = 0;; ++it) {
        __nanosleep(64);
        if (ld_acquire_cta(tag) >= want) return true;
        if ((it & 15) == 15) {
            if (abort_flag && *abort_flag) return false;
            if (clock64() - t0 > kWaitLimitCycles) {
                if (err) atomicOr(err, kErrWaitTimeout);
                if (abort_flag) *abort_flag = 1;
                return false;
            }
        }
    }
}

// Named CTA barriers (id 1..15; id 0 is __syncthreads). `count` counts threads
// and must be a multiple of 32; arrive does not wait (release), sync waits
// (acquire) for `count` arrivals in total.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int count) {
    asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// a / b for non-negative a, b: 32-bit division when a fits in 32 bits (the
// common case; 64-bit division is a long instruction sequence).
__host__ __device__ __forceinline__ long long div_nonneg(long long a, long long b) {
    if (((unsigned long long)a >> 32) == 0 && ((unsigned long long)b >> 32) == 0)
        return (long long)((unsigned)a / (unsigned)b);
    return a / b;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------- cluster -----------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %cluster_ctarank;" : "=r"(r));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
}

__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t cta) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(cta));
    return r;
}

// Bulk copy from this CTA's shared memory into a peer CTA's shared memory
// (both 32-bit shared::cluster addresses from mapa_shared for the peer side);
// completion is counted on the peer's mbarrier.
__device__ __forceinline__ void bulk_s2peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                            uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst_cluster),
        "r"(src_cta), "r"(bytes), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the source buffers of all committed bulk copies have been read.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ float4 ld_dsmem_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// ------------------------------- tcgen05 -----------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 in, fp32 acc).
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16. A (M=128 x K=16 bf16) is in
// TMEM: row m in lane m, K packed two bf16 per 32-bit column (8 columns).
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// This warp's 32 lanes each write 4 consecutive 32-bit columns of their own
// TMEM lane (lane quarter = warp % 4).
__device__ __forceinline__ void tmem_st4(uint32_t taddr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(a), "r"(b),
                 "r"(c), "r"(d)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// Arrive on `bar` once all previously issued tcgen05.mma of this thread finish.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory matrix descriptor for a K-major tile stored in the
// canonical 128-byte-swizzle layout: rows of 128 bytes (64 bf16), 8-row groups
// 1024 bytes apart, 16-byte chunk c of row r stored at chunk (c ^ (r & 7)).
// Tile base must be 1024-byte aligned. (Bit layout: start>>4 [0,14),
// LBO>>4 [16,30), SBO>>4 [32,46), version 1 at [46,48), layout 2 = 128B
// swizzle at [61,64).)
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;                 // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;       // SBO
    d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                 // 128-byte swizzle
    return d;
}

// Instruction descriptor: kind::f16, A = B = bf16, D = f32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Branch-free TCA-TBE row decode.
//
// One call decodes one row (8 consecutive elements along K) of one 8x8 small
// tile. Inputs are that row's bytes of the three code bitmaps (bit j = column
// j), the stream offsets of the row's first high-frequency byte and first
// fallback element, and two 8-byte exponent tables:
//   thb[c] = ((start_exp + c) mod 256) >> 1        (bf16 high byte, minus sign)
//   tlb[c] = ((start_exp + c) & 1) << 7            (bf16 low byte exponent bit)
// The result is four 32-bit words = 8 bf16 in column order, i.e. exactly the
// 16 bytes of the row segment.
//
// Work per row: the code nibbles X (nibble j = code of column j) are built from
// the three bitmap bytes with byte permutes of a constant (decode_row_words);
// the prefix-popcount selector for the packed sign/mantissa bytes is
// spread(indicator) * 0x11111110; everything else is byte permutes (prmt) and
// 3-input logic ops.
// ---------------------------------------------------------------------------
struct DecodeTables {
    uint32_t thb0, thb1, tlb0, tlb1;
};

__host__ __device__ inline DecodeTables make_decode_tables(int start_exp) {
    DecodeTables t;
    uint32_t hb[2] = {0, 0}, lb[2] = {0, 0};
    for (int c = 0; c < 8; ++c) {
        uint32_t e = (uint32_t)(start_exp + c) & 0xFFu;
        hb[c >> 2] |= (e >> 1) << (8 * (c & 3));
        lb[c >> 2] |= ((e & 1u) << 7) << (8 * (c & 3));
    }
    t.thb0 = hb[0]; t.thb1 = hb[1]; t.tlb0 = lb[0]; t.tlb1 = lb[1];
    return t;
}

// Shared-memory accesses on 32-bit shared addresses. The loads carry no memory
// clobber, so the compiler may overlap them with the stores of earlier rows;
// callers pass addresses derived through launder() after the barrier that
// makes the data valid (launder is volatile, so it cannot move above the wait,
// and every load depends on it).
__device__ __forceinline__ uint32_t launder(uint32_t a) {
    uint32_t r;
    asm volatile("mov.b32 %0, %1;" : "=r"(r) : "r"(a));
    return r;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
    uint2 v;
    asm("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}
__device__ __forceinline__ void sts16(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)v) : "memory");
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t s) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(s));
    return d;
}

// Bytes c & 3 .. (c & 3) + 3 of the 8-byte value {b, a} (a low): a funnel
// shift right by 8 (c & 3) bits that takes the byte offset itself.
__device__ __forceinline__ uint32_t prmt_f4e(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("prmt.b32.f4e %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ uint32_t lop_or_and(uint32_t a, uint32_t mask, uint32_t b) {
    return (a & mask) | b;  // compiles to a single LOP3
}

// Bit groups of the three bitmap words of a small tile's row half (w1, w2, w3:
// rows 4h .. 4h+3, one byte per row): for each bitmap, a holds groups 0 and 1
// (bits 0-1 and 2-3) of row r's byte as the two nibbles of byte r, and b
// groups 2 and 3 (bits 4-5 and 6-7). Five logic/shift ops per bitmap serve
// all four rows.
struct RowGroups {
    uint32_t a1, b1, a2, b2, a3, b3;
};
__device__ __forceinline__ void bit_groups(uint32_t w, uint32_t& a, uint32_t& b) {
    a = (w & 0x03030303u) | ((w << 2) & 0x30303030u);
    b = ((w >> 4) & 0x03030303u) | ((w >> 2) & 0x30303030u);
}
__device__ __forceinline__ RowGroups row_groups(uint32_t w1, uint32_t w2, uint32_t w3) {
    RowGroups g;
    bit_groups(w1, g.a1, g.b1);
    bit_groups(w2, g.a2, g.b2);
    bit_groups(w3, g.a3, g.b3);
    return g;
}

// Decode the high-frequency elements of one small-tile row (8 elements), row r
// (0..3) of the row half whose bit groups are g; fallback positions (code 0)
// receive junk that the caller patches. The spread of a bitmap byte c (nibble
// j = bit j) has byte k = {0x00, 0x01, 0x10, 0x11}[(c >> 2k) & 3], so one
// byte permute of the constant 0x11100100 produces it from a selector whose
// nibble k is bit group k of c; a second byte permute gathers that selector
// (bytes r of a and b) from the row half's bit groups.
__device__ __forceinline__ void decode_row_words(const RowGroups& g, uint32_t r, uint32_t win, const DecodeTables& t,
                                                 uint32_t (&o)[4]) {
    constexpr uint32_t kSpreadBytes = 0x11100100u;
    const uint32_t gsel = r | ((4u + r) << 4);
    const uint32_t s1 = prmt(kSpreadBytes, 0, prmt(g.a1, g.b1, gsel)),
                   s2 = prmt(kSpreadBytes, 0, prmt(g.a2, g.b2, gsel)),
                   s3 = prmt(kSpreadBytes, 0, prmt(g.a3, g.b3, gsel));
    const uint32_t X = s1 + (s2 << 1) + (s3 << 2);        // code nibbles
    const uint32_t sel = (s1 | s2 | s3) * 0x11111110u;    // hf-before-j nibbles
    const uint32_t wa = win & ~3u;
    const uint32_t q0 = lds32(wa), q1 = lds32(wa + 4), q2 = lds32(wa + 8);
    const uint32_t lo = prmt_f4e(q0, q1, win);   // the 8 bytes from `win` on
    const uint32_t hi = prmt_f4e(q1, q2, win);
    const uint32_t s_lo = prmt(lo, hi, sel);
    const uint32_t s_hi = prmt(lo, hi, sel >> 16);
    const uint32_t hb_lo = lop_or_and(s_lo, 0x80808080u, prmt(t.thb0, t.thb1, X));
    const uint32_t hb_hi = lop_or_and(s_hi, 0x80808080u, prmt(t.thb0, t.thb1, X >> 16));
    const uint32_t lb_lo = lop_or_and(s_lo, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X));
    const uint32_t lb_hi = lop_or_and(s_hi, 0x7F7F7F7Fu, prmt(t.tlb0, t.tlb1, X >> 16));
    o[0] = prmt(lb_lo, hb_lo, 0x5140);
    o[1] = prmt(lb_lo, hb_lo, 0x7362);
    o[2] = prmt(lb_hi, hb_hi, 0x5140);
    o[3] = prmt(lb_hi, hb_hi, 0x7362);
}

}  // namespace zs

// Host-side error helper: turn a CUDA error into a return code.
#define ZS_RETURN_IF_ERR(expr)                      \
    do {                                            \
        cudaError_t _e = (expr);                    \
        if (_e != cudaSuccess) return _e;           \
    } while (0)
