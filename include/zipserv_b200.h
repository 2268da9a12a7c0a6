/* Plain C ABI of libzipserv_b200.so (ctypes / cffi / cgo friendly).
 *
 * Every function returns a cudaError_t value as int (0 = success). Pointers
 * named d_* are device pointers; `stream` is a cudaStream_t (NULL = legacy
 * default stream). Nothing here synchronises the host or allocates device
 * memory; buffers are the caller's. Each
 * entry point cites the reference interface it replaces
 * (paths inside the reference project).
 */
#ifndef ZIPSERV_B200_H
#define ZIPSERV_B200_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Library version: major*10000 + minor*100 + patch. */
int zs_version(void);

/* Host exponent-window analysis.
 * Replaces kernel_benchmark/utils.h:189 analyzeExponentDistribution_BF16 (rule 0)
 * and the selection rule of kernel_benchmark/zipserv_decode_attention_ext.cu:65-133 (rule 1). */
int zs_analyze_exponents_host(const uint16_t* a, int64_t numel, int rule, int* top7);

/* Host encoder (multi-threaded), byte-identical to csrc/L_API.cu:559
 * InitBF16MatrixTripleBitmap_Reuse. Sizes: sm >= M*K + 16*#GT bytes,
 * full >= M*K + 8*#GT elements, bitmaps #ST = M*K/64 each, st_counts 2*#ST,
 * mt_off 2*#MT (#MT = M*K/1024), gt_off 2*(#GT+1); scalars4 receives
 * {max_hf, max_full, total_hf, total_full}. Temp memory is allocated on the host.
 * Returns 0, or cudaErrorInvalidValue / cudaErrorMemoryAllocation. */
int zs_encode_host(const uint16_t* a, int M, int K, const int* top7, uint8_t* sm, uint16_t* full,
                   uint64_t* b1, uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off,
                   int* scalars4);

/* Device scratch needed by zs_analyze_exponents (bytes). */
size_t zs_analyze_scratch_bytes(void);

/* GPU exponent-window analysis; writes 7 ints to d_top7 (stream ordered).
 * Replaces kernel_benchmark/zipserv_decode_attention_ext.cu:137 AnalyzeTopExponentsGPU
 * (rule 1) and gives the host rule of kernel_benchmark/utils.h:189 on the GPU (rule 0).
 * d_in must be 16-byte aligned. */
int zs_analyze_exponents(void* stream, const uint16_t* d_in, int64_t numel, int rule, void* d_scratch,
                         int* d_top7);

/* Device scratch needed by zs_encode for an M x K matrix (bytes). */
size_t zs_encode_scratch_bytes(int M, int K);

/* GPU encoder, byte-identical to the reference host encoder given the same top7.
 * Replaces csrc/L_API.cu:1355 InitBF16MatrixTripleBitmap_GPU. Output sizes as in
 * zs_encode_host; d_scalars4 (device) receives {max_hf, max_full, total_hf, total_full}. */
int zs_encode(void* stream, const uint16_t* d_in, int M, int K, const int* d_top7, uint8_t* d_sm,
              uint16_t* d_full, uint64_t* d_b1, uint64_t* d_b2, uint64_t* d_b3, int* d_st_counts,
              int* d_mt_off, int* d_gt_off, void* d_scratch, int* d_scalars4);

/* Dense decode, row-major M x K bf16 output.
 * Replaces csrc/L_API.cu:234 BF16TripleBitmap_Decompress_API. d_err (nullable)
 * receives error bits (1 = a wait timed out, 2 = an offset was out of range). */
int zs_decompress(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
                  const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off, const int* d_gt_off,
                  int max_hf, int max_full, int start_exp, uint16_t* d_out, int M, int K,
                  unsigned* d_err);

/* ZipGEMM: d_c[n*M + m] = sum_k W[m][k] * d_x[n*K + k] (bf16 in/out, fp32 accumulate).
 * Replaces csrc/L_API.cu:119 BF16TripleBitmap_MM_API. The K split is chosen by
 * the library: the K blocks of each 128-row output tile are split over the CTAs
 * of a thread-block cluster and the fp32 partial tiles are summed in-kernel
 * through distributed shared memory, in a fixed order (deterministic results,
 * no bf16 rounding of partials). split_k must be >= 1 and is otherwise
 * ignored. No device memory is allocated and nothing is synchronised, so calls
 * may be captured in CUDA graphs (the first call on a device sets kernel
 * attributes; make it outside capture). d_x must be 16-byte aligned, d_c
 * 8-byte aligned. */
int zs_zipgemm(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
               const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off, const int* d_gt_off,
               int max_hf, int max_full, int start_exp, const uint16_t* d_x, uint16_t* d_c, int M, int N,
               int K, int split_k, unsigned* d_err);

/* Row-parallel ZipGEMM with the all-reduce of its output fused into the
 * kernel's epilogue. New relative to the reference, which has no collectives;
 * it replaces zs_zipgemm followed by an NCCL all-reduce of d_c when W is split
 * by K over `world` GPUs (a tensor-parallel O or down projection).
 *
 * Every rank calls it with its own compressed K shard of W (M x K), its K
 * slice of X (N x K) and the same M and N; on return d_c holds, on every rank,
 * bf16(sum over ranks j in order 0..world-1 of bf16(W_j X_j^T)), bit-identical
 * across ranks. Words cross NVLink as 8-byte (two bf16 values, the call's
 * flag) pairs in 16-byte stores, and a CTA polls (bounded, about 2 s; then
 * error bit 1 in *d_err) its own buffer until the words it needs carry the
 * flag. With 2 ranks each CTA stores its rows into the peer's buffer and sums
 * both; from 3 ranks on, output tile t (128 rows) is summed by rank t % world,
 * which receives the other ranks' rows of it and stores the final rows back
 * into theirs (environment ZS_ALLREDUCE_SCHEME=all2all|owner overrides the
 * choice; every rank must see the same value).
 *
 * peer_bufs: host array of `world` device pointers: rank j's exchange buffer
 * of zs_zipgemm_allreduce_buffer_bytes(M, N, world) bytes, zeroed, opened on
 * this GPU (zs_peer_alloc on its owner, zs_peer_open here; own buffer at
 * [rank]), 256-byte aligned. d_epoch: this rank's zs_zipgemm_allreduce_counters
 * (M, N) unsigned counters (exchanges completed per tile), zeroed once, kept
 * between calls. All ranks must
 * issue the same sequence of calls with the same M, N. The grid must be
 * resident in one wave (it waits on the peers' CTAs of the same tile):
 * cudaErrorInvalidValue when M / 128 tiles exceed the co-resident clusters,
 * or when K < 128. world: 2..8. */
size_t zs_zipgemm_allreduce_buffer_bytes(int M, int N, int world);
size_t zs_zipgemm_allreduce_counters(int M, int N);
int zs_zipgemm_allreduce(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
                         const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off, const int* d_gt_off,
                         int max_hf, int max_full, int start_exp, const uint16_t* d_x, uint16_t* d_c, int M, int N,
                         int K, int world, int rank, void* const* peer_bufs, unsigned* d_epoch, unsigned* d_err);

/* Exchange buffers shared between the GPUs of one node (CUDA IPC). New
 * relative to the reference. zs_peer_alloc: cudaMalloc `bytes` on the current
 * device, zero them, and write the IPC handle (zs_peer_handle_bytes() bytes)
 * that other processes pass to zs_peer_open; free with zs_peer_free.
 * zs_peer_open maps a peer's buffer into this process (close with
 * zs_peer_close). */
size_t zs_peer_handle_bytes(void);
int zs_peer_alloc(size_t bytes, void** d_ptr, void* ipc_handle);
int zs_peer_open(const void* ipc_handle, void** d_ptr);
int zs_peer_close(void* d_ptr);
int zs_peer_free(void* d_ptr);

/* The split-KV factor zs_decode_attention picks when num_splits <= 0, for B
 * sequences of Hkv KV heads and up to max_seqlen tokens (a grid that fills the
 * SMs in few, full waves). New relative to the reference, whose FlashAttention
 * picks its own splits internally (FA flash_api.cpp num_splits_heuristic). */
int zs_decode_attention_default_splits(int B, int Hkv, int max_seqlen);

/* Workspace (device bytes) needed by zs_decode_attention for a split count
 * (0 when num_splits <= 1). */
size_t zs_decode_attention_workspace_bytes(int B, int Hq, int Hkv, int num_splits);

/* Compressed-KV decode attention, one query token per sequence:
 *   out[b][h] = softmax(q[b][h] . K[b][h/G]^T * softmax_scale) . V[b][h/G],  G = Hq / Hkv,
 * over the first d_seqlens[b] tokens. K and V are TCA-TBE compressed matrices
 * of B*Hkv*T_pad rows x D columns in head-major order (row (b*Hkv + h)*T_pad + t,
 * T_pad % 64 == 0, D == 128). k_ptrs / v_ptrs: host arrays of the 7 device
 * stream pointers {sign_mantissa, compressed_full, bitmap1, bitmap2, bitmap3,
 * tile_offsets_median, tile_offsets_global}; k_meta / v_meta: host arrays
 * {rows, cols, max_high_freq_count, max_full_count, start_exp}. q and out are
 * [B][Hq][D] bf16. max_seqlen bounds d_seqlens (host value). num_splits <= 0
 * picks the split-KV factor automatically; for more than one split d_ws must
 * hold zs_decode_attention_workspace_bytes(...) bytes. *splits_used (nullable)
 * receives the split count. Replaces the ZipServ decode path of FlashAttention
 * (FA csrc/flash_attn/flash_api.cpp:1346 mha_fwd_kvcache with zipserv_k/_v,
 * FA flash_attn/flash_attn_interface.py:1592 flash_attn_with_kvcache). */
int zs_decode_attention(void* stream, const uint16_t* d_q, const void* const* k_ptrs, const int* k_meta,
                        const void* const* v_ptrs, const int* v_meta, const int* d_seqlens, int B, int Hq, int Hkv,
                        int D, int T_pad, int max_seqlen, float softmax_scale, int num_splits, float* d_ws,
                        size_t ws_bytes, uint16_t* d_out, int* splits_used, unsigned* d_err);

/* Decode attention over an uncompressed, token-major K/V cache: d_k, d_v are
 * [B][T_rows][Hkv][D] bf16 (T_rows % 64 == 0, D == 128), 16-byte aligned;
 * everything else as zs_decode_attention (same kernel, every page read
 * dense). Serves the reference's token-major compressed layout (FA
 * flash_api.cpp:1512-1520, layout id 1) after zs_decompress has expanded it:
 * a token-major compressed matrix of B*T_rows*Hkv rows x D columns decodes to
 * exactly this [B][T_rows][Hkv][D] cache. */
int zs_decode_attention_dense(void* stream, const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                              const int* d_seqlens, int B, int Hq, int Hkv, int D, int T_rows, int max_seqlen,
                              float softmax_scale, int num_splits, float* d_ws, size_t ws_bytes, uint16_t* d_out,
                              int* splits_used, unsigned* d_err);

/* Allocation-free decode attention (no counterpart in the reference).
 * For callers that cannot allocate device memory when they run attention
 * (code running inside an allocator's own hooks, or deployments that forbid
 * cudaMalloc after start-up to keep a fixed memory budget): same inputs,
 * outputs and results as zs_decode_attention, but the split-KV workspace is a
 * fixed device array inside the library (2 MiB per GPU, held until exit), so
 * the caller passes no workspace and nothing is allocated. Returns
 * cudaErrorInvalidValue when B * Hq * splits * (D + 2) * 4 bytes exceeds
 * zs_decode_attention_noalloc_max_workspace_bytes(). The first call on a
 * device looks up the array's address on that device (and looks it up again
 * after the device's context changes, e.g. after cudaDeviceReset); make that
 * first call outside any stream capture. All calls share the array: calls that overlap on
 * the GPU (unordered streams) race; order them on one stream. */
size_t zs_decode_attention_noalloc_max_workspace_bytes(void);
int zs_decode_attention_noalloc(void* stream, const uint16_t* d_q, const void* const* k_ptrs, const int* k_meta,
                                const void* const* v_ptrs, const int* v_meta, const int* d_seqlens, int B, int Hq,
                                int Hkv, int D, int T_pad, int max_seqlen, float softmax_scale, int num_splits,
                                uint16_t* d_out, int* splits_used, unsigned* d_err);

/* ---- Paged compressed KV cache with online page append --------------------
 * The reference compresses a whole KV cache at once in its head-major layout
 * (kernel_benchmark/bench_zipserv_decode_attention.py:347-354) and, for online
 * compression, re-runs the matrix encoder pipeline
 * (bench_kv_cache_zipserv_compress_token_scaling.cu:1606-1647). Here a pool
 * holds fixed-window compressed pages of 64 tokens x 128 dims of one KV head
 * (two GTs each) at physical page slots P = block * Hkv + head; the streams of
 * each page are appended to shared stream pools at positions taken from a
 * device cursor, and page_off records them. All pointers are device memory. */
typedef struct ZsKvPool {
    uint8_t* d_sm;                 /* sign/mantissa stream pool, hf_capacity bytes, 16-byte aligned */
    uint16_t* d_full;              /* fallback stream pool, full_capacity elements, 16-byte aligned */
    uint64_t* d_b1, *d_b2, *d_b3;  /* [num_pages * 2 * 64] bitmaps */
    int* d_mt_off;                 /* [num_pages * 2 * 8] median-tile offsets */
    int* d_page_off;               /* [num_pages * 6]: {hf, fallback} starts of GT 0, GT 1 and the end */
    unsigned long long* d_cursor;  /* [4] (start at 0): next free hf byte, next free fallback element, and the
                                      largest padded hf / fallback length of a GT appended so far */
    int64_t hf_capacity, full_capacity;
    int num_pages;                 /* num_blocks * Hkv */
    int start_exp;                 /* (top[0] - 1) mod 256 of the window below */
    const int* d_top7;             /* the pool's fixed exponent window */
} ZsKvPool;

/* Compress whole pages of new tokens into the pool. d_x is token-major
 * [B][64 * npg][Hkv][D] bf16 (D = 128); page (b, j, h) goes to physical page
 * d_dst_pages[(b * npg + j) * Hkv + h] (negative: skipped). Encoding is
 * byte-identical to zs_encode of the 64 x 128 page with the pool's window.
 * A page that does not fit in the stream pools sets bit 2 in *d_err. */
int zs_kv_append_pages(void* stream, const ZsKvPool* pool, const uint16_t* d_x, int B, int npg, int Hkv, int D,
                       const int* d_dst_pages, unsigned* d_err);

/* Decode attention over paged compressed K/V (same outputs and workspace rules
 * as zs_decode_attention). Logical page g of sequence b is block
 * d_block_table[b * max_blocks + g]; d_seqlens[b] is the sequence length. When
 * d_tail_k / d_tail_v ([B][64][Hkv][D] bf16) are given, a sequence whose length
 * is not a multiple of 64 ends with a dense page read from them (its first
 * len % 64 tokens); otherwise every page must be in the pools. */
int zs_decode_attention_paged(void* stream, const uint16_t* d_q, const ZsKvPool* k, const ZsKvPool* v,
                              const int* d_block_table, int max_blocks, const int* d_seqlens, const uint16_t* d_tail_k,
                              const uint16_t* d_tail_v, int B, int Hq, int Hkv, int D, int max_seqlen,
                              float softmax_scale, int num_splits, float* d_ws, size_t ws_bytes, uint16_t* d_out,
                              int* splits_used, unsigned* d_err);

/* ---- On-disk TCA-TBE container (file format version 1) -------------------
 * No counterpart in the reference, which keeps no serialised compressed form
 * (its benchmarks re-encode the dense checkpoint at start-up,
 * kernel_benchmark/bench_zipserv_gemm_sweep.cu:290-345). The file holds the
 * arrays the encoders produce (csrc/L_API.cu:559-771 layout) with a CRC-32 per
 * array; all buffers here are HOST memory. Errors: 301 (cudaErrorFileNotFound)
 * when the file cannot be opened, 999 (cudaErrorUnknown) on a short read or
 * write, 1 (cudaErrorInvalidValue) for bad arguments, a foreign or damaged
 * file (magic, version, sizes, checksum). */
typedef struct ZsTcatbeInfo {
    int64_t rows, cols;
    int32_t start_exp, max_hf, max_full;
    int32_t top[7];
    int64_t total_hf, total_full;   /* valid lengths of the two streams */
    int32_t has_st_counts;          /* 1 when the small-tile counts are stored */
} ZsTcatbeInfo;

/* Write one compressed matrix. Array lengths follow from info: sm total_hf
 * bytes, full total_full elements, bitmaps rows*cols/64 words each, st_counts
 * 2*#ST ints (only when info->has_st_counts), mt_off 2*#MT, gt_off 2*(#GT+1). */
int zs_tcatbe_save(const char* path, const ZsTcatbeInfo* info, const uint8_t* sm, const uint16_t* full,
                   const uint64_t* b1, const uint64_t* b2, const uint64_t* b3, const int* st_counts,
                   const int* mt_off, const int* gt_off);
/* Read the header (sizes and scalars) so the caller can size its buffers. */
int zs_tcatbe_read_info(const char* path, ZsTcatbeInfo* info);
/* Read every array into caller buffers sized from zs_tcatbe_read_info and
 * verify the checksums; st_counts may be NULL to skip them. */
int zs_tcatbe_load(const char* path, ZsTcatbeInfo* info, uint8_t* sm, uint16_t* full, uint64_t* b1,
                   uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off);

#ifdef __cplusplus
}
#endif
#endif
