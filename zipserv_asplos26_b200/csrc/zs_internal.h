// Internal launchers shared between the .cu translation units of the library.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace zs {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Exponent-window rules.
//   0 = host rule (kernel_benchmark/utils.h:189 analyzeExponentDistribution_BF16)
//   1 = torch-extension rule (kernel_benchmark/zipserv_decode_attention_ext.cu:35)
enum WindowRule : int { kRuleHost = 0, kRuleExt = 1 };

// Scratch for launch_analyze: 256 x u64 counters + 1 u32 ticket (2056 bytes).
constexpr size_t kAnalyzeScratchBytes = 256 * 8 + 8;

cudaError_t launch_analyze(cudaStream_t s, const uint16_t* in, long long numel, int rule, void* scratch,
                           int* d_top);

// Per-GT scratch for launch_encode: 4 x (#GT + 1) ints.
cudaError_t launch_encode(cudaStream_t s, const uint16_t* in, int M, int K, const int* d_top, uint8_t* sm,
                          uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3, int* st_counts,
                          int* mt_off, int* gt_off, int* gt_hf_cnt, int* gt_full_cnt, int* hf_prefix,
                          int* full_prefix, int* d_max_hf, int* d_max_full, int* d_total_hf, int* d_total_full);

// Online KV page append into a page pool (see kv_append_kernel).
cudaError_t launch_kv_append(cudaStream_t s, const uint16_t* x, int B, int npg, int Hkv, int D,
                             const int* dst_pages, int num_pages, const int* d_top, uint8_t* sm, uint16_t* full,
                             uint64_t* b1, uint64_t* b2, uint64_t* b3, int* mt_off, int* page_off,
                             unsigned long long* cursor, long long hf_cap, long long full_cap, unsigned* err);

cudaError_t launch_decompress(cudaStream_t s, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                              const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                              int max_hf, int max_full, int start_exp, uint16_t* out, int M, int K,
                              unsigned* err);

cudaError_t launch_zipgemm(cudaStream_t s, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                           const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                           int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M,
                           int N, int K, int split_k, unsigned* err);

// Row-parallel ZipGEMM with the all-reduce of C over `world` GPUs fused into
// its epilogue (see zs_zipgemm_allreduce).
struct PeerExchange {
    int world, rank;
    uint16_t* recv[8];
    unsigned* epoch;
};
size_t zipgemm_allreduce_counters(int M, int N);
size_t zipgemm_allreduce_buffer_bytes(int M, int N, int world);
cudaError_t launch_zipgemm_allreduce(cudaStream_t s, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                                     const uint64_t* b2, const uint64_t* b3, const int* mt_off, const int* gt_off,
                                     int max_hf, int max_full, int start_exp, const uint16_t* X, uint16_t* C, int M,
                                     int N, int K, int world, int rank, void* const* peer_bufs, unsigned* epoch,
                                     unsigned* err);

// One TCA-TBE compressed matrix (device pointers + scalars).
struct AttnCompressed {
    const uint8_t* sm;
    const uint16_t* full;
    const uint64_t* b1;
    const uint64_t* b2;
    const uint64_t* b3;
    const int* mt_off;
    const int* gt_off;
    int rows, cols, max_hf, max_full, start_exp;
};

size_t attn_workspace_bytes(int B, int Hq, int Hkv, int num_splits);
int attn_default_splits(int B, int Hkv, int max_pages);

cudaError_t launch_attention(cudaStream_t s, const AttnCompressed& k, const AttnCompressed& v, const uint16_t* q,
                             const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int T_pad,
                             int max_seqlen, float softmax_scale, int num_splits, float* ws, size_t ws_bytes,
                             unsigned* err, int* splits_used);

// Paged compressed KV (see attn_decode_kernel): physical page of logical page g
// of sequence b and KV head h is block_table[b * max_blocks + g] * Hkv + h;
// page_off holds per physical page {hf, fallback} starts of its two GTs and
// the end. tail_k / tail_v (nullable, [B][64][Hkv][D] bf16) hold each
// sequence's last, not yet compressed, page when its length is not a
// multiple of 64.
struct AttnPaged {
    const int* block_table;
    int max_blocks, num_blocks;
    const int* k_page_off;
    const int* v_page_off;
    const uint16_t* tail_k;
    const uint16_t* tail_v;
    // nullable: {max padded hf bytes, max padded fallback elements} of a GT in
    // each pool, kept by the append kernel; lets the kernel size its page slots
    const unsigned long long* k_max;
    const unsigned long long* v_max;
};

cudaError_t launch_attention_paged(cudaStream_t s, const AttnCompressed& k, const AttnCompressed& v,
                                   const AttnPaged& pg, const uint16_t* q, const int* seqlens, uint16_t* out, int B,
                                   int Hq, int Hkv, int D, int max_seqlen, float softmax_scale, int num_splits,
                                   float* ws, size_t ws_bytes, unsigned* err, int* splits_used);

// Decode attention over an uncompressed token-major cache ([B][T_rows][Hkv][D]
// bf16, T_rows % 64 == 0): the same kernel with every page read dense.
struct AttnDense {
    const uint16_t* k;
    const uint16_t* v;
};
cudaError_t launch_attention_dense(cudaStream_t s, const uint16_t* k, const uint16_t* v, const uint16_t* q,
                                   const int* seqlens, uint16_t* out, int B, int Hq, int Hkv, int D, int T_rows,
                                   int max_seqlen, float softmax_scale, int num_splits, float* ws, size_t ws_bytes,
                                   unsigned* err, int* splits_used);

size_t attn_noalloc_ws_bytes();
cudaError_t launch_attention_noalloc(cudaStream_t s, const AttnCompressed& k, const AttnCompressed& v,
                                     const uint16_t* q, const int* seqlens, uint16_t* out, int B, int Hq, int Hkv,
                                     int D, int T_pad, int max_seqlen, float softmax_scale, int num_splits,
                                     unsigned* err, int* splits_used);

}  // namespace zs
