// C ABI (include/zipserv_b200.h) and the reference's GPU C++ ABI
// (include/L_API.cuh, same mangled names as the reference build/L_API.cuh).
#include <cstring>
#include <cstdlib>
#include <new>
#include <vector>

#include "L_API.cuh"
#include "zipserv_b200.h"
#include "zs_host.h"
#include "zs_internal.h"

extern "C" int zs_version(void) { return 100; }

extern "C" int zs_analyze_exponents_host(const uint16_t* a, int64_t numel, int rule, int* top7) {
    if (!a || !top7 || numel <= 0 || (rule != 0 && rule != 1)) return cudaErrorInvalidValue;
    zs::analyze_host(a, numel, rule, top7);
    return cudaSuccess;
}

extern "C" int zs_encode_host(const uint16_t* a, int M, int K, const int* top7, uint8_t* sm, uint16_t* full,
                              uint64_t* b1, uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off,
                              int* scalars4) {
    if (!a || !top7 || !sm || !full || !b1 || !b2 || !b3 || !st_counts || !mt_off || !gt_off || !scalars4)
        return cudaErrorInvalidValue;
    if (M <= 0 || K <= 0 || (M % 64) || (K % 64)) return cudaErrorInvalidValue;
    const size_t ngt = (size_t)(M / 64) * (K / 64);
    uint8_t* tsm = (uint8_t*)malloc(ngt * (4096 + 15));
    uint16_t* tfu = (uint16_t*)malloc(ngt * (4096 + 7) * 2);
    std::vector<int> c1, c2, o1, o2;
    try {
        c1.resize(ngt + 1); c2.resize(ngt + 1); o1.resize(ngt + 1); o2.resize(ngt + 1);
    } catch (const std::bad_alloc&) {
        free(tsm); free(tfu);
        return cudaErrorMemoryAllocation;
    }
    if (!tsm || !tfu) { free(tsm); free(tfu); return cudaErrorMemoryAllocation; }
    int r = zs::encode_host(a, M, K, top7, sm, full, b1, b2, b3, st_counts, mt_off, gt_off, tsm, tfu, c1.data(),
                            c2.data(), o1.data(), o2.data(), &scalars4[0], &scalars4[1], &scalars4[2],
                            &scalars4[3]);
    free(tsm);
    free(tfu);
    return r < 0 ? cudaErrorInvalidValue : cudaSuccess;
}

extern "C" size_t zs_analyze_scratch_bytes(void) { return zs::kAnalyzeScratchBytes; }

extern "C" int zs_analyze_exponents(void* stream, const uint16_t* d_in, int64_t numel, int rule, void* d_scratch,
                                    int* d_top7) {
    return zs::launch_analyze((cudaStream_t)stream, d_in, numel, rule, d_scratch, d_top7);
}

extern "C" size_t zs_encode_scratch_bytes(int M, int K) {
    if (M <= 0 || K <= 0) return 0;
    const size_t ngt = (size_t)(M / 64) * (K / 64);
    return 4 * (ngt + 1) * sizeof(int) + 64;
}

extern "C" int zs_encode(void* stream, const uint16_t* d_in, int M, int K, const int* d_top7, uint8_t* d_sm,
                         uint16_t* d_full, uint64_t* d_b1, uint64_t* d_b2, uint64_t* d_b3, int* d_st_counts,
                         int* d_mt_off, int* d_gt_off, void* d_scratch, int* d_scalars4) {
    if (!d_scratch || !d_scalars4 || M <= 0 || K <= 0) return cudaErrorInvalidValue;
    const size_t ngt = (size_t)(M / 64) * (K / 64);
    int* s = reinterpret_cast<int*>(d_scratch);
    return zs::launch_encode((cudaStream_t)stream, d_in, M, K, d_top7, d_sm, d_full, d_b1, d_b2, d_b3,
                             d_st_counts, d_mt_off, d_gt_off, s, s + (ngt + 1), s + 2 * (ngt + 1),
                             s + 3 * (ngt + 1), d_scalars4, d_scalars4 + 1, d_scalars4 + 2, d_scalars4 + 3);
}

extern "C" int zs_decompress(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
                             const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off, const int* d_gt_off,
                             int max_hf, int max_full, int start_exp, uint16_t* d_out, int M, int K,
                             unsigned* d_err) {
    return zs::launch_decompress((cudaStream_t)stream, d_sm, d_full, d_b1, d_b2, d_b3, d_mt_off, d_gt_off, max_hf,
                                 max_full, start_exp, d_out, M, K, d_err);
}

extern "C" int zs_zipgemm(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
                          const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off, const int* d_gt_off,
                          int max_hf, int max_full, int start_exp, const uint16_t* d_x, uint16_t* d_c, int M,
                          int N, int K, int split_k, unsigned* d_err) {
    return zs::launch_zipgemm((cudaStream_t)stream, d_sm, d_full, d_b1, d_b2, d_b3, d_mt_off, d_gt_off, max_hf,
                              max_full, start_exp, d_x, d_c, M, N, K, split_k, d_err);
}

extern "C" size_t zs_zipgemm_allreduce_buffer_bytes(int M, int N, int world) {
    return zs::zipgemm_allreduce_buffer_bytes(M, N, world);
}

extern "C" size_t zs_zipgemm_allreduce_counters(int M, int N) { return zs::zipgemm_allreduce_counters(M, N); }

extern "C" int zs_zipgemm_allreduce(void* stream, const uint8_t* d_sm, const uint16_t* d_full, const uint64_t* d_b1,
                                    const uint64_t* d_b2, const uint64_t* d_b3, const int* d_mt_off,
                                    const int* d_gt_off, int max_hf, int max_full, int start_exp, const uint16_t* d_x,
                                    uint16_t* d_c, int M, int N, int K, int world, int rank, void* const* peer_bufs,
                                    unsigned* d_epoch, unsigned* d_err) {
    return zs::launch_zipgemm_allreduce((cudaStream_t)stream, d_sm, d_full, d_b1, d_b2, d_b3, d_mt_off, d_gt_off,
                                        max_hf, max_full, start_exp, d_x, d_c, M, N, K, world, rank, peer_bufs,
                                        d_epoch, d_err);
}

extern "C" int zs_peer_alloc(size_t bytes, void** d_ptr, void* ipc_handle) {
    if (!d_ptr || !ipc_handle || bytes == 0) return cudaErrorInvalidValue;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return e;
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return e;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *d_ptr = p;
    return cudaSuccess;
}

extern "C" int zs_peer_open(const void* ipc_handle, void** d_ptr) {
    if (!ipc_handle || !d_ptr) return cudaErrorInvalidValue;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    return cudaIpcOpenMemHandle(d_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

extern "C" int zs_peer_close(void* d_ptr) { return cudaIpcCloseMemHandle(d_ptr); }

extern "C" int zs_peer_free(void* d_ptr) { return cudaFree(d_ptr); }

extern "C" size_t zs_peer_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int zs_decode_attention_dense(void* stream, const uint16_t* d_q, const uint16_t* d_k, const uint16_t* d_v,
                                         const int* d_seqlens, int B, int Hq, int Hkv, int D, int T_rows,
                                         int max_seqlen, float softmax_scale, int num_splits, float* d_ws,
                                         size_t ws_bytes, uint16_t* d_out, int* splits_used, unsigned* d_err) {
    return zs::launch_attention_dense((cudaStream_t)stream, d_k, d_v, d_q, d_seqlens, d_out, B, Hq, Hkv, D, T_rows,
                                      max_seqlen, softmax_scale, num_splits, d_ws, ws_bytes, d_err, splits_used);
}

extern "C" int zs_decode_attention_default_splits(int B, int Hkv, int max_seqlen) {
    if (B <= 0 || Hkv <= 0 || max_seqlen < 0) return 1;
    return zs::attn_default_splits(B, Hkv, (max_seqlen + 63) / 64);
}

extern "C" size_t zs_decode_attention_workspace_bytes(int B, int Hq, int Hkv, int num_splits) {
    return zs::attn_workspace_bytes(B, Hq, Hkv, num_splits);
}

static bool to_compressed(const void* const* ptrs, const int* meta, zs::AttnCompressed* c) {
    if (!ptrs || !meta) return false;
    c->sm = static_cast<const uint8_t*>(ptrs[0]);
    c->full = static_cast<const uint16_t*>(ptrs[1]);
    c->b1 = static_cast<const uint64_t*>(ptrs[2]);
    c->b2 = static_cast<const uint64_t*>(ptrs[3]);
    c->b3 = static_cast<const uint64_t*>(ptrs[4]);
    c->mt_off = static_cast<const int*>(ptrs[5]);
    c->gt_off = static_cast<const int*>(ptrs[6]);
    c->rows = meta[0];
    c->cols = meta[1];
    c->max_hf = meta[2];
    c->max_full = meta[3];
    c->start_exp = meta[4];
    return true;
}

extern "C" int zs_decode_attention(void* stream, const uint16_t* d_q, const void* const* k_ptrs, const int* k_meta,
                                   const void* const* v_ptrs, const int* v_meta, const int* d_seqlens, int B, int Hq,
                                   int Hkv, int D, int T_pad, int max_seqlen, float softmax_scale, int num_splits,
                                   float* d_ws, size_t ws_bytes, uint16_t* d_out, int* splits_used,
                                   unsigned* d_err) {
    zs::AttnCompressed k{}, v{};
    if (!to_compressed(k_ptrs, k_meta, &k) || !to_compressed(v_ptrs, v_meta, &v)) return cudaErrorInvalidValue;
    return zs::launch_attention((cudaStream_t)stream, k, v, d_q, d_seqlens, d_out, B, Hq, Hkv, D, T_pad, max_seqlen,
                                softmax_scale, num_splits, d_ws, ws_bytes, d_err, splits_used);
}

extern "C" size_t zs_decode_attention_noalloc_max_workspace_bytes(void) { return zs::attn_noalloc_ws_bytes(); }

extern "C" int zs_decode_attention_noalloc(void* stream, const uint16_t* d_q, const void* const* k_ptrs,
                                           const int* k_meta, const void* const* v_ptrs, const int* v_meta,
                                           const int* d_seqlens, int B, int Hq, int Hkv, int D, int T_pad,
                                           int max_seqlen, float softmax_scale, int num_splits, uint16_t* d_out,
                                           int* splits_used, unsigned* d_err) {
    zs::AttnCompressed k{}, v{};
    if (!to_compressed(k_ptrs, k_meta, &k) || !to_compressed(v_ptrs, v_meta, &v)) return cudaErrorInvalidValue;
    return zs::launch_attention_noalloc((cudaStream_t)stream, k, v, d_q, d_seqlens, d_out, B, Hq, Hkv, D, T_pad,
                                        max_seqlen, softmax_scale, num_splits, d_err, splits_used);
}

extern "C" int zs_kv_append_pages(void* stream, const ZsKvPool* pool, const uint16_t* d_x, int B, int npg, int Hkv,
                                  int D, const int* d_dst_pages, unsigned* d_err) {
    if (!pool) return cudaErrorInvalidValue;
    return zs::launch_kv_append((cudaStream_t)stream, d_x, B, npg, Hkv, D, d_dst_pages, pool->num_pages,
                                pool->d_top7, pool->d_sm, pool->d_full, pool->d_b1, pool->d_b2, pool->d_b3,
                                pool->d_mt_off, pool->d_page_off, pool->d_cursor, pool->hf_capacity,
                                pool->full_capacity, d_err);
}

static zs::AttnCompressed pool_view(const ZsKvPool& p) {
    zs::AttnCompressed c{};
    c.sm = p.d_sm;
    c.full = p.d_full;
    c.b1 = p.d_b1;
    c.b2 = p.d_b2;
    c.b3 = p.d_b3;
    c.mt_off = p.d_mt_off;
    c.gt_off = nullptr;
    c.rows = 0;
    c.cols = 128;
    c.max_hf = 4096;     // a page GT of the pool may hold up to 4096 hf bytes
    c.max_full = 4096;   // and up to 4096 fallback elements
    c.start_exp = p.start_exp;
    return c;
}

extern "C" int zs_decode_attention_paged(void* stream, const uint16_t* d_q, const ZsKvPool* k, const ZsKvPool* v,
                                         const int* d_block_table, int max_blocks, const int* d_seqlens,
                                         const uint16_t* d_tail_k, const uint16_t* d_tail_v, int B, int Hq, int Hkv,
                                         int D, int max_seqlen, float softmax_scale, int num_splits, float* d_ws,
                                         size_t ws_bytes, uint16_t* d_out, int* splits_used, unsigned* d_err) {
    if (!k || !v || Hkv <= 0 || k->num_pages != v->num_pages || k->num_pages % Hkv) return cudaErrorInvalidValue;
    zs::AttnPaged pg{};
    pg.block_table = d_block_table;
    pg.max_blocks = max_blocks;
    pg.num_blocks = k->num_pages / Hkv;
    pg.k_page_off = k->d_page_off;
    pg.v_page_off = v->d_page_off;
    pg.tail_k = d_tail_k;
    pg.tail_v = d_tail_v;
    pg.k_max = k->d_cursor + 2;
    pg.v_max = v->d_cursor + 2;
    return zs::launch_attention_paged((cudaStream_t)stream, pool_view(*k), pool_view(*v), pg, d_q, d_seqlens, d_out,
                                      B, Hq, Hkv, D, max_seqlen, softmax_scale, num_splits, d_ws, ws_bytes, d_err,
                                      splits_used);
}

// ---------------------- reference GPU ABI (C++ names) -----------------------
cudaError_t BF16TripleBitmap_MM_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                    const __nv_bfloat16* CompressedFull, const uint64_t* Bitmap1,
                                    const uint64_t* Bitmap2, const uint64_t* Bitmap3,
                                    const int* TileOffsets_Median, const int* TileOffsets_Global,
                                    const int max_high_freq_count, const int max_full_count,
                                    const uint8_t start_exp, const __nv_bfloat16* B, __nv_bfloat16* C,
                                    const int M_Global, const int N_Global, const int K_Global,
                                    __nv_bfloat16* Reduction_Workspace, int Split_K) {
    (void)Reduction_Workspace;
    return zs::launch_zipgemm(stream, SignMantissa, reinterpret_cast<const uint16_t*>(CompressedFull), Bitmap1,
                              Bitmap2, Bitmap3, TileOffsets_Median, TileOffsets_Global, max_high_freq_count,
                              max_full_count, start_exp, reinterpret_cast<const uint16_t*>(B),
                              reinterpret_cast<uint16_t*>(C), M_Global, N_Global, K_Global, Split_K, nullptr);
}

cudaError_t BF16TripleBitmap_Decompress_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                            const __nv_bfloat16* CompressedFull, const uint64_t* Bitmap1,
                                            const uint64_t* Bitmap2, const uint64_t* Bitmap3,
                                            const int* TileOffsets_Median, const int* TileOffsets_Global,
                                            const int max_high_freq_count, const int max_full_count,
                                            const uint8_t start_exp, __nv_bfloat16* Output, const int M_Global,
                                            const int K_Global) {
    return zs::launch_decompress(stream, SignMantissa, reinterpret_cast<const uint16_t*>(CompressedFull), Bitmap1,
                                 Bitmap2, Bitmap3, TileOffsets_Median, TileOffsets_Global, max_high_freq_count,
                                 max_full_count, start_exp, reinterpret_cast<uint16_t*>(Output), M_Global, K_Global,
                                 nullptr);
}

cudaError_t InitBF16MatrixTripleBitmap_GPU(cudaStream_t stream, const __nv_bfloat16* d_input, int M, int K,
                                           const int* d_top_exponents, uint8_t* d_sign_mantissa,
                                           __nv_bfloat16* d_compressed_full, uint64_t* d_bitmap1,
                                           uint64_t* d_bitmap2, uint64_t* d_bitmap3, int* d_tile_offsets,
                                           int* d_tile_offsets_median, int* d_tile_offsets_global,
                                           uint8_t* d_temp_sm, __nv_bfloat16* d_temp_full, int* d_gt_hf_count,
                                           int* d_gt_full_count, int* d_hf_offsets, int* d_full_offsets,
                                           int* d_max_hf_count, int* d_max_full_count, int* d_total_hf,
                                           int* d_total_full) {
    (void)d_temp_sm;
    (void)d_temp_full;
    return zs::launch_encode(stream, reinterpret_cast<const uint16_t*>(d_input), M, K, d_top_exponents,
                             d_sign_mantissa, reinterpret_cast<uint16_t*>(d_compressed_full), d_bitmap1, d_bitmap2,
                             d_bitmap3, d_tile_offsets, d_tile_offsets_median, d_tile_offsets_global, d_gt_hf_count,
                             d_gt_full_count, d_hf_offsets, d_full_offsets, d_max_hf_count, d_max_full_count,
                             d_total_hf, d_total_full);
}
