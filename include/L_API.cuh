// Drop-in C++ ABI of the ZipServ library, B200 build (libzipserv_b200.so).
//
// Same six functions, parameter types and (C++) name mangling as the
// reference header build/L_API.cuh:19-165, so code compiled against the
// reference header links against this library unchanged. Each declaration cites
// the reference declaration it replaces.
//
// Behavioural notes (differences are strictly additive):
//  * Inputs are validated on the host; bad shapes, null or misaligned pointers
//    return cudaErrorInvalidValue instead of launching.
//  * BF16TripleBitmap_MM_API splits K itself: the K blocks of each 128-row
//    output tile go to the CTAs of a thread-block cluster, whose fp32 partial
//    tiles are summed in the same kernel through distributed shared memory in
//    a fixed order (deterministic fp32 sums, no bf16 rounding of partials).
//    Split_K is accepted and ignored; Reduction_Workspace is not used and may
//    be nullptr. Like the reference, it allocates nothing.
//  * All device work is ordered on `stream`; nothing synchronises the host.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Reference: build/L_API.cuh:19-37 (csrc/L_API.cu:119).
cudaError_t BF16TripleBitmap_MM_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                    const __nv_bfloat16* CompressedFull, const uint64_t* Bitmap1,
                                    const uint64_t* Bitmap2, const uint64_t* Bitmap3,
                                    const int* TileOffsets_Median, const int* TileOffsets_Global,
                                    const int max_high_freq_count, const int max_full_count,
                                    const uint8_t start_exp, const __nv_bfloat16* B, __nv_bfloat16* C,
                                    const int M_Global, const int N_Global, const int K_Global,
                                    __nv_bfloat16* Reduction_Workspace, int Split_K);

// Reference: build/L_API.cuh:38-52 (csrc/L_API.cu:234).
cudaError_t BF16TripleBitmap_Decompress_API(cudaStream_t stream, const uint8_t* SignMantissa,
                                            const __nv_bfloat16* CompressedFull, const uint64_t* Bitmap1,
                                            const uint64_t* Bitmap2, const uint64_t* Bitmap3,
                                            const int* TileOffsets_Median, const int* TileOffsets_Global,
                                            const int max_high_freq_count, const int max_full_count,
                                            const uint8_t start_exp, __nv_bfloat16* Output, const int M_Global,
                                            const int K_Global);

// Reference: build/L_API.cuh:54-74 (csrc/L_API.cu:314). Outputs are malloc'ed;
// free them with free(). Returns #global tiles or -1.
__host__ int InitBF16MatrixTripleBitmap(__nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median,
                                        int tile_M_global, int tile_K, int tile_K_median, int tile_K_global,
                                        const int* top_exponents, uint8_t** sign_mantissa,
                                        __nv_bfloat16** compressed_full, uint64_t** bitmap1, uint64_t** bitmap2,
                                        uint64_t** bitmap3, int** TileOffsets, int** TileOffsets_median,
                                        int** TileOffsets_global, int& max_high_freq_count, int& max_full_count);

// Reference: build/L_API.cuh:77-110 (csrc/L_API.cu:559).
__host__ int InitBF16MatrixTripleBitmap_Reuse(__nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median,
                                              int tile_M_global, int tile_K, int tile_K_median, int tile_K_global,
                                              const int* top_exponents, uint8_t* sign_mantissa,
                                              __nv_bfloat16* compressed_full, uint64_t* bitmap1, uint64_t* bitmap2,
                                              uint64_t* bitmap3, int* TileOffsets, int* TileOffsets_median,
                                              int* TileOffsets_global, uint8_t* temp_sm, __nv_bfloat16* temp_full,
                                              int* gt_hf_count, int* gt_full_count, int* hf_offsets,
                                              int* full_offsets, int& max_high_freq_count, int& max_full_count,
                                              int& out_total_hf, int& out_total_full);

// Reference: build/L_API.cuh:113-144 (csrc/L_API.cu:804).
__host__ int InitBF16MatrixTripleBitmap_Reuse_SIMD(
    __nv_bfloat16* A_bf16, int M, int K, int tile_M, int tile_M_median, int tile_M_global, int tile_K,
    int tile_K_median, int tile_K_global, const int* top_exponents, uint8_t* sign_mantissa,
    __nv_bfloat16* compressed_full, uint64_t* bitmap1, uint64_t* bitmap2, uint64_t* bitmap3, int* TileOffsets,
    int* TileOffsets_median, int* TileOffsets_global, uint8_t* temp_sm, __nv_bfloat16* temp_full, int* gt_hf_count,
    int* gt_full_count, int* hf_offsets, int* full_offsets, int& max_high_freq_count, int& max_full_count,
    int& out_total_hf, int& out_total_full);

// Reference: build/L_API.cuh:146-165 (csrc/L_API.cu:1355). Device pointers.
// d_temp_sm / d_temp_full are not needed by this implementation (streams are
// compacted in shared memory) and may be nullptr; d_gt_*_count and
// d_*_offsets are used as scratch for the per-tile counts and prefixes.
cudaError_t InitBF16MatrixTripleBitmap_GPU(cudaStream_t stream, const __nv_bfloat16* d_input, int M, int K,
                                           const int* d_top_exponents, uint8_t* d_sign_mantissa,
                                           __nv_bfloat16* d_compressed_full, uint64_t* d_bitmap1,
                                           uint64_t* d_bitmap2, uint64_t* d_bitmap3, int* d_tile_offsets,
                                           int* d_tile_offsets_median, int* d_tile_offsets_global,
                                           uint8_t* d_temp_sm, __nv_bfloat16* d_temp_full, int* d_gt_hf_count,
                                           int* d_gt_full_count, int* d_hf_offsets, int* d_full_offsets,
                                           int* d_max_hf_count, int* d_max_full_count, int* d_total_hf,
                                           int* d_total_full);
