// TEST INFRASTRUCTURE ONLY -- extern "C" shims over the reference ZipServ
// library, compiled from the reference's own sources (csrc/L_API.cu and
// kernel_benchmark/utils.h) by oracle/Makefile into oracle/_ref/. Tests use it
// to produce golden fixtures and, on a GPU, to run the reference kernels on the
// same inputs as ours. The product never loads it.
#include "L_API.cuh"   // reference build/L_API.cuh
#include "utils.h"     // reference kernel_benchmark/utils.h
#include <cstdlib>
#include <cstring>

extern "C" {

// kernel_benchmark/utils.h:189 (host exponent-window rule)
void ref_analyze(const uint16_t* a, int M, int K, int* top) {
    analyzeExponentDistribution_BF16((__nv_bfloat16*)a, M, K, top, 7);
}

// kernel_benchmark/utils.h:101 (reference seeded matrix generator)
void ref_init_matrices(uint16_t* A, uint16_t* B, int M, int K, int N, unsigned seed) {
    init_host_matrices_bf16((__nv_bfloat16*)A, (__nv_bfloat16*)B, M, K, N, nullptr, seed);
}

// csrc/L_API.cu:314 (malloc-ing scalar encoder). Copies results into caller
// buffers and frees the reference's allocations.
int ref_encode_scalar(const uint16_t* a, int M, int K, const int* top,
                      uint8_t* sm, uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3,
                      int* st, int* mt, int* gt, int* max_hf, int* max_full) {
    uint8_t* p_sm; __nv_bfloat16* p_full; uint64_t *p1, *p2, *p3; int *p_st, *p_mt, *p_gt;
    int mh = 0, mf = 0;
    int ngt = InitBF16MatrixTripleBitmap((__nv_bfloat16*)a, M, K, 8, 16, 64, 8, 64, 64, top,
                                         &p_sm, &p_full, &p1, &p2, &p3, &p_st, &p_mt, &p_gt, mh, mf);
    if (ngt < 0) return ngt;
    int nst = M * K / 64, nmt = M * K / 1024;
    int thf = p_gt[2 * ngt], tfull = p_gt[2 * ngt + 1];
    memcpy(sm, p_sm, thf);
    memcpy(full, p_full, (size_t)tfull * 2);
    memcpy(b1, p1, (size_t)nst * 8); memcpy(b2, p2, (size_t)nst * 8); memcpy(b3, p3, (size_t)nst * 8);
    memcpy(st, p_st, (size_t)nst * 8); memcpy(mt, p_mt, (size_t)nmt * 8); memcpy(gt, p_gt, (size_t)(ngt + 1) * 8);
    free(p_sm); free(p_full); free(p1); free(p2); free(p3); free(p_st); free(p_mt); free(p_gt);
    *max_hf = mh; *max_full = mf;
    return ngt;
}

static int encode_reuse_common(bool simd, const uint16_t* a, int M, int K, const int* top,
                               uint8_t* sm, uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3,
                               int* st, int* mt, int* gt, int* max_hf, int* max_full,
                               int* total_hf, int* total_full) {
    int ngt = (M / 64) * (K / 64);
    uint8_t* tsm = (uint8_t*)malloc((size_t)ngt * (4096 + 15) + 16);
    uint16_t* tfu = (uint16_t*)malloc(((size_t)ngt * (4096 + 7) + 8) * 2);
    int* c1 = (int*)malloc(sizeof(int) * (ngt + 1));
    int* c2 = (int*)malloc(sizeof(int) * (ngt + 1));
    int* o1 = (int*)malloc(sizeof(int) * (ngt + 1));
    int* o2 = (int*)malloc(sizeof(int) * (ngt + 1));
    int mh = 0, mf = 0, th = 0, tf = 0, r;
    if (simd)
        r = InitBF16MatrixTripleBitmap_Reuse_SIMD((__nv_bfloat16*)a, M, K, 8, 16, 64, 8, 64, 64, top,
              sm, (__nv_bfloat16*)full, b1, b2, b3, st, mt, gt, tsm, (__nv_bfloat16*)tfu,
              c1, c2, o1, o2, mh, mf, th, tf);
    else
        r = InitBF16MatrixTripleBitmap_Reuse((__nv_bfloat16*)a, M, K, 8, 16, 64, 8, 64, 64, top,
              sm, (__nv_bfloat16*)full, b1, b2, b3, st, mt, gt, tsm, (__nv_bfloat16*)tfu,
              c1, c2, o1, o2, mh, mf, th, tf);
    free(tsm); free(tfu); free(c1); free(c2); free(o1); free(o2);
    *max_hf = mh; *max_full = mf; *total_hf = th; *total_full = tf;
    return r;
}

// csrc/L_API.cu:559 and :804
int ref_encode_reuse(const uint16_t* a, int M, int K, const int* top,
                     uint8_t* sm, uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3,
                     int* st, int* mt, int* gt, int* max_hf, int* max_full, int* th, int* tf) {
    return encode_reuse_common(false, a, M, K, top, sm, full, b1, b2, b3, st, mt, gt, max_hf, max_full, th, tf);
}
int ref_encode_simd(const uint16_t* a, int M, int K, const int* top,
                    uint8_t* sm, uint16_t* full, uint64_t* b1, uint64_t* b2, uint64_t* b3,
                    int* st, int* mt, int* gt, int* max_hf, int* max_full, int* th, int* tf) {
    return encode_reuse_common(true, a, M, K, top, sm, full, b1, b2, b3, st, mt, gt, max_hf, max_full, th, tf);
}

// csrc/L_API.cu:119 -- device pointers, caller's stream.
int ref_mm(void* stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
           const uint64_t* b2, const uint64_t* b3, const int* mt, const int* gt,
           int max_hf, int max_full, int start_exp, const uint16_t* B, uint16_t* C,
           int M, int N, int K, uint16_t* ws, int split_k) {
    return (int)BF16TripleBitmap_MM_API((cudaStream_t)stream, sm, (const __nv_bfloat16*)full, b1, b2, b3,
                                        mt, gt, max_hf, max_full, (uint8_t)start_exp,
                                        (const __nv_bfloat16*)B, (__nv_bfloat16*)C, M, N, K,
                                        (__nv_bfloat16*)ws, split_k);
}

// csrc/L_API.cu:234
int ref_decompress(void* stream, const uint8_t* sm, const uint16_t* full, const uint64_t* b1,
                   const uint64_t* b2, const uint64_t* b3, const int* mt, const int* gt,
                   int max_hf, int max_full, int start_exp, uint16_t* out, int M, int K) {
    return (int)BF16TripleBitmap_Decompress_API((cudaStream_t)stream, sm, (const __nv_bfloat16*)full,
                                                b1, b2, b3, mt, gt, max_hf, max_full, (uint8_t)start_exp,
                                                (__nv_bfloat16*)out, M, K);
}

int ref_sync() { return (int)cudaDeviceSynchronize(); }

}  // extern "C"
