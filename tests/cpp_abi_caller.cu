// A C++ caller of the drop-in ABI, written the way the reference's own callers
// use it (kernel_benchmark/test_mm.cu:749-819: host encode, H2D, MM_API;
// kernel_benchmark/test_decompress.cu:461-491: Decompress_API). It is compiled
// against include/L_API.cuh only and linked to libzipserv_b200.so, so the
// six C++-mangled entry points are resolved exactly as a program built against
// the reference header would resolve them. tests/test_gpu_cpp_abi.py builds and
// runs it and checks what it writes.
//
// usage: cpp_abi_caller <dir>
//   reads  <dir>/dims.txt (M K N), a.bin (M*K bf16), top.bin (7 int32), x.bin (N*K bf16)
//   writes <dir>/{scalar,reuse,simd,gpu}_<array>.bin for the four encoders,
//          <dir>/mm.bin (N*M bf16, column-major M x N) and <dir>/dec.bin (M*K bf16)
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "L_API.cuh"

#define CHECK(x)                                                                    \
    do {                                                                            \
        cudaError_t e_ = (x);                                                       \
        if (e_ != cudaSuccess) {                                                    \
            fprintf(stderr, "%s:%d %s -> %s\n", __FILE__, __LINE__, #x, cudaGetErrorString(e_)); \
            return 2;                                                               \
        }                                                                           \
    } while (0)

static std::string g_dir;

static bool read_file(const char* name, void* dst, size_t bytes) {
    FILE* f = fopen((g_dir + "/" + name).c_str(), "rb");
    if (!f) return false;
    const size_t n = fread(dst, 1, bytes, f);
    fclose(f);
    return n == bytes;
}

static bool write_file(const std::string& name, const void* src, size_t bytes) {
    FILE* f = fopen((g_dir + "/" + name).c_str(), "wb");
    if (!f) return false;
    const size_t n = fwrite(src, 1, bytes, f);
    fclose(f);
    return n == bytes;
}

// The encoder outputs, trimmed to their valid lengths.
static bool dump(const char* tag, int M, int K, const uint8_t* sm, const __nv_bfloat16* full, const uint64_t* b1,
                 const uint64_t* b2, const uint64_t* b3, const int* st, const int* mt, const int* gt, int max_hf,
                 int max_full) {
    const int ngt = (M / 64) * (K / 64), nst = M * K / 64, nmt = M * K / 1024;
    const int total_hf = gt[2 * ngt], total_full = gt[2 * ngt + 1];
    const std::string p = std::string(tag) + "_";
    const int scalars[2] = {max_hf, max_full};
    return write_file(p + "sign_mantissa.bin", sm, (size_t)total_hf) &&
           write_file(p + "full.bin", full, (size_t)total_full * 2) && write_file(p + "bitmap1.bin", b1, (size_t)nst * 8) &&
           write_file(p + "bitmap2.bin", b2, (size_t)nst * 8) && write_file(p + "bitmap3.bin", b3, (size_t)nst * 8) &&
           write_file(p + "st_counts.bin", st, (size_t)nst * 8) && write_file(p + "mt_offsets.bin", mt, (size_t)nmt * 8) &&
           write_file(p + "gt_offsets.bin", gt, (size_t)(ngt + 1) * 8) && write_file(p + "scalars.bin", scalars, 8);
}

int main(int argc, char** argv) {
    if (argc < 2) return 1;
    g_dir = argv[1];
    int M = 0, K = 0, N = 0;
    {
        FILE* f = fopen((g_dir + "/dims.txt").c_str(), "r");
        if (!f || fscanf(f, "%d %d %d", &M, &K, &N) != 3) return 1;
        fclose(f);
    }
    const int ngt = (M / 64) * (K / 64), nst = M * K / 64, nmt = M * K / 1024;
    std::vector<__nv_bfloat16> A((size_t)M * K), X((size_t)N * K);
    int top[7];
    if (!read_file("a.bin", A.data(), A.size() * 2) || !read_file("top.bin", top, sizeof(top)) ||
        !read_file("x.bin", X.data(), X.size() * 2))
        return 1;

    // 1. InitBF16MatrixTripleBitmap: the library allocates the outputs (malloc), the caller frees them
    {
        uint8_t* sm = nullptr;
        __nv_bfloat16* full = nullptr;
        uint64_t *b1 = nullptr, *b2 = nullptr, *b3 = nullptr;
        int *st = nullptr, *mt = nullptr, *gt = nullptr;
        int max_hf = 0, max_full = 0;
        const int r = InitBF16MatrixTripleBitmap(A.data(), M, K, 8, 16, 64, 8, 64, 64, top, &sm, &full, &b1, &b2, &b3,
                                                 &st, &mt, &gt, max_hf, max_full);
        if (r != ngt) { fprintf(stderr, "scalar encoder returned %d\n", r); return 3; }
        if (!dump("scalar", M, K, sm, full, b1, b2, b3, st, mt, gt, max_hf, max_full)) return 4;
        free(sm); free(full); free(b1); free(b2); free(b3); free(st); free(mt); free(gt);
    }

    // 2-3. _Reuse and _Reuse_SIMD: caller buffers (sizes as csrc/L_API.cu:559 expects)
    std::vector<uint8_t> sm((size_t)M * K + 16 * (size_t)ngt), tsm((size_t)ngt * (4096 + 15) + 16);
    std::vector<__nv_bfloat16> full((size_t)M * K + 8 * (size_t)ngt), tfull((size_t)ngt * (4096 + 7) + 8);
    std::vector<uint64_t> b1(nst), b2(nst), b3(nst);
    std::vector<int> st(2 * (size_t)nst), mt(2 * (size_t)nmt), gt(2 * ((size_t)ngt + 1));
    std::vector<int> c1(ngt + 1), c2(ngt + 1), o1(ngt + 1), o2(ngt + 1);
    for (int simd = 0; simd < 2; ++simd) {
        int max_hf = 0, max_full = 0, th = 0, tf = 0;
        auto fn = simd ? InitBF16MatrixTripleBitmap_Reuse_SIMD : InitBF16MatrixTripleBitmap_Reuse;
        const int r = fn(A.data(), M, K, 8, 16, 64, 8, 64, 64, top, sm.data(), full.data(), b1.data(), b2.data(),
                         b3.data(), st.data(), mt.data(), gt.data(), tsm.data(), tfull.data(), c1.data(), c2.data(),
                         o1.data(), o2.data(), max_hf, max_full, th, tf);
        if (r < 0 || th != gt[2 * ngt] || tf != gt[2 * ngt + 1]) { fprintf(stderr, "reuse encoder %d failed\n", simd); return 3; }
        if (!dump(simd ? "simd" : "reuse", M, K, sm.data(), full.data(), b1.data(), b2.data(), b3.data(), st.data(),
                  mt.data(), gt.data(), max_hf, max_full))
            return 4;
    }
    // the arrays of the last host encode feed the GPU calls below
    int host_max_hf = 0, host_max_full = 0;
    {
        int sc[2];
        if (!read_file("simd_scalars.bin", sc, 8)) return 4;
        host_max_hf = sc[0];
        host_max_full = sc[1];
    }

    cudaStream_t stream;
    CHECK(cudaStreamCreate(&stream));
    // 4. InitBF16MatrixTripleBitmap_GPU: every buffer on the device
    {
        __nv_bfloat16 *d_a, *d_full, *d_tfull;
        uint8_t *d_sm, *d_tsm;
        uint64_t *d_b1, *d_b2, *d_b3;
        int *d_top, *d_st, *d_mt, *d_gt, *d_c1, *d_c2, *d_o1, *d_o2, *d_sc;
        CHECK(cudaMalloc(&d_a, A.size() * 2));
        CHECK(cudaMalloc(&d_full, full.size() * 2));
        CHECK(cudaMalloc(&d_tfull, tfull.size() * 2));
        CHECK(cudaMalloc(&d_sm, sm.size()));
        CHECK(cudaMalloc(&d_tsm, tsm.size()));
        CHECK(cudaMalloc(&d_b1, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_b2, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_b3, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_top, 7 * 4));
        CHECK(cudaMalloc(&d_st, st.size() * 4));
        CHECK(cudaMalloc(&d_mt, mt.size() * 4));
        CHECK(cudaMalloc(&d_gt, gt.size() * 4));
        CHECK(cudaMalloc(&d_c1, (ngt + 1) * 4));
        CHECK(cudaMalloc(&d_c2, (ngt + 1) * 4));
        CHECK(cudaMalloc(&d_o1, (ngt + 1) * 4));
        CHECK(cudaMalloc(&d_o2, (ngt + 1) * 4));
        CHECK(cudaMalloc(&d_sc, 4 * 4));
        CHECK(cudaMemcpy(d_a, A.data(), A.size() * 2, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_top, top, sizeof(top), cudaMemcpyHostToDevice));
        CHECK(InitBF16MatrixTripleBitmap_GPU(stream, d_a, M, K, d_top, d_sm, d_full, d_b1, d_b2, d_b3, d_st, d_mt, d_gt,
                                             d_tsm, d_tfull, d_c1, d_c2, d_o1, d_o2, d_sc, d_sc + 1, d_sc + 2, d_sc + 3));
        CHECK(cudaStreamSynchronize(stream));
        int sc[4];
        CHECK(cudaMemcpy(sc, d_sc, sizeof(sc), cudaMemcpyDeviceToHost));
        std::vector<uint8_t> g_sm(sm.size());
        std::vector<__nv_bfloat16> g_full(full.size());
        std::vector<uint64_t> g_b1(nst), g_b2(nst), g_b3(nst);
        std::vector<int> g_st(st.size()), g_mt(mt.size()), g_gt(gt.size());
        CHECK(cudaMemcpy(g_sm.data(), d_sm, g_sm.size(), cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_full.data(), d_full, g_full.size() * 2, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_b1.data(), d_b1, (size_t)nst * 8, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_b2.data(), d_b2, (size_t)nst * 8, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_b3.data(), d_b3, (size_t)nst * 8, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_st.data(), d_st, g_st.size() * 4, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_mt.data(), d_mt, g_mt.size() * 4, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(g_gt.data(), d_gt, g_gt.size() * 4, cudaMemcpyDeviceToHost));
        if (!dump("gpu", M, K, g_sm.data(), g_full.data(), g_b1.data(), g_b2.data(), g_b3.data(), g_st.data(),
                  g_mt.data(), g_gt.data(), sc[0], sc[1]))
            return 4;
        cudaFree(d_a); cudaFree(d_full); cudaFree(d_tfull); cudaFree(d_sm); cudaFree(d_tsm); cudaFree(d_b1);
        cudaFree(d_b2); cudaFree(d_b3); cudaFree(d_top); cudaFree(d_st); cudaFree(d_mt); cudaFree(d_gt);
        cudaFree(d_c1); cudaFree(d_c2); cudaFree(d_o1); cudaFree(d_o2); cudaFree(d_sc);
    }

    // 5-6. MM_API and Decompress_API on the host-encoded arrays, uploaded as test_mm.cu does
    {
        uint8_t* d_sm;
        __nv_bfloat16 *d_full, *d_x, *d_c, *d_out;
        uint64_t *d_b1, *d_b2, *d_b3;
        int *d_mt, *d_gt;
        const int total_hf = gt[2 * ngt], total_full = gt[2 * ngt + 1];
        CHECK(cudaMalloc(&d_sm, (size_t)total_hf + 16));
        CHECK(cudaMalloc(&d_full, ((size_t)total_full + 8) * 2));
        CHECK(cudaMalloc(&d_b1, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_b2, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_b3, (size_t)nst * 8));
        CHECK(cudaMalloc(&d_mt, mt.size() * 4));
        CHECK(cudaMalloc(&d_gt, gt.size() * 4));
        CHECK(cudaMalloc(&d_x, X.size() * 2));
        CHECK(cudaMalloc(&d_c, (size_t)M * N * 2));
        CHECK(cudaMalloc(&d_out, A.size() * 2));
        CHECK(cudaMemcpy(d_sm, sm.data(), (size_t)total_hf, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_full, full.data(), (size_t)total_full * 2, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_b1, b1.data(), (size_t)nst * 8, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_b2, b2.data(), (size_t)nst * 8, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_b3, b3.data(), (size_t)nst * 8, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_mt, mt.data(), mt.size() * 4, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_gt, gt.data(), gt.size() * 4, cudaMemcpyHostToDevice));
        CHECK(cudaMemcpy(d_x, X.data(), X.size() * 2, cudaMemcpyHostToDevice));
        const uint8_t start_exp = (uint8_t)((top[0] - 1) & 0xFF);
        CHECK(BF16TripleBitmap_MM_API(stream, d_sm, d_full, d_b1, d_b2, d_b3, d_mt, d_gt, host_max_hf, host_max_full,
                                      start_exp, d_x, d_c, M, N, K, nullptr, 1));
        CHECK(BF16TripleBitmap_Decompress_API(stream, d_sm, d_full, d_b1, d_b2, d_b3, d_mt, d_gt, host_max_hf,
                                              host_max_full, start_exp, d_out, M, K));
        CHECK(cudaStreamSynchronize(stream));
        std::vector<__nv_bfloat16> Cc((size_t)M * N), D((size_t)M * K);
        CHECK(cudaMemcpy(Cc.data(), d_c, Cc.size() * 2, cudaMemcpyDeviceToHost));
        CHECK(cudaMemcpy(D.data(), d_out, D.size() * 2, cudaMemcpyDeviceToHost));
        if (!write_file("mm.bin", Cc.data(), Cc.size() * 2) || !write_file("dec.bin", D.data(), D.size() * 2)) return 4;
        cudaFree(d_sm); cudaFree(d_full); cudaFree(d_b1); cudaFree(d_b2); cudaFree(d_b3); cudaFree(d_mt);
        cudaFree(d_gt); cudaFree(d_x); cudaFree(d_c); cudaFree(d_out);
    }
    CHECK(cudaStreamDestroy(stream));
    printf("ok\n");
    return 0;
}
