// Host-side (CPU) codec entry points shared by host_encode.cpp and capi.cu.
#pragma once
#include <stdint.h>

namespace zs {
// Exponent-window analysis on the host; rule 0 = kernel_benchmark/utils.h:189,
// rule 1 = kernel_benchmark/zipserv_decode_attention_ext.cu:65-133.
void analyze_host(const uint16_t* a, long long n, int rule, int* top);

// Multi-threaded host encoder producing the reference's bytes. Temp slots:
// temp_sm #GT*(4096+15) bytes, temp_full #GT*(4096+7) elements; gt_hf / gt_full
// #GT ints; hf_pre / full_pre #GT+1 ints. Returns #GT or -1.
int encode_host(const uint16_t* a, int M, int K, const int* top, uint8_t* sm, uint16_t* full, uint64_t* b1,
                uint64_t* b2, uint64_t* b3, int* st_counts, int* mt_off, int* gt_off, uint8_t* temp_sm,
                uint16_t* temp_full, int* gt_hf, int* gt_full, int* hf_pre, int* full_pre, int* max_hf,
                int* max_full, int* total_hf, int* total_full);
}  // namespace zs
