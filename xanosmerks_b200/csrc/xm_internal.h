// Declarations shared between the library's translation units (not part of the C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Grouped tensor-core GEMM over fp16 activations already prepared (row-scaled):
// for each group g < G, rows [off[g], off[g] + cnt[g]) of a16 (P x K, fp16)
// times the Q4_K weight w[g] (N x K) -> y rows (P x N, fp32), scaled back by
// rowscale.  cnt/off are device arrays, h_w a host array of G <= 32 device
// pointers; max_rows bounds cnt[g] (grid size).
int qgemm_q4k_grouped(const __half* a16, const float* rowscale, int64_t P, int64_t K, int64_t N,
                      const uint8_t* const* h_w, const int* d_cnt, const int* d_off, int G, int64_t max_rows,
                      int64_t expect_rows, float* y, cudaStream_t st);
