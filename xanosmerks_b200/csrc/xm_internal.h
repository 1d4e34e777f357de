// Declarations shared between the library's translation units (not part of the C ABI).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

// Grouped tensor-core GEMM over fp16 activations already prepared (row-scaled):
// for each group g < G, rows [off[g], off[g] + cnt[g]) of a16 (P x K, fp16)
// times the weight w[g] (N x K, GGUF blocks of qtype) -> y rows (P x N, fp32),
// scaled back by rowscale.  cnt/off are device arrays, h_w a host array of
// G <= 32 device pointers; max_rows bounds cnt[g] (grid size).
int qgemm_grouped(int qtype, const __half* a16, const float* rowscale, int64_t P, int64_t K, int64_t N,
                  const uint8_t* const* h_w, const int* d_cnt, const int* d_off, int G, int64_t max_rows,
                  int64_t expect_rows, float* y, cudaStream_t st);
// Gate/up experts fused: y = act(a W1^T) * (a W3^T) per group (XM_ACT_* act),
// fp32 out.  Returns 1 (nothing launched) when the device cannot hold the
// kernel, so the caller can run the two projections separately.
int qgemm_grouped_gate_up(int qtype, int act, const __half* a16, const float* rowscale, int64_t P, int64_t K,
                          int64_t N, const uint8_t* const* h_w1, const uint8_t* const* h_w3, const int* d_cnt,
                          const int* d_off, int G, int64_t max_rows, int64_t expect_rows, float* y, cudaStream_t st);
// Whether the tensor-core GEMM takes weights of this type with rows of k
// elements (k a multiple of 256 and a row a multiple of 16 bytes).
bool qgemm_type_supported(int qtype, int64_t k);
// Bytes of one row of k weights of a block type (0: not block-quantized).
int64_t qgemm_row_bytes(int qtype, int64_t k);

// Generic integer-dot GEMV (Q4_K, Q5_K, Q6_K, Q8_0; k % 128 == 0, k <= 16384)
// over a group-major activation split in d_ws; y (+)= W x (+ bias).
bool gemv_kq_supported(int qtype, int64_t n, int64_t k, int64_t m);
int gemv_kq(int qtype, const uint8_t* W, int64_t n, int64_t k, int64_t m, const void* d_ws, const float* bias,
            float* y, int accumulate, cudaStream_t st);
// Group-major activation split of m rows of k values with an XM_PRO_* prologue.
int split_rows(const void* d_x, int x_dtype, int64_t m, int64_t k, int64_t x_stride, int prologue,
               const float* norm_w, float eps, void* d_ws, cudaStream_t st);
// Q4_K GEMV for 2..8 activation rows on the tensor cores (integer MMA): the
// per-row activation split (with an XM_PRO_* prologue) goes to d_ws, which must
// hold gemv_mma_split_bytes(k, m) bytes; y (+)= W x (+ bias).
bool gemv_mma_supported(int qtype, int64_t n, int64_t k, int64_t m);
int64_t gemv_mma_split_bytes(int64_t k, int64_t m);
int gemv_mma(const uint8_t* W, int64_t n, int64_t k, int64_t m, const void* d_x, int x_dtype, int64_t x_stride,
             int prologue, const float* norm_w, float eps, const float* bias, float* y, int accumulate, void* d_ws,
             cudaStream_t st);
