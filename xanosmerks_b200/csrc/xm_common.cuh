// Shared device/host helpers for the GGUF kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/xm_gguf.h"

#define XM_DEV __device__ __forceinline__

// ---------------------------------------------------------------------------
// Host-side error reporting: every entry point returns an XM_* status and
// leaves a human-readable message for xm_last_error() (thread-local).
// ---------------------------------------------------------------------------
int xm_set_error(int status, const char* fmt, ...);
int xm_check_launch(const char* what);

#define XM_TRY_CUDA(call)                                                   \
  do {                                                                      \
    cudaError_t e_ = (call);                                                \
    if (e_ != cudaSuccess)                                                  \
      return xm_set_error(XM_ERR_CUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// ---------------------------------------------------------------------------
// Byte-stream field readers.  GGUF records are packed (18, 22, 84, 110, 210 B
// ...), so fields are read bytewise unless the caller knows the alignment.
// ---------------------------------------------------------------------------
XM_DEV uint32_t rd_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
XM_DEV uint32_t rd_u32(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
// little-endian fp16 -> fp32 (exact; subnormals kept)
XM_DEV float rd_f16(const uint8_t* p) { return __half2float(__ushort_as_half((unsigned short)rd_u16(p))); }
XM_DEV float rd_f32(const uint8_t* p) { return __uint_as_float(rd_u32(p)); }

// Exact int -> float for |q| < 2^22 without the (quarter-rate) I2F unit:
// 0x4B400000 is 1.5 * 2^23, whose ulp is 1.
XM_DEV float i2f_small(int q) { return __int_as_float(0x4B400000 + q) - 12582912.0f; }

// 16-byte read-only global load that does not allocate in L1 (streamed bytes).
XM_DEV uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Copy bytes [src, src+bytes) of global memory into shared memory so that
// smem[mis + i] == src[i], mis = src & 15.  16-byte vector loads for chunks
// wholly inside the range, byte loads for the (at most two) ragged chunks.
// Returns mis.  All threads of the block participate; caller syncs.
XM_DEV int stage_bytes(uint8_t* smem, const uint8_t* src, int bytes, int tid, int nthreads) {
  const int mis = (int)((uintptr_t)src & 15);
  const uint8_t* asrc = src - mis;
  const int nchunks = (mis + bytes + 15) >> 4;
  for (int c = tid; c < nchunks; c += nthreads) {
    const int lo = c * 16, hi = lo + 16;
    if (lo >= mis && hi <= mis + bytes) {
      *reinterpret_cast<uint4*>(smem + lo) = ldg_stream_v4(asrc + lo);
    } else {
      const int a = lo > mis ? lo : mis;
      const int b = hi < mis + bytes ? hi : mis + bytes;
      for (int k = a; k < b; ++k) smem[k] = asrc[k];
    }
  }
  return mis;
}

template <typename T> XM_DEV float to_f32(T v);
template <> XM_DEV float to_f32<float>(float v) { return v; }
template <> XM_DEV float to_f32<__half>(__half v) { return __half2float(v); }
template <> XM_DEV float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

XM_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// ---------------------------------------------------------------------------
// mbarrier + bulk-copy (TMA, no multicast) helpers.  Every wait is bounded:
// after kSpinLimit polls the waiter records XM_DEVERR_TIMEOUT in the device
// error word and carries on, so a lost transfer turns into a host-visible
// error instead of a hung GPU.
// ---------------------------------------------------------------------------
#define XM_DEVERR_TIMEOUT 1
extern __device__ int g_xm_device_error;

XM_DEV uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

XM_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
XM_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
XM_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

XM_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

// global -> shared bulk copy completing on `bar`; 16-byte aligned src/dst, size % 16 == 0
XM_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

XM_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

constexpr uint32_t kSpinLimit = 1u << 24;

// Returns false (and records the timeout) if the phase did not complete in time.
XM_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  atomicOr(&g_xm_device_error, XM_DEVERR_TIMEOUT);
  return false;
}

XM_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded spin until a shared-memory word equals `want` (written by another
// warp of the CTA).  Used to make sure a ring slot is armed for the item a
// consumer holds before it waits on the slot's mbarrier parity: parity alone
// cannot tell lap L from lap L+2.
XM_DEV bool smem_wait_eq(const volatile int* p, int want) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (*p == want) return true;
  atomicOr(&g_xm_device_error, XM_DEVERR_TIMEOUT);
  return false;
}

// ---------------------------------------------------------------------------
// Row preparation of tensor-core GEMM activations: one 256-thread block per
// row, 4 consecutive values per thread per step (vector loads), the row's
// values converted to fp16 after division by a power of two that puts the
// row's largest magnitude in [2^14, 2^15) (exact for bf16 and fp16 input;
// keeps large and tiny rows inside fp16's range).
// ---------------------------------------------------------------------------
constexpr int kPrepThreads = 256;

// 4 consecutive values as fp32 (p 8-byte aligned for 16-bit types, 16-byte for fp32)
template <typename T> XM_DEV void ld4f(const T* p, float (&v)[4]);
template <> XM_DEV void ld4f<float>(const float* p, float (&v)[4]) {
  const float4 f = *reinterpret_cast<const float4*>(p);
  v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
}
template <> XM_DEV void ld4f<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(u.x << 16); v[1] = __uint_as_float(u.x & 0xFFFF0000u);
  v[2] = __uint_as_float(u.y << 16); v[3] = __uint_as_float(u.y & 0xFFFF0000u);
}
template <> XM_DEV void ld4f<__half>(const __half* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
  v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
}

// block-wide max / sum of one value per thread (kPrepThreads threads; red: 32 floats)
template <int NTH = kPrepThreads>
XM_DEV float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < NTH / 32; ++w) r = fmaxf(r, red[w]);
  __syncthreads();
  return r;
}
template <int NTH = kPrepThreads>
XM_DEV float block_sum(float v, float* red) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < NTH / 32; ++w) r += red[w];
  __syncthreads();
  return r;
}

// Expert activations (moe.py / primitives.py): silu x / (1 + exp(-x)), gelu
// (tanh form) 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))), relu
// max(x, 0), identity.  `act` is an XM_ACT_* id.
XM_DEV float xm_act(int act, float x) {
  if (act == XM_ACT_SILU) return x / (1.0f + expf(-x));
  if (act == XM_ACT_GELU) return 0.5f * x * (1.0f + tanhf(0.7978845608f * (x + 0.044715f * x * x * x)));
  if (act == XM_ACT_RELU) return fmaxf(x, 0.0f);
  return x;
}

// The power-of-two exponent s with amax / 2^s in [2^14, 2^15) (0 for zero or non-finite rows).
XM_DEV int fp16_row_shift(float amax) {
  int s = 0;
  if (amax > 0.f && amax < INFINITY) {
    int e;
    frexpf(amax, &e);           // amax = f * 2^e, f in [0.5, 1): amax in [2^(e-1), 2^e)
    s = (e - 1) - 14;
  }
  return s;
}

// One row: val(k, v) writes the 4 values at k (k % 4 == 0); out[k] = fp16(v / 2^s),
// *scale = 2^s.  Every thread of the block (NTH threads) calls it; K % 4 == 0.
template <int NTH, typename F>
XM_DEV void prep_row_fp16_n(F val, int K, __half* __restrict__ out, float* __restrict__ scale, float* red) {
  float amax = 0.f;
  for (int k = threadIdx.x * 4; k < K; k += NTH * 4) {
    float v[4];
    val(k, v);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3]))));
  }
  amax = block_max<NTH>(amax, red);
  const int s = fp16_row_shift(amax);
  const float inv = ldexpf(1.0f, -s);
  for (int k = threadIdx.x * 4; k < K; k += NTH * 4) {
    float v[4];
    val(k, v);
    const __half2 a = __floats2half2_rn(v[0] * inv, v[1] * inv), b = __floats2half2_rn(v[2] * inv, v[3] * inv);
    *reinterpret_cast<uint2*>(out + k) = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                                                    *reinterpret_cast<const uint32_t*>(&b));
  }
  if (threadIdx.x == 0) *scale = ldexpf(1.0f, s);
}
template <typename F>
XM_DEV void prep_row_fp16(F val, int K, __half* __restrict__ out, float* __restrict__ scale, float* red) {
  prep_row_fp16_n<kPrepThreads>(val, K, out, scale, red);
}
