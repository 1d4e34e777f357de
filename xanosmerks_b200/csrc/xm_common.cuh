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
