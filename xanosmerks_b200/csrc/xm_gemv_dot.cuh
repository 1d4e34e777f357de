// Small device helpers shared by the integer-dot GEMV kernels.
#pragma once

#include "xm_qtypes.cuh"

XM_DEV uint4 lds_v4(const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); }
XM_DEV uint32_t lds_u32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
XM_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
XM_DEV void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// byte i of w as an exact float (magic-number conversion, no I2F)
XM_DEV float byte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)i)) - 8388608.0f;
}
// signed byte i of w as an exact float
XM_DEV float sbyte_f(uint32_t w, int i) { return (float)(int8_t)((w >> (8 * i)) & 0xFF); }

XM_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {   // unsigned bytes of a x signed bytes of b
  int d;
  asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
XM_DEV int dp4a_ss(uint32_t a, uint32_t b, int c) {   // signed x signed
  return __dp4a((int)a, (int)b, c);
}

// NW consecutive 32-bit words starting at a 2-byte-aligned shared address:
// NW + 1 aligned loads, each pair joined with a funnel shift (shift 0 or 16).
template <int NW>
XM_DEV void lds_words(const uint8_t* p, uint32_t (&w)[NW]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t prev = lds_u32(base);
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    const uint32_t next = lds_u32(base + 4 * (i + 1));
    w[i] = __funnelshift_r(prev, next, sh);
    prev = next;
  }
}

inline int xm_sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Two-digit split of one 32-element activation group held one element per
// lane: x ~= t * (254*x0 + x1), t = max|x| / (127*254), x0, x1 in [-127, 127]
// (about 16 significant bits).  Also returns the fp32 sums of elements 0-15
// and 16-31, reduced in a fixed shuffle order so the result is deterministic.
XM_DEV void split_group(float v, int& x0, int& x1, float& t, float& s_lo, float& s_hi) {
  float amax = fabsf(v);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  float s = v;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  s_lo = __shfl_sync(0xffffffffu, s, 0);
  s_hi = __shfl_sync(0xffffffffu, s, 16);
  x0 = 0;
  x1 = 0;
  t = 0.f;
  if (amax > 0.f) {
    const float sc = amax / 127.0f;
    const float u = v * (1.0f / sc);
    const float r0 = rintf(u);
    x0 = (int)r0;
    x1 = max(-127, min(127, (int)rintf((u - r0) * 254.0f)));
    t = sc / 254.0f;
  }
}
