// Per-type GGUF block decoders (device).
//
// QT<type>::decode8(blk, e0, v) writes the exact fp32 values of elements
// e0 .. e0+7 (e0 % 8 == 0) of one block record `blk`: the value the reference
// computes before its final .astype(np.float16), with the same float32
// operation order (explicit __fmul_rn / __fadd_rn / __fsub_rn, so no FMA is
// contracted; the products are exact in every type except Q8_1 and Q8_K, where
// the rounding order matters).  Rounding that result with __float2half_rn
// (IEEE round-to-nearest-even, overflow to inf) gives the reference's fp16.
#pragma once

#include "xm_common.cuh"

enum : int {
  T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q4_1 = 3, T_Q5_0 = 6, T_Q5_1 = 7, T_Q8_0 = 8, T_Q8_1 = 9,
  T_Q2_K = 10, T_Q3_K = 11, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14, T_Q8_K = 15,
  T_I8 = 24, T_I16 = 25, T_I32 = 26, T_I64 = 27, T_BF16 = 30
};

template <int T> struct QT;

// Q4_0 (gguf_dequant.py:25-45): d @0, 16 nibble bytes @2; element i is the low
// nibble of byte i/2 for even i, the high nibble for odd i; (q - 8) * d.
template <> struct QT<T_Q4_0> {
  static constexpr int QK = 32, REC = 18;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f16(b);
#pragma unroll
    for (int t = 0; t < 8; t += 2) {
      const uint32_t q = b[2 + ((e0 + t) >> 1)];
      v[t] = __fmul_rn(i2f_small((int)(q & 15)) - 8.0f, d);
      v[t + 1] = __fmul_rn(i2f_small((int)(q >> 4)) - 8.0f, d);
    }
  }
};

// Q4_1 (gguf_dequant.py:51-72): d @0, m @2, nibbles @4 (interleaved); q*d + m.
template <> struct QT<T_Q4_1> {
  static constexpr int QK = 32, REC = 20;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f16(b), m = rd_f16(b + 2);
#pragma unroll
    for (int t = 0; t < 8; t += 2) {
      const uint32_t q = b[4 + ((e0 + t) >> 1)];
      v[t] = __fadd_rn(__fmul_rn(i2f_small((int)(q & 15)), d), m);
      v[t + 1] = __fadd_rn(__fmul_rn(i2f_small((int)(q >> 4)), d), m);
    }
  }
};

// Q5_0 (gguf_dequant.py:78-105): d @0, qh u32 @2, nibbles @6 (interleaved);
// bit i of qh is bit 4 of element i; (q - 16) * d.
template <> struct QT<T_Q5_0> {
  static constexpr int QK = 32, REC = 22;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f16(b);
    const uint32_t qh = rd_u32(b + 2);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int i = e0 + t;
      const uint32_t nib = (b[6 + (i >> 1)] >> ((i & 1) * 4)) & 15;
      const int q = (int)(nib | (((qh >> i) & 1) << 4)) - 16;
      v[t] = __fmul_rn(i2f_small(q), d);
    }
  }
};

// Q5_1 (gguf_dequant.py:111-137): d @0, m @2, qh @4, nibbles @8; q*d + m.
template <> struct QT<T_Q5_1> {
  static constexpr int QK = 32, REC = 24;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f16(b), m = rd_f16(b + 2);
    const uint32_t qh = rd_u32(b + 4);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int i = e0 + t;
      const uint32_t nib = (b[8 + (i >> 1)] >> ((i & 1) * 4)) & 15;
      const int q = (int)(nib | (((qh >> i) & 1) << 4));
      v[t] = __fadd_rn(__fmul_rn(i2f_small(q), d), m);
    }
  }
};

// Q8_0 (gguf_dequant.py:143-156): d @0, 32 x int8 @2; q * d.
template <> struct QT<T_Q8_0> {
  static constexpr int QK = 32, REC = 34;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f16(b);
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(i2f_small((int)(int8_t)b[2 + e0 + t]), d);
  }
};

// Q8_1 as the reference lays it out (gguf_dequant.py:162-176): fp32 d @0,
// fp32 m @4, 32 x int8 @8; (q * d) + m with two roundings.
template <> struct QT<T_Q8_1> {
  static constexpr int QK = 32, REC = 40;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f32(b), m = rd_f32(b + 4);
#pragma unroll
    for (int t = 0; t < 8; ++t)
      v[t] = __fadd_rn(__fmul_rn(i2f_small((int)(int8_t)b[8 + e0 + t]), d), m);
  }
};

// Q2_K (gguf_dequant.py:183-223): scales[16] @0, qs[64] @16, d @80, dmin @82.
// Output 128h + 32j + 16p + l: sc = scales[8h + 2j + p],
// q = (qs[32h + 16p + l] >> 2j) & 3, value (d*(sc&15))*q - dmin*(sc>>4).
// All products are exact in fp32; the one rounding is the subtraction, as in
// the reference's float64-then-float32 evaluation.
template <> struct QT<T_Q2_K> {
  static constexpr int QK = 256, REC = 84;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const int h = e0 >> 7, r = e0 & 127, j = r >> 5, p = (r >> 4) & 1, l0 = r & 15;
    const uint32_t sc = b[8 * h + 2 * j + p];
    const float dl = __fmul_rn(rd_f16(b + 80), i2f_small((int)(sc & 15)));
    const float ml = __fmul_rn(rd_f16(b + 82), i2f_small((int)(sc >> 4)));
    const uint8_t* q = b + 16 + 32 * h + 16 * p + l0;
#pragma unroll
    for (int t = 0; t < 8; ++t)
      v[t] = __fsub_rn(__fmul_rn(dl, i2f_small((int)((q[t] >> (2 * j)) & 3))), ml);
  }
};

// Q3_K (gguf_dequant.py:233-293): hmask[32] @0, qs[64] @32, scales12 @96,
// d @108.  Scale i (0..15) is unpacked with the kmask1/kmask2 shuffle of
// gguf_dequant.py:247-262; output 128h + 32j + 16p + l uses scale 8h+2j+p,
// q = ((qs[32h + 16p + l] >> 2j) & 3) - (hmask[16p + l] bit (4h+j) ? 0 : 4);
// value (d * (sc - 32)) * q, exact.
template <> struct QT<T_Q3_K> {
  static constexpr int QK = 256, REC = 110;
  XM_DEV static int scale(const uint8_t* s, int i) {
    // bytes of the four u32 words after the shuffle
    if (i < 4) return (s[i] & 15) | (((s[8 + i] >> 0) & 3) << 4);
    if (i < 8) return (s[i] & 15) | (((s[8 + i - 4] >> 2) & 3) << 4);
    if (i < 12) return (s[i - 8] >> 4) | (((s[8 + i - 8] >> 4) & 3) << 4);
    return (s[i - 8] >> 4) | (((s[8 + i - 12] >> 6) & 3) << 4);
  }
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const int h = e0 >> 7, r = e0 & 127, j = r >> 5, p = (r >> 4) & 1, l0 = r & 15;
    const int sc = scale(b + 96, 8 * h + 2 * j + p);
    const float dl = __fmul_rn(rd_f16(b + 108), i2f_small(sc - 32));
    const uint32_t mbit = 1u << (4 * h + j);
    const uint8_t* q = b + 32 + 32 * h + 16 * p + l0;
    const uint8_t* hm = b + 16 * p + l0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int qq = (int)((q[t] >> (2 * j)) & 3) - ((hm[t] & mbit) ? 0 : 4);
      v[t] = __fmul_rn(dl, i2f_small(qq));
    }
  }
};

// 6-bit scale/min pair j of the 12 packed bytes (gguf_dequant.py:299-306).
XM_DEV void k4_scale_min(const uint8_t* s, int j, int& sc, int& mn) {
  if (j < 4) {
    sc = s[j] & 63;
    mn = s[j + 4] & 63;
  } else {
    sc = (s[j + 4] & 15) | ((s[j - 4] >> 6) << 4);
    mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
  }
}

// Q4_K (gguf_dequant.py:309-341): d @0, dmin @2, scales12 @4, qs[128] @16.
// Sub-block s: q = (qs[32*(s/2) + l] >> 4*(s%2)) & 15;
// value (d*sc[s])*q - dmin*mn[s].
template <> struct QT<T_Q4_K> {
  static constexpr int QK = 256, REC = 144;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const int s = e0 >> 5, l0 = e0 & 31;
    int sc, mn;
    k4_scale_min(b + 4, s, sc, mn);
    const float d1 = __fmul_rn(rd_f16(b), i2f_small(sc));
    const float m1 = __fmul_rn(rd_f16(b + 2), i2f_small(mn));
    const uint8_t* q = b + 16 + 32 * (s >> 1) + l0;
    const int sh = 4 * (s & 1);
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __fsub_rn(__fmul_rn(d1, i2f_small((q[t] >> sh) & 15)), m1);
  }
};

// Q5_K (gguf_dequant.py:347-386): d @0, dmin @2, scales12 @4, qh[32] @16,
// qs[128] @48.  The reference's high bit for element l of sub-block s is bit l
// of the little-endian u32 qh[4*(s/2) .. 4*(s/2)+3] (gguf_dequant.py:372-381);
// value (d*sc[s])*(q + 16*hb) - dmin*mn[s].
template <> struct QT<T_Q5_K> {
  static constexpr int QK = 256, REC = 176;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const int s = e0 >> 5, l0 = e0 & 31, g = s >> 1;
    int sc, mn;
    k4_scale_min(b + 4, s, sc, mn);
    const float d1 = __fmul_rn(rd_f16(b), i2f_small(sc));
    const float m1 = __fmul_rn(rd_f16(b + 2), i2f_small(mn));
    const uint32_t qh = rd_u32(b + 16 + 4 * g);
    const uint8_t* q = b + 48 + 32 * g + l0;
    const int sh = 4 * (s & 1);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int qq = (int)((q[t] >> sh) & 15) + 16 * (int)((qh >> (l0 + t)) & 1);
      v[t] = __fsub_rn(__fmul_rn(d1, i2f_small(qq)), m1);
    }
  }
};

// Q6_K (gguf_dequant.py:392-436): ql[128] @0, qh[64] @128, int8 sc[16] @192,
// d @208.  Output 128h + 32i + l: low nibble (i < 2) or high nibble (i >= 2)
// of ql[64h + 32*(i&1) + l], bits 2i..2i+1 of qh[32h + l] as bits 4-5, minus
// 32; value (d * sc[8h + l/16 + 2i]) * q, exact.
template <> struct QT<T_Q6_K> {
  static constexpr int QK = 256, REC = 210;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const int h = e0 >> 7, r = e0 & 127, i = r >> 5, l0 = r & 31;
    const float ds = __fmul_rn(rd_f16(b + 208), i2f_small((int)(int8_t)b[192 + 8 * h + (l0 >> 4) + 2 * i]));
    const uint8_t* ql = b + 64 * h + 32 * (i & 1) + l0;
    const uint8_t* qh = b + 128 + 32 * h + l0;
    const int nsh = 4 * (i >> 1), hsh = 2 * i;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const int q = (int)(((ql[t] >> nsh) & 15) | (((qh[t] >> hsh) & 3) << 4)) - 32;
      v[t] = __fmul_rn(ds, i2f_small(q));
    }
  }
};

// Q8_K (gguf_dequant.py:442-455): fp32 d @0, int8 qs[256] @4, bsums ignored.
template <> struct QT<T_Q8_K> {
  static constexpr int QK = 256, REC = 292;
  XM_DEV static void decode8(const uint8_t* b, int e0, float* v) {
    const float d = rd_f32(b);
#pragma unroll
    for (int t = 0; t < 8; ++t) v[t] = __fmul_rn(i2f_small((int)(int8_t)b[4 + e0 + t]), d);
  }
};

// Calls F.template operator()<T>() for the runtime type id; returns false for
// types that are not block-quantized.
template <typename F>
inline bool dispatch_quant(int qtype, F&& f) {
  switch (qtype) {
    case T_Q4_0: f.template operator()<T_Q4_0>(); return true;
    case T_Q4_1: f.template operator()<T_Q4_1>(); return true;
    case T_Q5_0: f.template operator()<T_Q5_0>(); return true;
    case T_Q5_1: f.template operator()<T_Q5_1>(); return true;
    case T_Q8_0: f.template operator()<T_Q8_0>(); return true;
    case T_Q8_1: f.template operator()<T_Q8_1>(); return true;
    case T_Q2_K: f.template operator()<T_Q2_K>(); return true;
    case T_Q3_K: f.template operator()<T_Q3_K>(); return true;
    case T_Q4_K: f.template operator()<T_Q4_K>(); return true;
    case T_Q5_K: f.template operator()<T_Q5_K>(); return true;
    case T_Q6_K: f.template operator()<T_Q6_K>(); return true;
    case T_Q8_K: f.template operator()<T_Q8_K>(); return true;
    default: return false;
  }
}

// Host-side geometry (qk, record bytes); false if unknown.
bool host_qtype_geometry(int qtype, int* qk, int* rec);
