// Word-level decoders of GGUF block records to the reference's fp16 weight
// values, shared by the prefill GEMM (decoded weights written to tensor
// memory) and the standalone dequantization kernel.
//
// Every value is the fp32 value of gguf_dequant.py's unpacker (for Q4_K,
// (d * sc) * q - dmin * mn with exact products), rounded once to fp16; the
// integer codes become floats exactly through a byte permute into the
// 2^23 exponent pattern.
#pragma once
#include "xm_qtypes.cuh"

namespace xm_decode {

// byte i of w as an exact float
XM_DEV float byte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)i)) - 8388608.0f;
}

// NW consecutive 32-bit words at a 2-byte-aligned shared address: 16-byte
// loads of the units that hold them, then funnel shifts.  Reads up to 15
// bytes past the last word.  Fastest when the offset in the 16-byte unit
// (p & 15) is the same for every thread of the warp (one branch taken).
template <int NW>
XM_DEV void smem_words16(const uint8_t* p, uint32_t (&w)[NW]) {
  constexpr int NU = (NW * 4 + 15 + 15) / 16;     // 16-byte units that can hold NW words at any offset
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint4* base = reinterpret_cast<const uint4*>(a & ~(uintptr_t)15);
  uint32_t u[NU * 4];
#pragma unroll
  for (int i = 0; i < NU; ++i) {
    const uint4 v = base[i];
    u[4 * i] = v.x;
    u[4 * i + 1] = v.y;
    u[4 * i + 2] = v.z;
    u[4 * i + 3] = v.w;
  }
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  const int o = (int)((a >> 2) & 3);
  // o is warp-uniform: one branch, each with constant register indices
#define XM_SW16(O)                                                          \
  _Pragma("unroll") for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(u[(O) + i], u[(O) + i + 1], sh)
  if (o == 0) {
    XM_SW16(0);
  } else if (o == 1) {
    XM_SW16(1);
  } else if (o == 2) {
    XM_SW16(2);
  } else {
    XM_SW16(3);
  }
#undef XM_SW16
}

// Four bytes of w (codes b0..b3) as exact floats b - bias, in two pairs:
// 2^23 + b by byte permute into the exponent pattern, minus (2^23 + bias).
XM_DEV void bytes_minus(uint32_t w, float bias, float2& lo, float2& hi) {
  const float2 mg = make_float2(-(8388608.0f + bias), -(8388608.0f + bias));
  lo = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u)),
                              __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7651u))), mg);
  hi = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7652u)),
                              __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7653u))), mg);
}

XM_DEV uint32_t half2_bits(float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Register forms of the item decoders: hv[4c + t] = the fp16 pair of weights
// (8c + 2t, 8c + 2t + 1) of item h (weights 32h .. 32h+31 of K step j).
XM_DEV void q4k_item_regs(const uint8_t* rec, int j, int h, uint32_t (&hv)[16]) {
  const uint4 hd = *reinterpret_cast<const uint4*>(rec);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * j);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * j);
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const uint32_t A = hd.y, B = hd.z, C = hd.w;
  const int sub = 2 * j + h;
  const uint32_t scw = sub < 4 ? (A & 0x3F3F3F3Fu) : ((C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u));
  const uint32_t mnw = sub < 4 ? (B & 0x3F3F3F3Fu) : (((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u));
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  const float d1 = __fmul_rn(d, byte_f(scw, sub & 3));       // exact (11-bit x 6-bit)
  const float m1 = __fmul_rn(dmin, byte_f(mnw, sub & 3));
  const float2 dd = make_float2(d1, d1), mm = make_float2(-m1, -m1);
  const int sh = 4 * h;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    float2 lo, hi;
    bytes_minus((qw[w] >> sh) & 0x0F0F0F0Fu, 0.0f, lo, hi);
    // d1*q is exact, so one rounding of d1*q - m1 is the reference's fp32 value
    hv[2 * w] = half2_bits(__ffma2_rn(dd, lo, mm));
    hv[2 * w + 1] = half2_bits(__ffma2_rn(dd, hi, mm));
  }
}

XM_DEV void q6k_item_regs(const uint8_t* rec, int j, int h, uint32_t (&hv)[16]) {
  const int hh = j >> 1, i = 2 * (j & 1) + h;
  uint32_t ql[8], qh[8];
  smem_words16<8>(rec + 64 * hh + 32 * (i & 1), ql);
  smem_words16<8>(rec + 128 + 32 * hh, qh);
  const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(rec + 208)));
  const float ds0 = d * (float)(int8_t)rec[192 + 8 * hh + 2 * i];       // exact (11-bit x 8-bit)
  const float ds1 = d * (float)(int8_t)rec[192 + 8 * hh + 2 * i + 1];
  const int nsh = 4 * (i >> 1), hsh = 2 * i;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const float ds = w < 4 ? ds0 : ds1;       // weights 0-15 and 16-31 of the item
    const float2 dd = make_float2(ds, ds);
    const uint32_t q = ((ql[w] >> nsh) & 0x0F0F0F0Fu) | (((qh[w] >> hsh) & 0x03030303u) << 4);
    float2 lo, hi;
    bytes_minus(q, 32.0f, lo, hi);
    hv[2 * w] = half2_bits(__fmul2_rn(lo, dd));
    hv[2 * w + 1] = half2_bits(__fmul2_rn(hi, dd));
  }
}

XM_DEV void q5k_item_regs(const uint8_t* rec, int j, int h, uint32_t (&hv)[16]) {
  const uint4 hd = *reinterpret_cast<const uint4*>(rec);
  const int sub = 2 * j + h;
  const uint32_t A = hd.y, B = hd.z, C = hd.w;
  const uint32_t scw = sub < 4 ? (A & 0x3F3F3F3Fu) : ((C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u));
  const uint32_t mnw = sub < 4 ? (B & 0x3F3F3F3Fu) : (((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u));
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  const float d1 = __fmul_rn(d, byte_f(scw, sub & 3));
  const float m1 = __fmul_rn(dmin, byte_f(mnw, sub & 3));
  const float2 dd = make_float2(d1, d1), mm = make_float2(-m1, -m1);
  const uint32_t qh32 = *reinterpret_cast<const uint32_t*>(rec + 16 + 4 * j);
  const uint4 q0 = *reinterpret_cast<const uint4*>(rec + 48 + 32 * j);
  const uint4 q1 = *reinterpret_cast<const uint4*>(rec + 64 + 32 * j);
  const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const int sh = 4 * h;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const uint32_t fifth = (((qh32 >> (4 * w)) & 0xFu) * 0x02040810u) & 0x10101010u;
    float2 lo, hi;
    bytes_minus(((qw[w] >> sh) & 0x0F0F0F0Fu) | fifth, 0.0f, lo, hi);
    hv[2 * w] = half2_bits(__ffma2_rn(dd, lo, mm));
    hv[2 * w + 1] = half2_bits(__ffma2_rn(dd, hi, mm));
  }
}

XM_DEV void q8_0_item_regs(const uint8_t* col, int j, int h, uint32_t (&hv)[16]) {
  const uint8_t* rec = col + (2 * j + h) * 34;
  const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(rec)));
  const float2 dd = make_float2(d, d);
  uint32_t qw[8];
  smem_words16<8>(rec + 2, qw);
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    float2 lo, hi;
    bytes_minus(qw[w] ^ 0x80808080u, 128.0f, lo, hi);   // signed byte b: (b + 128) - 128
    hv[2 * w] = half2_bits(__fmul2_rn(lo, dd));
    hv[2 * w + 1] = half2_bits(__fmul2_rn(hi, dd));
  }
}

template <int T>
XM_DEV void generic_item_regs(const uint8_t* col, int j, int h, uint32_t (&hv)[16]) {
  using Q = QT<T>;
  const uint8_t* rec = Q::QK == 256 ? col : col + (2 * j + h) * Q::REC;
  const int e0 = Q::QK == 256 ? 64 * j + 32 * h : 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float v[8];
    Q::decode8(rec, e0 + 8 * c, v);
#pragma unroll
    for (int p = 0; p < 4; ++p) hv[4 * c + p] = half2_bits(make_float2(v[2 * p], v[2 * p + 1]));
  }
}

template <int T>
XM_DEV void item_regs(const uint8_t* rec, int j, int h, uint32_t (&hv)[16]) {
  if constexpr (T == T_Q4_K) q4k_item_regs(rec, j, h, hv);
  else if constexpr (T == T_Q6_K) q6k_item_regs(rec, j, h, hv);
  else if constexpr (T == T_Q5_K) q5k_item_regs(rec, j, h, hv);
  else if constexpr (T == T_Q8_0) q8_0_item_regs(rec, j, h, hv);
  else generic_item_regs<T>(rec, j, h, hv);
}

}  // namespace xm_decode
