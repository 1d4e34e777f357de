// Integer-dot GEMV for Q4_K, Q5_K, Q6_K and Q8_0 weights, y[m][n] = sum_k
// x[m][k] * W[n][k] for 1 <= m <= 8 and any row length K (K % 128 == 0,
// K <= 16384), plus the activation prologues the decoder layers need.
//
// Numerics are those of the Q4_K kernels: x is split per 32-element group
// into two int8 digit planes, x ~= t * (254*X0 + X1), and each weight's
// integer code is multiplied against both planes with dp4a (exact in int32);
// the per-(sub-)block scales and offsets are applied once per 16 or 32
// weights in fp32:
//   Q4_K / Q5_K  sub-block of 32: d*sc * t*P - dmin*mn * sum(x)
//   Q6_K         half-block of 16: d*sc * (t*P - 32 * sum(x))   (codes 0..63)
//   Q8_0         block of 32:      d * t*P                      (signed codes)
//
// Structure (one CTA per SM): a producer warp streams whole rows into a ring
// of shared-memory slots with cp.async.bulk (no multicast), R rows per copy;
// 8 consumer warps (224 registers per thread) take work items from shared
// counters.  A row is cut into "units" of 128 elements (a half super-block, or
// four Q8_0 blocks); rows of more than 32 units are cut into P = 2 or 4 parts,
// and consumer warp w always serves part w % P, so with one activation row the
// digits of the lane's unit stay in registers for the whole kernel.  A work
// item is one part of RI = 2 * 32 / L rows (L lanes per row, one unit per
// lane, two rows per lane: two independent dot products share the digits);
// the P partial sums of a row meet in shared memory and the warp that finishes
// last adds them in part order (deterministic).  With 2..8 activation rows the
// digits live in shared memory instead.
#include <algorithm>

#include "xm_gemv_dot.cuh"
#include "xm_internal.h"

namespace {

constexpr int kKqConsumers = 8;    // + the producer: 288 threads, up to 224 registers each
constexpr int kKqThreads = (kKqConsumers + 1) * 32;
constexpr int kUnitX = 336;       // shared bytes per (activation row, unit): 256 B digits, 4 x float4, 16 B pad
constexpr int kPieceBytes = 64;   // digits per 32-element group in the split workspace
constexpr int kMaxSlots = 64;
constexpr int kCtlBytes = 1536;   // full[64], empty[64] mbarriers; slot tags[64]; part counters[4]
constexpr int kMaxSmem = 227 * 1024;

// ---------------------------------------------------------------------------
// Per-type unit decoders.  load() pulls the unit's weight bytes out of the
// shared-memory ring into registers.  dot2() returns the dot products of two
// units (two rows, same columns) with one activation row's digits of the
// unit's four 32-element groups (x[j]: words 0-7 plane 0, 8-15 plane 1; ts[j] =
// (t, s_lo, s_hi, s32)).  The integer loops run word-major over all groups and
// both rows, so every dp4a chain is at most 4-8 deep and 16-32 chains are
// independent.
// ---------------------------------------------------------------------------
template <int T> struct Unit;

// Q4_K (gguf_dequant.py:309-341): unit h of a record = sub-blocks 4h..4h+3,
// codes in qs[64h .. 64h+63] (low nibble: even sub-block, high: odd).
template <> struct Unit<T_Q4_K> {
  float d, dmin;
  uint32_t scw, mnw, qs[16];
  XM_DEV static const uint8_t* rec(const uint8_t* row, int u) { return row + (u >> 1) * 144; }
  XM_DEV void load(const uint8_t* r, int h) {
    const uint4 hd = lds_v4(r);
    d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
    dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    scw = h == 0 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
    mnw = h == 0 ? (hd.z & 0x3F3F3F3Fu) : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = lds_v4(r + 16 + 64 * h + 16 * i);
      qs[4 * i] = v.x; qs[4 * i + 1] = v.y; qs[4 * i + 2] = v.z; qs[4 * i + 3] = v.w;
    }
  }
  XM_DEV static void dot2(const Unit (&w)[2], const uint32_t (&x)[4][16], const float4 (&ts)[4], float (&out)[2]) {
    int D[2][4][2];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) D[r][j][0] = D[r][j][1] = 0;
#pragma unroll
    for (int wd = 0; wd < 8; ++wd)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t q = w[r].qs[8 * (j >> 1) + wd];
          const uint32_t v = (j & 1) ? (q & 0xF0F0F0F0u) : (q & 0x0F0F0F0Fu);   // odd: 16x the code
          D[r][j][0] = dp4a_us(v, x[j][wd], D[r][j][0]);
          D[r][j][1] = dp4a_us(v, x[j][8 + wd], D[r][j][1]);
        }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float P = __int2float_rn(254 * D[r][j][0] + D[r][j][1]);
        a = fmaf(byte_f(w[r].scw, j) * ((j & 1) ? 0.0625f * ts[j].x : ts[j].x), P, a);
        b = fmaf(byte_f(w[r].mnw, j), ts[j].w, b);
      }
      out[r] = w[r].d * a - w[r].dmin * b;
    }
  }
};

// Q5_K (gguf_dequant.py:347-386) with the reference's high-bit layout: bit l
// of the little-endian u32 qh[4*(s/2) ..] is the fifth bit of element l of
// sub-blocks s and s+1 alike (gguf_dequant.py:372-381).
template <> struct Unit<T_Q5_K> {
  float d, dmin;
  uint32_t scw, mnw, qh[2], qs[16];
  XM_DEV static const uint8_t* rec(const uint8_t* row, int u) { return row + (u >> 1) * 176; }
  XM_DEV void load(const uint8_t* r, int h) {
    const uint4 hd = lds_v4(r);
    d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
    dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
    scw = h == 0 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u));
    mnw = h == 0 ? (hd.z & 0x3F3F3F3Fu) : (((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u));
    const uint2 hw = *reinterpret_cast<const uint2*>(r + 16 + 8 * h);
    qh[0] = hw.x;
    qh[1] = hw.y;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = lds_v4(r + 48 + 64 * h + 16 * i);
      qs[4 * i] = v.x; qs[4 * i + 1] = v.y; qs[4 * i + 2] = v.z; qs[4 * i + 3] = v.w;
    }
  }
  XM_DEV static void dot2(const Unit (&w)[2], const uint32_t (&x)[4][16], const float4 (&ts)[4], float (&out)[2]) {
    int D[2][4][2];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) D[r][j][0] = D[r][j][1] = 0;
#pragma unroll
    for (int wd = 0; wd < 8; ++wd)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t q = w[r].qs[8 * (j >> 1) + wd];
          const uint32_t nib = (j & 1) ? ((q >> 4) & 0x0F0F0F0Fu) : (q & 0x0F0F0F0Fu);
          // bits 4wd..4wd+3 of the high-bit word -> bit 4 of bytes 0..3 (partial products do not overlap)
          const uint32_t fifth = (((w[r].qh[j >> 1] >> (4 * wd)) & 0xFu) * 0x02040810u) & 0x10101010u;
          const uint32_t v = nib | fifth;
          D[r][j][0] = dp4a_us(v, x[j][wd], D[r][j][0]);
          D[r][j][1] = dp4a_us(v, x[j][8 + wd], D[r][j][1]);
        }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.f, b = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float P = __int2float_rn(254 * D[r][j][0] + D[r][j][1]);
        a = fmaf(byte_f(w[r].scw, j) * ts[j].x, P, a);
        b = fmaf(byte_f(w[r].mnw, j), ts[j].w, b);
      }
      out[r] = w[r].d * a - w[r].dmin * b;
    }
  }
};

// Q6_K (gguf_dequant.py:392-436): unit h = elements 128h .. 128h+127.  Group j
// of the unit takes the low (j < 2) or high nibble of ql[64h + 32(j&1) + l],
// bits 2j, 2j+1 of qh[32h + l] as bits 4-5, and the int8 scales sc[8h + 2j]
// (l < 16) and sc[8h + 2j + 1] (l >= 16).  Records are 210 bytes, so fields
// are read with aligned 32-bit loads joined by funnel shifts.
template <> struct Unit<T_Q6_K> {
  float d;
  uint32_t ql[16], qh[8], sc[2];
  XM_DEV static const uint8_t* rec(const uint8_t* row, int u) { return row + (u >> 1) * 210; }
  XM_DEV void load(const uint8_t* r, int h) {
    lds_words<16>(r + 64 * h, ql);
    lds_words<8>(r + 128 + 32 * h, qh);
    lds_words<2>(r + 192 + 8 * h, sc);
    d = __half2float(*reinterpret_cast<const __half*>(r + 208));
  }
  XM_DEV static void dot2(const Unit (&w)[2], const uint32_t (&x)[4][16], const float4 (&ts)[4], float (&out)[2]) {
    int D[2][4][2][2];   // [row][group][half of 16][plane]
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) D[r][j][0][0] = D[r][j][0][1] = D[r][j][1][0] = D[r][j][1][1] = 0;
#pragma unroll
    for (int wd = 0; wd < 8; ++wd)
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const uint32_t l0 = w[r].ql[wd], l1 = w[r].ql[8 + wd], hq = w[r].qh[wd];
        const uint32_t v[4] = {(l0 & 0x0F0F0F0Fu) | ((hq << 4) & 0x30303030u),
                               (l1 & 0x0F0F0F0Fu) | ((hq << 2) & 0x30303030u),
                               ((l0 >> 4) & 0x0F0F0F0Fu) | (hq & 0x30303030u),
                               ((l1 >> 4) & 0x0F0F0F0Fu) | ((hq >> 2) & 0x30303030u)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          D[r][j][wd >> 2][0] = dp4a_us(v[j], x[j][wd], D[r][j][wd >> 2][0]);
          D[r][j][wd >> 2][1] = dp4a_us(v[j], x[j][8 + wd], D[r][j][wd >> 2][1]);
        }
      }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float PA = __int2float_rn(254 * D[r][j][0][0] + D[r][j][0][1]);
        const float PB = __int2float_rn(254 * D[r][j][1][0] + D[r][j][1][1]);
        const float sa = sbyte_f(w[r].sc[j >> 1], (2 * j) & 3), sb = sbyte_f(w[r].sc[j >> 1], (2 * j + 1) & 3);
        a = fmaf(sa, fmaf(ts[j].x, PA, -32.0f * ts[j].y), a);
        a = fmaf(sb, fmaf(ts[j].x, PB, -32.0f * ts[j].z), a);
      }
      out[r] = w[r].d * a;
    }
  }
};

// Q8_0 (gguf_dequant.py:143-156): a unit is four 34-byte blocks, block j =
// group j: fp16 d, then 32 signed codes.
template <> struct Unit<T_Q8_0> {
  float d[4];
  uint32_t qs[4][8];
  XM_DEV static const uint8_t* rec(const uint8_t* row, int u) { return row + u * 136; }
  XM_DEV void load(const uint8_t* r, int) {
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      d[b] = __half2float(*reinterpret_cast<const __half*>(r + 34 * b));
      lds_words<8>(r + 34 * b + 2, qs[b]);
    }
  }
  XM_DEV static void dot2(const Unit (&w)[2], const uint32_t (&x)[4][16], const float4 (&ts)[4], float (&out)[2]) {
    int D[2][4][2];
#pragma unroll
    for (int r = 0; r < 2; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) D[r][j][0] = D[r][j][1] = 0;
#pragma unroll
    for (int wd = 0; wd < 8; ++wd)
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          D[r][j][0] = dp4a_ss(w[r].qs[j][wd], x[j][wd], D[r][j][0]);
          D[r][j][1] = dp4a_ss(w[r].qs[j][wd], x[j][8 + wd], D[r][j][1]);
        }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      float a = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) a = fmaf(w[r].d[j] * ts[j].x, __int2float_rn(254 * D[r][j][0] + D[r][j][1]), a);
      out[r] = a;
    }
  }
};

struct KqArgs {
  const uint8_t* W;
  float* y;
  const float* bias;
  const int8_t* pieces;   // group-major split: [m][G][64]
  const float4* ts;       // [m][G]
  int N, RB, U, P, UP, L, R, S, slot_bytes, G, accumulate, max_rows;
};

template <int T, int M>
__global__ void __launch_bounds__(kKqThreads, 1) k_qgemv_kq(const __grid_constant__ KqArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + kMaxSlots;
  int* slot_tag = reinterpret_cast<int*>(empty + kMaxSlots);
  int* part_next = slot_tag + kMaxSlots;
  uint8_t* ring = sm + kCtlBytes;
  uint8_t* xs = ring + (size_t)a.S * a.slot_bytes;                                  // M > 1: [M][U][kUnitX]
  float* part = reinterpret_cast<float*>(xs + (M > 1 ? (size_t)M * a.U * kUnitX : 0));  // P > 1: [rows][P][M]
  int* row_cnt = reinterpret_cast<int*>(part + (a.P > 1 ? (size_t)a.max_rows * a.P * M : 0));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nchunks_all = (a.N + a.R - 1) / a.R;
  const int q0 = (int)((int64_t)nchunks_all * blockIdx.x / gridDim.x);
  const int q1 = (int)((int64_t)nchunks_all * (blockIdx.x + 1) / gridDim.x);
  const int rb = q0 * a.R;
  const int nrows = min(a.N, q1 * a.R) - rb;
  const int nch = q1 - q0;
  const int RL = 32 / a.L;          // rows covered by the warp's lanes at once
  const int RI = 2 * RL;             // rows per work item (each lane takes two)
  const int ngroups = (nrows + RI - 1) / RI;
  grid_dep_launch();   // the next kernel only prefetches its weights before its own wait

  if (tid == 0) {
    for (int i = 0; i < a.S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], (a.R / RI) * a.P);   // one arrival per work item
      slot_tag[i] = -1;
    }
    for (int p = 0; p < 4; ++p) part_next[p] = 0;
    fence_mbar_init();
  }
  if (a.P > 1)
    for (int i = tid; i < a.max_rows; i += kKqThreads) row_cnt[i] = 0;
  __syncthreads();

  if (warp == kKqConsumers) {
    // producer: weights only, so it does not wait for the preceding kernel
    if (lane == 0) {
      for (int q = 0; q < nch; ++q) {
        const int slot = q % a.S;
        if (q >= a.S) mbar_wait_bounded(&empty[slot], (uint32_t)(((q / a.S) - 1) & 1));
        *(volatile int*)&slot_tag[slot] = q;
        const int rows = min(a.R, nrows - q * a.R);
        const uint32_t bytes = (uint32_t)rows * (uint32_t)a.RB;
        const uint32_t bulk = bytes & ~15u;
        const uint8_t* src = a.W + (int64_t)(rb + q * a.R) * a.RB;
        uint8_t* dst = ring + (size_t)slot * a.slot_bytes;
        for (uint32_t i = bulk; i < bytes; ++i) dst[i] = src[i];   // ragged tail of the last rows (< 16 B)
        mbar_arrive_expect_tx(&full[slot], bulk);
        if (bulk) bulk_g2s(dst, src, bulk, &full[slot]);
      }
    }
    return;
  }

  const int p = warp % a.P;
  const int c = lane % a.L;
  const int u = p * a.UP + c;
  const bool uvalid = c < a.UP && u < a.U;
  const int h = u & 1;

  grid_dep_wait();   // the activation split is written by the preceding kernel
  uint32_t xr[4][16];
  float4 tr[4];
  if constexpr (M == 1) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (uvalid) {
        const uint4* src = reinterpret_cast<const uint4*>(a.pieces + (int64_t)(4 * u + j) * kPieceBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = src[i];
          xr[j][4 * i] = v.x; xr[j][4 * i + 1] = v.y; xr[j][4 * i + 2] = v.z; xr[j][4 * i + 3] = v.w;
        }
        tr[j] = a.ts[4 * u + j];
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) xr[j][i] = 0;
        tr[j] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
  } else {
    const int nchunk = M * a.U * 20;   // 16 digit chunks + 4 (t, sums) per (row, unit)
    for (int i = tid; i < nchunk; i += kKqConsumers * 32) {
      const int mu = i / 20, k = i - mu * 20;
      const int m = mu / a.U, uu = mu - m * a.U;
      uint4 v;
      if (k < 16)
        v = *reinterpret_cast<const uint4*>(a.pieces + ((int64_t)m * a.G + 4 * uu) * kPieceBytes + 16 * k);
      else
        v = *reinterpret_cast<const uint4*>(&a.ts[(int64_t)m * a.G + 4 * uu + (k - 16)]);
      *reinterpret_cast<uint4*>(xs + (size_t)mu * kUnitX + 16 * k) = v;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kKqConsumers * 32) : "memory");   // consumer warps only
  }

  // a work item: rows row0 + lane/L and row0 + lane/L + RL (two independent
  // dot products per lane), one part of each
  for (;;) {
    int gi = 0;
    if (lane == 0) gi = atomicAdd(&part_next[p], 1);
    gi = __shfl_sync(0xffffffffu, gi, 0);
    if (gi >= ngroups) break;
    const int row0 = gi * RI, q = row0 / a.R, slot = q % a.S;
    smem_wait_eq(&slot_tag[slot], q);   // armed for this chunk, not the previous lap
    mbar_wait_bounded(&full[slot], (uint32_t)((q / a.S) & 1));
    const int rowA = row0 + lane / a.L, rowB = rowA + RL;
    const bool okA = uvalid && rowA < nrows, okB = uvalid && rowB < nrows;
    const uint8_t* base = ring + (size_t)slot * a.slot_bytes;
    Unit<T> w2[2];
    if (okA) w2[0].load(Unit<T>::rec(base + (size_t)(rowA - q * a.R) * a.RB, u), h);
    if (okB) w2[1].load(Unit<T>::rec(base + (size_t)(rowB - q * a.R) * a.RB, u), h);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);   // every lane holds its weights in registers
    float accA[M], accB[M];
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float o2[2];
      if constexpr (M == 1) {
        Unit<T>::dot2(w2, xr, tr, o2);
      } else {
        // lanes past the row's last unit read unit 0 (their result is dropped)
        const uint8_t* xu = xs + ((size_t)m * a.U + (uvalid ? u : 0)) * kUnitX;
        uint32_t x[4][16];
        float4 t4[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = lds_v4(xu + 64 * j + 16 * i);
            x[j][4 * i] = v.x; x[j][4 * i + 1] = v.y; x[j][4 * i + 2] = v.z; x[j][4 * i + 3] = v.w;
          }
          t4[j] = *reinterpret_cast<const float4*>(xu + 256 + 16 * j);
        }
        Unit<T>::dot2(w2, x, t4, o2);
      }
      accA[m] = okA ? o2[0] : 0.f;
      accB[m] = okB ? o2[1] : 0.f;
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float va = accA[m], vb = accB[m];
      for (int o = a.L >> 1; o > 0; o >>= 1) {
        va += __shfl_xor_sync(0xffffffffu, va, o);
        vb += __shfl_xor_sync(0xffffffffu, vb, o);
      }
      accA[m] = va;
      accB[m] = vb;
    }
    if (c == 0) {
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int row = k ? rowB : rowA;
        if (row >= nrows) continue;
        const int64_t grow = rb + row;
        if (a.P == 1) {
#pragma unroll
          for (int m = 0; m < M; ++m) {
            float v = (k ? accB[m] : accA[m]) + (a.bias ? a.bias[grow] : 0.f);
            if (a.accumulate) v = a.y[(int64_t)m * a.N + grow] + v;
            a.y[(int64_t)m * a.N + grow] = v;
          }
        } else {
#pragma unroll
          for (int m = 0; m < M; ++m) part[((size_t)row * a.P + p) * M + m] = k ? accB[m] : accA[m];
          __threadfence_block();
          if (atomicAdd(&row_cnt[row], 1) == a.P - 1) {
            __threadfence_block();
#pragma unroll
            for (int m = 0; m < M; ++m) {
              const volatile float* pr = part + (size_t)row * a.P * M + m;
              float v = pr[0];
              for (int pp = 1; pp < a.P; ++pp) v += pr[pp * M];
              v += a.bias ? a.bias[grow] : 0.f;
              if (a.accumulate) v = a.y[(int64_t)m * a.N + grow] + v;
              a.y[(int64_t)m * a.N + grow] = v;
            }
          }
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Activation split with a prologue, one CTA per activation row:
//   XM_PRO_NONE     v = x
//   XM_PRO_RMSNORM  v = (x / sqrt(mean(x^2) + eps)) * w   (ops.py:107-123, primitives.py:20-23)
//   XM_PRO_SWIGLU   v = silu(x[:K]) * x[K:2K]             (forward.py:97-98, primitives.py:37-44)
// Output: the group-major split (digits [m][G][64], (t, s_lo, s_hi, s32) [m][G]).
// ---------------------------------------------------------------------------
// Grid (rows, ceil(G / kSplitGroups)): each CTA splits kSplitGroups groups of
// its row (with RMSNorm every CTA first reduces the whole row, 16-56 KB from L2).
constexpr int kSplitGroups = 16;

template <typename XT, int PRO>
__global__ void __launch_bounds__(256) k_split_rows(const XT* __restrict__ x, int64_t x_stride, int K,
                                                    const float* __restrict__ norm_w, float eps,
                                                    int8_t* __restrict__ pieces, float4* __restrict__ ts) {
  __shared__ float red[8];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const XT* xr = x + (int64_t)m * x_stride;
  const int G = K / 32;
  const int g_begin = blockIdx.y * kSplitGroups, g_end = min(G, g_begin + kSplitGroups);
  float rms = 1.f;
  if constexpr (PRO == XM_PRO_RMSNORM) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += 256) {
      const float v = to_f32(xr[i]);
      ss = fmaf(v, v, ss);
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    rms = sqrtf(tot / (float)K + eps);
  }
  for (int g = g_begin + warp; g < g_end; g += 8) {
    const int k = g * 32 + lane;
    float v;
    if constexpr (PRO == XM_PRO_SWIGLU) {
      const float gt = to_f32(xr[k]), up = to_f32(xr[K + k]);
      v = gt / (1.0f + expf(-gt)) * up;
    } else if constexpr (PRO == XM_PRO_RMSNORM) {
      v = (to_f32(xr[k]) / rms) * norm_w[k];
    } else {
      v = to_f32(xr[k]);
    }
    int x0, x1;
    float t, s_lo, s_hi;
    split_group(v, x0, x1, t, s_lo, s_hi);
    const int64_t grp = (int64_t)m * G + g;
    pieces[grp * kPieceBytes + lane] = (int8_t)x0;
    pieces[grp * kPieceBytes + 32 + lane] = (int8_t)x1;
    if (lane == 0) ts[grp] = make_float4(t, s_lo, s_hi, s_lo + s_hi);
  }
}

// Launch with programmatic dependent launch allowed (the kernel calls griddepcontrol.wait
// before it reads anything the preceding kernel writes).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int T, int M>
int launch_kq(const KqArgs& a, int smem, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemv_kq<T, M>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
    if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv: smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int nchunks = (a.N + a.R - 1) / a.R;
  const int grid = std::min(xm_sm_count(), nchunks);
  cudaError_t e = launch_pdl(k_qgemv_kq<T, M>, dim3(grid), dim3(kKqThreads), smem, st, a);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemv(integer, generic)");
}

template <int T>
int launch_kq_m(int64_t m, const KqArgs& a, int smem, cudaStream_t st) {
  switch (m) {
    case 1: return launch_kq<T, 1>(a, smem, st);
    case 2: return launch_kq<T, 2>(a, smem, st);
    case 3: return launch_kq<T, 3>(a, smem, st);
    case 4: return launch_kq<T, 4>(a, smem, st);
    case 5: return launch_kq<T, 5>(a, smem, st);
    case 6: return launch_kq<T, 6>(a, smem, st);
    case 7: return launch_kq<T, 7>(a, smem, st);
    default: return launch_kq<T, 8>(a, smem, st);
  }
}

int rec_bytes(int qtype) {
  switch (qtype) {
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q8_0: return 34;
    default: return 0;
  }
}
int qk_of(int qtype) { return qtype == T_Q8_0 ? 32 : 256; }

// Geometry of a launch; false if the shape does not fit the kernel.
bool plan(int qtype, int64_t n, int64_t k, int64_t m, KqArgs& a, int& smem) {
  const int rec = rec_bytes(qtype);
  if (!rec || k % 128 || k > 16384 || k % qk_of(qtype) || m < 1 || m > 8) return false;
  const int U = (int)(k / 128);
  const int P = U <= 32 ? 1 : U <= 64 ? 2 : 4;
  const int UP = (U + P - 1) / P;
  int L = 1;
  while (L < UP) L <<= 1;
  const int RI = 2 * (32 / L);   // rows per work item
  const int64_t RB = k / qk_of(qtype) * rec;
  int r0 = 1;
  while ((r0 * RB) % 16) r0 <<= 1;
  int R = std::max(r0, RI);
  if (R * RB < 8192) R *= (int)std::max<int64_t>(1, 8192 / (R * RB));
  const int64_t slot_bytes = R * RB;
  const int64_t nchunks = (n + R - 1) / R;
  const int grid = (int)std::min<int64_t>(xm_sm_count(), nchunks);
  const int64_t max_rows = (nchunks + grid - 1) / grid * R;
  const int64_t xs = m > 1 ? m * U * kUnitX : 0;
  const int64_t part = P > 1 ? max_rows * P * m * 4 + max_rows * 4 : 0;
  const int64_t room = kMaxSmem - kCtlBytes - xs - part - 16;
  const int64_t S = std::min<int64_t>(kMaxSlots, room / slot_bytes);
  if (S < 2 || n >= (1ll << 31)) return false;
  a.N = (int)n;
  a.RB = (int)RB;
  a.U = U;
  a.P = P;
  a.UP = UP;
  a.L = L;
  a.R = R;
  a.S = (int)S;
  a.slot_bytes = (int)slot_bytes;
  a.G = (int)(k / 32);
  a.max_rows = (int)max_rows;
  smem = (int)(kCtlBytes + S * slot_bytes + xs + part + 16);
  return true;
}

}  // namespace

bool gemv_kq_supported(int qtype, int64_t n, int64_t k, int64_t m) {
  KqArgs a{};
  int smem = 0;
  return m >= 1 && m <= 8 && plan(qtype, n, k, 1, a, smem);
}

int gemv_kq(int qtype, const uint8_t* W, int64_t n, int64_t k, int64_t m, const void* d_ws, const float* bias,
            float* y, int accumulate, cudaStream_t st) {
  // rows of x are independent: when the digits of all m rows do not fit in
  // shared memory, run the largest row groups that do (each streams W again)
  int64_t ms = m;
  KqArgs a{};
  int smem = 0;
  while (ms > 1 && !plan(qtype, n, k, ms, a, smem)) --ms;
  if (!plan(qtype, n, k, ms, a, smem))
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemv: shape n=%lld k=%lld has no integer-path plan", (long long)n,
                        (long long)k);
  const int64_t G = k / 32;
  const int8_t* pieces = (const int8_t*)d_ws;
  const float4* ts = (const float4*)((const uint8_t*)d_ws + m * G * kPieceBytes);
  for (int64_t m0 = 0; m0 < m; m0 += ms) {
    const int64_t mm = std::min(ms, m - m0);
    if (!plan(qtype, n, k, mm, a, smem))
      return xm_set_error(XM_ERR_UNSUPPORTED, "qgemv: no integer-path plan for %lld rows", (long long)mm);
    a.W = W;
    a.y = y + m0 * n;
    a.bias = bias;
    a.pieces = pieces + m0 * G * kPieceBytes;
    a.ts = ts + m0 * G;
    a.accumulate = accumulate;
    int rc;
    switch (qtype) {
      case T_Q4_K: rc = launch_kq_m<T_Q4_K>(mm, a, smem, st); break;
      case T_Q5_K: rc = launch_kq_m<T_Q5_K>(mm, a, smem, st); break;
      case T_Q6_K: rc = launch_kq_m<T_Q6_K>(mm, a, smem, st); break;
      default: rc = launch_kq_m<T_Q8_0>(mm, a, smem, st); break;
    }
    if (rc) return rc;
  }
  return XM_OK;
}

int split_rows(const void* d_x, int x_dtype, int64_t m, int64_t k, int64_t x_stride, int prologue,
               const float* norm_w, float eps, void* d_ws, cudaStream_t st) {
  int8_t* pieces = (int8_t*)d_ws;
  float4* ts = (float4*)((uint8_t*)d_ws + m * (k / 32) * kPieceBytes);
  cudaError_t e = cudaSuccess;
  const dim3 grid((unsigned)m, (unsigned)((k / 32 + kSplitGroups - 1) / kSplitGroups)), block(256);
#define XM_SPLIT(XT)                                                                                            \
  switch (prologue) {                                                                                           \
    case XM_PRO_RMSNORM:                                                                                        \
      e = launch_pdl(k_split_rows<XT, XM_PRO_RMSNORM>, grid, block, 0, st, (const XT*)d_x, x_stride, (int)k,     \
                     norm_w, eps, pieces, ts);                                                                  \
      break;                                                                                                    \
    case XM_PRO_SWIGLU:                                                                                         \
      e = launch_pdl(k_split_rows<XT, XM_PRO_SWIGLU>, grid, block, 0, st, (const XT*)d_x, x_stride, (int)k,      \
                     norm_w, eps, pieces, ts);                                                                  \
      break;                                                                                                    \
    default:                                                                                                    \
      e = launch_pdl(k_split_rows<XT, XM_PRO_NONE>, grid, block, 0, st, (const XT*)d_x, x_stride, (int)k, norm_w, \
                     eps, pieces, ts);                                                                          \
  }
  if (x_dtype == XM_DT_F32) {
    XM_SPLIT(float)
  } else if (x_dtype == XM_DT_BF16) {
    XM_SPLIT(__nv_bfloat16)
  } else {
    XM_SPLIT(__half)
  }
#undef XM_SPLIT
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "split_rows launch: %s", cudaGetErrorString(e));
  return xm_check_launch("split_rows");
}
