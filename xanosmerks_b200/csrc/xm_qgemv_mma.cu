// Q4_K GEMV for 2..8 activation rows on the tensor cores (integer MMA).
//
// With several activation rows the dp4a path multiplies every weight once per
// row and plane and re-reads the activation digits for every weight row; here
// one warp-wide integer MMA (mma.sync m16n8k32, u8 weight codes x s8
// activation digits, s32 accumulators) covers 16 weight rows x 32 elements (one
// Q4_K sub-block) x 4 activation rows x 2 digit planes, so activation digits
// are read once per 16 weight rows.
//
// Activations are split per row (not per 32-element group) into two int8
// planes, x ~= t * (254*X0 + X1), t = max|x_row| / (127*254), plus the fp32
// sum of x over every 32-element sub-block; so that the sub-block scales can
// be applied in integer arithmetic:
//   y[r][m] = sum over super-blocks of
//             d_r * t_m * (254 * sum_s sc_rs * D0_rsm + sum_s sc_rs * D1_rsm)
//             - dmin_r * sum_s mn_rs * xsum_ms
// with D0/D1 the MMA dot products of the 4-bit codes against the planes
// (exact in int32; sum_s sc*D stays below 2^25 per super-block).
//
// Fragment layout (PTX m16n8k32 .u8/.s8): lane (g = lane/4, q = lane%4) holds
// A bytes at K slots 4q..4q+3 and 16+4q..16+4q+3 of rows g and g+8, B bytes at
// the same K slots of column g, and D columns 2q, 2q+1 of rows g, g+8.  The K
// order inside a sub-block is free as long as A and B agree: slot 4q+i holds
// element 8q+i and slot 16+4q+i element 8q+4+i, so both operands are one
// 8-byte load of 8 consecutive elements.  Columns are (activation row,
// plane) pairs: column 2j + p = row 4*tile + j, plane p, so a lane's two D
// columns are the two planes of one activation row.
//
// The split runs in its own kernel (k_split_tok, one CTA per row and 512
// columns) so that it is done once, not once per GEMV CTA.
//
// Structure: a producer warp copies 16-row tiles into a ring of shared-memory
// slots (one bulk copy per row, padded pitch), 8 consumer warps; a tile's K
// range is cut into P parts (warp w serves part w % P) when the matrix has too
// few tiles to occupy every warp, and the parts' partial sums meet in shared
// memory in part order.  Activation digits of the whole row length stay in
// shared memory for the whole kernel.
#include <algorithm>

#include "xm_gemv_dot.cuh"
#include "xm_internal.h"

namespace {

constexpr int kMmaConsumers = 8;
constexpr int kMmaThreads = (kMmaConsumers + 1) * 32;
constexpr int kTileRows = 16;
constexpr int kMaxSlots = 16;
constexpr int kCtlBytes = 1024;
constexpr int kRec = 144;
constexpr int kMaxSmemMma = 227 * 1024;

XM_DEV void mma_u8s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

struct MmaArgs {
  const uint8_t* W;
  float* y;
  const float* bias;
  const int8_t* planes;   // [M][2][K] activation digits
  const float* tscale;    // [M]
  const float* xsum;      // [M][K/32]
  int N, K, M, P, S, pitch, slot_bytes, xcol, accumulate, max_tiles;
};

// Activation value k of row xr under the prologue (x, RMSNorm, SwiGLU of [gate | up]).
template <typename XT, int PRO>
XM_DEV float pro_value(const XT* xr, int K, int k, float rms, const float* norm_w) {
  if constexpr (PRO == XM_PRO_SWIGLU) {
    const float gt = to_f32(xr[k]), up = to_f32(xr[K + k]);
    return gt / (1.0f + expf(-gt)) * up;
  } else if constexpr (PRO == XM_PRO_RMSNORM) {
    return (to_f32(xr[k]) / rms) * norm_w[k];
  } else {
    return to_f32(xr[k]);
  }
}

// Per-row activation split.  Grid (rows, K / kSliceK): every CTA of a row
// reduces the whole row (sum of squares for RMSNorm, max |v|; for RMSNorm
// max|v| = max|x*w| / rms) in the same order, so all of them derive the same
// scale t = max|v| / (127*254), then writes the digits of v / t and the fp32
// sub-block sums of its slice: planes[m][0|1][k], tscale[m], xsum[m][k/32].
constexpr int kSliceK = 512;

template <typename XT, int PRO>
__global__ void __launch_bounds__(256) k_split_tok(const XT* __restrict__ x, int64_t x_stride, int K,
                                                   const float* __restrict__ norm_w, float eps,
                                                   int8_t* __restrict__ planes, float* __restrict__ tscale,
                                                   float* __restrict__ xsum) {
  __shared__ float red[2][8];
  grid_dep_wait();
  grid_dep_launch();
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const XT* xr = x + (int64_t)m * x_stride;
  float ss = 0.f, mx = 0.f;
  for (int k = tid; k < K; k += 256) {
    if constexpr (PRO == XM_PRO_RMSNORM) {
      const float xv = to_f32(xr[k]);
      ss = fmaf(xv, xv, ss);
      mx = fmaxf(mx, fabsf(xv * norm_w[k]));
    } else {
      mx = fmaxf(mx, fabsf(pro_value<XT, PRO>(xr, K, k, 1.f, norm_w)));
    }
  }
  ss = warp_sum(ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) {
    red[0][warp] = ss;
    red[1][warp] = mx;
  }
  __syncthreads();
  float tot = 0.f, amax = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    tot += red[0][w];
    amax = fmaxf(amax, red[1][w]);
  }
  const float rms = PRO == XM_PRO_RMSNORM ? sqrtf(tot / (float)K + eps) : 1.f;
  if (PRO == XM_PRO_RMSNORM) amax = amax / rms;
  const float sc = amax > 0.f ? amax / 127.0f : 0.f;
  const float inv = amax > 0.f ? 1.0f / sc : 0.f;
  if (blockIdx.y == 0 && tid == 0) tscale[m] = sc / 254.0f;
  // this CTA's slice: 8 consecutive elements per thread, 4 threads per 32-element sub-block
  int8_t* p0 = planes + (int64_t)m * 2 * K;
  int8_t* p1 = p0 + K;
  const int kb = blockIdx.y * kSliceK, ke = min(K, kb + kSliceK);
  for (int k0 = kb + tid * 8; k0 < ke; k0 += 256 * 8) {
    uint32_t w0[2] = {0, 0}, w1[2] = {0, 0};
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = pro_value<XT, PRO>(xr, K, k0 + e, rms, norm_w);
      sum += v;
      const float u = v * inv;
      const float r0 = rintf(u);
      const int x0 = max(-127, min(127, (int)r0));
      const int x1 = max(-127, min(127, (int)rintf((u - r0) * 254.0f)));
      w0[e >> 2] |= (uint32_t)(x0 & 0xFF) << (8 * (e & 3));
      w1[e >> 2] |= (uint32_t)(x1 & 0xFF) << (8 * (e & 3));
    }
    *reinterpret_cast<uint2*>(p0 + k0) = make_uint2(w0[0], w0[1]);
    *reinterpret_cast<uint2*>(p1 + k0) = make_uint2(w1[0], w1[1]);
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((k0 & 31) == 0) xsum[(int64_t)m * (K / 32) + k0 / 32] = sum;
  }
}

template <int NT>
__global__ void __launch_bounds__(kMmaThreads, 1) k_qgemv_q4k_mma(const __grid_constant__ MmaArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(sm);
  uint64_t* empty = full + kMaxSlots;
  int* slot_tag = reinterpret_cast<int*>(empty + kMaxSlots);
  int* part_cnt = slot_tag + kMaxSlots;
  uint8_t* ring = sm + kCtlBytes;
  uint8_t* xs = ring + (size_t)a.S * a.slot_bytes;                       // [8*NT columns][xcol]
  float* ts = reinterpret_cast<float*>(xs + (size_t)8 * NT * a.xcol);    // [4*NT]
  float* xsum = ts + 4 * NT;                                             // [4*NT][K/32]
  float* part = xsum + (size_t)4 * NT * (a.K / 32);                      // [S][P][16 rows][4*NT]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int ntiles_all = (a.N + kTileRows - 1) / kTileRows;
  const int t0 = (int)((int64_t)ntiles_all * blockIdx.x / gridDim.x);
  const int t1 = (int)((int64_t)ntiles_all * (blockIdx.x + 1) / gridDim.x);
  const int ntiles = t1 - t0;
  const int nb = a.K / 256;
  const int64_t row_bytes = (int64_t)nb * kRec;
  grid_dep_launch();

  if (tid == 0) {
    for (int i = 0; i < a.S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], a.P);
      slot_tag[i] = -1;
      part_cnt[i] = 0;
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kMmaConsumers) {
    // producer: the rows of one tile per slot, one bulk copy per row into the padded pitch
    if (lane == 0) {
      for (int q = 0; q < ntiles; ++q) {
        const int slot = q % a.S;
        if (q >= a.S) mbar_wait_bounded(&empty[slot], (uint32_t)(((q / a.S) - 1) & 1));
        *(volatile int*)&slot_tag[slot] = q;
        const int r0 = (t0 + q) * kTileRows;
        const int rows = min(kTileRows, a.N - r0);
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(rows * row_bytes));
        uint8_t* dst = ring + (size_t)slot * a.slot_bytes;
        for (int r = 0; r < rows; ++r)
          bulk_g2s(dst + (size_t)r * a.pitch, a.W + (int64_t)(r0 + r) * row_bytes, (uint32_t)row_bytes, &full[slot]);
      }
    }
    return;
  }

  // stage the activation digits (zero columns for absent rows), scales and sub-block sums
  grid_dep_wait();
  {
    const int ncol = 8 * NT;
    const int chunks = a.K / 16;
    for (int i = tid; i < ncol * chunks; i += kMmaConsumers * 32) {
      const int n = i / chunks, c = i % chunks;
      const int m = n >> 1, p = n & 1;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (m < a.M) v = *reinterpret_cast<const uint4*>(a.planes + ((int64_t)m * 2 + p) * a.K + 16 * c);
      *reinterpret_cast<uint4*>(xs + (size_t)n * a.xcol + 16 * c) = v;
    }
    for (int i = tid; i < 4 * NT * (a.K / 32); i += kMmaConsumers * 32) {
      const int m = i / (a.K / 32);
      xsum[i] = m < a.M ? a.xsum[i] : 0.f;
    }
    if (tid < 4 * NT) ts[tid] = tid < a.M ? a.tscale[tid] : 0.f;
    asm volatile("bar.sync 1, %0;" ::"r"(kMmaConsumers * 32) : "memory");
  }

  const int g = lane >> 2, q4 = lane & 3;
  const int p = warp % a.P;
  const int wpp = kMmaConsumers / a.P;
  const int sb_per_part = nb / a.P;
  const int sb0 = p * sb_per_part;
  for (int tq = warp / a.P; tq < ntiles; tq += wpp) {
    const int slot = tq % a.S;
    smem_wait_eq(&slot_tag[slot], tq);
    mbar_wait_bounded(&full[slot], (uint32_t)((tq / a.S) & 1));
    const uint8_t* rowg = ring + (size_t)slot * a.slot_bytes + (size_t)g * a.pitch;
    const uint8_t* rowh = rowg + (size_t)8 * a.pitch;
    float acc[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) acc[nt][0] = acc[nt][1] = 0.f;
    for (int sb = sb0; sb < sb0 + sb_per_part; ++sb) {
      const uint8_t* rg = rowg + sb * kRec;
      const uint8_t* rh = rowh + sb * kRec;
      const uint4 hg = lds_v4(rg), hh = lds_v4(rh);
      // 6-bit scales / mins of the 8 sub-blocks, bytes 0-3 in *_lo, 4-7 in *_hi
      const uint32_t scg_lo = hg.y & 0x3F3F3F3Fu, mng_lo = hg.z & 0x3F3F3F3Fu;
      const uint32_t scg_hi = (hg.w & 0x0F0F0F0Fu) | ((hg.y >> 2) & 0x30303030u);
      const uint32_t mng_hi = ((hg.w >> 4) & 0x0F0F0F0Fu) | ((hg.z >> 2) & 0x30303030u);
      const uint32_t sch_lo = hh.y & 0x3F3F3F3Fu, mnh_lo = hh.z & 0x3F3F3F3Fu;
      const uint32_t sch_hi = (hh.w & 0x0F0F0F0Fu) | ((hh.y >> 2) & 0x30303030u);
      const uint32_t mnh_hi = ((hh.w >> 4) & 0x0F0F0F0Fu) | ((hh.z >> 2) & 0x30303030u);
      int S0[NT][2], S1[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) S0[nt][0] = S0[nt][1] = S1[nt][0] = S1[nt][1] = 0;
#pragma unroll
      for (int pr = 0; pr < 4; ++pr) {
        const uint2 wg = *reinterpret_cast<const uint2*>(rg + 16 + 32 * pr + 8 * q4);
        const uint2 wh = *reinterpret_cast<const uint2*>(rh + 16 + 32 * pr + 8 * q4);
        const uint32_t alo[4] = {wg.x & 0x0F0F0F0Fu, wh.x & 0x0F0F0F0Fu, wg.y & 0x0F0F0F0Fu, wh.y & 0x0F0F0F0Fu};
        const uint32_t ahi[4] = {(wg.x >> 4) & 0x0F0F0F0Fu, (wh.x >> 4) & 0x0F0F0F0Fu, (wg.y >> 4) & 0x0F0F0F0Fu,
                                 (wh.y >> 4) & 0x0F0F0F0Fu};
        const int s_lo = 2 * pr, s_hi = 2 * pr + 1;   // sub-blocks of this pair
        const int scg0 = (int)((s_lo < 4 ? scg_lo : scg_hi) >> (8 * (s_lo & 3)) & 0xFF);
        const int scg1 = (int)((s_hi < 4 ? scg_lo : scg_hi) >> (8 * (s_hi & 3)) & 0xFF);
        const int sch0 = (int)((s_lo < 4 ? sch_lo : sch_hi) >> (8 * (s_lo & 3)) & 0xFF);
        const int sch1 = (int)((s_hi < 4 ? sch_lo : sch_hi) >> (8 * (s_hi & 3)) & 0xFF);
        const int kb = sb * 256 + 32 * s_lo + 8 * q4;   // element offset of this lane's 8 codes (low sub-block)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          const uint8_t* xc = xs + (size_t)(8 * nt + g) * a.xcol;
          const uint2 blo = *reinterpret_cast<const uint2*>(xc + kb);
          const uint2 bhi = *reinterpret_cast<const uint2*>(xc + kb + 32);
          int dlo[4], dhi[4];
          mma_u8s8(dlo, alo, blo.x, blo.y);
          mma_u8s8(dhi, ahi, bhi.x, bhi.y);
          S0[nt][0] += scg0 * dlo[0] + scg1 * dhi[0];
          S1[nt][0] += scg0 * dlo[1] + scg1 * dhi[1];
          S0[nt][1] += sch0 * dlo[2] + sch1 * dhi[2];
          S1[nt][1] += sch0 * dlo[3] + sch1 * dhi[3];
        }
      }
      const float dg = __half2float(__ushort_as_half((unsigned short)(hg.x & 0xFFFF)));
      const float dming = __half2float(__ushort_as_half((unsigned short)(hg.x >> 16)));
      const float dh = __half2float(__ushort_as_half((unsigned short)(hh.x & 0xFFFF)));
      const float dminh = __half2float(__ushort_as_half((unsigned short)(hh.x >> 16)));
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int tok = 4 * nt + q4;
        const float t = ts[tok];
        const float* xsb = xsum + (size_t)tok * (a.K / 32) + sb * 8;
        const float4 xa = *reinterpret_cast<const float4*>(xsb), xb = *reinterpret_cast<const float4*>(xsb + 4);
        const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
        float mg = 0.f, mh = 0.f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          mg = fmaf(byte_f(s < 4 ? mng_lo : mng_hi, s & 3), xv[s], mg);
          mh = fmaf(byte_f(s < 4 ? mnh_lo : mnh_hi, s & 3), xv[s], mh);
        }
        acc[nt][0] += dg * t * fmaf(254.0f, (float)S0[nt][0], (float)S1[nt][0]) - dming * mg;
        acc[nt][1] += dh * t * fmaf(254.0f, (float)S0[nt][1], (float)S1[nt][1]) - dminh * mh;
      }
    }
    // rows g, g+8 of the tile; activation rows 4nt + q4
    const int rbase = (t0 + tq) * kTileRows;
    if (a.P == 1) {
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = rbase + g + 8 * h, tok = 4 * nt + q4;
          if (row < a.N && tok < a.M) {
            float v = acc[nt][h] + (a.bias ? a.bias[row] : 0.f);
            float* yp = a.y + (int64_t)tok * a.N + row;
            if (a.accumulate) v += *yp;
            *yp = v;
          }
        }
    } else {
      float* pp = part + (((size_t)slot * a.P + p) * kTileRows) * (4 * NT);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) pp[(g + 8 * h) * (4 * NT) + 4 * nt + q4] = acc[nt][h];
      __threadfence_block();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = atomicAdd(&part_cnt[slot], 1) == a.P - 1;
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence_block();
        for (int i = lane; i < kTileRows * 4 * NT; i += 32) {
          const int r = i / (4 * NT), tok = i % (4 * NT);
          const volatile float* src = part + ((size_t)slot * a.P * kTileRows + r) * (4 * NT) + tok;
          float v = src[0];
          for (int pp2 = 1; pp2 < a.P; ++pp2) v += src[(size_t)pp2 * kTileRows * 4 * NT];
          const int row = rbase + r;
          if (row < a.N && tok < a.M) {
            v += a.bias ? a.bias[row] : 0.f;
            float* yp = a.y + (int64_t)tok * a.N + row;
            if (a.accumulate) v += *yp;
            *yp = v;
          }
        }
        __syncwarp();
        if (lane == 0) part_cnt[slot] = 0;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }
  }
}

bool plan_mma(int64_t n, int64_t k, int64_t m, MmaArgs& a, int& smem, int& grid) {
  if (m < 2 || m > 8 || k % 256 || k < 256 || n < 1 || n >= (1ll << 31)) return false;
  const int NT = m <= 4 ? 1 : 2;
  const int nb = (int)(k / 256);
  const int64_t row_bytes = (int64_t)nb * kRec;
  // padded row pitch: 32 bytes past a multiple of 128, so the 8-byte fragment
  // loads of rows g = 0..3 (and 4..7) fall on distinct banks
  const int64_t pitch = (row_bytes + 127) / 128 * 128 + 32;
  const int64_t slot_bytes = kTileRows * pitch;
  const int64_t xcol = (k + 127) / 128 * 128 + 32;
  const int ntiles = (int)((n + kTileRows - 1) / kTileRows);
  grid = std::min(xm_sm_count(), ntiles);
  const int tiles_per_cta = (ntiles + grid - 1) / grid;
  int P = 1;
  while (P < 8 && tiles_per_cta * P < kMmaConsumers && nb % (2 * P) == 0) P *= 2;
  const int64_t fixed = kCtlBytes + 8LL * NT * xcol + 16LL * NT + 4LL * NT * (k / 32) * 4 + 16;
  int64_t S = 0;
  for (S = kMaxSlots; S >= 2; --S)
    if (fixed + S * slot_bytes + S * P * kTileRows * 4 * NT * 4 <= kMaxSmemMma) break;
  if (S < 2) return false;
  a.N = (int)n;
  a.K = (int)k;
  a.M = (int)m;
  a.P = P;
  a.S = (int)S;
  a.pitch = (int)pitch;
  a.slot_bytes = (int)slot_bytes;
  a.xcol = (int)xcol;
  smem = (int)(fixed + S * slot_bytes + S * P * kTileRows * 4 * NT * 4);
  return true;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_mma(void (*kernel)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, Args... args) {
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

template <int NT>
int launch_mma(const MmaArgs& a, int smem, int grid, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemv_q4k_mma<NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmemMma);
    if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv mma: smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  cudaError_t e = launch_pdl_mma(k_qgemv_q4k_mma<NT>, dim3(grid), dim3(kMmaThreads), smem, st, a);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv mma launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemv(tensor-core, m 2..8)");
}

template <typename XT>
cudaError_t launch_split_tok(int prologue, int64_t m, const XT* x, int64_t x_stride, int64_t k, const float* norm_w,
                             float eps, int8_t* planes, float* tscale, float* xsum, cudaStream_t st) {
  const dim3 grid((unsigned)m, (unsigned)((k + kSliceK - 1) / kSliceK));
  switch (prologue) {
    case XM_PRO_RMSNORM:
      return launch_pdl_mma(k_split_tok<XT, XM_PRO_RMSNORM>, grid, dim3(256), 0, st, x, x_stride, (int)k, norm_w, eps,
                            planes, tscale, xsum);
    case XM_PRO_SWIGLU:
      return launch_pdl_mma(k_split_tok<XT, XM_PRO_SWIGLU>, grid, dim3(256), 0, st, x, x_stride, (int)k, norm_w, eps,
                            planes, tscale, xsum);
    default:
      return launch_pdl_mma(k_split_tok<XT, XM_PRO_NONE>, grid, dim3(256), 0, st, x, x_stride, (int)k, norm_w, eps,
                            planes, tscale, xsum);
  }
}

}  // namespace

bool gemv_mma_supported(int qtype, int64_t n, int64_t k, int64_t m) {
  MmaArgs a{};
  int smem = 0, grid = 0;
  return qtype == T_Q4_K && plan_mma(n, k, m, a, smem, grid);
}

int64_t gemv_mma_split_bytes(int64_t k, int64_t m) { return m * 2 * k + (m * 4 + 255) / 256 * 256 + m * (k / 32) * 4; }

int gemv_mma(const uint8_t* W, int64_t n, int64_t k, int64_t m, const void* d_x, int x_dtype, int64_t x_stride,
             int prologue, const float* norm_w, float eps, const float* bias, float* y, int accumulate, void* d_ws,
             cudaStream_t st) {
  MmaArgs a{};
  int smem = 0, grid = 0;
  if (!plan_mma(n, k, m, a, smem, grid))
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemv mma: no plan for n=%lld k=%lld m=%lld", (long long)n, (long long)k,
                        (long long)m);
  int8_t* planes = (int8_t*)d_ws;
  float* tscale = (float*)((uint8_t*)d_ws + m * 2 * k);
  float* xsum = (float*)((uint8_t*)tscale + (m * 4 + 255) / 256 * 256);
  cudaError_t e;
  if (x_dtype == XM_DT_F32)
    e = launch_split_tok<float>(prologue, m, (const float*)d_x, x_stride, k, norm_w, eps, planes, tscale, xsum, st);
  else if (x_dtype == XM_DT_BF16)
    e = launch_split_tok<__nv_bfloat16>(prologue, m, (const __nv_bfloat16*)d_x, x_stride, k, norm_w, eps, planes,
                                        tscale, xsum, st);
  else
    e = launch_split_tok<__half>(prologue, m, (const __half*)d_x, x_stride, k, norm_w, eps, planes, tscale, xsum, st);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "split_tok launch: %s", cudaGetErrorString(e));
  int rc = xm_check_launch("split_tok");
  if (rc) return rc;
  a.W = W;
  a.y = y;
  a.bias = bias;
  a.planes = planes;
  a.tscale = tscale;
  a.xsum = xsum;
  a.accumulate = accumulate;
  return m <= 4 ? launch_mma<1>(a, smem, grid, st) : launch_mma<2>(a, smem, grid, st);
}
