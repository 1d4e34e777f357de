// K2: fused dequant-GEMV for decode, y[m][n] = sum_k x[m][k] * W[n][k], m <= 8.
//
// Two code paths:
//
// * Integer-dot path (Q4_K): the activation row is first split into 32-element
//   groups and written as two int8 digits per element, x ~= t * (254*X0 + X1)
//   with t = max|x_group| / (127*254) -- about 16 significant bits, far inside
//   the fp32 tolerance of the matmul -- plus the exact fp32 group sums.  The
//   GEMV then multiplies the raw 4-bit codes against both digit planes with
//   dp4a (four products per instruction, exact in int32), and applies the
//   per-sub-block scale d*sc and the offset dmin*mn*sum(x) once per 32
//   elements in fp32.  Unpacking costs 3 integer ops per 8 weights, so the
//   kernel stays bound by HBM rather than by instruction issue.
//
// * Exact path (all other types, and any shape the integer path does not
//   take): each weight is decoded to the reference's fp16 value and multiplied
//   in fp32.  Slower; it is the fallback and the cross-check.
#include <algorithm>
#include <mutex>
#include <type_traits>

#include "xm_gemv_dot.cuh"
#include "xm_internal.h"

namespace {

constexpr int kThreads = 256;
constexpr int kPieceBytes = 64;  // per 32-element group: 32 x X0, 32 x X1

// ---------------------------------------------------------------------------
// Activation split: one warp per 32-element group.
// pieces[(m*G + g)*64 + i] = X0_i, [+32 + i] = X1_i ; ts[m*G + g] = (t, sum_lo16, sum_hi16, sum32)
// ---------------------------------------------------------------------------
// Lane-major layout (one activation row of 4096 = 128 groups, used by the
// K = 4096 single-row kernel): lane l of that kernel owns groups 4l..4l+3; its
// 16-byte digit chunk q (X0 bytes 0-15, 16-31, X1 bytes 0-15, 16-31) of group
// 4l+i sits at ((4i + q) * 32 + l) * 16, and (t, sum32) at 8192 + (32i + l) * 8,
// so that a warp reading one chunk per lane touches 512 contiguous bytes.
constexpr int kLaneMajorBytes = 8192 + 1024;

template <typename XT>
__global__ void __launch_bounds__(kThreads) k_split_x(const XT* __restrict__ x, int64_t mg, int G,
                                                      int8_t* __restrict__ pieces, float4* __restrict__ ts,
                                                      int8_t* __restrict__ lane_major) {
  const int lane = threadIdx.x & 31;
  const int64_t grp = ((int64_t)blockIdx.x * kThreads + threadIdx.x) >> 5;
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (grp >= mg) return;
  const float v = to_f32(x[grp * 32 + lane]);
  int x0, x1;
  float t, s_lo, s_hi;
  split_group(v, x0, x1, t, s_lo, s_hi);
  pieces[grp * kPieceBytes + lane] = (int8_t)x0;
  pieces[grp * kPieceBytes + 32 + lane] = (int8_t)x1;
  if (lane == 0) ts[grp] = make_float4(t, s_lo, s_hi, s_lo + s_hi);
  if (lane_major) {
    const int L = (int)(grp >> 2), i = (int)(grp & 3);
    lane_major[((4 * i + (lane >> 4)) * 32 + L) * 16 + (lane & 15)] = (int8_t)x0;
    lane_major[((4 * i + 2 + (lane >> 4)) * 32 + L) * 16 + (lane & 15)] = (int8_t)x1;
    if (lane == 0) reinterpret_cast<float2*>(lane_major + 8192)[32 * i + L] = make_float2(t, s_lo + s_hi);
  }
}

XM_DEV uint4 ldg_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

XM_DEV uint32_t byte_of(uint32_t w, int i) { return (w >> (8 * i)) & 0xFF; }

// y = v, or y += v for the residual-add (accumulate) form
XM_DEV void store_out(float* p, float v, int accumulate) {
  if (accumulate) v += *p;
  *p = v;
}

// ---------------------------------------------------------------------------
// Q4_K integer-dot GEMV.  A warp serves 4 rows; 8 lanes per row, lane cl
// handles super-blocks c = cl, cl+8, ... of its row.  The 4 rows of a warp read
// the same activation digits in the same instruction (one L1 wavefront).
// ---------------------------------------------------------------------------
template <int M>
__global__ void __launch_bounds__(kThreads) k_qgemv_q4k_dp4a(const uint8_t* __restrict__ W, int N, int nb,
                                                             const int8_t* __restrict__ pieces,
                                                             const float4* __restrict__ ts,
                                                             const float* __restrict__ bias, float* __restrict__ y,
                                                             int accumulate) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int slot = lane >> 3, cl = lane & 7;
  const int G = nb * 8;  // 32-element groups per row
  const int64_t nwarps = (int64_t)gridDim.x * (kThreads / 32);
  for (int64_t r0 = ((int64_t)blockIdx.x * (kThreads / 32) + warp) * 4; r0 < N; r0 += nwarps * 4) {
    const int64_t row = r0 + slot;
    const bool valid = row < N;
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int c = cl; c < nb; c += 8) {
      const uint8_t* blk = W + ((valid ? row : 0) * (int64_t)nb + c) * 144;
      const uint4 hd = ldg_v4(blk);
      const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
      // 6-bit scales and mins of the 8 sub-blocks, one byte each
      const uint32_t A = hd.y, B = hd.z, C = hd.w;
      const uint32_t sc_lo = A & 0x3F3F3F3Fu, mn_lo = B & 0x3F3F3F3Fu;
      const uint32_t sc_hi = (C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u);
      const uint32_t mn_hi = ((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 qa = ldg_v4(blk + 16 + 32 * j);
        const uint4 qb = ldg_v4(blk + 32 + 32 * j);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const int sa = 2 * j, sb = 2 * j + 1;
        const float scA = (float)byte_of(sa < 4 ? sc_lo : sc_hi, sa & 3);
        const float scB = (float)byte_of(sb < 4 ? sc_lo : sc_hi, sb & 3);
        const float mnA = (float)byte_of(sa < 4 ? mn_lo : mn_hi, sa & 3);
        const float mnB = (float)byte_of(sb < 4 ? mn_lo : mn_hi, sb & 3);
        const float d1A = d * scA, d1B = d * scB, m1A = dmin * mnA, m1B = dmin * mnB;
        const int g = c * 8 + sa;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const int8_t* pa = pieces + ((int64_t)m * G + g) * kPieceBytes;
          const uint4 a0 = ldg_v4(pa), a1 = ldg_v4(pa + 16), a2 = ldg_v4(pa + 32), a3 = ldg_v4(pa + 48);
          const uint4 b0 = ldg_v4(pa + 64), b1 = ldg_v4(pa + 80), b2 = ldg_v4(pa + 96), b3 = ldg_v4(pa + 112);
          const uint32_t xa0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const uint32_t xa1[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
          const uint32_t xb0[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const uint32_t xb1[8] = {b2.x, b2.y, b2.z, b2.w, b3.x, b3.y, b3.z, b3.w};
          int DA0 = 0, DA1 = 0, DB0 = 0, DB1 = 0;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const int lo = (int)(q[w] & 0x0F0F0F0Fu);
            const int hi = (int)((q[w] >> 4) & 0x0F0F0F0Fu);
            DA0 = __dp4a(lo, (int)xa0[w], DA0);
            DA1 = __dp4a(lo, (int)xa1[w], DA1);
            DB0 = __dp4a(hi, (int)xb0[w], DB0);
            DB1 = __dp4a(hi, (int)xb1[w], DB1);
          }
          const float4 tA = ts[(int64_t)m * G + g], tB = ts[(int64_t)m * G + g + 1];
          const float PA = __int2float_rn(254 * DA0 + DA1), PB = __int2float_rn(254 * DB0 + DB1);
          acc[m] += (d1A * tA.x) * PA - m1A * tA.w;
          acc[m] += (d1B * tB.x) * PB - m1B * tB.w;
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      float v = acc[m];
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      if (cl == 0 && valid) store_out(&y[(int64_t)m * N + row], v + (bias ? bias[row] : 0.f), accumulate);
    }
  }
}

int sm_count() { return xm_sm_count(); }

// ---------------------------------------------------------------------------
// Q4_K integer-dot GEMV, TMA-staged (the main decode kernel).
//
// One CTA of kGemvWarps warps per SM owns a contiguous, balanced range of
// rows.  Every warp runs its own pipeline: a ring of kGemvStages slots of 32
// super-block records (4,608 bytes), filled by cp.async.bulk (TMA, no
// multicast) and completing on the slot's mbarrier.  A stage is RW = 32/LPR
// rows x LPR super-blocks (a K-chunk); lane l works on super-block
// (row l/LPR, column l%LPR), reading the 144-byte record from shared memory
// at a 144-byte lane stride (conflict-free).  Warps take row groups from a
// shared counter, so the CTA's rows are balanced dynamically and no warp ever
// waits on another.  The activation digits of the whole row stay resident in
// shared memory, 656 bytes per super-block column (512 B digits, 128 B
// (t, sums), 16 B pad: neighbouring columns fall 4 banks apart).
// Launched with programmatic dependent launch: the weight prefetch is issued
// before griddepcontrol.wait, so it overlaps the kernel that produced x.
// ---------------------------------------------------------------------------
constexpr int kGemvWarps = 16;
constexpr int kGemvThreads = kGemvWarps * 32;
constexpr int kGemvStages = 2;
constexpr int kSlotBytes = 32 * 144;
constexpr int kColStride = 656;


struct GemvSmem {
  int next_group;
  int slot_group[kGemvWarps][kGemvStages];
  int slot_chunk[kGemvWarps][kGemvStages];
};

template <int M, int LPR>
__global__ void __launch_bounds__(kGemvThreads, 1) k_qgemv_q4k_tma(const uint8_t* __restrict__ W, int N, int nb,
                                                                   const int8_t* __restrict__ pieces,
                                                                   const float4* __restrict__ ts,
                                                                   const float* __restrict__ bias,
                                                                   float* __restrict__ y, int accumulate) {
  constexpr int RW = 32 / LPR;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* slots = smem;                                                // [warps][stages][kSlotBytes]
  uint8_t* xs = smem + kGemvWarps * kGemvStages * kSlotBytes;           // [M][nb][kColStride]
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + (size_t)M * nb * kColStride);  // [warps][stages]
  GemvSmem* ctl = reinterpret_cast<GemvSmem*>(full + kGemvWarps * kGemvStages);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = nb * 8;

  const int64_t rb = (int64_t)N * blockIdx.x / gridDim.x;
  const int64_t re = (int64_t)N * (blockIdx.x + 1) / gridDim.x;
  const int ngroups = (int)((re - rb + RW - 1) / RW);
  const int nchunks = (nb + LPR - 1) / LPR;

  if (tid == 0) {
    for (int i = 0; i < kGemvWarps * kGemvStages; ++i) mbar_init(&full[i], 1);
    ctl->next_group = 0;
    fence_mbar_init();
  }
  __syncthreads();

  uint8_t* my_slots = slots + warp * kGemvStages * kSlotBytes;
  uint64_t* my_full = full + warp * kGemvStages;
  // issue-side generator, identical in every lane of the warp
  int gi = -1, ki = nchunks - 1;
  int issued = 0;
  auto issue_next = [&]() -> bool {
    if (ki == nchunks - 1) {
      int g = 0;
      if (lane == 0) g = atomicAdd(&ctl->next_group, 1);
      g = __shfl_sync(0xffffffffu, g, 0);
      if (g >= ngroups) return false;
      gi = g;
      ki = 0;
    } else {
      ++ki;
    }
    const int slot = issued % kGemvStages;
    if (lane == 0) {
      const int64_t r0 = rb + (int64_t)gi * RW;
      const int R = (int)min((int64_t)RW, re - r0);
      const int c0 = ki * LPR, cc = min(LPR, nb - c0);
      ctl->slot_group[warp][slot] = gi;
      ctl->slot_chunk[warp][slot] = ki;
      uint8_t* buf = my_slots + slot * kSlotBytes;
      mbar_arrive_expect_tx(&my_full[slot], (uint32_t)(R * cc * 144));
      for (int r = 0; r < R; ++r)
        bulk_g2s(buf + r * LPR * 144, W + ((r0 + r) * nb + c0) * 144, (uint32_t)(cc * 144), &my_full[slot]);
    }
    ++issued;
    return true;
  };
  bool more = true;
  for (int i = 0; i < kGemvStages && more; ++i) more = issue_next();

  grid_dep_wait();  // x digits are written by the preceding kernel
  for (int i = tid; i < M * G * 4; i += kGemvThreads) {          // 16-byte digit chunks
    const int m = i / (G * 4), rem = i - m * (G * 4), g = rem >> 2, q = rem & 3;
    const uint4 v = *reinterpret_cast<const uint4*>(pieces + ((int64_t)m * G + g) * kPieceBytes + q * 16);
    *reinterpret_cast<uint4*>(xs + ((size_t)m * nb + (g >> 3)) * kColStride + (g & 7) * 64 + q * 16) = v;
  }
  for (int i = tid; i < M * G; i += kGemvThreads) {
    const int m = i / G, g = i - m * G;
    *reinterpret_cast<float4*>(xs + ((size_t)m * nb + (g >> 3)) * kColStride + 512 + (g & 7) * 16) =
        ts[(int64_t)m * G + g];
  }
  __syncthreads();

  const int lr = lane / LPR, lc = lane % LPR;
  float acc[M];
#pragma unroll
  for (int m = 0; m < M; ++m) acc[m] = 0.f;

  for (int s = 0; s < issued; ++s) {
    const int slot = s % kGemvStages;
    mbar_wait_bounded(&my_full[slot], (uint32_t)((s / kGemvStages) & 1));
    const int g = ctl->slot_group[warp][slot], kc = ctl->slot_chunk[warp][slot];
    const int64_t r0 = rb + (int64_t)g * RW;
    const int c = kc * LPR + lc;
    if (r0 + lr < re && c < nb) {
      const uint8_t* blk = my_slots + slot * kSlotBytes + lane * 144;
      const uint4 hd = lds_v4(blk);
      const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
      const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
      const uint32_t A = hd.y, B = hd.z, C = hd.w;
      // 6-bit scales / mins, one byte per sub-block: [0..3] in *_lo, [4..7] in *_hi
      const uint32_t sc_lo = A & 0x3F3F3F3Fu, mn_lo = B & 0x3F3F3F3Fu;
      const uint32_t sc_hi = (C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u);
      const uint32_t mn_hi = ((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 qa = lds_v4(blk + 16 + 32 * j);
        const uint4 qb = lds_v4(blk + 32 + 32 * j);
        const uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
        const uint32_t scw = j < 2 ? sc_lo : sc_hi, mnw = j < 2 ? mn_lo : mn_hi;
        const int bA = (2 * j) & 3, bB = (2 * j + 1) & 3;
        const float d1A = d * byte_f(scw, bA), d1B = d * byte_f(scw, bB);
        const float m1A = dmin * byte_f(mnw, bA), m1B = dmin * byte_f(mnw, bB);
#pragma unroll
        for (int m = 0; m < M; ++m) {
          const uint8_t* col = xs + ((size_t)m * nb + c) * kColStride;
          const uint8_t* pa = col + j * 128;
          const uint4 a0 = lds_v4(pa), a1 = lds_v4(pa + 16), a2 = lds_v4(pa + 32), a3 = lds_v4(pa + 48);
          const uint4 b0 = lds_v4(pa + 64), b1 = lds_v4(pa + 80), b2 = lds_v4(pa + 96), b3 = lds_v4(pa + 112);
          const uint32_t xa0[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const uint32_t xa1[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
          const uint32_t xb0[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
          const uint32_t xb1[8] = {b2.x, b2.y, b2.z, b2.w, b3.x, b3.y, b3.z, b3.w};
          int DA0 = 0, DA1 = 0, DB0 = 0, DB1 = 0;
#pragma unroll
          for (int w = 0; w < 8; ++w) {
            const int lo = (int)(q[w] & 0x0F0F0F0Fu);
            const int hi = (int)((q[w] >> 4) & 0x0F0F0F0Fu);
            DA0 = __dp4a(lo, (int)xa0[w], DA0);
            DA1 = __dp4a(lo, (int)xa1[w], DA1);
            DB0 = __dp4a(hi, (int)xb0[w], DB0);
            DB1 = __dp4a(hi, (int)xb1[w], DB1);
          }
          const float4 tA = *reinterpret_cast<const float4*>(col + 512 + (2 * j) * 16);
          const float4 tB = *reinterpret_cast<const float4*>(col + 512 + (2 * j + 1) * 16);
          const float PA = __int2float_rn(254 * DA0 + DA1), PB = __int2float_rn(254 * DB0 + DB1);
          acc[m] = fmaf(d1A * tA.x, PA, acc[m]) - m1A * tA.w;
          acc[m] = fmaf(d1B * tB.x, PB, acc[m]) - m1B * tB.w;
        }
      }
    }
    if (kc == nchunks - 1) {
      // row group done: reduce over the LPR lanes of each row (contiguous)
#pragma unroll
      for (int m = 0; m < M; ++m) {
        float v = acc[m];
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lc == 0 && r0 + lr < re)
          store_out(&y[(int64_t)m * N + r0 + lr], v + (bias ? bias[r0 + lr] : 0.f), accumulate);
        acc[m] = 0.f;
      }
    }
    __syncwarp();  // all lanes are done reading the slot
    if (more) more = issue_next();
  }
  grid_dep_launch();
}

// ---------------------------------------------------------------------------
// Q4_K GEMV for one activation row and K = 4096 (16 super-blocks per row):
// the decode shape of every Q4_K projection of the Llama-7B-class layer.
//
// Warp-specialised.  A producer warp streams the CTA's rows into a 20-slot
// shared-memory ring, four rows (9,216 B) per cp.async.bulk (TMA without
// multicast; copies this large keep HBM busy, 2 KB copies do not), refilling
// a slot as soon as its rows have been taken (full/empty mbarrier pair per
// slot).  15 consumer warps take row pairs in order from a shared counter and
// work on both rows at once (two independent dependency chains, one shuffle
// tree for both sums).  Lane (c, h) = (lane/2, lane%2) always handles
// sub-block pairs 2h, 2h+1 of super-block column c, so its 4 activation-digit
// groups and their (t, sums) sit in registers for the whole kernel (filled
// once from a lane-major copy in shared memory) and the inner loop reads only
// weights.  Low nibbles go to dp4a as q & 0x0F0F0F0F; high nibbles as
// q & 0xF0F0F0F0 (unsigned x signed dp4a, 16x the value; the 1/16 folds into
// the sub-block scale), which saves the shift.
// ---------------------------------------------------------------------------
constexpr int kWsConsumers = 15;   // + the producer: 16 warps, so the register budget is 128 per thread
constexpr int kWsThreads = (kWsConsumers + 1) * 32;
// 20 slots (184 KB): a CTA's whole share of an 11008 x 4096 matrix (75 rows,
// 171 KB) is in flight before the consumers finish their activation prologue
constexpr int kWsSlots = 20;
constexpr int kWsRowsPerSlot = 4;
constexpr int kWsEarlyChunks = 6;  // copies issued before the activation row arrives
constexpr int kRowBytes4096 = 16 * 144;
constexpr int kWsSlotBytes = kWsRowsPerSlot * kRowBytes4096;
// slots | lane-major split | barriers and counters | (fused form) the raw fp32/bf16 row of x
// (barriers 41 x 8 B + counter + 20 slot tags = 412 B, rounded up so that the
// row of x behind it keeps the 16-byte alignment a bulk copy needs)
constexpr int kWsCtlBytes = 512;
static_assert((2 * kWsSlots + 1) * 8 + (kWsSlots + 1) * 4 <= kWsCtlBytes, "control block");
static_assert((kWsSlots * kWsSlotBytes + kLaneMajorBytes + kWsCtlBytes) % 16 == 0, "x row alignment");
// + 64 B behind the row of x for the RMSNorm partial sums
constexpr int kWsSmem = kWsSlots * kWsSlotBytes + kLaneMajorBytes + kWsCtlBytes + 4096 * 4 + 64;


// Partial dot of one row's 128 weights (sub-block pairs 2h, 2h+1 of column c)
// with this lane's digits: returns d*sum(sc*t*P) - dmin*sum(mn*sum_x).
XM_DEV float q4k_lane_dot(uint4 hd, uint4 q0, uint4 q1, uint4 q2, uint4 q3, int h, const uint32_t (&xd)[4][16],
                          const float (&tx)[4], const float (&tw)[4]) {
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  const uint32_t A = hd.y, B = hd.z, C = hd.w;
  const uint32_t scw = h == 0 ? (A & 0x3F3F3F3Fu) : ((C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u));
  const uint32_t mnw = h == 0 ? (B & 0x3F3F3F3Fu) : (((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u));
  const uint32_t qw[2][8] = {{q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w},
                             {q2.x, q2.y, q2.z, q2.w, q3.x, q3.y, q3.z, q3.w}};
  float acc = 0.f, macc = 0.f;
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const uint32_t* xa = xd[2 * jj];
    const uint32_t* xb = xd[2 * jj + 1];
    int DA0 = 0, DA1 = 0, DB0 = 0, DB1 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const uint32_t lo = qw[jj][w] & 0x0F0F0F0Fu;
      const uint32_t hi = qw[jj][w] & 0xF0F0F0F0u;
      DA0 = dp4a_us(lo, xa[w], DA0);
      DA1 = dp4a_us(lo, xa[8 + w], DA1);
      DB0 = dp4a_us(hi, xb[w], DB0);
      DB1 = dp4a_us(hi, xb[8 + w], DB1);
    }
    const float PA = __int2float_rn(254 * DA0 + DA1), PB = __int2float_rn(254 * DB0 + DB1);
    acc = fmaf(byte_f(scw, 2 * jj) * tx[2 * jj], PA, acc);
    acc = fmaf(byte_f(scw, 2 * jj + 1) * (0.0625f * tx[2 * jj + 1]), PB, acc);
    macc = fmaf(byte_f(mnw, 2 * jj), tw[2 * jj], macc);
    macc = fmaf(byte_f(mnw, 2 * jj + 1), tw[2 * jj + 1], macc);
  }
  return d * acc - dmin * macc;
}

// The activation split written by the consumer warps straight into the
// lane-major shared-memory layout (the fused form of k_split_x for one row of
// 4096).  Threads 0..255 work: thread t takes half (t&1) -- 16 elements -- of
// 32-element group t>>1, so each thread writes whole 16-byte digit chunks and
// the only cross-thread step is one shuffle for the group max and one for the
// sum.  `x` is a shared-memory copy of the row.  With norm_w the row is first
// RMS-normalised, v = (x / sqrt(mean(x^2) + eps)) * norm_w (ops.py:115-117);
// every consumer thread must then call this (it holds a consumer-only barrier).
template <typename XT>
XM_DEV void split_row4096_to_smem(const XT* x, uint8_t* xsm, int tid, const float* norm_w, float eps, float* red) {
  const bool work = tid < 256;
  const int g = tid >> 1, half = tid & 1;
  float v[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) v[e] = work ? to_f32(x[g * 32 + half * 16 + e]) : 0.f;
  if (norm_w) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) ss = fmaf(v[e], v[e], ss);
    ss = warp_sum(ss);
    if ((tid & 31) == 0 && work) red[tid >> 5] = ss;
    asm volatile("bar.sync 1, %0;" ::"r"(kWsConsumers * 32) : "memory");
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) tot += red[w];
    const float rms = sqrtf(tot / 4096.0f + eps);
    if (work) {
      const float4* nw = reinterpret_cast<const float4*>(norm_w + g * 32 + half * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 w4 = nw[q];
        v[4 * q] = (v[4 * q] / rms) * w4.x;
        v[4 * q + 1] = (v[4 * q + 1] / rms) * w4.y;
        v[4 * q + 2] = (v[4 * q + 2] / rms) * w4.z;
        v[4 * q + 3] = (v[4 * q + 3] / rms) * w4.w;
      }
    }
  }
  if (!work) return;
  float amax = 0.f, s = 0.f;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    amax = fmaxf(amax, fabsf(v[e]));
    s += v[e];
  }
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const float s_other = __shfl_xor_sync(0xffffffffu, s, 1);
  uint32_t w0[4] = {0, 0, 0, 0}, w1[4] = {0, 0, 0, 0};
  float t = 0.f;
  if (amax > 0.f) {
    const float sc = amax / 127.0f;
    const float inv = 1.0f / sc;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float u = v[e] * inv;
      const float r0 = rintf(u);
      const int x0 = (int)r0;
      const int x1 = max(-127, min(127, (int)rintf((u - r0) * 254.0f)));
      w0[e >> 2] |= (uint32_t)(x0 & 0xFF) << (8 * (e & 3));
      w1[e >> 2] |= (uint32_t)(x1 & 0xFF) << (8 * (e & 3));
    }
    t = sc / 254.0f;
  }
  const int L = g >> 2, i = g & 3;
  *reinterpret_cast<uint4*>(xsm + ((4 * i + half) * 32 + L) * 16) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
  *reinterpret_cast<uint4*>(xsm + ((4 * i + 2 + half) * 32 + L) * 16) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
  if (half == 0) *reinterpret_cast<float2*>(xsm + 8192 + (32 * i + L) * 8) = make_float2(t, s + s_other);
}

// XT = void: the split comes from a workspace written by k_split_x (lane-major);
// otherwise x itself is read and split in the prologue.  ACC: y += W x (the
// residual add) instead of y = W x; a template flag so that the plain form
// never reads y.
template <typename XT, bool ACC>
__global__ void __launch_bounds__(kWsThreads, 1) k_qgemv_q4k_k4096_m1(const uint8_t* __restrict__ W, int N,
                                                                      const void* __restrict__ xin,
                                                                      const float* __restrict__ norm_w, float eps,
                                                                      const float* __restrict__ bias,
                                                                      float* __restrict__ y) {
  extern __shared__ __align__(128) uint8_t ws_smem[];
  uint8_t* slots = ws_smem;                                            // [kWsSlots][kWsSlotBytes]
  uint8_t* xsm = ws_smem + kWsSlots * kWsSlotBytes;                    // lane-major digits
  uint64_t* full = reinterpret_cast<uint64_t*>(xsm + kLaneMajorBytes); // [kWsSlots]
  uint64_t* empty = full + kWsSlots;                                   // [kWsSlots]
  uint64_t* xbar = empty + kWsSlots;
  int* next_item = reinterpret_cast<int*>(xbar + 1);
  int* slot_chunk = next_item + 1;                                     // [kWsSlots]: chunk the slot is armed for
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int rb = (int)((int64_t)N * blockIdx.x / gridDim.x);
  const int re = (int)((int64_t)N * (blockIdx.x + 1) / gridDim.x);
  const int nrows = re - rb;
  const int nchunks = (nrows + kWsRowsPerSlot - 1) / kWsRowsPerSlot;
  const int npairs = (nrows + 1) / 2;
  // The next kernel may start at once: before its griddepcontrol.wait it only
  // streams its own weights.
  grid_dep_launch();

  if (tid == 0) {
    for (int i = 0; i < kWsSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kWsRowsPerSlot / 2);   // one arrival per row pair
      slot_chunk[i] = -1;
    }
    mbar_init(xbar, 1);
    *next_item = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kWsConsumers) {
    // producer: the first kWsEarlyChunks copies need no wait on the preceding
    // kernel (weights only); the rest are queued behind the activation row,
    // so that the row's copy does not wait behind the whole weight stream
    if (lane == 0) {
      for (int q = 0; q < nchunks; ++q) {
        if (q == kWsEarlyChunks) {
          grid_dep_wait();
          mbar_wait_bounded(xbar, 0);   // the activation (or its split) has landed
        }
        const int slot = q % kWsSlots;
        if (q >= kWsSlots) mbar_wait_bounded(&empty[slot], (uint32_t)(((q / kWsSlots) - 1) & 1));
        *(volatile int*)&slot_chunk[slot] = q;   // the previous lap of this slot is fully consumed
        const int rows = min(kWsRowsPerSlot, nrows - q * kWsRowsPerSlot);
        mbar_arrive_expect_tx(&full[slot], (uint32_t)(rows * kRowBytes4096));
        bulk_g2s(slots + slot * kWsSlotBytes, W + (int64_t)(rb + q * kWsRowsPerSlot) * kRowBytes4096,
                 (uint32_t)(rows * kRowBytes4096), &full[slot]);
      }
    }
    return;
  }

  grid_dep_wait();  // x (or its split) is produced by the preceding kernel
  if constexpr (std::is_same<XT, void>::value) {
    if (tid == 0) {
      mbar_arrive_expect_tx(xbar, kLaneMajorBytes);
      bulk_g2s(xsm, xin, kLaneMajorBytes, xbar);
    }
    mbar_wait_bounded(xbar, 0);
  } else {
    // one bulk copy brings the whole row (8 KB bf16 / 16 KB fp32) in a single latency
    XT* xrow = reinterpret_cast<XT*>(xsm + kLaneMajorBytes + kWsCtlBytes);
    if (tid == 0) {
      mbar_arrive_expect_tx(xbar, 4096 * sizeof(XT));
      bulk_g2s(xrow, xin, 4096 * sizeof(XT), xbar);
    }
    mbar_wait_bounded(xbar, 0);
    split_row4096_to_smem<XT>(xrow, xsm, tid, norm_w, eps, reinterpret_cast<float*>(xrow + 4096));
    asm volatile("bar.sync 1, %0;" ::"r"(kWsConsumers * 32) : "memory");   // consumer warps only
  }
  const int c = lane >> 1, h = lane & 1;
  uint32_t xd[4][16];
  float tx[4], tw[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = lds_v4(xsm + ((4 * i + q) * 32 + lane) * 16);
      xd[i][4 * q] = v.x; xd[i][4 * q + 1] = v.y; xd[i][4 * q + 2] = v.z; xd[i][4 * q + 3] = v.w;
    }
    const float2 t2 = *reinterpret_cast<const float2*>(xsm + 8192 + (32 * i + lane) * 8);
    tx[i] = t2.x;
    tw[i] = t2.y;
  }

  for (;;) {
    int p = 0;
    if (lane == 0) p = atomicAdd(next_item, 1);
    p = __shfl_sync(0xffffffffu, p, 0);
    if (p >= npairs) break;
    const int q = p >> 1, slot = q % kWsSlots;
    const int r = 2 * p;                         // first row (CTA-relative)
    const bool two = r + 1 < nrows;
    // row pairs are taken out of order across warps: make sure the slot is
    // armed for this chunk (not for its previous lap) before the parity wait
    smem_wait_eq(&slot_chunk[slot], q);
    mbar_wait_bounded(&full[slot], (uint32_t)((q / kWsSlots) & 1));
    const uint8_t* b0 = slots + slot * kWsSlotBytes + (r % kWsRowsPerSlot) * kRowBytes4096 + c * 144;
    const uint8_t* b1 = b0 + (two ? kRowBytes4096 : 0);
    const uint4 hd0 = lds_v4(b0), hd1 = lds_v4(b1);
    const uint4 a0 = lds_v4(b0 + 16 + 64 * h), a1 = lds_v4(b0 + 32 + 64 * h);
    const uint4 a2 = lds_v4(b0 + 48 + 64 * h), a3 = lds_v4(b0 + 64 + 64 * h);
    const uint4 c0 = lds_v4(b1 + 16 + 64 * h), c1 = lds_v4(b1 + 32 + 64 * h);
    const uint4 c2 = lds_v4(b1 + 48 + 64 * h), c3 = lds_v4(b1 + 64 + 64 * h);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);   // both rows are in registers
    const float v0 = q4k_lane_dot(hd0, a0, a1, a2, a3, h, xd, tx, tw);
    const float v1 = q4k_lane_dot(hd1, c0, c1, c2, c3, h, xd, tx, tw);
    // one shuffle tree for both rows: after the first step lanes 0-15 carry row 0, 16-31 row 1
    const bool upper = lane >= 16;
    float v = __shfl_xor_sync(0xffffffffu, upper ? v0 : v1, 16) + (upper ? v1 : v0);
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0 || (lane == 16 && two)) {
      const int row = rb + r + (lane >> 4);
      const float o = v + (bias ? bias[row] : 0.f);
      if constexpr (ACC) y[row] += o; else y[row] = o;
    }
  }
}

template <typename XT, bool ACC>
int launch_q4k_k4096_m1_impl(const uint8_t* W, int64_t N, const void* xin, const float* norm_w, float eps,
                             const float* bias, float* y, cudaStream_t st) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemv_q4k_k4096_m1<XT, ACC>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         kWsSmem);
    if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv: smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int grid = (int)std::min<int64_t>(sm_count(), (N + 1) / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kWsThreads);
  cfg.dynamicSmemBytes = kWsSmem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_qgemv_q4k_k4096_m1<XT, ACC>, W, (int)N, xin, norm_w, eps, bias, y);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv launch: %s", cudaGetErrorString(e));
  return XM_OK;
}

template <typename XT>
int launch_q4k_k4096_m1(const uint8_t* W, int64_t N, const void* xin, const float* norm_w, float eps,
                        const float* bias, float* y, int accumulate, cudaStream_t st) {
  return accumulate ? launch_q4k_k4096_m1_impl<XT, true>(W, N, xin, norm_w, eps, bias, y, st)
                    : launch_q4k_k4096_m1_impl<XT, false>(W, N, xin, norm_w, eps, bias, y, st);
}

int q4k_tma_smem(int64_t m, int64_t nb) {
  return kGemvWarps * kGemvStages * kSlotBytes + (int)(m * nb * kColStride) +
         kGemvWarps * kGemvStages * 8 + (int)sizeof(GemvSmem) + 16;
}

// ---------------------------------------------------------------------------
// Exact path: one warp per row; the row is staged through shared memory in
// chunks, each weight decoded to the reference's fp16 value and multiplied
// with fp32 x.
// ---------------------------------------------------------------------------
template <typename XT>
XM_DEV void load_x8(const XT* p, float* v);
template <>
XM_DEV void load_x8<float>(const float* p, float* v) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
template <>
XM_DEV void load_x8<__nv_bfloat16>(const __nv_bfloat16* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}
template <>
XM_DEV void load_x8<__half>(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}

template <int T, int M, typename XT>
__global__ void __launch_bounds__(kThreads) k_qgemv_exact(const uint8_t* __restrict__ W, int64_t N, int64_t K,
                                                          const XT* __restrict__ x, const float* __restrict__ bias,
                                                          float* __restrict__ y) {
  using Q = QT<T>;
  constexpr int CHUNK_BLOCKS = 1024 / Q::QK;  // 1024 elements per chunk
  constexpr int CHUNK_BYTES = CHUNK_BLOCKS * Q::REC;
  // per-warp slice; the stride is a multiple of 16 so that every slice keeps
  // the 16-byte alignment stage_bytes' vector stores need (210- and 110-byte
  // records would otherwise leave odd warps' slices 8-byte aligned)
  constexpr int WARP_STRIDE = (CHUNK_BYTES + 32 + 15) / 16 * 16;
  __shared__ __align__(16) uint8_t sm[kThreads / 32][WARP_STRIDE];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t nb = K / Q::QK;
  const int64_t rb = nb * Q::REC;
  uint8_t* wsm = sm[warp];
  for (int64_t row = (int64_t)blockIdx.x * (kThreads / 32) + warp; row < N;
       row += (int64_t)gridDim.x * (kThreads / 32)) {
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int64_t b0 = 0; b0 < nb; b0 += CHUNK_BLOCKS) {
      const int cb = (int)min((int64_t)CHUNK_BLOCKS, nb - b0);
      __syncwarp();
      const int mis = stage_bytes(wsm, W + row * rb + b0 * Q::REC, cb * Q::REC, lane, 32);
      __syncwarp();
      const int ngroups = cb * (Q::QK / 8);
      for (int gi = lane; gi < ngroups; gi += 32) {
        const int blk = gi / (Q::QK / 8), e0 = (gi % (Q::QK / 8)) * 8;
        float w[8];
        Q::decode8(wsm + mis + blk * Q::REC, e0, w);
#pragma unroll
        for (int t = 0; t < 8; ++t) w[t] = __half2float(__float2half_rn(w[t]));
        const int64_t k0 = (b0 + blk) * Q::QK + e0;
#pragma unroll
        for (int m = 0; m < M; ++m) {
          float xv[8];
          load_x8<XT>(x + m * K + k0, xv);
#pragma unroll
          for (int t = 0; t < 8; ++t) acc[m] = fmaf(w[t], xv[t], acc[m]);
        }
      }
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const float v = warp_sum(acc[m]);
      if (lane == 0) y[m * N + row] = v + (bias ? bias[row] : 0.f);
    }
  }
}


template <int M>
struct ExactLaunch {
  const uint8_t* W; int64_t N, K; const void* x; int x_dtype; const float* bias; float* y; cudaStream_t st;
  template <int T>
  void operator()() {
    const int64_t want = (N + 7) / 8;
    const unsigned grid = (unsigned)std::min<int64_t>(want, (int64_t)sm_count() * 8);
    if (x_dtype == XM_DT_F32)
      k_qgemv_exact<T, M, float><<<grid, kThreads, 0, st>>>(W, N, K, (const float*)x, bias, y);
    else if (x_dtype == XM_DT_BF16)
      k_qgemv_exact<T, M, __nv_bfloat16><<<grid, kThreads, 0, st>>>(W, N, K, (const __nv_bfloat16*)x, bias, y);
    else
      k_qgemv_exact<T, M, __half><<<grid, kThreads, 0, st>>>(W, N, K, (const __half*)x, bias, y);
  }
};

template <int M>
void launch_exact(int qtype, const uint8_t* W, int64_t N, int64_t K, const void* x, int x_dtype, const float* bias,
                  float* y, cudaStream_t st) {
  ExactLaunch<M> l{W, N, K, x, x_dtype, bias, y, st};
  dispatch_quant(qtype, l);
}

template <int M>
void launch_q4k(const uint8_t* W, int64_t N, int64_t nb, const int8_t* pieces, const float4* ts, const float* bias,
                float* y, int accumulate, cudaStream_t st) {
  const int64_t warps = (N + 3) / 4;
  const unsigned grid = (unsigned)std::min<int64_t>((warps + 7) / 8, (int64_t)sm_count() * 4);
  k_qgemv_q4k_dp4a<M><<<grid, kThreads, 0, st>>>(W, (int)N, (int)nb, pieces, ts, bias, y, accumulate);
}

}  // namespace

// Workspace for the activation split: 64 B of digits + 16 B of (t, sums) per
// 32-element group of x (group-major), and for a single row of 4096 also the
// lane-major copy that the K = 4096 Q4_K kernel reads (9,216 B behind it).
extern "C" int64_t xm_qgemv_workspace_size(int64_t k, int64_t m) {
  if (k <= 0 || m <= 0 || (k % 32)) return 0;
  return m * (k / 32) * (kPieceBytes + 16) + (m == 1 && k == 4096 ? kLaneMajorBytes : 0);
}

namespace {

bool integer_path_type(int qtype) {
  return qtype == T_Q4_K || qtype == T_Q5_K || qtype == T_Q6_K || qtype == T_Q8_0;
}

// The single-row K = 4096 Q4_K kernel reads the lane-major layout; every other
// integer-path kernel reads the group-major one.
bool lane_major_shape(int64_t m, int64_t k) { return m == 1 && k == 4096; }

// Whether the integer path takes this type and shape (the Q4_K kernels take
// any k % 256 == 0; the generic kernel has its own limits).
bool integer_path(int qtype, int64_t n, int64_t k, int64_t m) {
  if (qtype == T_Q4_K) return true;
  return integer_path_type(qtype) && gemv_kq_supported(qtype, n, k, m);
}

int8_t* lane_major_part(const void* d_ws, int64_t m, int64_t k) {
  return (int8_t*)d_ws + m * (k / 32) * (kPieceBytes + 16);
}

int split_activation(const void* d_x, int x_dtype, int64_t m, int64_t k, void* d_ws, cudaStream_t st) {
  const int G = (int)(k / 32);
  int8_t* pieces = (int8_t*)d_ws;
  float4* ts = (float4*)((uint8_t*)d_ws + m * G * kPieceBytes);
  int8_t* lm = lane_major_shape(m, k) ? lane_major_part(d_ws, m, k) : nullptr;
  const int64_t groups = m * G;
  const unsigned sgrid = (unsigned)((groups * 32 + kThreads - 1) / kThreads);
  if (x_dtype == XM_DT_F32)
    k_split_x<float><<<sgrid, kThreads, 0, st>>>((const float*)d_x, groups, G, pieces, ts, lm);
  else if (x_dtype == XM_DT_BF16)
    k_split_x<__nv_bfloat16><<<sgrid, kThreads, 0, st>>>((const __nv_bfloat16*)d_x, groups, G, pieces, ts, lm);
  else
    k_split_x<__half><<<sgrid, kThreads, 0, st>>>((const __half*)d_x, groups, G, pieces, ts, lm);
  return xm_check_launch("split_activation");
}

int choose_lpr(int64_t nb) {
  // power of two <= 32 with the least idle columns (ties -> larger)
  int best = 1;
  int64_t best_waste = 1 << 30;
  for (int c = 1; c <= 32; c <<= 1) {
    const int64_t waste = (nb + c - 1) / c * c - nb;
    if (waste <= best_waste) { best = c; best_waste = waste; }
  }
  return best;
}

template <int M, int LPR>
int launch_q4k_tma_lpr(const uint8_t* W, int64_t N, int64_t nb, const int8_t* pieces, const float4* ts,
                       const float* bias, float* y, int accumulate, cudaStream_t st) {
  const int smem = q4k_tma_smem(M, nb);
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(k_qgemv_q4k_tma<M, LPR>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         227 * 1024);
    if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv: smem attribute: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int grid = (int)std::min<int64_t>(sm_count(), N);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_qgemv_q4k_tma<M, LPR>, W, (int)N, (int)nb, pieces, ts, bias, y,
                                     accumulate);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv launch: %s", cudaGetErrorString(e));
  return XM_OK;
}

template <int M>
int launch_q4k_tma(const uint8_t* W, int64_t N, int64_t nb, const int8_t* pieces, const float4* ts, const float* bias,
                   float* y, int accumulate, cudaStream_t st) {
  switch (choose_lpr(nb)) {
    case 1: return launch_q4k_tma_lpr<M, 1>(W, N, nb, pieces, ts, bias, y, accumulate, st);
    case 2: return launch_q4k_tma_lpr<M, 2>(W, N, nb, pieces, ts, bias, y, accumulate, st);
    case 4: return launch_q4k_tma_lpr<M, 4>(W, N, nb, pieces, ts, bias, y, accumulate, st);
    case 8: return launch_q4k_tma_lpr<M, 8>(W, N, nb, pieces, ts, bias, y, accumulate, st);
    case 16: return launch_q4k_tma_lpr<M, 16>(W, N, nb, pieces, ts, bias, y, accumulate, st);
    default: return launch_q4k_tma_lpr<M, 32>(W, N, nb, pieces, ts, bias, y, accumulate, st);
  }
}

constexpr int kMaxTmaSmem = 227 * 1024;

// GEMV from an activation split already in the workspace.  `lane_major`: the
// workspace also holds the lane-major copy (split_activation writes it for a
// single row of 4096).
int gemv_presplit(int qtype, const uint8_t* W, int64_t n, int64_t k, int64_t m, const void* d_ws, bool lane_major,
                  const float* bias, float* y, int accumulate, cudaStream_t st) {
  if (qtype != T_Q4_K) return gemv_kq(qtype, W, n, k, m, d_ws, bias, y, accumulate, st);
  const int G = (int)(k / 32);
  const int8_t* pieces = (const int8_t*)d_ws;
  const float4* ts = (const float4*)((const uint8_t*)d_ws + m * G * kPieceBytes);
  const int64_t nb = k / 256;
  if (lane_major && lane_major_shape(m, k)) {
    const int rc = launch_q4k_k4096_m1<void>(W, n, lane_major_part(d_ws, m, k), nullptr, 0.f, bias, y, accumulate,
                                             st);
    if (rc) return rc;
    return xm_check_launch("qgemv(integer, k4096 m1)");
  }
  if (q4k_tma_smem(m, nb) <= kMaxTmaSmem) {
    int rc = XM_OK;
    switch (m) {
      case 1: rc = launch_q4k_tma<1>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 2: rc = launch_q4k_tma<2>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 3: rc = launch_q4k_tma<3>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 4: rc = launch_q4k_tma<4>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 5: rc = launch_q4k_tma<5>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 6: rc = launch_q4k_tma<6>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      case 7: rc = launch_q4k_tma<7>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
      default: rc = launch_q4k_tma<8>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    }
    if (rc) return rc;
    return xm_check_launch("qgemv(integer, tma)");
  }
  if (gemv_kq_supported(qtype, n, k, m)) return gemv_kq(qtype, W, n, k, m, d_ws, bias, y, accumulate, st);
  switch (m) {
    case 1: launch_q4k<1>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 2: launch_q4k<2>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 3: launch_q4k<3>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 4: launch_q4k<4>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 5: launch_q4k<5>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 6: launch_q4k<6>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    case 7: launch_q4k<7>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
    default: launch_q4k<8>(W, n, nb, pieces, ts, bias, y, accumulate, st); break;
  }
  return xm_check_launch("qgemv(integer)");
}

int check_gemv_args(const char* who, int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, int64_t m,
                    int64_t* nb_out) {
  int qk = 0, rec = 0;
  if (!host_qtype_geometry(qtype, &qk, &rec) || qk == 1)
    return xm_set_error(XM_ERR_UNSUPPORTED, "%s: type id %d is not a block-quantized type", who, qtype);
  if (m < 1 || m > 8) return xm_set_error(XM_ERR_INVALID, "%s: m=%lld outside 1..8", who, (long long)m);
  if (n < 0 || k <= 0 || k % qk)
    return xm_set_error(XM_ERR_INVALID, "%s: k=%lld is not a positive multiple of %d", who, (long long)k, qk);
  if (k % 32) return xm_set_error(XM_ERR_INVALID, "%s: k must be a multiple of 32", who);
  if (n >= (1ll << 31)) return xm_set_error(XM_ERR_INVALID, "%s: n too large", who);
  const int64_t nb = k / qk;
  if (n * nb * rec > w_bytes)
    return xm_set_error(XM_ERR_INVALID, "%s: weight needs %lld bytes, got %lld", who, (long long)(n * nb * rec),
                        (long long)w_bytes);
  if (n > 0 && !d_w) return xm_set_error(XM_ERR_INVALID, "%s: null weight pointer", who);
  *nb_out = nb;
  return XM_OK;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int exact_path(int qtype, const uint8_t* W, int64_t n, int64_t k, const void* d_x, int x_dtype, int64_t m,
               const float* bias, float* y, cudaStream_t st) {
  switch (m) {
    case 1: launch_exact<1>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 2: launch_exact<2>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 3: launch_exact<3>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 4: launch_exact<4>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 5: launch_exact<5>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 6: launch_exact<6>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    case 7: launch_exact<7>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
    default: launch_exact<8>(qtype, W, n, k, d_x, x_dtype, bias, y, st); break;
  }
  return xm_check_launch("qgemv(exact)");
}

template <typename XT>
int launch_k4096_fused(const uint8_t* W, int64_t n, const void* x, const float* norm_w, float eps, const float* bias,
                       float* y, int accumulate, cudaStream_t st) {
  const int rc = launch_q4k_k4096_m1<XT>(W, n, x, norm_w, eps, bias, y, accumulate, st);
  if (rc) return rc;
  return xm_check_launch("qgemv(integer, k4096 m1, fused split)");
}

int k4096_fused(int x_dtype, const uint8_t* W, int64_t n, const void* x, const float* norm_w, float eps,
                const float* bias, float* y, int accumulate, cudaStream_t st) {
  if (x_dtype == XM_DT_F32) return launch_k4096_fused<float>(W, n, x, norm_w, eps, bias, y, accumulate, st);
  if (x_dtype == XM_DT_BF16) return launch_k4096_fused<__nv_bfloat16>(W, n, x, norm_w, eps, bias, y, accumulate, st);
  return launch_k4096_fused<__half>(W, n, x, norm_w, eps, bias, y, accumulate, st);
}

}  // namespace

extern "C" int xm_split_activation(const void* d_x, int x_dtype, int64_t m, int64_t k, void* d_workspace,
                                   int64_t workspace_bytes, void* stream) {
  if (m < 1 || m > 8 || k <= 0 || k % 32)
    return xm_set_error(XM_ERR_INVALID, "split_activation: need 1 <= m <= 8 and k a positive multiple of 32");
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "split_activation: bad x dtype %d", x_dtype);
  if (!d_x || !d_workspace) return xm_set_error(XM_ERR_INVALID, "split_activation: null pointer");
  if (workspace_bytes < xm_qgemv_workspace_size(k, m) || !aligned16(d_workspace))
    return xm_set_error(XM_ERR_INVALID, "split_activation: workspace too small or not 16-byte aligned");
  return split_activation(d_x, x_dtype, m, k, d_workspace, (cudaStream_t)stream);
}

extern "C" int xm_qgemv_presplit(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, int64_t m,
                                 const void* d_workspace, int64_t workspace_bytes, const float* d_bias, float* d_y,
                                 void* stream) {
  int64_t nb = 0;
  int rc = check_gemv_args("qgemv_presplit", qtype, d_w, w_bytes, n, k, m, &nb);
  if (rc) return rc;
  if (!integer_path(qtype, n, k, m))
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemv_presplit: type id %d has no integer-dot path for this shape",
                        qtype);
  if (!aligned16(d_w)) return xm_set_error(XM_ERR_INVALID, "qgemv_presplit: weight not 16-byte aligned");
  if (!d_workspace || workspace_bytes < xm_qgemv_workspace_size(k, m) || !aligned16(d_workspace))
    return xm_set_error(XM_ERR_INVALID, "qgemv_presplit: workspace too small or not 16-byte aligned");
  if (n == 0) return XM_OK;
  if (!d_y) return xm_set_error(XM_ERR_INVALID, "qgemv_presplit: null output");
  return gemv_presplit(qtype, (const uint8_t*)d_w, n, k, m, d_workspace, true, d_bias, d_y, 0, (cudaStream_t)stream);
}

extern "C" int xm_qgemv(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                        int x_dtype, int64_t m, const float* d_bias, float* d_y, void* d_workspace,
                        int64_t workspace_bytes, void* stream) {
  int64_t nb = 0;
  int rc = check_gemv_args("qgemv", qtype, d_w, w_bytes, n, k, m, &nb);
  if (rc) return rc;
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "qgemv: bad x dtype %d", x_dtype);
  if (n == 0) return XM_OK;
  if (!d_x || !d_y) return xm_set_error(XM_ERR_INVALID, "qgemv: null pointer");
  if (!aligned16(d_x)) return xm_set_error(XM_ERR_INVALID, "qgemv: x not 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const uint8_t* W = (const uint8_t*)d_w;
  if (qtype == T_Q4_K && lane_major_shape(m, k) && aligned16(d_w))
    // one row of 4096: the split is done inside the GEMV, no workspace needed
    return k4096_fused(x_dtype, W, n, d_x, nullptr, 0.f, d_bias, d_y, 0, st);
  const bool ws_ok =
      d_workspace && workspace_bytes >= xm_qgemv_workspace_size(k, m) && aligned16(d_workspace);
  if (ws_ok && aligned16(d_w) && m >= 2 && gemv_mma_supported(qtype, n, k, m) &&
      workspace_bytes >= gemv_mma_split_bytes(k, m))
    return gemv_mma(W, n, k, m, d_x, x_dtype, k, XM_PRO_NONE, nullptr, 0.f, d_bias, d_y, 0, d_workspace, st);
  if (ws_ok && aligned16(d_w) && integer_path(qtype, n, k, m)) {
    rc = split_activation(d_x, x_dtype, m, k, d_workspace, st);
    if (rc) return rc;
    return gemv_presplit(qtype, W, n, k, m, d_workspace, true, d_bias, d_y, 0, st);
  }
  return exact_path(qtype, W, n, k, d_x, x_dtype, m, d_bias, d_y, st);
}

extern "C" int xm_qgemv_ex(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                           int x_dtype, int64_t m, int64_t x_stride, int prologue, const float* d_norm_w, float eps,
                           const float* d_bias, float* d_y, int accumulate, void* d_workspace,
                           int64_t workspace_bytes, void* stream) {
  int64_t nb = 0;
  int rc = check_gemv_args("qgemv_ex", qtype, d_w, w_bytes, n, k, m, &nb);
  if (rc) return rc;
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "qgemv_ex: bad x dtype %d", x_dtype);
  if (prologue != XM_PRO_NONE && prologue != XM_PRO_RMSNORM && prologue != XM_PRO_SWIGLU)
    return xm_set_error(XM_ERR_INVALID, "qgemv_ex: unknown prologue %d", prologue);
  if (prologue == XM_PRO_RMSNORM && !d_norm_w) return xm_set_error(XM_ERR_INVALID, "qgemv_ex: RMSNorm needs weights");
  if (x_stride < (prologue == XM_PRO_SWIGLU ? 2 * k : k))
    return xm_set_error(XM_ERR_INVALID, "qgemv_ex: x_stride %lld too small", (long long)x_stride);
  if (n == 0) return XM_OK;
  if (!d_x || !d_y) return xm_set_error(XM_ERR_INVALID, "qgemv_ex: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const uint8_t* W = (const uint8_t*)d_w;
  if (qtype == T_Q4_K && lane_major_shape(m, k) && prologue != XM_PRO_SWIGLU && aligned16(d_w) && aligned16(d_x) &&
      (prologue != XM_PRO_RMSNORM || aligned16(d_norm_w)))
    return k4096_fused(x_dtype, W, n, d_x, prologue == XM_PRO_RMSNORM ? d_norm_w : nullptr, eps, d_bias, d_y,
                       accumulate, st);
  const bool ws_ok =
      d_workspace && workspace_bytes >= xm_qgemv_workspace_size(k, m) && aligned16(d_workspace);
  if (ws_ok && aligned16(d_w) && m >= 2 && gemv_mma_supported(qtype, n, k, m) &&
      workspace_bytes >= gemv_mma_split_bytes(k, m))
    return gemv_mma(W, n, k, m, d_x, x_dtype, x_stride, prologue, d_norm_w, eps, d_bias, d_y, accumulate,
                    d_workspace, st);
  if (ws_ok && aligned16(d_w) && integer_path(qtype, n, k, m)) {
    rc = split_rows(d_x, x_dtype, m, k, x_stride, prologue, d_norm_w, eps, d_workspace, st);
    if (rc) return rc;
    return gemv_presplit(qtype, W, n, k, m, d_workspace, false, d_bias, d_y, accumulate, st);
  }
  if (prologue == XM_PRO_NONE && !accumulate && x_stride == k && aligned16(d_x))
    return exact_path(qtype, W, n, k, d_x, x_dtype, m, d_bias, d_y, st);
  return xm_set_error(XM_ERR_UNSUPPORTED,
                      "qgemv_ex: prologues and accumulate need the integer-dot path (Q4_K/Q5_K/Q6_K/Q8_0, "
                      "16-byte aligned weights and a workspace)");
}

// Exact-path-only entry (used to cross-check the integer path on the same
// inputs): always the fp16-exact kernel, whatever the type and shape.
extern "C" int xm_qgemv_exact(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                              int x_dtype, int64_t m, const float* d_bias, float* d_y, void* stream) {
  int64_t nb = 0;
  int rc = check_gemv_args("qgemv_exact", qtype, d_w, w_bytes, n, k, m, &nb);
  if (rc) return rc;
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "qgemv_exact: bad x dtype %d", x_dtype);
  if (n == 0) return XM_OK;
  if (!d_x || !d_y) return xm_set_error(XM_ERR_INVALID, "qgemv_exact: null pointer");
  if (!aligned16(d_x)) return xm_set_error(XM_ERR_INVALID, "qgemv_exact: x not 16-byte aligned");
  return exact_path(qtype, (const uint8_t*)d_w, n, k, d_x, x_dtype, m, d_bias, d_y, (cudaStream_t)stream);
}

// ---------------------------------------------------------------------------
// Allocation-free GEMV.
//
// Some callers cannot allocate device memory at all: code running under a
// runtime that owns the device allocator (a host program that hands this
// library only the tensors it already has), an environment that forbids
// cudaMalloc after start-up, or a plugin that must not grow the process's
// device footprint per call.  For them, xm_qgemv_noalloc keeps the
// activation split (the only scratch the decode GEMV needs) in a fixed
// array compiled into this library instead of a caller-supplied workspace.
//
// The array is a file-scope __device__ variable, so every GPU that loads the
// library holds its own copy, kNoAllocScratchBytes long, until the process
// exits.  Its host-side name is only a stand-in for the device address, so the
// address is fetched with cudaGetSymbolAddress once per device (with that
// device current), on the first call made on that device; that first call
// should therefore happen before any stream capture.  Calls share the array:
// two calls whose kernels overlap on the GPU (different streams, no ordering
// between them) race on it.  Every call rewrites all of the split it later
// reads, so nothing in the array has to start at zero.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kNoAllocScratchBytes = 8 * (16384 / 32) * (kPieceBytes + 16);   // m <= 8, k <= 16384: 320 KiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct NoAllocTable {
  std::mutex mu;
  void* ptr[64] = {};
};
NoAllocTable& noalloc_table() {
  static NoAllocTable t;
  return t;
}
}  // namespace

extern "C" int xm_qgemv_noalloc(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                                const void* d_x, int x_dtype, int64_t m, const float* d_bias, float* d_y,
                                void* stream) {
  const int64_t need = xm_qgemv_workspace_size(k, m);
  if (need > kNoAllocScratchBytes)
    return xm_set_error(XM_ERR_INVALID,
                        "qgemv_noalloc: m=%lld, k=%lld needs %lld bytes of split scratch; the built-in array holds "
                        "%lld (m <= 8 with k <= 16384)",
                        (long long)m, (long long)k, (long long)need, (long long)kNoAllocScratchBytes);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemv_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= 64) return xm_set_error(XM_ERR_INVALID, "qgemv_noalloc: device id %d out of range", dev);
  void* scratch = nullptr;
  {
    NoAllocTable& t = noalloc_table();
    std::lock_guard<std::mutex> lock(t.mu);
    if (!t.ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p)
        return xm_set_error(XM_ERR_CUDA, "qgemv_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      t.ptr[dev] = p;
    }
    scratch = t.ptr[dev];
  }
  return xm_qgemv(qtype, d_w, w_bytes, n, k, d_x, x_dtype, m, d_bias, d_y, scratch, kNoAllocScratchBytes, stream);
}
