// K3: fused dequant-GEMM for prefill on 5th-generation tensor cores.
//
//   y[m][n] = sum_k x[m][k] * W[n][k]   (fp32 out), W in GGUF blocks of any
//   of the twelve block-quantized types (Q4_0 ... Q8_K).
//
// Numerics.  Every weight is decoded to the reference's fp16 value (the fp32
// value of gguf_dequant.py's unpacker, e.g. d*sc*q - dmin*mn for Q4_K,
// rounded once to fp16), so B is exact.  The
// activation is converted to fp16 after scaling each row by a power of two
// chosen from the row's largest magnitude (k_prep_rows): bf16 input converts
// exactly, and the scale keeps rows with large or tiny values inside fp16's
// range.  tcgen05.mma kind::f16 multiplies fp16 x fp16 exactly and
// accumulates in fp32 in tensor memory; the epilogue multiplies each row by
// its scale (exact).  The result therefore differs from the reference's
// fp32 `x @ W.T` only in summation order (and, for fp32 x, in x's fp16
// rounding).
//
// Three kernels:
//  * k_qgemm_tm<T> (the default, every block type T): persistent CTA pairs on
//    tcgen05 cta_group::2 computing y^T = W x^T: the decoded weights are the
//    M = 256 operand, written by decode warps straight into tensor memory,
//    the activations the N operand, TMA-staged in shared memory; the
//    epilogue writes y with bulk tensor stores.  Dense and grouped (MoE)
//    modes.  Its own comment block below has the details.
//  * k_qgemm_pair<T>: the same pairs with the activations as the M operand
//    and the decoded weights staged in shared memory; used when a device
//    cannot hold the tensor-memory-A kernel.
//  * k_qgemm_q4k_tc (Q4_K only): one CTA per output tile of MT*128 rows x BN
//    columns, used when a device cannot hold a CTA pair of the chosen size:
//   warp 0      TMA producer of the activation tiles (fp16, 128-byte swizzle,
//               2-D tensor map, no multicast).
//   warp 1      allocates tensor memory and issues tcgen05.mma (one thread).
//   warps 2-17  decode the weight blocks into the fp16 B tile of each
//               64-wide K step, written straight into the UMMA K-major
//               128-byte-swizzled layout, then run the epilogue.
// Pipelines are mbarrier rings with bounded waits.
#include <cuda.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "xm_internal.h"
#include "xm_qtypes.cuh"
#include "xm_decode.cuh"

namespace {
using namespace xm_decode;

constexpr int kMaxStages = 8;                  // ring depth: as many stages as shared memory holds
constexpr int kBK = 64;                        // K elements per stage (one 128-byte swizzle atom of fp16)
constexpr int kATileBytes = 128 * kBK * 2;     // one 128-row A box
constexpr int kDequantWarps = 16;
constexpr int kThreads = (2 + kDequantWarps) * 32;

XM_DEV void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 / TMA helpers
// ---------------------------------------------------------------------------
XM_DEV void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

XM_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
XM_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

XM_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

XM_DEV void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Wait for an mbarrier phase, testing once without suspending first (the
// common case on the MMA thread is that the stage is already full).
XM_DEV void mbar_wait_fast(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  if (!ok) mbar_wait_bounded(bar, parity);
}

XM_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
XM_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
XM_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor: K-major operand in the 128-byte swizzle
// layout (8-row groups 1024 bytes apart, 16-byte chunks XOR-ed by row % 8).
XM_DEV uint64_t smem_desc_sw128(const void* p) {
  const uint64_t addr = smem_u32(p);
  uint64_t d = 0;
  d |= (addr >> 4) & 0x3FFFull;            // start address
  d |= (uint64_t)1 << 16;                  // leading byte offset (16 B; unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;        // stride byte offset: 8-row group pitch
  d |= (uint64_t)1 << 46;                  // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                  // 128-byte swizzle
  return d;
}

// Instruction descriptor: fp16 x fp16 -> fp32, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int n) {
  return (1u << 4)                       // D format f32
         | (0u << 7) | (0u << 10)        // A, B format f16
         | ((uint32_t)(n >> 3) << 17)    // N >> 3
         | ((uint32_t)(128 >> 4) << 24); // M >> 4
}

// ---------------------------------------------------------------------------
// Activation preparation: fp16 copy of pro(x) with a power-of-two scale per
// row (prep_row_fp16: one block per row, vector loads).  rowscale[m] = 2^s
// with the row's max magnitude in [2^14, 2^15) after division by 2^s (s may
// be negative for small rows).
// PRO is an XM_PRO_* prologue, applied in fp32 in the reference's order:
//   XM_PRO_RMSNORM  v = (x / sqrt(mean(x^2) + eps)) * norm_w   (ops.py:115-117)
//   XM_PRO_SWIGLU   v = silu(x[:K]) * x[K:2K]                  (forward.py:97-98)
// `ldx` is the row pitch of x in elements.  NTH threads per block: 256, or
// 1024 when the rows are too few to occupy the device (a decode step's 4-8
// rows), so that each row's two passes are short.
// ---------------------------------------------------------------------------
template <typename XT, int PRO, int NTH = kPrepThreads>
__global__ void __launch_bounds__(NTH) k_prep_rows(const XT* __restrict__ x, int M, int K, int64_t ldx,
                                                            const float* __restrict__ norm_w, float eps,
                                                            __half* __restrict__ x16, float* __restrict__ rowscale) {
  __shared__ float red[32];
  const int row = blockIdx.x;
  const XT* xr = x + (int64_t)row * ldx;
  float rms = 1.f;
  if constexpr (PRO == XM_PRO_RMSNORM) {
    float ss = 0.f;
    for (int k = threadIdx.x * 4; k < K; k += NTH * 4) {
      float v[4];
      ld4f<XT>(xr + k, v);
      ss = fmaf(v[0], v[0], fmaf(v[1], v[1], fmaf(v[2], v[2], fmaf(v[3], v[3], ss))));
    }
    rms = sqrtf(block_sum<NTH>(ss, red) / (float)K + eps);
  }
  prep_row_fp16_n<NTH>(
      [&](int k, float (&v)[4]) {
        ld4f<XT>(xr + k, v);
        if constexpr (PRO == XM_PRO_RMSNORM) {
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = (v[i] / rms) * norm_w[k + i];
        } else if constexpr (PRO == XM_PRO_SWIGLU) {
          float u[4];
          ld4f<XT>(xr + K + k, u);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i] = v[i] / (1.0f + expf(-v[i])) * u[i];
        }
      },
      K, x16 + (int64_t)row * K, rowscale + row, red);
}

// Plain RMSNorm of rows (one warp per row), fp32 out: the norm of
// FusedRMSNormLinearOp for weights whose matmul has no fused prologue.
template <typename XT>
__global__ void __launch_bounds__(256) k_rmsnorm_rows(const XT* __restrict__ x, int M, int K, int64_t ldx,
                                                      const float* __restrict__ norm_w, float eps,
                                                      float* __restrict__ out) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const XT* xr = x + (int64_t)warp * ldx;
  float ss = 0.f;
  for (int k = lane; k < K; k += 32) {
    const float v = to_f32(xr[k]);
    ss = fmaf(v, v, ss);
  }
  const float rms = sqrtf(warp_sum(ss) / (float)K + eps);
  float* o = out + (int64_t)warp * K;
  for (int k = lane; k < K; k += 32) o[k] = (to_f32(xr[k]) / rms) * norm_w[k];
}

// ---------------------------------------------------------------------------
// The GEMM kernel.
// ---------------------------------------------------------------------------
// Grouped mode (MoE experts): group g = blockIdx.z multiplies rows
// [off[g], off[g] + cnt[g]) of the activation with weight w[g]; the row
// ranges come from the device-side expert sort, so they are read after the
// grid dependency resolves and CTAs past the end of their group exit at once.
constexpr int kMaxGroups = 32;
struct GemmGroups {
  int n;                               // 0: single GEMM
  const int* cnt;
  const int* off;
  const uint8_t* w[kMaxGroups];        // passed by value: no device-side pointer table to build
};

struct GemmSmem {
  uint64_t full[kMaxStages], ab_empty[kMaxStages];   // full: A bytes + one arrival per decode warp
  uint64_t acc_full;
  uint32_t tmem_base;
};

// One decode item: 32 weights (sub-block 2j+h of row n in K step kt) as raw bytes.
struct RawItem {
  uint4 hd;        // d, dmin, 12 scale bytes
  uint4 q0, q1;    // the 32 qs bytes of sub-block pair j
};

XM_DEV RawItem load_item(const uint8_t* W, int64_t row_bytes, int n, int N, int kt) {
  RawItem it;
  const int nn = n < N ? n : N - 1;                    // rows past N decode a valid row; the epilogue drops them
  const uint8_t* blk = W + (int64_t)nn * row_bytes + (int64_t)(kt >> 2) * 144;
  const int j = kt & 3;
  it.hd = ldg_stream_v4(blk);
  it.q0 = ldg_stream_v4(blk + 16 + 32 * j);
  it.q1 = ldg_stream_v4(blk + 32 + 32 * j);
  return it;
}

// Decode chunks c0 .. c0+NC-1 (8 weights each) of sub-block 2j+h of one row
// into fp16 and store them into the swizzled B row (n: the row's index within
// its 8-row swizzle group pattern).  qw holds the qs words of those chunks,
// two per chunk; hd is the record's 16-byte header.
template <int NC>
XM_DEV void decode_part(const uint4& hd, const uint32_t (&qw)[2 * NC], int h, int j, int c0, uint8_t* row, int n) {
  const uint32_t A = hd.y, B = hd.z, C = hd.w;
  const int sub = 2 * j + h;
  const uint32_t scw = sub < 4 ? (A & 0x3F3F3F3Fu) : ((C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u));
  const uint32_t mnw = sub < 4 ? (B & 0x3F3F3F3Fu) : (((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u));
  const float d = __half2float(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
  const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
  const float d1 = __fmul_rn(d, byte_f(scw, sub & 3));       // exact (11-bit x 6-bit)
  const float m1 = __fmul_rn(dmin, byte_f(mnw, sub & 3));
  const float2 dd = make_float2(d1, d1), mm = make_float2(-m1, -m1), mg = make_float2(-8388608.0f, -8388608.0f);
  const int sh = 4 * h;
#pragma unroll
  for (int c = 0; c < NC; ++c) {          // chunk c0 + c: weights 8(c0+c) .. 8(c0+c)+7 of the sub-block
    uint32_t hv[4];
#pragma unroll
    for (int wv = 0; wv < 2; ++wv) {
      const uint32_t nib = (qw[2 * c + wv] >> sh) & 0x0F0F0F0Fu;
#pragma unroll
      for (int p = 0; p < 2; ++p) {
        // 2^23 + q as floats (magic exponent), minus 2^23: exact small integers
        float2 q = make_float2(__uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7650u | (2 * p))),
                               __uint_as_float(__byte_perm(nib, 0x4B000000u, 0x7650u | (2 * p + 1))));
        q = __fadd2_rn(q, mg);
        // d1*q is exact, so one rounding of d1*q - m1 is the reference's fp32 value
        const float2 v = __ffma2_rn(dd, q, mm);
        const __half2 hh = __floats2half2_rn(v.x, v.y);
        hv[2 * wv + p] = *reinterpret_cast<const uint32_t*>(&hh);
      }
    }
    const int chunk = 4 * h + c0 + c;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (n & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

// One whole item (all 4 chunks of the sub-block).
XM_DEV void decode_item(const RawItem& it, int h, int j, uint8_t* row, int n) {
  const uint32_t qw[8] = {it.q0.x, it.q0.y, it.q0.z, it.q0.w, it.q1.x, it.q1.y, it.q1.z, it.q1.w};
  decode_part<4>(it.hd, qw, h, j, 0, row, n);
}

__global__ void __launch_bounds__(kThreads, 1)
    k_qgemm_q4k_tc(const __grid_constant__ CUtensorMap map_a, const uint8_t* __restrict__ W0, int M, int N,
                   int K, int MT, int BN, int kStages, const float* __restrict__ rowscale,
                   const float* __restrict__ bias, float* __restrict__ y, int acc, GemmGroups groups) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned carve-up: A stages | B stages | control
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_stage_bytes = MT * kATileBytes;
  const int b_stage_bytes = BN * kBK * 2;
  uint8_t* sA = base;
  uint8_t* sB = sA + kStages * a_stage_bytes;
  GemmSmem* ctl = reinterpret_cast<GemmSmem*>(sB + kStages * b_stage_bytes);
  const int64_t row_bytes = (int64_t)(K / 256) * 144;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * BN;
  int mlo = 0, mhi = M;
  const uint8_t* W = W0;
  if (groups.n) {
    grid_dep_wait();                   // counts and offsets come from the preceding sort kernel
    const int g = blockIdx.z;
    mlo = groups.off[g];
    mhi = mlo + groups.cnt[g];
    W = groups.w[g];
  }
  const int m0 = mlo + blockIdx.y * (MT * 128);
  if (m0 >= mhi) return;               // whole CTA: nothing of this group left
  const int nkt = K / kBK;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&ctl->full[i], 1 + kDequantWarps);
      mbar_init(&ctl->ab_empty[i], 1);
    }
    mbar_init(&ctl->acc_full, 1);
    fence_mbar_init();
  }
  uint32_t ncols = 32;
  while (ncols < (uint32_t)(MT * BN)) ncols <<= 1;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl->tmem_base)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      grid_dep_wait();   // the prepared activation comes from the preceding kernel
      for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % kStages;
        if (kt >= kStages) mbar_wait_bounded(&ctl->ab_empty[s], (uint32_t)(((kt / kStages) - 1) & 1));
        mbar_arrive_expect_tx(&ctl->full[s], (uint32_t)a_stage_bytes);
        for (int mt = 0; mt < MT; ++mt)
          tma_load_2d(sA + s * a_stage_bytes + mt * kATileBytes, &map_a, kt * kBK, m0 + mt * 128, &ctl->full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(BN);
      // descriptors of stage 0; stage s and K sub-step kk only move the start
      // address (16-byte units): + s*stage_bytes/16 + kk*2
      const uint64_t a0 = smem_desc_sw128(sA), b0 = smem_desc_sw128(sB);
      int s = 0;
      uint32_t ph = 0;
      for (int kt = 0; kt < nkt; ++kt) {
        mbar_wait_fast(&ctl->full[s], ph);
        tc_fence_after();
        const uint64_t as = a0 + (uint64_t)((s * a_stage_bytes) >> 4);
        const uint64_t bs = b0 + (uint64_t)((s * b_stage_bytes) >> 4);
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            tc_mma_f16(tmem + (uint32_t)(mt * BN), as + (uint64_t)((mt * kATileBytes) >> 4) + 2 * kk, bs + 2 * kk,
                       idesc, (kt | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&ctl->ab_empty[s]);   // frees the stage once these MMAs have read it
        if (++s == kStages) { s = 0; ph ^= 1u; }
      }
      tc_commit(&ctl->acc_full);
    }
  } else {
    // ---------------- dequant producers ----------------
    const int dt = (warp - 2) * 32 + lane;       // 0..511: one item (row dt/2, half dt&1) per K step
    const int h = dt & 1;
    const int n = dt >> 1;
    const bool active = n < BN;
    // block bytes are prefetched kPre K steps ahead into a register ring
    // (the loads come from L2; one step of lookahead left the warps waiting)
    constexpr int kPre = 3;
    RawItem ring[kPre];
#pragma unroll
    for (int u = 0; u < kPre; ++u)
      if (u < nkt && active) ring[u] = load_item(W, row_bytes, n0 + n, N, u);
    for (int kt0 = 0; kt0 < nkt; kt0 += kPre) {
#pragma unroll
      for (int u = 0; u < kPre; ++u) {
        const int kt = kt0 + u;
        if (kt < nkt) {
          const RawItem cur = ring[u];
          if (kt + kPre < nkt && active) ring[u] = load_item(W, row_bytes, n0 + n, N, kt + kPre);
          const int s = kt % kStages;
          if (kt >= kStages) mbar_wait_bounded(&ctl->ab_empty[s], (uint32_t)(((kt / kStages) - 1) & 1));
          if (active) decode_item(cur, h, kt & 3, sB + s * b_stage_bytes + n * 128, n);
          fence_proxy_async_smem();    // generic-proxy writes -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->full[s]);
        }
      }
    }
    // ---------------- epilogue ----------------
    // tcgen05.ld gives each lane 32 consecutive columns of its own row; a
    // per-warp padded shared-memory tile turns that into row-contiguous
    // 128-byte stores (lane-per-row stores scattered 4 bytes over 32 rows and
    // held every CTA on its SM for tens of microseconds while they drained).
    mbar_wait_bounded(&ctl->acc_full, 0);
    tc_fence_after();
    const int sp = warp & 3;                     // TMEM sub-partition this warp may read
    const int quarter = (warp - 2) >> 2;         // four warps per sub-partition split the columns
    float* tile = reinterpret_cast<float*>(sA) + (warp - 2) * (32 * 33);   // operand stages are free now
    const int nchunks = BN / 32;
    for (int mt = 0; mt < MT; ++mt) {
      const int mrow0 = m0 + mt * 128 + sp * 32;
      for (int ch = quarter; ch < nchunks; ch += 4) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(sp * 32) << 16) + (uint32_t)(mt * BN + ch * 32), v);
        tmem_ld_wait();
        const float rs = (mrow0 + lane) < mhi ? rowscale[mrow0 + lane] : 0.f;
#pragma unroll
        for (int t = 0; t < 32; ++t) tile[lane * 33 + t] = __uint_as_float(v[t]) * rs;
        __syncwarp();
        const int nn = n0 + ch * 32 + lane;
        const float bv = (bias && nn < N) ? bias[nn] : 0.f;
        for (int r = 0; r < 32; ++r) {
          const int m = mrow0 + r;
          if (m < mhi && nn < N) {
            float* yp = y + (int64_t)m * N + nn;
            const float o = tile[r * 33 + lane] + bv;
            *yp = acc ? *yp + o : o;
          }
        }
        __syncwarp();
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Persistent CTA-pair GEMM (prefill and MoE expert GEMMs).
//
// A cluster of two CTAs on neighbouring SMs computes 256-row output tiles
// with tcgen05.mma.cta_group::2 (M = 256): CTA r of the pair holds activation
// rows [128r, 128r+128) of the tile and decodes its half of every N = BN
// weight block (output columns [r*BN/2, (r+1)*BN/2) of that block), so each
// SM decodes half of the B operand that the 256-row MMA consumes and reads
// only its own halves from shared memory.  Tiles go round-robin over the
// pairs (order: pair_tile).
//
// Per CTA (2 + 16 + 4 + 1 warps):
//   warp 0      TMA producer of the fp16 activation box (64 K x 128 rows,
//               128-byte swizzle) of every 64-wide K step.  Rank 1's
//               activation box completes on rank 0's barrier (cta_group::2
//               form of the tensor load; no multicast).
//   warp 22     TMA producer of the raw block records of the CTA's weight
//               rows, one 256-wide K column per stage (ColGeom<T>: a box of BB
//               bytes x BN/2 rows per N half, starting at the column's first
//               byte rounded down to 16 -- TMA's alignment rule -- and wide
//               enough for the column at any of its offsets); a thread of its
//               own so that the next column is requested as soon as a raw
//               slot is free.
//   warp 1      TMEM allocation (both ranks); rank 0 issues the MMAs.
//   warps 2-17  decode, two groups of 8 warps taking turns by K step: one
//               thread per (row, 32-weight sub-block) item, from the staged
//               records into the swizzled B half of its CTA.
//   warps 18-21 epilogue: TMEM -> row scale (+ bias) -> y, one TMEM
//               sub-partition each, while the MMA fills the other accumulator.
// Every per-step loop keeps its ring position and phase in running counters:
// those loops run on single threads, where an integer division per step
// costs more than the step's synchronisation.
//
// Barriers (all waits bounded; a timeout sets the device error word and later
// waits give up at once, so a lost arrival ends the kernel instead of hanging):
//   wfull/wempty[RW]   raw record ring (TMA bytes / 16 decode-warp arrivals)
//   ofull[S]           (rank 0 only) operand stage of both CTAs: the two
//                      producers' expect-tx arrivals and TMA bytes + the 8 + 8
//                      warps of the decode group that owns the step
//   oempty[S]          MMA commit, multicast to both CTAs
//   acc_full[2]        MMA commit after the tile's last K step, both CTAs
//   acc_empty[2]       (rank 0) 4 + 4 epilogue warps of the two CTAs
// Remote arrivals use the default (release, CTA-scope) semantics: a
// cluster-scope release costs ~200 ns per arrival here against ~50 ns.
// ---------------------------------------------------------------------------
constexpr int kPairEpiWarps = 4;
// warps: TMA producer of the activation tiles, MMA issuer, DW decode warps,
// the epilogue warps, and the TMA producer of the raw weight records
constexpr int pair_threads(int dw) { return (2 + dw + kPairEpiWarps + 1) * 32; }
constexpr int kMaxRawStages = 2;
constexpr int kEpiTileFloats = 32 * 33;        // per-warp padded 32 x 32 staging tile

// Staging geometry of one 256-wide K column of a weight row of type T: CB
// bytes in the row (one Q4_K record; eight Q8_0 records; ...).  Column kb
// starts at byte kb*CB of its row, which is 16-byte aligned only when CB is a
// multiple of 16; its offset inside the 16-byte unit is a multiple of
// gcd(CB, 16), at most MIS.  The TMA box (BB bytes per row, 16-bit elements)
// starts at the rounded-down address and covers CB + MIS bytes, rounded up
// to an odd number of 16-byte units: rows BB bytes apart then fall on
// distinct 16-byte bank groups for 8 consecutive rows, so the decoders'
// 16-byte shared loads (one row per thread) are conflict-free.
constexpr int gcd16(int v) { return (v & 15) == 0 ? 16 : (v & 7) == 0 ? 8 : (v & 3) == 0 ? 4 : (v & 1) == 0 ? 2 : 1; }
template <int T>
struct ColGeom {
  static constexpr int QK = QT<T>::QK, REC = QT<T>::REC;
  static constexpr int CB = REC * (256 / QK);
  static constexpr int MIS = (CB & 15) == 0 ? 0 : 16 - gcd16(CB);
  static constexpr int BB0 = (CB + MIS + 15) / 16 * 16;
  static constexpr int BB = (BB0 / 16) % 2 ? BB0 : BB0 + 16;
  static_assert(BB / 2 <= 256, "TMA box width");
};

// NW consecutive 32-bit words at a 2-byte-aligned shared address: NW + 1
// aligned loads joined by funnel shifts (shift 0 or 16).
template <int NW>
XM_DEV void smem_words(const uint8_t* p, uint32_t (&w)[NW]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
  const uint32_t sh = (uint32_t)(a & 3) * 8;
  uint32_t prev = base[0];
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    const uint32_t next = base[i + 1];
    w[i] = __funnelshift_r(prev, next, sh);
    prev = next;
  }
}

// Q6_K item (gguf_dequant.py:392-436): weights 64j + 32h + l, l = 0..31, of the
// record at `rec` (2-byte aligned): half hh = j/2 of the super-block, quarter
// i = 2(j%2) + h; code = nibble i/2 of ql[64hh + 32(i%2) + l] | bits 2i..2i+1 of
// qh[32hh + l] << 4; value (d * sc[8hh + 2i + l/16]) * (code - 32) -- an exact
// product, rounded once to fp16 as the reference's astype does.
XM_DEV void decode_q6k_item(const uint8_t* rec, int j, int h, uint8_t* row, int n) {
  const int hh = j >> 1, i = 2 * (j & 1) + h;
  uint32_t ql[8], qh[8];
  smem_words<8>(rec + 64 * hh + 32 * (i & 1), ql);
  smem_words<8>(rec + 128 + 32 * hh, qh);
  const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(rec + 208)));
  const float ds0 = d * (float)(int8_t)rec[192 + 8 * hh + 2 * i];       // exact (11-bit x 8-bit)
  const float ds1 = d * (float)(int8_t)rec[192 + 8 * hh + 2 * i + 1];
  const int nsh = 4 * (i >> 1), hsh = 2 * i;
#pragma unroll
  for (int c = 0; c < 4; ++c) {               // chunk c: weights 8c .. 8c+7 of the item (words 2c, 2c+1)
    const float ds = c < 2 ? ds0 : ds1;
    const float2 dd = make_float2(ds, ds);
    uint32_t hv[4];
#pragma unroll
    for (int wv = 0; wv < 2; ++wv) {
      const int w = 2 * c + wv;
      const uint32_t q = ((ql[w] >> nsh) & 0x0F0F0F0Fu) | (((qh[w] >> hsh) & 0x03030303u) << 4);
      float2 lo, hi;
      bytes_minus(q, 32.0f, lo, hi);
      hv[2 * wv] = half2_bits(__fmul2_rn(lo, dd));
      hv[2 * wv + 1] = half2_bits(__fmul2_rn(hi, dd));
    }
    const int chunk = 4 * h + c;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (n & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

// Q5_K item (gguf_dequant.py:347-386, with the reference's high-bit layout):
// sub-block s = 2j + h, weights l = 0..31: code = nibble h of qs[48 + 32j + l]
// + 16 * (bit l of the little-endian u32 at 16 + 4j); value (d*sc_s)*code -
// dmin*mn_s with one rounding (the products are exact).  The record is
// 16-byte aligned (176-byte records, 16-byte aligned columns).
XM_DEV void decode_q5k_item(const uint8_t* rec, int j, int h, uint8_t* row, int n) {
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
  for (int c = 0; c < 4; ++c) {
    uint32_t hv[4];
#pragma unroll
    for (int wv = 0; wv < 2; ++wv) {
      const int w = 2 * c + wv;
      // bits 4w..4w+3 of the high-bit word -> bit 4 of bytes 0..3 (the partial products do not overlap)
      const uint32_t fifth = (((qh32 >> (4 * w)) & 0xFu) * 0x02040810u) & 0x10101010u;
      const uint32_t q = ((qw[w] >> sh) & 0x0F0F0F0Fu) | fifth;
      float2 lo, hi;
      bytes_minus(q, 0.0f, lo, hi);
      hv[2 * wv] = half2_bits(__ffma2_rn(dd, lo, mm));
      hv[2 * wv + 1] = half2_bits(__ffma2_rn(dd, hi, mm));
    }
    const int chunk = 4 * h + c;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (n & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

// Q8_0 item (gguf_dequant.py:143-156): record 2j + h of the 256-wide column
// (34 bytes, 2-byte aligned): int8(q) * d, an exact product rounded once.
XM_DEV void decode_q8_0_item(const uint8_t* col, int j, int h, uint8_t* row, int n) {
  const uint8_t* rec = col + (2 * j + h) * 34;
  const float d = __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short*>(rec)));
  const float2 dd = make_float2(d, d);
  uint32_t qw[8];
  smem_words<8>(rec + 2, qw);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t hv[4];
#pragma unroll
    for (int wv = 0; wv < 2; ++wv) {
      float2 lo, hi;
      bytes_minus(qw[2 * c + wv] ^ 0x80808080u, 128.0f, lo, hi);   // signed byte b: (b + 128) - 128
      hv[2 * wv] = half2_bits(__fmul2_rn(lo, dd));
      hv[2 * wv + 1] = half2_bits(__fmul2_rn(hi, dd));
    }
    const int chunk = 4 * h + c;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (n & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

// One decode item of a type without a hand-tuned decoder: weights 32h .. 32h+31
// of K step j (64 weights) of one row, from the staged column `col`, rounded
// to fp16 (the reference's values) and stored as four 16-byte chunks into the
// swizzled B row (n: the row's index for the swizzle pattern).
template <int T>
XM_DEV void decode_item_generic(const uint8_t* col, int j, int h, uint8_t* row, int n) {
  using Q = QT<T>;
  const uint8_t* rec = Q::QK == 256 ? col : col + (2 * j + h) * Q::REC;
  const int e0 = Q::QK == 256 ? 64 * j + 32 * h : 0;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    float v[8];
    Q::decode8(rec, e0 + 8 * c, v);
    uint32_t hv[4];
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const __half2 hh = __floats2half2_rn(v[2 * p], v[2 * p + 1]);
      hv[p] = *reinterpret_cast<const uint32_t*>(&hh);
    }
    const int chunk = 4 * h + c;
    *reinterpret_cast<uint4*>(row + ((chunk ^ (n & 7)) << 4)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
  }
}

struct PairSmem {
  uint64_t wfull[kMaxRawStages], wempty[kMaxRawStages];
  uint64_t ofull[kMaxStages], oempty[kMaxStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
};

XM_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cta address -> shared::cluster address of the same variable in CTA `rank`
XM_DEV uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
XM_DEV void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
XM_DEV void mbar_arrive_expect_tx_remote(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(bytes)
               : "memory");
}
XM_DEV bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
               : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}
// Bounded wait.  A non-blocking test first: most waits find the phase already
// complete, and try_wait costs noticeably more than test_wait even then.
// Gives up at once when another wait anywhere has recorded a timeout.
// Barriers that count arrivals from the peer CTA are waited on with the
// default (CTA-scope) acquire, as in the established 2-SM MMA pipelines: the
// peer's arrivals follow its proxy fence, and the mbarrier phase completion
// orders them before the MMAs issued after tcgen05.fence::after_thread_sync.
XM_DEV bool pair_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_test_wait(bar, parity)) return true;
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && *reinterpret_cast<volatile int*>(&g_xm_device_error)) return false;
  }
  atomicOr(&g_xm_device_error, XM_DEVERR_TIMEOUT);
  return false;
}
// 2-D tensor load into this CTA's shared memory whose completion is counted
// on an mbarrier of either CTA of the pair (no multicast)
XM_DEV void tma_load_2d_pair(void* dst, const CUtensorMap* map, int c0, int c1, uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(bar_cluster_addr)
      : "memory");
}
XM_DEV void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
XM_DEV void tc2_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` (same shared offset) in both CTAs of the pair once the
// previously issued MMAs have completed
XM_DEV void tc2_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(smem_u32(bar)), "h"((uint16_t)3)
      : "memory");
}
__host__ __device__ constexpr uint32_t idesc_f16_f32_m256(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

// Weight tensor maps and (grouped mode) the device-side row ranges of the
// groups.  NMAP = 1: one dense GEMM; NMAP = kMaxGroups: group g multiplies
// activation rows [off[g], off[g] + cnt[g]) with weight g.
template <int NMAP>
struct PairW {
  CUtensorMap map[NMAP];
  const int* cnt;
  const int* off;
  int groups;
};

struct PairTile {
  int g, am0, mhi, col0;   // group, first activation row of the 256-row tile, row limit, first output column
};

// Tile t of the round-robin order.  Dense: m-fastest, so the pairs that run
// together share a weight column tile in L2.  Grouped: n-fastest within
// (group, m tile), so the tiles past a group's row count (skipped, identically
// by every role) form whole runs and the real tiles spread evenly over pairs.
template <int NMAP>
XM_DEV bool pair_tile(const PairW<NMAP>& pw, int t, int M, int TM, int TN, int width, PairTile& pt) {
  if (NMAP == 1) {
    pt.g = 0;
    pt.am0 = (t % TM) * 256;
    pt.mhi = M;
    pt.col0 = (t / TM) * width;
    return true;
  }
  const int nt = t % TN, r = t / TN;
  const int mt = r % TM, g = r / TM;
  const int lo = pw.off[g], cnt = pw.cnt[g];
  pt.g = g;
  pt.am0 = lo + mt * 256;
  pt.mhi = lo + cnt;
  pt.col0 = nt * width;
  return mt * 256 < cnt;
}

// NH = 1: tile 256 x BN, two accumulators (the epilogue of one tile overlaps
// the main loop of the next).  NH = 2: tile 256 x 2BN as two N = BN MMAs into
// one accumulator of 2BN columns (fewer, wider tiles for mid-size M).
template <int T, int DW, int NMAP>
__global__ void __launch_bounds__(pair_threads(DW), 1)
    k_qgemm_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ PairW<NMAP> pw, int M, int N,
                 int K, int BN, int NH, int S, int RW, int TM, const float* __restrict__ rowscale,
                 const float* __restrict__ bias, float* __restrict__ y, int acc) {
  using CG = ColGeom<T>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int hb = BN >> 1;                         // rows of each N half this CTA decodes
  const int rows = NH * hb;                       // weight rows decoded by this CTA per K step
  const int width = NH * BN;                      // output columns of a tile
  const int ostage = kATileBytes + rows * 128;    // [A 128 x 64 fp16 | B half 0 | B half 1], 1024-byte multiples
  const int wstage = rows * CG::BB;               // the CTA's staged bytes of one 256-wide K column
  uint8_t* sO = base;
  uint8_t* sW = sO + S * ostage;
  float* sEpi = reinterpret_cast<float*>(sW + RW * wstage);
  PairSmem* ctl = reinterpret_cast<PairSmem*>(sEpi + kPairEpiWarps * kEpiTileFloats);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int TN = (N + width - 1) / width;
  const int NT = TM * TN * (NMAP == 1 ? 1 : pw.groups);   // tiles
  const int KB = K >> 8, nkt = K / kBK;
  const int nacc = NH == 1 ? 2 : 1;               // accumulators of `width` columns in TMEM

  if (tid == 0) {
    for (int i = 0; i < RW; ++i) {
      mbar_init(&ctl->wfull[i], 1);
      mbar_init(&ctl->wempty[i], DW);
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl->ofull[i], 2 + 2 * 8);       // rank 0 only: 2 producers + 8 warps of one decode group per CTA
      mbar_init(&ctl->oempty[i], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], 1);
      mbar_init(&ctl->acc_empty[b], 2 * kPairEpiWarps);
    }
    fence_mbar_init();
  }
  constexpr uint32_t kCols = 512;                 // nacc * width <= 512 columns
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl->tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();                             // barriers of both CTAs initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  // the group row ranges (and the prepared activation) come from the preceding kernel
  if (NMAP > 1) grid_dep_wait();

  // Ring positions advance incrementally (no division on the per-step paths,
  // which run on single threads).  Waits on an "empty" barrier use the
  // opposite parity, so the first lap passes at once.
  if (warp == 0) {
    // ---------------- TMA producer: activation tiles ----------------
    if (lane == 0) {
      grid_dep_wait();
      const uint32_t leader_ofull = mapa_shared(smem_u32(&ctl->ofull[0]), 0);
      uint32_t s = 0, ph = 0;
      for (int t = pair; t < NT; t += npairs) {
        PairTile pt;
        if (!pair_tile(pw, t, M, TM, TN, width, pt)) continue;
        const int am = pt.am0 + (int)rank * 128;
        int ka = 0;
        for (int kb = 0; kb < KB; ++kb) {
          for (int j = 0; j < 4; ++j, ka += kBK) {
            pair_wait(&ctl->oempty[s], ph ^ 1);
            if (rank == 0) {
              mbar_arrive_expect_tx(&ctl->ofull[s], (uint32_t)kATileBytes);
              tma_load_2d(sO + s * ostage, &map_a, ka, am, &ctl->ofull[s]);
            } else {
              mbar_arrive_expect_tx_remote(leader_ofull + 8u * s, (uint32_t)kATileBytes);
              tma_load_2d_pair(sO + s * ostage, &map_a, ka, am, leader_ofull + 8u * s);
            }
            if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer ----------------
      const uint32_t idesc = idesc_f16_f32_m256(BN);
      const uint64_t a0 = smem_desc_sw128(sO), b0 = smem_desc_sw128(sO + kATileBytes);
      const uint64_t step = (uint64_t)(ostage >> 4), bhalf = (uint64_t)((hb * 128) >> 4);
      uint32_t s = 0, ph = 0, it = 0;
      uint64_t off = 0;
      for (int t = pair; t < NT; t += npairs) {
        PairTile pt;
        if (!pair_tile(pw, t, M, TM, TN, width, pt)) continue;
        const uint32_t b = nacc == 2 ? (it & 1) : 0u, u = nacc == 2 ? (it >> 1) : it;
        pair_wait(&ctl->acc_empty[b], (u & 1) ^ 1);
        tc_fence_after();
        const uint32_t d = tmem + b * (uint32_t)width;
        for (int kt = 0; kt < nkt; ++kt) {
          pair_wait(&ctl->ofull[s], ph);
          tc_fence_after();
          for (int h = 0; h < NH; ++h) {
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              tc2_mma_f16(d + (uint32_t)(h * BN), a0 + off + 2 * kk, b0 + off + h * bhalf + 2 * kk, idesc,
                          (kt | kk) != 0 ? 1u : 0u);
          }
          tc2_commit_pair(&ctl->oempty[s]);      // both CTAs may refill the stage once these MMAs are done
          off += step;
          if (++s == (uint32_t)S) { s = 0; ph ^= 1; off = 0; }
        }
        tc2_commit_pair(&ctl->acc_full[b]);
        ++it;
      }
    }
  } else if (warp < 2 + DW) {
    // ---------------- decode ----------------
    // DW / 8 groups of 8 warps take turns by K step (group g decodes the steps
    // q with q % groups == g), so several stages are decoded at once.  In a
    // group, one thread decodes one (row, sub-block) item; 128 rows per pass,
    // a CTA with 2 x 128 rows takes two passes.
    constexpr int kGroups = DW / 8;
    const int grp = (warp - 2) >> 3;
    const int dt = ((warp - 2) & 7) * 32 + lane;
    const int h = dt & 1, n = dt >> 1;
    const uint32_t leader_ofull = mapa_shared(smem_u32(&ctl->ofull[0]), 0);
    uint32_t s = (uint32_t)grp, ph = 0, rs = 0, rph = 0;   // this group's first step is q = grp (< S)
    for (int t = pair; t < NT; t += npairs) {
      PairTile pt;
      if (!pair_tile(pw, t, M, TM, TN, width, pt)) continue;
      for (int kb = 0; kb < KB; ++kb) {
        pair_wait(&ctl->wfull[rs], rph);
        const int mis = (kb * CG::CB) & 15;       // the column's offset in its staged box (0 for Q4_K)
        [[maybe_unused]] uint4 hd[2];
        if constexpr (T == T_Q4_K) {
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int rl = p * 128 + n;
            if (rl < rows) hd[p] = *reinterpret_cast<const uint4*>(sW + rs * wstage + rl * CG::BB);
          }
        }
        for (int j = grp; j < 4; j += kGroups) {
          pair_wait(&ctl->oempty[s], ph ^ 1);
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int rl = p * 128 + n;
            if (rl < rows) {
              const int half = rl >= hb ? 1 : 0, rr = rl - half * hb;
              const uint8_t* rec = sW + rs * wstage + rl * CG::BB + mis;
              uint8_t* dst = sO + s * ostage + kATileBytes + half * hb * 128 + rr * 128;
              if constexpr (T == T_Q4_K) {
                const uint4 q0 = *reinterpret_cast<const uint4*>(rec + 16 + 32 * j);
                const uint4 q1 = *reinterpret_cast<const uint4*>(rec + 32 + 32 * j);
                const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
                decode_part<4>(hd[p], qw, h, j, 0, dst, rr);
              } else if constexpr (T == T_Q6_K) {
                decode_q6k_item(rec, j, h, dst, rr);
              } else if constexpr (T == T_Q5_K) {
                decode_q5k_item(rec, j, h, dst, rr);
              } else if constexpr (T == T_Q8_0) {
                decode_q8_0_item(rec, j, h, dst, rr);
              } else {
                decode_item_generic<T>(rec, j, h, dst, rr);
              }
            }
          }
          fence_proxy_async_smem();               // generic-proxy writes -> visible to the tensor core
          __syncwarp();
          if (lane == 0) {
            if (rank == 0)
              mbar_arrive(&ctl->ofull[s]);
            else
              mbar_arrive_remote(leader_ofull + 8u * s);
          }
          s += kGroups;                           // next step of this group
          if (s >= (uint32_t)S) { s -= (uint32_t)S; ph ^= 1; }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&ctl->wempty[rs]);
        if (++rs == (uint32_t)RW) { rs = 0; rph ^= 1; }
      }
    }
  } else if (warp == 2 + DW + kPairEpiWarps) {
    // ---------------- TMA producer: raw weight records ----------------
    // A thread of its own, so that the next super-block column is requested
    // as soon as a raw slot is free rather than behind the activation tiles
    // (whose loads wait for the MMA to release operand stages).
    if (lane == 0) {
      uint32_t rs = 0, rph = 0;
      for (int t = pair; t < NT; t += npairs) {
        PairTile pt;
        if (!pair_tile(pw, t, M, TM, TN, width, pt)) continue;
        const CUtensorMap* wmap = &pw.map[NMAP == 1 ? 0 : pt.g];
        const int wn = pt.col0 + (int)rank * hb;
        for (int kb = 0; kb < KB; ++kb) {
          pair_wait(&ctl->wempty[rs], rph ^ 1);
          mbar_arrive_expect_tx(&ctl->wfull[rs], (uint32_t)wstage);
          const int wx = ((kb * CG::CB) & ~15) >> 1;   // 16-byte aligned start, in 16-bit elements
          for (int h = 0; h < NH; ++h)
            tma_load_2d(sW + rs * wstage + h * hb * CG::BB, wmap, wx, wn + h * BN, &ctl->wfull[rs]);
          if (++rs == (uint32_t)RW) { rs = 0; rph ^= 1; }
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    grid_dep_wait();                              // row scales come from the preceding kernel
    const int ew = warp - 2 - DW;                 // 0..3
    const int sp = warp & 3;                      // TMEM sub-partition this warp may read
    float* tile = sEpi + ew * kEpiTileFloats;
    const uint32_t leader_acc_empty = mapa_shared(smem_u32(&ctl->acc_empty[0]), 0);
    uint32_t it = 0;
    for (int t = pair; t < NT; t += npairs) {
      PairTile pt;
      if (!pair_tile(pw, t, M, TM, TN, width, pt)) continue;
      const uint32_t b = nacc == 2 ? (it & 1) : 0u, u = nacc == 2 ? (it >> 1) : it;
      pair_wait(&ctl->acc_full[b], u & 1);
      tc_fence_after();
      const int mrow0 = pt.am0 + (int)rank * 128 + sp * 32;
      const float rsc = (mrow0 + lane) < pt.mhi ? rowscale[mrow0 + lane] : 0.f;
      for (int ch = 0; ch < width / 32; ++ch) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t)(sp * 32) << 16) + b * (uint32_t)width + (uint32_t)(ch * 32), v);
        tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 32; ++c) tile[lane * 33 + c] = __uint_as_float(v[c]) * rsc;
        __syncwarp();
        const int nn = pt.col0 + ch * 32 + lane;
        const float bv = (bias && nn < N) ? bias[nn] : 0.f;
        for (int r = 0; r < 32; ++r) {
          const int m = mrow0 + r;
          if (m < pt.mhi && nn < N) {
            float* yp = y + (int64_t)m * N + nn;
            const float o = tile[r * 33 + lane] + bv;
            *yp = acc ? *yp + o : o;
          }
        }
        __syncwarp();
      }
      tc_fence_before();                          // this warp's TMEM reads are complete
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&ctl->acc_empty[b]);
        else
          mbar_arrive_remote(leader_acc_empty + 8u * b);
      }
      ++it;
    }
  }
  tc_fence_before();
  cluster_sync_all();                             // no arrival or MMA read of the peer's memory is outstanding
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Tensor-memory-A GEMM (CTA pairs): the decoded weights never touch shared
// memory.  The product is computed transposed, D[feature][token] =
// sum_k W[feature][k] * x[token][k]: the weights are the A operand of
// tcgen05.mma, written by the decode warps straight into tensor memory with
// tcgen05.st (lane = weight row, 32-bit column = two consecutive K values),
// and the fp16 activation is the B operand, TMA-staged in shared memory
// (128-byte swizzle, K-major).  Per K step and CTA, shared memory then carries
// only the activation tile and the raw weight records; in the CTA-pair kernel
// above it also carries the decoded B tile (written by the decode warps and
// read by both tensor cores), which measured as the limit of that kernel.
//
// A pair covers 256 weight rows (rank r: rows 128r..128r+127 of the tile, in
// its own tensor memory) and NT tokens (rank r stages tokens NT/2 r ..
// NT/2 (r+1) - 1 of the B operand).  One pipeline stage is 128 K values: 8
// MMAs (K = 16 each) per barrier wait, since a wait on the issuing thread
// costs about as much as issuing two MMAs and small-N MMAs are issue-bound.
// Tensor memory (512 columns per CTA): nacc accumulators of NT columns, then
// S stages of 64 columns of A (128 K values x 128 rows).  With one accumulator
// of more than 128 columns (nacc = 0, "ping-pong": S = 4 and 4 | K/128), the
// accumulator of tile t and the A stages swap halves on every tile: D_t in
// columns 256 (t & 1) .. +NT, stage s of tile t in 256 (1 - (t & 1)) + 64 s,
// which is where chunks 2s, 2s + 1 of D_(t-1) lie; the epilogue frees each
// 64-column slot (col_free[s]) as soon as it has read it, and the decode warps
// wait for that before the first write of the slot in a tile, so the next
// tile's main loop runs while the epilogue drains.
//
// Warps (24 per CTA):
//   0        TMA producer of the activation tiles, two 64-K boxes per stage
//            (rank 1's complete on rank 0's barrier, cta_group::2 form of the
//            tensor load; no multicast)
//   1        tensor-memory allocation (both ranks); rank 0 issues the MMAs
//   2        TMA producer of the raw weight records (one 256-wide K column of
//            128 rows per ring slot, ColGeom<T> boxes)
//   3        idle
//   4-19     decode: warp 4 + 8g + 4h + q decodes K step j = 2g + h (64
//            weights) of every 256-wide column for the rows of lane quarter q
//            (the tensor-memory lanes warp q (mod 4) may access): stage 2c + g
//            of column c, its A columns 32h .. 32h + 31, two tcgen05.st of 16
//            columns per thread (one row each)
//   20-23    epilogue: tcgen05.ld of 32 tokens per thread (its row = one
//            output feature), row scale of each token, bias, bulk tensor
//            stores of 32 x 32 boxes
// Barriers (all waits bounded):
//   ofull[S]   (rank 0) both producers' expect-tx arrivals and TMA bytes + the
//              8 + 8 decode warps of the group that owns the stage
//   oempty[S]  MMA commit, multicast to both CTAs (frees the B stage and the A
//              columns of the stage)
//   wfull/wempty[RW]  raw record ring (TMA bytes / 16 decode-warp arrivals)
//   acc_full[2], acc_empty[2] as in the CTA-pair kernel
// ---------------------------------------------------------------------------
constexpr int kTmDecodeWarps = 16;
constexpr int kTmThreads = (4 + kTmDecodeWarps + kPairEpiWarps) * 32;
constexpr int kTmMaxStages = 6;
constexpr int kTmStageK = 128;              // K values per pipeline stage
constexpr int kTmRows = 128;                // weight rows per CTA
constexpr int kTmEpiBox = 32 * 32;          // fp32 output box: 32 tokens x 32 features
constexpr double kTmDualStageClk = 1000.0;  // host cost model: one 128-K stage with two MMA threads

constexpr int kTmMaxRaw = 6;                // raw record ring slots (256-wide K columns), as shared memory allows

struct TmSmem {
  uint64_t wfull[kTmMaxRaw], wempty[kTmMaxRaw];
  uint64_t ofull[kTmMaxStages], oempty[kTmMaxStages];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t col_free[4];            // ping-pong mode: the epilogue has read these 64 columns of the last tile
  uint32_t tmem_base;
};

XM_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
XM_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bulk tensor store / reduce-add of a shared-memory box to global memory, and
// the bulk-group waits that guard the reuse of the box.
XM_DEV void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(map), "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}
XM_DEV void tma_store_3d(const CUtensorMap* map, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%1, %2, %3}], [%4];"
               ::"l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(src))
               : "memory");
}
XM_DEV void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];"
               ::"l"(map), "r"(c0), "r"(c1), "r"(smem_u32(src))
               : "memory");
}
XM_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
XM_DEV void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
XM_DEV void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// The 8 MMAs of one 128-K stage (K = 16 each) in one instruction block, so
// that the issuing thread, which shares its scheduler with decode warps, runs
// as few instructions as possible: A columns a + 8k, B descriptors {blo +
// boff_k, bhi} (the low word holds the start address field, which the
// offsets never carry out of), accumulate into D except for the first MMA
// when `first` is set.
XM_DEV void tc2_mma_stage128(uint32_t d, uint32_t a, uint32_t blo, uint32_t bhi, uint32_t bh, uint32_t idesc,
                             uint32_t first) {
  asm volatile(
      "{\n"
      " .reg .pred p0, p1;\n"
      " .reg .b32 l;\n"
      " .reg .b64 bd;\n"
      " setp.eq.b32 p0, %6, 0;\n"
      " setp.eq.b32 p1, %6, %6;\n"
      " mov.b64 bd, {%2, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], bd, %5, p0;\n"
      " add.u32 l, %2, 2;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], bd, %5, p1;\n"
      " add.u32 l, %2, 4;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%8], bd, %5, p1;\n"
      " add.u32 l, %2, 6;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%9], bd, %5, p1;\n"
      " add.u32 l, %2, %4;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%10], bd, %5, p1;\n"
      " add.u32 l, l, 2;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%11], bd, %5, p1;\n"
      " add.u32 l, l, 2;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%12], bd, %5, p1;\n"
      " add.u32 l, l, 2;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%13], bd, %5, p1;\n"
      "}"
      ::"r"(d), "r"(a), "r"(blo), "r"(bhi), "r"(bh), "r"(idesc), "r"(first), "r"(a + 8u), "r"(a + 16u),
        "r"(a + 24u), "r"(a + 32u), "r"(a + 40u), "r"(a + 48u), "r"(a + 56u)
      : "memory");
}

// Half a stage (K steps 4h .. 4h + 3: one 64-K box) for the dual-issue mode:
// A columns a + 8k, B descriptors {blo + 2k, bhi}.
XM_DEV void tc2_mma_half64(uint32_t d, uint32_t a, uint32_t blo, uint32_t bhi, uint32_t idesc, uint32_t first) {
  asm volatile(
      "{\n"
      " .reg .pred p0, p1;\n"
      " .reg .b32 l;\n"
      " .reg .b64 bd;\n"
      " setp.eq.b32 p0, %5, 0;\n"
      " setp.eq.b32 p1, %5, %5;\n"
      " mov.b64 bd, {%2, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], bd, %4, p0;\n"
      " add.u32 l, %2, 2;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%6], bd, %4, p1;\n"
      " add.u32 l, %2, 4;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%7], bd, %4, p1;\n"
      " add.u32 l, %2, 6;\n mov.b64 bd, {l, %3};\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%8], bd, %4, p1;\n"
      "}"
      ::"r"(d), "r"(a), "r"(blo), "r"(bhi), "r"(idesc), "r"(first), "r"(a + 8u), "r"(a + 16u), "r"(a + 24u)
      : "memory");
}

// Gate/up epilogue, one warp pair (gate warp: lanes = w1 rows, up warp: the
// same features' w3 rows) and one 32-token chunk: each warp evaluates
// act(gate) * up for 16 tokens, the gate warp for tokens 0-15 (its own gate
// values, the up values from `xu`), the up warp for 16-31 (the gate values
// from `xg`, its own up values); o[c - c0] = the result for token c.  Only the
// epilogue warps evaluate the activation, beside busy decode warps, so SiLU
// uses the fast exponential and division intrinsics (a few ulp from x / (1 +
// exp(-x)) in fp32; 0 for x -> -inf).
template <int ACT>
XM_DEV float gate_act(float x) {
  if constexpr (ACT == XM_ACT_SILU) return __fdividef(x, 1.0f + __expf(-x));
  else return xm_act(ACT, x);
}
template <int ACT>
XM_DEV void gate_up_half(const uint32_t (&v)[32], float rs, bool gate, const float* xg, const float* xu,
                         float (&o)[16]) {
  if (gate) {
#pragma unroll
    for (int c = 0; c < 16; ++c)
      o[c] = gate_act<ACT>(__uint_as_float(v[c]) * __shfl_sync(~0u, rs, c)) * xu[c * 32];
  } else {
#pragma unroll
    for (int c = 0; c < 16; ++c)
      o[c] = gate_act<ACT>(xg[c * 32]) * (__uint_as_float(v[16 + c]) * __shfl_sync(~0u, rs, 16 + c));
  }
}
XM_DEV void named_bar(int id, int threads) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory"); }

// Tile t of the tensor-memory-A kernel: token tile (fastest, so that the
// pairs that run together share a weight tile in L2) and weight tile of W
// output features (256; 128 in gate/up mode).
template <int NMAP>
XM_DEV bool tm_tile(const PairW<NMAP>& pw, int t, int M, int TM, int TW, int NT, int W, PairTile& pt) {
  if (NMAP == 1) {
    pt.g = 0;
    pt.am0 = (t % TM) * NT;
    pt.mhi = M;
    pt.col0 = (t / TM) * W;
    return true;
  }
  const int wt = t % TW, r = t / TW;
  const int mt = r % TM, g = r / TM;
  const int lo = pw.off[g], cnt = pw.cnt[g];
  pt.g = g;
  pt.am0 = lo + mt * NT;
  pt.mhi = lo + cnt;
  pt.col0 = wt * W;
  return mt * NT < cnt;
}

// GU (gate/up mode, grouped): each CTA's 128 MMA rows are 64 rows of w1 (map
// pw; tensor-memory lanes 0-63) and the same 64 rows of w3 (map pw3; lanes
// 64-127), so the epilogue warps of lane quarters q and q + 2 hold the gate
// and up accumulators of the same features and combine them through shared
// memory: y = act(gate) * up, 128 features per CTA pair.
template <int T, int NMAP, bool GU, bool DUAL = false>
__global__ void __launch_bounds__(kTmThreads, 1)
    k_qgemm_tm(const __grid_constant__ CUtensorMap map_b, const __grid_constant__ PairW<NMAP> pw,
               const __grid_constant__ PairW<NMAP> pw3, const __grid_constant__ CUtensorMap map_y, int y_tma,
               const __grid_constant__ CUtensorMap map_p, int ksplit, float* __restrict__ part, int M, int N, int K,
               int NT, int nacc, int S, int RW, int TM, const float* __restrict__ rowscale,
               const float* __restrict__ bias, float* __restrict__ y, int acc, int act) {
  using CG = ColGeom<T>;
  constexpr bool dual = DUAL;
  constexpr int TWID = GU ? kTmRows : 2 * kTmRows;   // output features per tile
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bhalf = (NT / 2) * 128;               // this CTA's NT/2 tokens x 64 K of fp16, 128-byte swizzled
  const int bstage = 2 * bhalf;                   // one stage: two such boxes
  const int wstage = kTmRows * CG::BB;            // the CTA's staged bytes of one 256-wide K column
  uint8_t* sB = base;
  float* sE = reinterpret_cast<float*>(sB + S * bstage);           // epilogue boxes: 2 per epilogue warp
  float* sU = sE + kPairEpiWarps * 2 * kTmEpiBox;                   // gate/up: per warp pair 2 x [16][32]
  uint8_t* sW = reinterpret_cast<uint8_t*>(sU + (GU ? 2 * kTmEpiBox : 0));
  TmSmem* ctl = reinterpret_cast<TmSmem*>(sW + RW * wstage);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int TW = (N + TWID - 1) / TWID;
  const int NTILES = TM * TW * (NMAP == 1 ? 1 : pw.groups);
  const int KB = K >> 8;
  // split-K: unit u = tile (u % NTILES) x K part (u / NTILES); part sp covers
  // the 256-wide columns [kcol(sp), kcol(sp + 1)), an even number of them
  const int NUNITS = NTILES * ksplit;
  auto kcol = [&](int sp) { return ksplit == 1 ? (sp ? KB : 0) : 2 * ((KB >> 1) * sp / ksplit); };
  const bool pp = nacc == 0;                      // ping-pong accumulator (see above)
  constexpr int nd = dual ? 2 : 1;                // dual issue: two MMA threads, two partial accumulators per tile
  const int accw = nd * NT;                       // tensor-memory columns of one tile's accumulator(s)
  const uint32_t a_col0 = (uint32_t)(nacc * accw);   // first tensor-memory column of the A stages (nacc > 0)

  if (tid == 0) {
    for (int i = 0; i < RW; ++i) {
      mbar_init(&ctl->wfull[i], 1);
      mbar_init(&ctl->wempty[i], kTmDecodeWarps);
    }
    for (int i = 0; i < S; ++i) {
      mbar_init(&ctl->ofull[i], 2 + 2 * 8);       // rank 0 only: 2 producers + 8 decode warps per CTA
      mbar_init(&ctl->oempty[i], nd);             // one commit per MMA thread
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&ctl->acc_full[b], nd);
      mbar_init(&ctl->acc_empty[b], 2 * kPairEpiWarps);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&ctl->col_free[i], kPairEpiWarps);   // this CTA's epilogue warps
    fence_mbar_init();
  }
  constexpr uint32_t kCols = 512;
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&ctl->tmem_base)),
                 "r"(kCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  cluster_sync_all();                             // barriers of both CTAs initialised, tensor memory allocated
  tc_fence_after();
  const uint32_t tmem = ctl->tmem_base;
  if (NMAP > 1) grid_dep_wait();                  // the group row ranges come from the preceding kernel

  if (warp == 0) {
    // ---------------- TMA producer: activation tiles (B) ----------------
    if (lane == 0) {
      grid_dep_wait();
      const uint32_t leader_ofull = mapa_shared(smem_u32(&ctl->ofull[0]), 0);
      uint32_t s = 0, ph = 0;
      for (int u = pair; u < NUNITS; u += npairs) {
        const int t = u % NTILES, sp = u / NTILES;
        PairTile pt;
        if (!tm_tile(pw, t, M, TM, TW, NT, TWID, pt)) continue;
        const int bm = pt.am0 + (int)rank * (NT / 2);
        for (int ks = 2 * kcol(sp); ks < 2 * kcol(sp + 1); ++ks) {
          pair_wait(&ctl->oempty[s], ph ^ 1);
          uint8_t* dst = sB + s * bstage;
          if (rank == 0) {
            mbar_arrive_expect_tx(&ctl->ofull[s], (uint32_t)bstage);
            tma_load_2d(dst, &map_b, ks * kTmStageK, bm, &ctl->ofull[s]);
            tma_load_2d(dst + bhalf, &map_b, ks * kTmStageK + kBK, bm, &ctl->ofull[s]);
          } else {
            mbar_arrive_expect_tx_remote(leader_ofull + 8u * s, (uint32_t)bstage);
            tma_load_2d_pair(dst, &map_b, ks * kTmStageK, bm, leader_ofull + 8u * s);
            tma_load_2d_pair(dst + bhalf, &map_b, ks * kTmStageK + kBK, bm, leader_ofull + 8u * s);
          }
          if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
        }
      }
    }
  } else if (warp == 1 || (warp == 3 && dual)) {
    if (lane == 0 && rank == 0) {
      // ---------------- MMA issuer(s) ----------------
      // Dual issue: warp 1 issues K steps 0-3 of every stage into the tile's
      // first accumulator and warp 3 steps 4-7 into the second (the epilogue
      // adds the two); each thread commits its own MMAs.
      const uint32_t hsel = warp == 3 ? 1u : 0u;
      const uint32_t idesc = idesc_f16_f32_m256(NT);
      const uint64_t b0 = smem_desc_sw128(sB);
      const uint64_t bstep = (uint64_t)(bstage >> 4), bh = (uint64_t)(bhalf >> 4);
      uint32_t s = 0, ph = 0, it = 0;
      for (int un = pair; un < NUNITS; un += npairs) {
        const int t = un % NTILES, sp = un / NTILES;
        PairTile pt;
        if (!tm_tile(pw, t, M, TM, TW, NT, TWID, pt)) continue;
        const uint32_t b = nacc != 1 ? (it & 1) : 0u, u = nacc != 1 ? (it >> 1) : it;
        if (!pp) pair_wait(&ctl->acc_empty[b], (u & 1) ^ 1);   // (ping-pong: the decode warps' col_free waits)
        tc_fence_after();
        const uint32_t d = pp ? tmem + (it & 1u) * 256u : tmem + b * (uint32_t)accw + hsel * (uint32_t)NT;
        const uint32_t abase = pp ? tmem + ((it & 1u) ^ 1u) * 256u : tmem + a_col0;
        const int ks0 = 2 * kcol(sp), ks1 = 2 * kcol(sp + 1);
        for (int ks = ks0; ks < ks1; ++ks) {
          pair_wait(&ctl->ofull[s], ph);
          tc_fence_after();
          const uint64_t bs = b0 + s * bstep;
          if constexpr (dual)
            tc2_mma_half64(d, abase + s * 64u + hsel * 32u, (uint32_t)bs + hsel * (uint32_t)bh, (uint32_t)(bs >> 32),
                           idesc, ks == ks0 ? 1u : 0u);
          else
            tc2_mma_stage128(d, abase + s * 64u, (uint32_t)bs, (uint32_t)(bs >> 32), (uint32_t)bh, idesc,
                             ks == ks0 ? 1u : 0u);
          tc2_commit_pair(&ctl->oempty[s]);      // both CTAs may refill the stage once these MMAs are done
          if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
        }
        tc2_commit_pair(&ctl->acc_full[b]);
        ++it;
      }
    }
  } else if (warp == 2) {
    // ---------------- TMA producer: raw weight records ----------------
    if (lane == 0) {
      uint32_t rs = 0, rph = 0;
      for (int u = pair; u < NUNITS; u += npairs) {
        const int t = u % NTILES, sp = u / NTILES;
        PairTile pt;
        if (!tm_tile(pw, t, M, TM, TW, NT, TWID, pt)) continue;
        const CUtensorMap* wmap = &pw.map[NMAP == 1 ? 0 : pt.g];
        const CUtensorMap* wmap3 = &pw3.map[NMAP == 1 ? 0 : pt.g];
        const int wn = pt.col0 + (GU ? (int)rank * (kTmRows / 2) : (int)rank * kTmRows);
        for (int kb = kcol(sp); kb < kcol(sp + 1); ++kb) {
          pair_wait(&ctl->wempty[rs], rph ^ 1);
          mbar_arrive_expect_tx(&ctl->wfull[rs], (uint32_t)wstage);
          const int wx = ((kb * CG::CB) & ~15) >> 1;   // 16-byte aligned start, in 16-bit elements
          tma_load_2d(sW + rs * wstage, wmap, wx, wn, &ctl->wfull[rs]);
          if (GU) tma_load_2d(sW + rs * wstage + (kTmRows / 2) * CG::BB, wmap3, wx, wn, &ctl->wfull[rs]);
          if (++rs == (uint32_t)RW) { rs = 0; rph ^= 1; }
        }
      }
    }
  } else if (warp >= 4 && warp < 4 + kTmDecodeWarps) {
    // ---------------- decode into tensor memory ----------------
    const int grp = (warp - 4) >> 3;              // stages 2c + grp of the columns c
    const int hs = ((warp - 4) >> 2) & 1;         // 64-K half of the stage
    const int j = 2 * grp + hs;                   // K step of each 256-wide column decoded by this warp
    const int quarter = warp & 3;                 // the tensor-memory lanes this warp may access
    const int row = quarter * 32 + lane;          // this thread's weight row in the CTA's 128
    const uint32_t leader_ofull = mapa_shared(smem_u32(&ctl->ofull[0]), 0);
    const uint32_t lane0 = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(hs * 32);
    uint32_t s = (uint32_t)grp, ph = 0, rs = 0, rph = 0;   // this group's first stage is q = grp (< S)
    uint32_t it = 0;
    for (int u = pair; u < NUNITS; u += npairs) {
      const int t = u % NTILES, sp = u / NTILES;
      PairTile pt;
      if (!tm_tile(pw, t, M, TM, TW, NT, TWID, pt)) continue;
      const uint32_t lane_addr = lane0 + (pp ? ((it & 1u) ^ 1u) * 256u : a_col0);
      const int kb0 = kcol(sp);
      for (int kb = kb0; kb < kcol(sp + 1); ++kb) {
        pair_wait(&ctl->wfull[rs], rph);
        const int mis = (kb * CG::CB) & 15;       // the column's offset in its staged box (0 for Q4_K)
        const uint8_t* rec = sW + rs * wstage + row * CG::BB + mis;
        // decode both 32-weight items first (one pass over the record bytes),
        // then wait for the tensor-memory columns
        uint32_t hv[16], hv1[16];
        item_regs<T>(rec, j, 0, hv);
        item_regs<T>(rec, j, 1, hv1);
        pair_wait(&ctl->oempty[s], ph ^ 1);       // the MMAs that read these columns are done
        // ping-pong: the first write of a slot in a tile also waits for the
        // epilogue of the previous tile to have read these columns
        if (pp && it > 0 && kb - kb0 < 2) pair_wait(&ctl->col_free[s], (it - 1u) & 1u);
        tc_fence_after();
        tmem_st16(lane_addr + s * 64u, hv);
        tmem_st16(lane_addr + s * 64u + 16u, hv1);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          if (rank == 0)
            mbar_arrive(&ctl->ofull[s]);
          else
            mbar_arrive_remote(leader_ofull + 8u * s);
          mbar_arrive(&ctl->wempty[rs]);
        }
        s += 2;                                   // this group's stage of the next column
        if (s >= (uint32_t)S) { s -= (uint32_t)S; ph ^= 1; }
        if (++rs == (uint32_t)RW) { rs = 0; rph ^= 1; }
      }
      ++it;
    }
  } else if (warp >= 4 + kTmDecodeWarps) {
    // ---------------- epilogue ----------------
    // Thread = output feature, tcgen05.ld column = token.  A 32-token chunk is
    // scaled (row scale of each token, broadcast by shuffle), biased, written
    // as a [token][feature] box into shared memory and sent to y by one bulk
    // tensor store (or reduce-add when accumulating); the tensor map clips
    // the box at M and N.  A chunk that crosses the end of its group's rows
    // (grouped mode: the next rows belong to another group), or any chunk when
    // y's row pitch is not a multiple of 16 bytes, is stored element-wise.
    grid_dep_wait();                              // row scales come from the preceding kernel
    const int quarter = warp & 3;
    float* box0 = sE + quarter * 2 * kTmEpiBox;
    uint32_t nb = 0;
    const uint32_t leader_acc_empty = mapa_shared(smem_u32(&ctl->acc_empty[0]), 0);
    uint32_t it = 0;
    for (int un = pair; un < NUNITS; un += npairs) {
      const int t = un % NTILES, sp = un / NTILES;
      PairTile pt;
      if (!tm_tile(pw, t, M, TM, TW, NT, TWID, pt)) continue;
      const uint32_t b = nacc != 1 ? (it & 1) : 0u, u = nacc != 1 ? (it >> 1) : it;
      // a K part's partial sums go to part[sp] (row-scaled; the bias and the
      // residual add come in the ordered reduction)
      float* const ydst = ksplit > 1 ? part + (int64_t)sp * M * N : y;
      const int uacc = ksplit > 1 ? 0 : acc;
      const uint32_t dcol = pp ? (it & 1u) * 256u : b * (uint32_t)accw;
      uint32_t rel = 0;                           // ping-pong: 64-column slots released so far
      const int f0 = pt.col0 + (GU ? (int)rank * (kTmRows / 2) + (quarter & 1) * 32 : (int)rank * kTmRows + quarter * 32);
      const int f = f0 + lane;                    // this thread's output feature
      const bool fok = f < N;
      const int nch = NT / 32;
      // row scales of the tile's tokens and the bias do not depend on the
      // accumulator: read them before waiting for it
      float rsv[8];
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int tok = pt.am0 + ch * 32 + lane;
        rsv[ch] = (ch < nch && tok < pt.mhi) ? rowscale[tok] : 0.f;
      }
      const float bv = (bias && fok && ksplit == 1) ? bias[f] : 0.f;
      pair_wait(&ctl->acc_full[b], u & 1);
      tc_fence_after();
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        const int tok0 = pt.am0 + ch * 32;
        if (ch >= nch || tok0 >= pt.mhi) break;
        uint32_t v[32];
        const uint32_t tq = tmem + ((uint32_t)(quarter * 32) << 16) + dcol + (uint32_t)(ch * 32);
        tmem_ld32(tq, v);
        if constexpr (dual) {                     // add the second issuer's partial sums
#pragma unroll
          for (int hh = 0; hh < 4; ++hh) {
            uint32_t w2[8];
            tmem_ld8(tq + (uint32_t)NT + (uint32_t)(hh * 8), w2);
            tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < 8; ++c)
              v[hh * 8 + c] = __float_as_uint(__uint_as_float(v[hh * 8 + c]) + __uint_as_float(w2[c]));
          }
        }
        tmem_ld_wait();
        if (pp && (ch & 1)) {                     // chunks 2s, 2s + 1 read: slot s may take A of the next tile
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&ctl->col_free[ch >> 1]);
          rel = (uint32_t)(ch >> 1) + 1u;
        }
        const float rs = rsv[ch];
        if constexpr (GU) {
          const int wp = quarter & 1;            // warp pair: gate warp wp, up warp wp + 2
          const bool gate = quarter < 2;
          float* xg = sU + wp * kTmEpiBox;       // [16][32]: the gate values of tokens 16-31
          float* xu = xg + kTmEpiBox / 2;        // [16][32]: the up values of tokens 0-15
          if (gate) {
#pragma unroll
            for (int c = 16; c < 32; ++c) xg[(c - 16) * 32 + lane] = __uint_as_float(v[c]) * __shfl_sync(~0u, rs, c);
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) xu[c * 32 + lane] = __uint_as_float(v[c]) * __shfl_sync(~0u, rs, c);
          }
          const bool tma_ok = y_tma && (NMAP == 1 || tok0 + 32 <= pt.mhi);
          float* box = sE + wp * 2 * kTmEpiBox + nb * kTmEpiBox;   // the pair's output box
          if (tma_ok && gate && lane == 0) bulk_wait_read1();
          named_bar(2 + wp, 64);
          float o[16];
          if (act == XM_ACT_SILU)
            gate_up_half<XM_ACT_SILU>(v, rs, gate, xg + lane, xu + lane, o);
          else if (act == XM_ACT_GELU)
            gate_up_half<XM_ACT_GELU>(v, rs, gate, xg + lane, xu + lane, o);
          else if (act == XM_ACT_RELU)
            gate_up_half<XM_ACT_RELU>(v, rs, gate, xg + lane, xu + lane, o);
          else
            gate_up_half<XM_ACT_IDENTITY>(v, rs, gate, xg + lane, xu + lane, o);
          const int c0 = gate ? 0 : 16;
          if (tma_ok) {
#pragma unroll
            for (int c = 0; c < 16; ++c) box[(c0 + c) * 32 + lane] = o[c];
            fence_proxy_async_smem();
            named_bar(2 + wp, 64);                // both halves written (and xg / xu read)
            if (gate && lane == 0) {
              tma_store_2d(&map_y, box, f0, tok0);
              bulk_commit();
            }
            nb ^= 1;
          } else {
#pragma unroll
            for (int c = 0; c < 16; ++c) {
              const int tok = tok0 + c0 + c;
              if (tok < pt.mhi && fok) y[(int64_t)tok * N + f] = o[c];
            }
            named_bar(2 + wp, 64);                // xg / xu read before the next chunk writes them
          }
          continue;
        }
        const float vs = rs;
        if ((ksplit > 1 || y_tma) && (NMAP == 1 || tok0 + 32 <= pt.mhi)) {
          float* box = box0 + nb * kTmEpiBox;
          if (lane == 0) bulk_wait_read1();       // the store issued from this box two chunks ago has read it
          __syncwarp();
#pragma unroll
          for (int c = 0; c < 32; ++c) box[c * 32 + lane] = __uint_as_float(v[c]) * __shfl_sync(~0u, vs, c) + bv;
          fence_proxy_async_smem();               // generic-proxy writes -> visible to the bulk copy
          __syncwarp();
          if (lane == 0) {
            if (ksplit > 1)
              tma_store_3d(&map_p, box, f0, tok0, sp);
            else if (acc)
              tma_reduce_add_2d(&map_y, box, f0, tok0);
            else
              tma_store_2d(&map_y, box, f0, tok0);
            bulk_commit();
          }
          nb ^= 1;
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float o = __uint_as_float(v[c]) * __shfl_sync(~0u, vs, c) + bv;
            const int tok = tok0 + c;
            if (tok < pt.mhi && fok) {
              float* yp = ydst + (int64_t)tok * N + f;
              if (uacc)
                *yp += o;
              else
                *yp = o;
            }
          }
        }
      }
      tc_fence_before();                          // this warp's tensor-memory reads are complete
      __syncwarp();
      if (lane == 0) {
        if (pp) {
          for (; rel < 4u; ++rel) mbar_arrive(&ctl->col_free[rel]);   // slots of chunks this tile did not have
        } else if (rank == 0) {
          mbar_arrive(&ctl->acc_empty[b]);
        } else {
          mbar_arrive_remote(leader_acc_empty + 8u * b);
        }
      }
      ++it;
    }
    if (lane == 0) bulk_wait_all();               // every store has completed before the CTA exits
    __syncwarp();
  }
  tc_fence_before();
  cluster_sync_all();                             // no arrival or MMA read of the peer's memory is outstanding
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kCols) : "memory");
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

int sm_count_dev() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

struct TileCfg {
  int MT, BN, stages;
};

int stages_for(int MT, int BN) {
  const int per = MT * kATileBytes + BN * kBK * 2;
  const int avail = 227 * 1024 - 1024 - (int)sizeof(GemmSmem);
  return std::max(2, std::min(kMaxStages, avail / per));
}

// Output tile shape: MT*128 rows x BN columns.  MT = 2 once there are 256
// rows (each decoded B tile then serves 256 activation rows; MT*BN <= 512
// tensor-memory columns), and BN (a multiple of 16, <= 256) as large as the
// SM count allows: the activation is re-read once per column tile.
TileCfg choose_tile(int64_t M, int64_t N, int64_t K, int sms) {
  (void)K;
  const int MT = M > 128 ? 2 : 1;
  const int64_t tm = (M + MT * 128 - 1) / (MT * 128);
  int64_t bn = (N * tm + sms - 1) / sms;                  // one wave if possible
  bn = (bn + 31) / 32 * 32;                               // the epilogue moves 32-column chunks
  bn = std::max<int64_t>(64, std::min<int64_t>(256, bn));
  return {MT, (int)bn, stages_for(MT, (int)bn)};
}

}  // namespace

namespace {
int encode_a16(CUtensorMap* map, const __half* a16, int64_t rows, int64_t k, int box_rows = 128) {
  EncodeTiledFn encode = get_encode();
  if (!encode) return xm_set_error(XM_ERR_CUDA, "qgemm: cuTensorMapEncodeTiled unavailable");
  const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
  const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(a16), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return xm_set_error(XM_ERR_CUDA, "qgemm: activation tensor map (%d)", (int)r);
  return XM_OK;
}

int launch_gemm(const CUtensorMap& map_a, const uint8_t* w, int64_t m, int64_t n, int64_t k, TileCfg cfg,
                dim3 grid, const float* rowscale, const float* bias, float* y, int acc, const GemmGroups& groups,
                cudaStream_t st) {
  const int smem = 1024 + cfg.stages * (cfg.MT * kATileBytes + cfg.BN * kBK * 2) + (int)sizeof(GemmSmem);
  cudaError_t e = cudaFuncSetAttribute(k_qgemm_q4k_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = dim3(kThreads);
  lc.dynamicSmemBytes = smem;
  lc.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  e = cudaLaunchKernelEx(&lc, k_qgemm_q4k_tc, map_a, w, (int)m, (int)n, (int)k, cfg.MT, cfg.BN, cfg.stages, rowscale,
                         bias, y, acc, groups);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemm");
}

// ---- CTA-pair kernel ----
#ifndef XM_PAIR_DW
#define XM_PAIR_DW 16   // decode warps per CTA: groups of 8 that take turns by K step
#endif
constexpr int kPairDW = XM_PAIR_DW;
static_assert(kPairDW == 8 || kPairDW == 16, "decode warps");
constexpr int kPairRaw = 2;                     // raw record stages (double buffer)

struct PairCfg {
  int BN, NH, S, RW, smem;
};

int pair_smem_bytes(int BN, int NH, int S, int RW, int BB) {
  const int rows = NH * (BN / 2);
  return 1024 + S * (kATileBytes + rows * 128) + RW * rows * BB + kPairEpiWarps * kEpiTileFloats * 4 +
         (int)sizeof(PairSmem);
}

// Deepest operand ring that fits; S = 0 if fewer than 3 stages fit.
PairCfg pair_stages(int BN, int NH, int BB) {
  int S = kMaxStages;
  while (S > 2 && pair_smem_bytes(BN, NH, S, kPairRaw, BB) > 227 * 1024) --S;
  if (S < 3) S = 0;
  return {BN, NH, S, kPairRaw, pair_smem_bytes(BN, NH, S, kPairRaw, BB)};
}

template <int T, int NMAP>
const void* pair_kernel() {
  return reinterpret_cast<const void*>(k_qgemm_pair<T, kPairDW, NMAP>);
}

// How many CTA pairs of a kernel, block size and shared-memory size can be
// resident at once (0 if the device cannot launch it); cached per device,
// kernel and size.
int cluster_capacity(const void* fn, int threads, int smem) {
  struct Key {
    int dev;
    const void* fn;
    int smem;
  };
  static std::mutex mu;
  static Key keys[256];
  static int vals[256];
  static int used = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lock(mu);
    for (int i = 0; i < used; ++i)
      if (keys[i].dev == dev && keys[i].fn == fn && keys[i].smem == smem) return vals[i];
  }
  int n = 0;
  if (smem > 0 && cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(2);
    lc.blockDim = dim3(threads);
    lc.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &lc) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  std::lock_guard<std::mutex> lock(mu);
  if (used < 256) {
    keys[used] = Key{dev, fn, smem};
    vals[used] = n;
    ++used;
  }
  return n;
}

int pair_capacity(const void* fn, const PairCfg& cfg) {
  return cfg.S >= 3 ? cluster_capacity(fn, pair_threads(kPairDW), cfg.smem) : 0;
}

// Tile shape for `mtiles` 256-row tiles of output width n: BN (multiple of 32,
// <= 256) and NH (1: double-buffered accumulators; 2: one accumulator of 2BN
// columns).  Estimated time per pair: rounds x main loop (MMA per K step plus
// a fixed cost) plus the epilogues that do not overlap.
PairCfg choose_pair(int64_t mtiles, int64_t n, int64_t k, int pairs, int BB) {
  PairCfg best{0, 0, 0, 0, 0};
  double best_t = 1e30;
  const double nkt = (double)(k / kBK);
  for (int nh = 1; nh <= 2; ++nh)
    for (int bn = 256; bn >= 32; bn -= 32) {
      if (nh == 2 && bn < 128) continue;
      const PairCfg c = pair_stages(bn, nh, BB);
      if (c.S < 3) continue;
      const int width = nh * bn;
      const int64_t tiles = mtiles * ((n + width - 1) / width);
      const double rounds = (double)((tiles + pairs - 1) / pairs);
      const double main_us = nkt * (0.26 * width / 256.0 + 0.06);
      const double epi_us = width * 0.0128;
      const double t = rounds * main_us + (nh == 2 ? rounds : 1.0) * epi_us;
      if (t < best_t) {
        best_t = t;
        best = c;
      }
    }
  return best;
}

// Bytes of one weight row of type T (k a multiple of 256).  The pair kernel
// moves rows with a 2-D tensor map, whose row pitch must be a multiple of 16.
template <int T>
int64_t pair_row_bytes(int64_t k) {
  return (k / 256) * ColGeom<T>::CB;
}

template <int T>
int encode_w_records(CUtensorMap* map, const uint8_t* w, int64_t n, int64_t k, int rows_per_box,
                     int64_t pitch = 0) {
  EncodeTiledFn encode = get_encode();
  if (!encode) return xm_set_error(XM_ERR_CUDA, "qgemm: cuTensorMapEncodeTiled unavailable");
  // rows `pitch` bytes apart (0: packed rows); the bytes past a row's records are never decoded
  const int64_t row_bytes = pitch ? pitch : pair_row_bytes<T>(k);
  const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 2), (cuuint64_t)n};
  const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  const cuuint32_t box[2] = {(cuuint32_t)(ColGeom<T>::BB / 2), (cuuint32_t)rows_per_box};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint8_t*>(w), dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return xm_set_error(XM_ERR_CUDA, "qgemm: weight tensor map (%d)", (int)r);
  return XM_OK;
}

template <int T, int NMAP>
int launch_pair(const CUtensorMap& map_a, const PairW<NMAP>& pw, int64_t m, int64_t n, int64_t k, int tm,
                const PairCfg& cfg, int pairs, const float* rowscale, const float* bias, float* y, int acc,
                cudaStream_t st) {
  const void* fn = pair_kernel<T, NMAP>();
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, cfg.smem);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)(2 * pairs));
  lc.blockDim = dim3(pair_threads(kPairDW));
  lc.dynamicSmemBytes = cfg.smem;
  lc.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 2;
  e = cudaLaunchKernelEx(&lc, k_qgemm_pair<T, kPairDW, NMAP>, map_a, pw, (int)m, (int)n, (int)k, cfg.BN, cfg.NH,
                         cfg.S, cfg.RW, tm, rowscale, bias, y, acc);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm pair launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemm pair");
}

// Dense GEMM on the CTA-pair kernel.  Returns 1 (nothing launched) when the
// device cannot hold a pair, so the caller can use the single-CTA kernel.
template <int T>
int launch_pair_gemm(const CUtensorMap& map_a, const uint8_t* w, int64_t m, int64_t n, int64_t k,
                     const float* rowscale, const float* bias, float* y, int acc, cudaStream_t st) {
  constexpr int BB = ColGeom<T>::BB;
  const void* fn = pair_kernel<T, 1>();
  const int cap = pair_capacity(fn, pair_stages(256, 1, BB));
  if (cap < 1) return 1;
  const int64_t mtiles = (m + 255) / 256;
  const PairCfg cfg = choose_pair(mtiles, n, k, cap, BB);
  if (cfg.S < 3) return 1;
  const int cap_cfg = pair_capacity(fn, cfg);
  if (cap_cfg < 1) return 1;
  PairW<1> pw{};
  int rc = encode_w_records<T>(&pw.map[0], w, n, k, cfg.BN / 2);
  if (rc) return rc;
  pw.groups = 1;
  const int64_t tiles = mtiles * ((n + cfg.NH * cfg.BN - 1) / (cfg.NH * cfg.BN));
  const int pairs = (int)std::min<int64_t>(tiles, cap_cfg);
  return launch_pair<T, 1>(map_a, pw, m, n, k, (int)mtiles, cfg, pairs, rowscale, bias, y, acc, st);
}

// Grouped GEMM (MoE experts) on the CTA-pair kernel; 1 if not possible.
template <int T>
int launch_pair_grouped(const CUtensorMap& map_a, const uint8_t* const* h_w, const int* d_cnt, const int* d_off, int G,
                        int64_t P, int64_t n, int64_t k, int64_t max_rows, int64_t expect_rows,
                        const float* rowscale, float* y, cudaStream_t st) {
  constexpr int BB = ColGeom<T>::BB;
  const void* fn = pair_kernel<T, kMaxGroups>();
  const int cap = pair_capacity(fn, pair_stages(256, 1, BB));
  if (cap < 1) return 1;
  const PairCfg cfg = choose_pair((int64_t)G * ((expect_rows + 255) / 256), n, k, cap, BB);
  if (cfg.S < 3) return 1;
  const int cap_cfg = pair_capacity(fn, cfg);
  if (cap_cfg < 1) return 1;
  PairW<kMaxGroups> pw{};
  for (int g = 0; g < G; ++g) {
    int rc = encode_w_records<T>(&pw.map[g], h_w[g], n, k, cfg.BN / 2);
    if (rc) return rc;
  }
  pw.cnt = d_cnt;
  pw.off = d_off;
  pw.groups = G;
  const int tm = (int)((max_rows + 255) / 256);
  const int64_t tiles = (int64_t)G * tm * ((n + cfg.NH * cfg.BN - 1) / (cfg.NH * cfg.BN));
  const int pairs = (int)std::min<int64_t>(tiles, cap_cfg);
  return launch_pair<T, kMaxGroups>(map_a, pw, P, n, k, tm, cfg, pairs, rowscale, nullptr, y, 0, st);
}

// ---- tensor-memory-A kernel ----
constexpr int kTmMaxSplit = 4;              // K parts at most (dense GEMM)

// Partial planes of a split-K launch, [ks][rows][n] fp32, as a 3-D tensor
// map with 32 x 32 x 1 boxes, so that a box is clipped at the end of its own
// plane's rows.
bool encode_part_map(CUtensorMap* map, const float* part, int64_t rows, int64_t n, int ks) {
  if ((n * 4) % 16 || ((uintptr_t)part & 15)) return false;
  EncodeTiledFn encode = get_encode();
  if (!encode) return false;
  const cuuint64_t dims[3] = {(cuuint64_t)n, (cuuint64_t)rows, (cuuint64_t)ks};
  const cuuint64_t strides[2] = {(cuuint64_t)n * 4, (cuuint64_t)(rows * n * 4)};
  const cuuint32_t box[3] = {32, 32, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(part), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Ordered reduction of the K parts: y = [y +] ((part[0] + part[1] + ...) +
// bias), the same association as the unsplit epilogue (y [+]= acc + bias)
// with the accumulator summed part by part; n % 4 == 0.
__global__ void __launch_bounds__(256) k_splitk_reduce(const float* __restrict__ part, int ks, int64_t mn, int n,
                                                       const float* __restrict__ bias, float* __restrict__ y,
                                                       int acc) {
  const int64_t n4 = mn >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = __ldcs(reinterpret_cast<const float4*>(part) + i);
    for (int p = 1; p < ks; ++p) {
      const float4 v = __ldcs(reinterpret_cast<const float4*>(part + (int64_t)p * mn) + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    if (bias) {
      const int f = (int)((i * 4) % n);
      const float4 b = *reinterpret_cast<const float4*>(bias + f);
      s.x += b.x;
      s.y += b.y;
      s.z += b.z;
      s.w += b.w;
    }
    float4* yp = reinterpret_cast<float4*>(y) + i;
    if (acc) {
      const float4 o = *yp;
      s.x = o.x + s.x;
      s.y = o.y + s.y;
      s.z = o.z + s.z;
      s.w = o.w + s.w;
    }
    *yp = s;
  }
}

struct TmCfg {
  int NT, nacc, S, RW, smem, dual;
  int ks = 1;                      // K parts (split-K units per output tile)
};

int tm_smem_bytes(int NT, int S, int RW, int BB, bool gu = false) {
  return 1024 + S * (NT / 2) * 256 + kPairEpiWarps * 2 * kTmEpiBox * 4 + (gu ? 2 * kTmEpiBox * 4 : 0) +
         RW * kTmRows * BB + (int)sizeof(TmSmem);
}

// fp32 output [rows][n] as a tensor map with 32 x 32 boxes; false when the
// row pitch is not a multiple of 16 bytes (element-wise stores then).
bool encode_y_map(CUtensorMap* map, const float* y, int64_t rows, int64_t n) {
  if ((n * 4) % 16 || ((uintptr_t)y & 15)) return false;
  EncodeTiledFn encode = get_encode();
  if (!encode) return false;
  const cuuint64_t dims[2] = {(cuuint64_t)n, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)n * 4};
  const cuuint32_t box[2] = {32, 32};
  const cuuint32_t es[2] = {1, 1};
  return encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(y), dims, strides, box, es,
                CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Token-tile options: NT a multiple of 32 (<= 256); two accumulators where
// they fit beside 4 A stages (so the epilogue of one tile overlaps the next
// tile's main loop), then as many A stages (<= 6) as tensor and shared memory
// hold, then as many raw record slots (2 .. kTmMaxRaw) as the rest of shared
// memory holds: the record ring is what keeps a pair fed when the MMAs of a
// stage are short (narrow tiles), since each slot waits one HBM round trip.
// S = 0 if fewer than 3 stages fit.  Dual issue doubles a tile's accumulator
// columns (two partial sums of NT columns) and has no ping-pong form.
TmCfg tm_stages(int NT, int BB, bool gu = false, bool pp_ok = false, bool dual = false) {
  const int accw = dual ? 2 * NT : NT;
  const int nacc = 2 * accw + 4 * 64 <= 512 ? 2 : 1;
  auto raw_slots = [&](int S) {
    int RW = kPairRaw;
    while (RW < kTmMaxRaw && tm_smem_bytes(NT, S, RW + 1, BB, gu) <= 227 * 1024) ++RW;
    return RW;
  };
  // one accumulator: ping-pong halves when 4 stages fit (nacc = 0)
  if (!dual && nacc == 1 && pp_ok && tm_smem_bytes(NT, 4, kPairRaw, BB, gu) <= 227 * 1024) {
    const int RW = raw_slots(4);
    return {NT, 0, 4, RW, tm_smem_bytes(NT, 4, RW, BB, gu), 0, 1};
  }
  int S = std::min(kTmMaxStages, (512 - nacc * accw) / 64);
  while (S >= 3 && tm_smem_bytes(NT, S, kPairRaw, BB, gu) > 227 * 1024) --S;
  if (S < 3) S = 0;
  const int RW = S ? raw_slots(S) : kPairRaw;
  return {NT, nacc, S, RW, tm_smem_bytes(NT, S, RW, BB, gu), dual ? 1 : 0, 1};
}

template <int T, int NMAP, bool GU = false, bool DUAL = false>
const void* tm_kernel() {
  return reinterpret_cast<const void*>(k_qgemm_tm<T, NMAP, GU, DUAL>);
}

// Token tile for m rows (per group) and n output features: estimated clocks
// per pair = rounds x (main loop + the epilogues that do not overlap it).  A
// 128-K stage costs the larger of its MMA time (4 NT clocks) and the decode
// of 128 rows x 128 K beside it (~1000-1120 clocks measured, the MMA thread's
// issue included; ~1000 with two MMA threads); the epilogue ~1400 + 20 NT
// clocks (+ 10 NT for the second partial sum), hidden behind the next tile
// except with one non-ping-pong accumulator.  K parts (ks > 1, at most
// max_ks, dense only) cut each tile's K loop into ks units so that more pairs
// work when the tiles are few: each unit pays a pipeline fill (~4000 clocks)
// and an epilogue, and the ordered reduction reads the ks partial planes
// (~2600 bytes per clock) after a launch (~6000 clocks).
TmCfg choose_tm(int64_t m, int64_t groups, int64_t n, int64_t k, int pairs, int BB, bool gu = false,
                bool dual_ok = false, int max_ks = 1) {
  TmCfg best{0, 0, 0, 0, 0, 0, 1};
  double best_t = 1e30;
  const int64_t kcols = k / 256;
  const bool pp_ok = (k / kTmStageK) % 4 == 0;
  const int64_t tw = gu ? (n + kTmRows - 1) / kTmRows : (n + 255) / 256;
  for (int nt = 256; nt >= 32; nt -= 32) {
    if (nt > 32 && nt - 32 >= m) continue;      // a smaller tile already holds every row
    for (int dual = 0; dual < (dual_ok ? 2 : 1); ++dual) {
      const TmCfg c = tm_stages(nt, BB, gu, pp_ok, dual != 0);
      if (c.S < 3) continue;
      const int64_t tiles = groups * tw * ((m + nt - 1) / nt);
      for (int ks = 1; ks <= max_ks; ++ks) {
        if (ks > 1 && (kcols % 2 || ks > kcols / 2)) break;
        const int64_t units = tiles * ks;
        const double rounds = (double)((units + pairs - 1) / pairs);
        const double stages = 2.0 * (ks == 1 ? (double)kcols : 2.0 * (double)((kcols / 2 + ks - 1) / ks));
        const double main_clk = stages * std::max(dual ? kTmDualStageClk : 1120.0, 4.0 * nt + 90.0) +
                                (ks > 1 ? 4000.0 : 0.0);
        const double epi_clk = 1400.0 + (dual ? 30.0 : 20.0) * nt;
        double t = rounds * main_clk + (c.nacc == 1 ? rounds : 1.0) * epi_clk;
        if (ks > 1) t += 6000.0 + (double)(ks + 2) * (double)(m * n) * 4.0 / 2600.0;
        if (t < best_t * 0.97 || (t < best_t && ks == 1)) {   // a split must win clearly
          best_t = t;
          best = c;
          best.ks = ks;
        }
      }
    }
  }
  return best;
}

template <int T, int NMAP, bool GU = false>
int launch_tm(const CUtensorMap& map_b, const PairW<NMAP>& pw, const PairW<NMAP>& pw3, int64_t m, int64_t n,
              int64_t k, int tm, const TmCfg& cfg, int pairs, const float* rowscale, const float* bias, float* y,
              int acc, int act, cudaStream_t st, const CUtensorMap* map_p = nullptr, float* part = nullptr) {
  const void* fn = tm_kernel<T, NMAP, GU>();
  if constexpr (NMAP == 1 && !GU)
    if (cfg.dual) fn = tm_kernel<T, 1, false, true>();
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, cfg.smem);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm: smem attribute: %s", cudaGetErrorString(e));
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3((unsigned)(2 * pairs));
  lc.blockDim = dim3(kTmThreads);
  lc.dynamicSmemBytes = cfg.smem;
  lc.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 2;
  CUtensorMap map_y;
  memset(&map_y, 0, sizeof(map_y));
  const int y_tma = encode_y_map(&map_y, y, m, n) ? 1 : 0;
  CUtensorMap mp;
  if (map_p)
    mp = *map_p;
  else
    memset(&mp, 0, sizeof(mp));
  const int ksplit = map_p ? cfg.ks : 1;
  if constexpr (NMAP == 1 && !GU) {
    if (cfg.dual)
      e = cudaLaunchKernelEx(&lc, k_qgemm_tm<T, 1, false, true>, map_b, pw, pw3, map_y, y_tma, mp, ksplit, part,
                             (int)m, (int)n, (int)k, cfg.NT, cfg.nacc, cfg.S, cfg.RW, tm, rowscale, bias, y, acc, act);
    else
      e = cudaLaunchKernelEx(&lc, k_qgemm_tm<T, 1, false, false>, map_b, pw, pw3, map_y, y_tma, mp, ksplit, part,
                             (int)m, (int)n, (int)k, cfg.NT, cfg.nacc, cfg.S, cfg.RW, tm, rowscale, bias, y, acc, act);
  } else {
    e = cudaLaunchKernelEx(&lc, k_qgemm_tm<T, NMAP, GU>, map_b, pw, pw3, map_y, y_tma, mp, 1, (float*)nullptr,
                           (int)m, (int)n, (int)k, cfg.NT, cfg.nacc, cfg.S, cfg.RW, tm, rowscale, bias, y, acc, act);
  }
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm tm launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemm tm");
}

// Dense GEMM on the tensor-memory-A kernel; 1 (nothing launched) if the
// device cannot hold it.
template <int T>
int launch_tm_gemm(const __half* a16, const uint8_t* w, int64_t m, int64_t n, int64_t k, const float* rowscale,
                   const float* bias, float* y, int acc, cudaStream_t st, float* part = nullptr,
                   int64_t part_bytes = 0, int64_t w_pitch = 0) {
  constexpr int BB = ColGeom<T>::BB;
  const void* fn = tm_kernel<T, 1>();
  const TmCfg probe = tm_stages(128, BB);
  const int cap = cluster_capacity(fn, kTmThreads, probe.smem);
  if (cap < 1) return 1;
  // K parts need room for their partial planes and 16-byte output rows
  int max_ks = 1;
  if (part && n % 4 == 0 && !((uintptr_t)y & 15) && !((uintptr_t)bias & 15))
    while (max_ks < kTmMaxSplit && (int64_t)(max_ks + 1) * m * n * 4 <= part_bytes) ++max_ks;
  const TmCfg cfg = choose_tm(m, 1, n, k, cap, BB, false, true, max_ks);
  if (cfg.S < 3) return 1;
  const int cap_cfg = cluster_capacity(fn, kTmThreads, cfg.smem);
  if (cap_cfg < 1) return 1;
  CUtensorMap map_b;
  int rc = encode_a16(&map_b, a16, m, k, cfg.NT / 2);
  if (rc) return rc;
  PairW<1> pw{};
  rc = encode_w_records<T>(&pw.map[0], w, n, k, kTmRows, w_pitch);
  if (rc) return rc;
  pw.groups = 1;
  const int64_t tm = (m + cfg.NT - 1) / cfg.NT;
  const int64_t tiles = tm * ((n + 255) / 256);
  const int pairs = (int)std::min<int64_t>(tiles * cfg.ks, cap_cfg);
  if (cfg.ks == 1) return launch_tm<T, 1>(map_b, pw, pw, m, n, k, (int)tm, cfg, pairs, rowscale, bias, y, acc, 0, st);
  CUtensorMap map_p;
  if (!encode_part_map(&map_p, part, m, n, cfg.ks))
    return launch_tm<T, 1>(map_b, pw, pw, m, n, k, (int)tm, TmCfg{cfg.NT, cfg.nacc, cfg.S, cfg.RW, cfg.smem, cfg.dual, 1},
                           (int)std::min<int64_t>(tiles, cap_cfg), rowscale, bias, y, acc, 0, st);
  rc = launch_tm<T, 1>(map_b, pw, pw, m, n, k, (int)tm, cfg, pairs, rowscale, bias, y, acc, 0, st, &map_p, part);
  if (rc) return rc;
  const int64_t mn4 = m * n / 4;
  const unsigned rgrid = (unsigned)std::min<int64_t>((mn4 + 255) / 256, 148 * 8);
  k_splitk_reduce<<<rgrid, 256, 0, st>>>(part, cfg.ks, m * n, (int)n, bias, y, acc);
  return xm_check_launch("qgemm split-K reduction");
}

template <int T>
int launch_tm_grouped(const __half* a16, const uint8_t* const* h_w, const int* d_cnt, const int* d_off, int G,
                      int64_t P, int64_t n, int64_t k, int64_t max_rows, int64_t expect_rows, const float* rowscale,
                      float* y, cudaStream_t st) {
  constexpr int BB = ColGeom<T>::BB;
  const void* fn = tm_kernel<T, kMaxGroups>();
  const TmCfg probe = tm_stages(128, BB);
  const int cap = cluster_capacity(fn, kTmThreads, probe.smem);
  if (cap < 1) return 1;
  const TmCfg cfg = choose_tm(expect_rows, G, n, k, cap, BB);
  if (cfg.S < 3) return 1;
  const int cap_cfg = cluster_capacity(fn, kTmThreads, cfg.smem);
  if (cap_cfg < 1) return 1;
  CUtensorMap map_b;
  int rc = encode_a16(&map_b, a16, P, k, cfg.NT / 2);
  if (rc) return rc;
  PairW<kMaxGroups> pw{};
  for (int g = 0; g < G; ++g) {
    rc = encode_w_records<T>(&pw.map[g], h_w[g], n, k, kTmRows);
    if (rc) return rc;
  }
  pw.cnt = d_cnt;
  pw.off = d_off;
  pw.groups = G;
  const int tm = (int)((max_rows + cfg.NT - 1) / cfg.NT);
  const int64_t tiles = (int64_t)G * tm * ((n + 255) / 256);
  const int pairs = (int)std::min<int64_t>(tiles, cap_cfg);
  return launch_tm<T, kMaxGroups>(map_b, pw, pw, P, n, k, tm, cfg, pairs, rowscale, nullptr, y, 0, 0, st);
}

// Gate/up experts on the tensor-memory-A kernel: y = act(x W1^T) * (x W3^T)
// per group (rows [off[g], off[g] + cnt[g])); 1 if the device cannot hold it.
template <int T>
int launch_tm_grouped_gu(const __half* a16, const uint8_t* const* h_w1, const uint8_t* const* h_w3, const int* d_cnt,
                         const int* d_off, int G, int64_t P, int64_t n, int64_t k, int64_t max_rows,
                         int64_t expect_rows, const float* rowscale, int act, float* y, cudaStream_t st) {
  constexpr int BB = ColGeom<T>::BB;
  const void* fn = tm_kernel<T, kMaxGroups, true>();
  const TmCfg probe = tm_stages(128, BB, true);
  const int cap = cluster_capacity(fn, kTmThreads, probe.smem);
  if (cap < 1) return 1;
  const TmCfg cfg = choose_tm(expect_rows, G, n, k, cap, BB, true);
  if (cfg.S < 3) return 1;
  const int cap_cfg = cluster_capacity(fn, kTmThreads, cfg.smem);
  if (cap_cfg < 1) return 1;
  CUtensorMap map_b;
  int rc = encode_a16(&map_b, a16, P, k, cfg.NT / 2);
  if (rc) return rc;
  PairW<kMaxGroups> pw1{}, pw3{};
  for (int g = 0; g < G; ++g) {
    if ((rc = encode_w_records<T>(&pw1.map[g], h_w1[g], n, k, kTmRows / 2))) return rc;
    if ((rc = encode_w_records<T>(&pw3.map[g], h_w3[g], n, k, kTmRows / 2))) return rc;
  }
  pw1.cnt = pw3.cnt = d_cnt;
  pw1.off = pw3.off = d_off;
  pw1.groups = pw3.groups = G;
  const int tm = (int)((max_rows + cfg.NT - 1) / cfg.NT);
  const int64_t tiles = (int64_t)G * tm * ((n + kTmRows - 1) / kTmRows);
  const int pairs = (int)std::min<int64_t>(tiles, cap_cfg);
  return launch_tm<T, kMaxGroups, true>(map_b, pw1, pw3, P, n, k, tm, cfg, pairs, rowscale, nullptr, y, 0, act, st);
}

// Runtime type id -> the launchers above (dispatch_quant calls operator()<T>).
struct PairDense {
  const CUtensorMap* map_a;
  const uint8_t* w;
  int64_t m, n, k;
  const float *rowscale, *bias;
  float* y;
  int acc;
  cudaStream_t st;
  const __half* a16;
  float* part;                     // split-K partial planes (workspace beyond the activation), or null
  int64_t part_bytes;
  int64_t w_pitch;                 // weight row pitch in bytes (0: packed rows)
  int rc = 1;
  template <int T>
  void operator()() {
    // tensor-memory-A kernel; the CTA-pair kernel where the device cannot hold it (packed rows only)
    rc = launch_tm_gemm<T>(a16, w, m, n, k, rowscale, bias, y, acc, st, part, part_bytes, w_pitch);
    if (rc == 1 && w_pitch) rc = xm_set_error(XM_ERR_UNSUPPORTED, "qgemm: pitched weights need the CTA-pair kernel");
    if (rc == 1) rc = launch_pair_gemm<T>(*map_a, w, m, n, k, rowscale, bias, y, acc, st);
  }
};

struct PairGrouped {
  const CUtensorMap* map_a;
  const uint8_t* const* h_w;
  const int *cnt, *off;
  int G;
  int64_t P, n, k, max_rows, expect_rows;
  const float* rowscale;
  float* y;
  cudaStream_t st;
  const __half* a16;
  int rc = 1;
  template <int T>
  void operator()() {
    rc = launch_tm_grouped<T>(a16, h_w, cnt, off, G, P, n, k, max_rows, expect_rows, rowscale, y, st);
    if (rc == 1)
      rc = launch_pair_grouped<T>(*map_a, h_w, cnt, off, G, P, n, k, max_rows, expect_rows, rowscale, y, st);
  }
};

struct TmGroupedGU {
  const __half* a16;
  const uint8_t *const *w1, *const *w3;
  const int *cnt, *off;
  int G;
  int64_t P, n, k, max_rows, expect_rows;
  const float* rowscale;
  int act;
  float* y;
  cudaStream_t st;
  int rc = 1;
  template <int T>
  void operator()() {
    rc = launch_tm_grouped_gu<T>(a16, w1, w3, cnt, off, G, P, n, k, max_rows, expect_rows, rowscale, act, y, st);
  }
};

struct RowBytes {
  int64_t k;
  int64_t bytes = 0;
  template <int T>
  void operator()() {
    bytes = pair_row_bytes<T>(k);
  }
};
}  // namespace

// Bytes of one row of k weights of a block type, or 0 for a type that is not
// block-quantized.
int64_t qgemm_row_bytes(int qtype, int64_t k) {
  RowBytes rb{k};
  return dispatch_quant(qtype, rb) ? rb.bytes : 0;
}

bool qgemm_type_supported(int qtype, int64_t k) {
  if (k < 256 || k % 256) return false;
  const int64_t rb = qgemm_row_bytes(qtype, k);
  return rb > 0 && rb % 16 == 0;
}

int qgemm_grouped(int qtype, const __half* a16, const float* rowscale, int64_t P, int64_t K, int64_t N,
                  const uint8_t* const* h_w, const int* d_cnt, const int* d_off, int G, int64_t max_rows,
                  int64_t expect_rows, float* y, cudaStream_t st) {
  if (K % 256 || K < 256 || N < 1 || P < 1 || G < 1 || G > kMaxGroups)
    return xm_set_error(XM_ERR_INVALID, "grouped qgemm: bad shape");
  if (!qgemm_type_supported(qtype, K))
    return xm_set_error(XM_ERR_UNSUPPORTED, "grouped qgemm: type id %d rows of k=%lld are not 16-byte multiples", qtype,
                        (long long)K);
  CUtensorMap map_a;
  int rc = encode_a16(&map_a, a16, P, K);
  if (rc) return rc;
  PairGrouped pg{&map_a, h_w, d_cnt, d_off, G, P, N, K, max_rows, expect_rows, rowscale, y, st, a16};
  dispatch_quant(qtype, pg);
  if (pg.rc != 1) return pg.rc;
  if (qtype != T_Q4_K)
    return xm_set_error(XM_ERR_UNSUPPORTED, "grouped qgemm: this device cannot hold the CTA-pair kernel");
  GemmGroups groups{};
  groups.n = G;
  groups.cnt = d_cnt;
  groups.off = d_off;
  for (int g = 0; g < G; ++g) groups.w[g] = h_w[g];
  // tile shape for the expected rows per group, grid for the worst case
  TileCfg cfg = choose_tile(expect_rows, N * G, K, sm_count_dev());
  const dim3 grid((unsigned)((N + cfg.BN - 1) / cfg.BN), (unsigned)((max_rows + cfg.MT * 128 - 1) / (cfg.MT * 128)),
                  (unsigned)G);
  return launch_gemm(map_a, nullptr, P, N, K, cfg, grid, rowscale, nullptr, y, 0, groups, st);
}

int qgemm_grouped_gate_up(int qtype, int act, const __half* a16, const float* rowscale, int64_t P, int64_t K,
                          int64_t N, const uint8_t* const* h_w1, const uint8_t* const* h_w3, const int* d_cnt,
                          const int* d_off, int G, int64_t max_rows, int64_t expect_rows, float* y, cudaStream_t st) {
  if (K % 256 || K < 256 || N < 1 || P < 1 || G < 1 || G > kMaxGroups)
    return xm_set_error(XM_ERR_INVALID, "grouped gate/up qgemm: bad shape");
  if (!qgemm_type_supported(qtype, K))
    return xm_set_error(XM_ERR_UNSUPPORTED, "grouped gate/up qgemm: type id %d rows of k=%lld are not 16-byte "
                        "multiples", qtype, (long long)K);
  TmGroupedGU g{a16, h_w1, h_w3, d_cnt, d_off, G, P, N, K, max_rows, expect_rows, rowscale, act, y, st};
  dispatch_quant(qtype, g);
  return g.rc;
}

extern "C" int64_t xm_qgemm_workspace_size(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  return ((m * k * 2 + 255) / 256) * 256 + m * 4;
}

namespace {
// the split-K partial planes start after the activation and its row scales
int64_t qgemm_part_offset(int64_t m, int64_t k) {
  return ((m * k * 2 + 255) / 256) * 256 + ((m * 4 + 255) / 256) * 256;
}
constexpr int64_t kSplitMaxMN = int64_t(1) << 23;   // split-K only for outputs of at most 8M elements
}  // namespace

extern "C" int64_t xm_qgemm_workspace_size_n(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || k <= 0 || n <= 0) return 0;
  if (m * n > kSplitMaxMN) return xm_qgemm_workspace_size(m, k);
  return qgemm_part_offset(m, k) + (int64_t)kTmMaxSplit * m * n * 4;
}

namespace {
template <typename XT, int NTH>
void launch_prep_n(const void* x, int prologue, int64_t m, int64_t k, int64_t ldx, const float* norm_w, float eps,
                   __half* x16, float* rowscale, cudaStream_t st) {
  const unsigned pgrid = (unsigned)m;        // one block per row
  const XT* xt = (const XT*)x;
  if (prologue == XM_PRO_RMSNORM)
    k_prep_rows<XT, XM_PRO_RMSNORM, NTH><<<pgrid, NTH, 0, st>>>(xt, (int)m, (int)k, ldx, norm_w, eps, x16, rowscale);
  else if (prologue == XM_PRO_SWIGLU)
    k_prep_rows<XT, XM_PRO_SWIGLU, NTH><<<pgrid, NTH, 0, st>>>(xt, (int)m, (int)k, ldx, norm_w, eps, x16, rowscale);
  else
    k_prep_rows<XT, XM_PRO_NONE, NTH><<<pgrid, NTH, 0, st>>>(xt, (int)m, (int)k, ldx, norm_w, eps, x16, rowscale);
}
template <typename XT>
void launch_prep(const void* x, int prologue, int64_t m, int64_t k, int64_t ldx, const float* norm_w, float eps,
                 __half* x16, float* rowscale, cudaStream_t st) {
  if (m < 2 * sm_count_dev())
    launch_prep_n<XT, 1024>(x, prologue, m, k, ldx, norm_w, eps, x16, rowscale, st);
  else
    launch_prep_n<XT, kPrepThreads>(x, prologue, m, k, ldx, norm_w, eps, x16, rowscale, st);
}
}  // namespace

namespace {
int qgemm_ex_impl(int qtype, const void* d_w, int64_t w_pitch, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                  int x_dtype, int64_t m, int64_t x_stride, int prologue, const float* d_norm_w, float eps,
                  const float* d_bias, float* d_y, int accumulate, void* d_workspace, int64_t workspace_bytes,
                  void* stream) {
  int qk = 0, rec = 0;
  if (!host_qtype_geometry(qtype, &qk, &rec) || qk == 1)
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemm: type id %d is not a block-quantized type", qtype);
  if (m < 1 || n < 1 || k < 256 || k % 256)
    return xm_set_error(XM_ERR_INVALID, "qgemm: need m, n >= 1 and k a positive multiple of 256");
  if (m > (1 << 30) || n > (1 << 30) || k > (1 << 24)) return xm_set_error(XM_ERR_INVALID, "qgemm: shape too large");
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "qgemm: bad x dtype %d", x_dtype);
  if (prologue != XM_PRO_NONE && prologue != XM_PRO_RMSNORM && prologue != XM_PRO_SWIGLU)
    return xm_set_error(XM_ERR_INVALID, "qgemm: unknown prologue %d", prologue);
  if (prologue == XM_PRO_RMSNORM && !d_norm_w) return xm_set_error(XM_ERR_INVALID, "qgemm: RMSNorm needs weights");
  if (x_stride < (prologue == XM_PRO_SWIGLU ? 2 * k : k))
    return xm_set_error(XM_ERR_INVALID, "qgemm: x_stride %lld too small", (long long)x_stride);
  const int64_t row_bytes = qgemm_row_bytes(qtype, k);
  if (w_pitch && (w_pitch < row_bytes || w_pitch % 16))
    return xm_set_error(XM_ERR_INVALID, "qgemm: row pitch %lld must be a multiple of 16 and at least the row's %lld "
                        "bytes", (long long)w_pitch, (long long)row_bytes);
  const int64_t need_w = w_pitch ? (n - 1) * w_pitch + row_bytes : n * row_bytes;
  if (need_w > w_bytes)
    return xm_set_error(XM_ERR_INVALID, "qgemm: weight needs %lld bytes, got %lld", (long long)need_w,
                        (long long)w_bytes);
  if (!w_pitch && row_bytes % 16)
    return xm_set_error(XM_ERR_UNSUPPORTED,
                        "qgemm: a row of type id %d with k=%lld is %lld bytes, not a multiple of 16 (tensor-map "
                        "pitch); use the GEMV on row groups, or rows padded to a 16-byte pitch",
                        qtype, (long long)k, (long long)row_bytes);
  if (!d_w || !d_x || !d_y || !d_workspace) return xm_set_error(XM_ERR_INVALID, "qgemm: null pointer");
  if (((uintptr_t)d_w & 15) || ((uintptr_t)d_workspace & 255) || ((uintptr_t)d_x & 15))
    return xm_set_error(XM_ERR_INVALID, "qgemm: weight/x must be 16-byte and workspace 256-byte aligned");
  if (workspace_bytes < xm_qgemm_workspace_size(m, k))
    return xm_set_error(XM_ERR_INVALID, "qgemm: workspace too small");
  cudaStream_t st = (cudaStream_t)stream;

  __half* x16 = (__half*)d_workspace;
  float* rowscale = (float*)((uint8_t*)d_workspace + ((m * k * 2 + 255) / 256) * 256);
  if (x_dtype == XM_DT_F32)
    launch_prep<float>(d_x, prologue, m, k, x_stride, d_norm_w, eps, x16, rowscale, st);
  else if (x_dtype == XM_DT_BF16)
    launch_prep<__nv_bfloat16>(d_x, prologue, m, k, x_stride, d_norm_w, eps, x16, rowscale, st);
  else
    launch_prep<__half>(d_x, prologue, m, k, x_stride, d_norm_w, eps, x16, rowscale, st);
  int rc = xm_check_launch("qgemm prep");
  if (rc) return rc;

  CUtensorMap map_a;
  rc = encode_a16(&map_a, x16, m, k);
  if (rc) return rc;
  float* part = nullptr;
  int64_t part_bytes = 0;
  if (m * n <= kSplitMaxMN && workspace_bytes > qgemm_part_offset(m, k)) {
    part = (float*)((uint8_t*)d_workspace + qgemm_part_offset(m, k));
    part_bytes = workspace_bytes - qgemm_part_offset(m, k);
  }
  PairDense pd{&map_a, (const uint8_t*)d_w, m, n, k, rowscale, d_bias, d_y, accumulate ? 1 : 0, st, x16, part,
               part_bytes, w_pitch};
  dispatch_quant(qtype, pd);
  if (pd.rc != 1) return pd.rc;
  if (qtype != T_Q4_K)
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemm: this device cannot hold the CTA-pair kernel");
  if (w_pitch) return xm_set_error(XM_ERR_UNSUPPORTED, "qgemm: pitched weights need the CTA-pair kernel");
  const TileCfg cfg = choose_tile(m, n, k, sm_count_dev());
  const dim3 grid((unsigned)((n + cfg.BN - 1) / cfg.BN), (unsigned)((m + cfg.MT * 128 - 1) / (cfg.MT * 128)));
  return launch_gemm(map_a, (const uint8_t*)d_w, m, n, k, cfg, grid, rowscale, d_bias, d_y, accumulate ? 1 : 0,
                     GemmGroups{}, st);
}
}  // namespace

extern "C" int xm_qgemm_ex(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                           int x_dtype, int64_t m, int64_t x_stride, int prologue, const float* d_norm_w, float eps,
                           const float* d_bias, float* d_y, int accumulate, void* d_workspace,
                           int64_t workspace_bytes, void* stream) {
  return qgemm_ex_impl(qtype, d_w, 0, w_bytes, n, k, d_x, x_dtype, m, x_stride, prologue, d_norm_w, eps, d_bias, d_y,
                       accumulate, d_workspace, workspace_bytes, stream);
}

extern "C" int xm_qgemm_ex_pitched(int qtype, const void* d_w, int64_t w_row_pitch, int64_t w_bytes, int64_t n,
                                   int64_t k, const void* d_x, int x_dtype, int64_t m, int64_t x_stride, int prologue,
                                   const float* d_norm_w, float eps, const float* d_bias, float* d_y, int accumulate,
                                   void* d_workspace, int64_t workspace_bytes, void* stream) {
  if (w_row_pitch <= 0) return xm_set_error(XM_ERR_INVALID, "qgemm: row pitch must be positive");
  return qgemm_ex_impl(qtype, d_w, w_row_pitch, w_bytes, n, k, d_x, x_dtype, m, x_stride, prologue, d_norm_w, eps,
                       d_bias, d_y, accumulate, d_workspace, workspace_bytes, stream);
}

extern "C" int xm_qgemm(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                        int x_dtype, int64_t m, const float* d_bias, float* d_y, void* d_workspace,
                        int64_t workspace_bytes, void* stream) {
  return xm_qgemm_ex(qtype, d_w, w_bytes, n, k, d_x, x_dtype, m, k, XM_PRO_NONE, nullptr, 0.f, d_bias, d_y, 0,
                     d_workspace, workspace_bytes, stream);
}

extern "C" int xm_rmsnorm(const void* d_x, int x_dtype, int64_t m, int64_t k, int64_t x_stride, const float* d_norm_w,
                          float eps, float* d_out, void* stream) {
  if (m < 0 || k < 1 || x_stride < k) return xm_set_error(XM_ERR_INVALID, "rmsnorm: bad sizes");
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "rmsnorm: bad x dtype %d", x_dtype);
  if (m == 0) return XM_OK;
  if (!d_x || !d_norm_w || !d_out) return xm_set_error(XM_ERR_INVALID, "rmsnorm: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((m * 32 + 255) / 256);
  if (x_dtype == XM_DT_F32)
    k_rmsnorm_rows<float><<<grid, 256, 0, st>>>((const float*)d_x, (int)m, (int)k, x_stride, d_norm_w, eps, d_out);
  else if (x_dtype == XM_DT_BF16)
    k_rmsnorm_rows<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)d_x, (int)m, (int)k, x_stride,
                                                         d_norm_w, eps, d_out);
  else
    k_rmsnorm_rows<__half><<<grid, 256, 0, st>>>((const __half*)d_x, (int)m, (int)k, x_stride, d_norm_w, eps, d_out);
  return xm_check_launch("rmsnorm");
}
