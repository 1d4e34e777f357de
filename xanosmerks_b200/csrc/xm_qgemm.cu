// K3: fused dequant-GEMM for prefill on 5th-generation tensor cores.
//
//   y[m][n] = sum_k x[m][k] * W[n][k]   (fp32 out), W in GGUF Q4_K blocks.
//
// Numerics.  Every weight is decoded to the reference's fp16 value (the fp32
// value d*sc*q - dmin*mn rounded once to fp16), so B is exact.  The
// activation is converted to fp16 after scaling each row by a power of two
// chosen from the row's largest magnitude (k_prep_rows): bf16 input converts
// exactly, and the scale keeps rows with large or tiny values inside fp16's
// range.  tcgen05.mma kind::f16 multiplies fp16 x fp16 exactly and
// accumulates in fp32 in tensor memory; the epilogue multiplies each row by
// its scale (exact).  The result therefore differs from the reference's
// fp32 `x @ W.T` only in summation order (and, for fp32 x, in x's fp16
// rounding).
//
// Structure (one CTA per output tile of MT*128 rows x BN columns):
//   warp 0      TMA producer: activation tiles (fp16, 128-byte swizzle, 2-D
//               tensor map) and raw Q4_K super-blocks (BN rows x 144 B per
//               super-block column, 2-D tensor map over the byte stream); no
//               multicast anywhere.
//   warp 1      allocates tensor memory and issues tcgen05.mma (one thread).
//   warps 2-9   decode the raw super-block into the fp16 B tile of each
//               64-wide K step, written straight into the UMMA K-major
//               128-byte-swizzled layout; afterwards they run the epilogue
//               (tcgen05.ld -> row scale -> y).
// Pipelines are mbarrier rings with bounded waits.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "xm_qtypes.cuh"

namespace {

constexpr int kStages = 3;
constexpr int kBK = 64;                        // K elements per stage (one 128-byte swizzle atom of fp16)
constexpr int kATileBytes = 128 * kBK * 2;     // one 128-row A box
constexpr int kDequantWarps = 8;
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
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}"
      ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

XM_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
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

// byte i of w as an exact float
XM_DEV float byte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | (uint32_t)i)) - 8388608.0f;
}

// ---------------------------------------------------------------------------
// Activation preparation: fp16 copy of x with a power-of-two scale per row.
// One warp per row.  rowscale[m] = 2^s with the row's max magnitude in
// [2^14, 2^15) after division by 2^s (s may be negative for small rows).
// ---------------------------------------------------------------------------
template <typename XT>
__global__ void __launch_bounds__(256) k_prep_rows(const XT* __restrict__ x, int M, int K, __half* __restrict__ x16,
                                                   float* __restrict__ rowscale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const XT* xr = x + (int64_t)warp * K;
  float amax = 0.f;
  for (int k = lane; k < K; k += 32) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  int s = 0;
  if (amax > 0.f && amax < INFINITY) {
    int e;
    frexpf(amax, &e);           // amax = f * 2^e, f in [0.5, 1): amax in [2^(e-1), 2^e)
    s = (e - 1) - 14;           // amax / 2^s in [2^14, 2^15)
  }
  const float inv = ldexpf(1.0f, -s);
  __half* o = x16 + (int64_t)warp * K;
  for (int k = lane; k < K; k += 32) o[k] = __float2half_rn(to_f32(xr[k]) * inv);
  if (lane == 0) rowscale[warp] = ldexpf(1.0f, s);
}

// ---------------------------------------------------------------------------
// The GEMM kernel.
// ---------------------------------------------------------------------------
struct GemmSmem {
  uint64_t a_full[kStages], b_full[kStages], ab_empty[kStages];
  uint64_t raw_full[2], raw_empty[2];
  uint64_t acc_full;
  uint32_t tmem_base;
};

__global__ void __launch_bounds__(kThreads, 1)
    k_qgemm_q4k_tc(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w, int M, int N,
                   int K, int MT, int BN, const float* __restrict__ rowscale, const float* __restrict__ bias,
                   float* __restrict__ y) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned carve-up: A stages | B stages | raw W (x2) | control
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int a_stage_bytes = MT * kATileBytes;
  const int b_stage_bytes = BN * kBK * 2;
  const int raw_bytes = BN * 144;
  uint8_t* sA = base;
  uint8_t* sB = sA + kStages * a_stage_bytes;
  uint8_t* sRaw = sB + kStages * b_stage_bytes;
  GemmSmem* ctl = reinterpret_cast<GemmSmem*>(sRaw + ((2 * raw_bytes + 15) & ~15));

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * BN;
  const int m0 = blockIdx.y * (MT * 128);
  const int nkt = K / kBK;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&ctl->a_full[i], 1);
      mbar_init(&ctl->b_full[i], kDequantWarps);
      mbar_init(&ctl->ab_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&ctl->raw_full[i], 1);
      mbar_init(&ctl->raw_empty[i], kDequantWarps);
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
        if ((kt & 3) == 0) {
          const int sb = kt >> 2, r = sb & 1;
          if (sb >= 2) mbar_wait_bounded(&ctl->raw_empty[r], (uint32_t)(((sb >> 1) - 1) & 1));
          mbar_arrive_expect_tx(&ctl->raw_full[r], (uint32_t)raw_bytes);
          tma_load_2d(sRaw + r * raw_bytes, &map_w, sb * 144, n0, &ctl->raw_full[r]);
        }
        const int s = kt % kStages;
        if (kt >= kStages) mbar_wait_bounded(&ctl->ab_empty[s], (uint32_t)(((kt / kStages) - 1) & 1));
        mbar_arrive_expect_tx(&ctl->a_full[s], (uint32_t)a_stage_bytes);
        for (int mt = 0; mt < MT; ++mt)
          tma_load_2d(sA + s * a_stage_bytes + mt * kATileBytes, &map_a, kt * kBK, m0 + mt * 128, &ctl->a_full[s]);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_f16_f32(BN);
      for (int kt = 0; kt < nkt; ++kt) {
        const int s = kt % kStages;
        const uint32_t ph = (uint32_t)((kt / kStages) & 1);
        mbar_wait_bounded(&ctl->a_full[s], ph);
        mbar_wait_bounded(&ctl->b_full[s], ph);
        tc_fence_after();
        const uint8_t* a = sA + s * a_stage_bytes;
        const uint8_t* b = sB + s * b_stage_bytes;
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = smem_desc_sw128(a + mt * kATileBytes + kk * 32);
            const uint64_t bd = smem_desc_sw128(b + kk * 32);
            tc_mma_f16(tmem + (uint32_t)(mt * BN), ad, bd, idesc, (kt | kk) != 0 ? 1u : 0u);
          }
        }
        tc_commit(&ctl->ab_empty[s]);   // frees the stage once these MMAs have read it
      }
      tc_commit(&ctl->acc_full);
    }
  } else {
    // ---------------- dequant producers ----------------
    const int dw = warp - 2;                     // 0..7
    const int dt = dw * 32 + lane;               // 0..255
    const int items = BN * 4;                    // (row, 16-element quarter) per K step
    for (int kt = 0; kt < nkt; ++kt) {
      const int sb = kt >> 2, j = kt & 3, r = sb & 1;
      if (j == 0) mbar_wait_bounded(&ctl->raw_full[r], (uint32_t)((sb >> 1) & 1));
      const int s = kt % kStages;
      if (kt >= kStages) mbar_wait_bounded(&ctl->ab_empty[s], (uint32_t)(((kt / kStages) - 1) & 1));
      const uint8_t* raw = sRaw + r * raw_bytes;
      uint8_t* bt = sB + s * b_stage_bytes;
      for (int it = dt; it < items; it += kDequantWarps * 32) {
        const int n = it >> 2, qd = it & 3;      // elements 16*qd .. 16*qd+15 of this K step
        const uint8_t* blk = raw + n * 144;
        const uint32_t hw = *reinterpret_cast<const uint32_t*>(blk);
        const uint32_t A = *reinterpret_cast<const uint32_t*>(blk + 4);
        const uint32_t B = *reinterpret_cast<const uint32_t*>(blk + 8);
        const uint32_t C = *reinterpret_cast<const uint32_t*>(blk + 12);
        const int sub = 2 * j + (qd >> 1);       // sub-block 2j (low nibbles) or 2j+1 (high)
        const uint32_t scw = sub < 4 ? (A & 0x3F3F3F3Fu) : ((C & 0x0F0F0F0Fu) | ((A >> 2) & 0x30303030u));
        const uint32_t mnw = sub < 4 ? (B & 0x3F3F3F3Fu) : (((C >> 4) & 0x0F0F0F0Fu) | ((B >> 2) & 0x30303030u));
        const float d = __half2float(__ushort_as_half((unsigned short)(hw & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hw >> 16)));
        const float d1 = __fmul_rn(d, byte_f(scw, sub & 3));
        const float m1 = __fmul_rn(dmin, byte_f(mnw, sub & 3));
        const uint4 qv = *reinterpret_cast<const uint4*>(blk + 16 + 32 * j + 16 * (qd & 1));
        const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
        const int sh = (qd >> 1) * 4;
        uint32_t h[8];
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const uint32_t w = qw[t >> 1] >> (16 * (t & 1));          // bytes 2t, 2t+1 of the 16
          const float q0 = (float)((w >> sh) & 15u), q1 = (float)((w >> (8 + sh)) & 15u);
          const __half2 hv = __floats2half2_rn(__fsub_rn(__fmul_rn(d1, q0), m1), __fsub_rn(__fmul_rn(d1, q1), m1));
          h[t] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        // K-major 128-byte swizzle: row n, 16-byte chunk c stored at chunk c ^ (n & 7)
        uint8_t* row = bt + n * 128;
        const int c0 = 2 * qd, c1 = 2 * qd + 1;
        *reinterpret_cast<uint4*>(row + ((c0 ^ (n & 7)) << 4)) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(row + ((c1 ^ (n & 7)) << 4)) = make_uint4(h[4], h[5], h[6], h[7]);
      }
      fence_proxy_async_smem();    // generic-proxy writes -> visible to the tensor core
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&ctl->b_full[s]);
        if (j == 3) mbar_arrive(&ctl->raw_empty[r]);
      }
    }
    // ---------------- epilogue ----------------
    mbar_wait_bounded(&ctl->acc_full, 0);
    tc_fence_after();
    const int sp = warp & 3;                     // TMEM sub-partition this warp may read
    const int half = (warp - 2) >> 2;            // two warps per sub-partition split the columns
    const int nchunks = BN / 16;
    for (int mt = 0; mt < MT; ++mt) {
      const int m = m0 + mt * 128 + sp * 32 + lane;
      const float rs = m < M ? rowscale[m] : 0.f;
      for (int ch = half; ch < nchunks; ch += 2) {
        uint32_t v[16];
        tmem_ld16(tmem + ((uint32_t)(sp * 32) << 16) + (uint32_t)(mt * BN + ch * 16), v);
        tmem_ld_wait();
        const int nn = n0 + ch * 16;
        if (m < M) {
          float* yr = y + (int64_t)m * N + nn;
#pragma unroll
          for (int t = 0; t < 16; ++t)
            if (nn + t < N) yr[t] = __uint_as_float(v[t]) * rs + (bias ? bias[nn + t] : 0.f);
        }
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
  int MT, BN;
};

// Output tile shape: MT*128 rows x BN columns (BN a multiple of 16, MT*BN <=
// 512 tensor-memory columns), picked to minimise the estimated makespan
// (waves of tiles over the SMs, each tile's MMA and decode work) with a
// penalty for re-reading x once per column tile.
TileCfg choose_tile(int64_t M, int64_t N, int64_t K, int sms) {
  TileCfg best{1, 128};
  double best_t = 1e30;
  for (int MT = 1; MT <= 2; ++MT)
    for (int BN = 32; BN <= 256; BN += 16) {
      if (MT * BN > 512) continue;
      const int64_t a_stage = (int64_t)MT * kATileBytes, b_stage = (int64_t)BN * kBK * 2;
      if (kStages * (a_stage + b_stage) + 2 * BN * 144 + 1024 + 256 > 227 * 1024) continue;
      const int64_t tn = (N + BN - 1) / BN, tm = (M + MT * 128 - 1) / (MT * 128);
      const int64_t tiles = tn * tm;
      const int64_t waves = (tiles + sms - 1) / sms;
      const double mma = (double)MT * 128 * BN * K;            // MACs per tile
      const double deq = (double)BN * K * 6.0;                 // decode work per tile (MAC-equivalents)
      const double t = waves * std::max(mma / 4096.0, deq / 64.0) + (double)tn * M * K * 2 / 8e4;
      if (t < best_t) { best_t = t; best = {MT, BN}; }
    }
  return best;
}

}  // namespace

extern "C" int64_t xm_qgemm_workspace_size(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0) return 0;
  return ((m * k * 2 + 255) / 256) * 256 + m * 4;
}

extern "C" int xm_qgemm(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k, const void* d_x,
                        int x_dtype, int64_t m, const float* d_bias, float* d_y, void* d_workspace,
                        int64_t workspace_bytes, void* stream) {
  if (qtype != T_Q4_K)
    return xm_set_error(XM_ERR_UNSUPPORTED, "qgemm: type id %d has no tensor-core path yet", qtype);
  if (m < 1 || n < 1 || k < 256 || k % 256)
    return xm_set_error(XM_ERR_INVALID, "qgemm: need m, n >= 1 and k a positive multiple of 256");
  if (m > (1 << 30) || n > (1 << 30) || k > (1 << 24)) return xm_set_error(XM_ERR_INVALID, "qgemm: shape too large");
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "qgemm: bad x dtype %d", x_dtype);
  const int64_t row_bytes = (k / 256) * 144;
  if (n * row_bytes > w_bytes)
    return xm_set_error(XM_ERR_INVALID, "qgemm: weight needs %lld bytes, got %lld", (long long)(n * row_bytes),
                        (long long)w_bytes);
  if (!d_w || !d_x || !d_y || !d_workspace) return xm_set_error(XM_ERR_INVALID, "qgemm: null pointer");
  if (((uintptr_t)d_w & 15) || ((uintptr_t)d_workspace & 255) || ((uintptr_t)d_x & 15))
    return xm_set_error(XM_ERR_INVALID, "qgemm: weight/x must be 16-byte and workspace 256-byte aligned");
  if (workspace_bytes < xm_qgemm_workspace_size(m, k))
    return xm_set_error(XM_ERR_INVALID, "qgemm: workspace too small");
  EncodeTiledFn encode = get_encode();
  if (!encode) return xm_set_error(XM_ERR_CUDA, "qgemm: cuTensorMapEncodeTiled unavailable");
  cudaStream_t st = (cudaStream_t)stream;

  __half* x16 = (__half*)d_workspace;
  float* rowscale = (float*)((uint8_t*)d_workspace + ((m * k * 2 + 255) / 256) * 256);
  const unsigned pgrid = (unsigned)((m * 32 + 255) / 256);
  if (x_dtype == XM_DT_F32)
    k_prep_rows<float><<<pgrid, 256, 0, st>>>((const float*)d_x, (int)m, (int)k, x16, rowscale);
  else if (x_dtype == XM_DT_BF16)
    k_prep_rows<__nv_bfloat16><<<pgrid, 256, 0, st>>>((const __nv_bfloat16*)d_x, (int)m, (int)k, x16, rowscale);
  else
    k_prep_rows<__half><<<pgrid, 256, 0, st>>>((const __half*)d_x, (int)m, (int)k, x16, rowscale);
  int rc = xm_check_launch("qgemm prep");
  if (rc) return rc;

  const TileCfg cfg = choose_tile(m, n, k, sm_count_dev());
  CUtensorMap map_a, map_w;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)m};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, 128};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = encode(&map_a, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return xm_set_error(XM_ERR_CUDA, "qgemm: activation tensor map (%d)", (int)r);
  }
  {
    const cuuint64_t dims[2] = {(cuuint64_t)row_bytes, (cuuint64_t)n};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {144, (cuuint32_t)cfg.BN};
    const cuuint32_t es[2] = {1, 1};
    CUresult r = encode(&map_w, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(d_w), dims, strides, box, es,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return xm_set_error(XM_ERR_CUDA, "qgemm: weight tensor map (%d)", (int)r);
  }
  const int smem = 1024 + kStages * (cfg.MT * kATileBytes + cfg.BN * kBK * 2) + ((2 * cfg.BN * 144 + 15) & ~15) +
                   (int)sizeof(GemmSmem);
  cudaError_t e = cudaFuncSetAttribute(k_qgemm_q4k_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm: smem attribute: %s", cudaGetErrorString(e));
  const dim3 grid((unsigned)((n + cfg.BN - 1) / cfg.BN), (unsigned)((m + cfg.MT * 128 - 1) / (cfg.MT * 128)));
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
  e = cudaLaunchKernelEx(&lc, k_qgemm_q4k_tc, map_a, map_w, (int)m, (int)n, (int)k, cfg.MT, cfg.BN,
                         (const float*)rowscale, d_bias, d_y);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "qgemm launch: %s", cudaGetErrorString(e));
  return xm_check_launch("qgemm");
}
