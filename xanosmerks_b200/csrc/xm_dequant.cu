// K1: standalone GGUF dequantization (raw block bytes -> fp16 / fp32).
//
// HBM-bound.  Each CTA stages the contiguous byte range of its blocks into
// shared memory with 16-byte L1-bypassing loads (records of 18/22/84/110/210 B
// are not 16-byte aligned, so every thread reading its own fields from global
// memory would issue many narrow loads), then every thread decodes groups of
// 8 consecutive elements and writes them with one 16-byte (fp16) or two
// 16-byte (fp32) stores, fully coalesced.
#include "xm_decode.cuh"

namespace {

constexpr int kThreads = 256;

template <int T>
struct DequantCfg {
  // blocks per CTA: 4096 elements per CTA
  static constexpr int BPC = 4096 / QT<T>::QK;
  static constexpr int SMEM = BPC * QT<T>::REC + 16;
};

XM_DEV void store8(__half* out, const float* v) {
  __half2 h0 = __floats2half2_rn(v[0], v[1]);
  __half2 h1 = __floats2half2_rn(v[2], v[3]);
  __half2 h2 = __floats2half2_rn(v[4], v[5]);
  __half2 h3 = __floats2half2_rn(v[6], v[7]);
  uint4 u;
  u.x = *reinterpret_cast<uint32_t*>(&h0);
  u.y = *reinterpret_cast<uint32_t*>(&h1);
  u.z = *reinterpret_cast<uint32_t*>(&h2);
  u.w = *reinterpret_cast<uint32_t*>(&h3);
  *reinterpret_cast<uint4*>(out) = u;
}

XM_DEV void store8(float* out, const float* v) {
  reinterpret_cast<float4*>(out)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(out)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

template <int T, typename OutT>
__global__ void __launch_bounds__(kThreads) k_dequant(const uint8_t* __restrict__ raw, int64_t n_blocks,
                                                      OutT* __restrict__ out) {
  using Q = QT<T>;
  constexpr int BPC = DequantCfg<T>::BPC;
  __shared__ __align__(16) uint8_t sm[DequantCfg<T>::SMEM];
  const int64_t b0 = (int64_t)blockIdx.x * BPC;
  const int nb = (int)min((int64_t)BPC, n_blocks - b0);
  const int mis = stage_bytes(sm, raw + b0 * Q::REC, nb * Q::REC, threadIdx.x, kThreads);
  __syncthreads();
  const uint8_t* base = sm + mis;
  constexpr int GPB = Q::QK / 8;  // groups of 8 per block
  const int ngroups = nb * GPB;
  OutT* o = out + b0 * Q::QK;
  for (int g = threadIdx.x; g < ngroups; g += kThreads) {
    const int blk = g / GPB, e0 = (g % GPB) * 8;
    float v[8];
    Q::decode8(base + blk * Q::REC, e0, v);
    store8(o + (int64_t)blk * Q::QK + e0, v);
  }
}

// fp16 output, 16-byte-aligned input whose element count is a multiple of
// 256: one thread per 32-element item (a quarter-record of a 256-element
// super-block, or one of eight 32-element records), decoded word-wise
// (xm_decode) into 16 fp16 pairs and written with four 16-byte stores.  A CTA
// stages 32 consecutive 256-element columns (8192 elements).
constexpr int kItemCols = 32;
template <int T>
struct ItemCfg {
  static constexpr int CB = QT<T>::REC * (256 / QT<T>::QK);   // bytes of one 256-element column
  static constexpr int SMEM = kItemCols * CB + 32;            // + slack for the 16-byte over-read
};

template <int T>
__global__ void __launch_bounds__(kThreads) k_dequant_items(const uint8_t* __restrict__ raw, int64_t n_cols,
                                                            __half* __restrict__ out) {
  constexpr int CB = ItemCfg<T>::CB;
  __shared__ __align__(16) uint8_t sm[ItemCfg<T>::SMEM];
  const int64_t c0 = (int64_t)blockIdx.x * kItemCols;
  const int nc = (int)min((int64_t)kItemCols, n_cols - c0);
  stage_bytes(sm, raw + c0 * CB, nc * CB, threadIdx.x, kThreads);   // 16-byte aligned source: no offset
  __syncthreads();
  const int col = threadIdx.x >> 3, it = threadIdx.x & 7;
  if (col >= nc) return;
  uint32_t hv[16];
  xm_decode::item_regs<T>(sm + col * CB, it >> 1, it & 1, hv);
  uint4* o = reinterpret_cast<uint4*>(out + (c0 + col) * 256 + 32 * it);
#pragma unroll
  for (int q = 0; q < 4; ++q) o[q] = make_uint4(hv[4 * q], hv[4 * q + 1], hv[4 * q + 2], hv[4 * q + 3]);
}

// Plain (non-block) types, one element per thread-iteration.
template <typename OutT>
XM_DEV void put(OutT* o, int64_t i, float v);
template <>
XM_DEV void put<__half>(__half* o, int64_t i, float v) { o[i] = __float2half_rn(v); }
template <>
XM_DEV void put<float>(float* o, int64_t i, float v) { o[i] = v; }

template <typename OutT>
__global__ void k_plain(int qtype, const uint8_t* __restrict__ raw, int64_t n, OutT* __restrict__ out) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    switch (qtype) {
      case T_F16: {
        const __half h = reinterpret_cast<const __half*>(raw)[i];
        if constexpr (sizeof(OutT) == 2) out[i] = h; else put(out, i, __half2float(h));
        break;
      }
      case T_F32: put(out, i, reinterpret_cast<const float*>(raw)[i]); break;
      case T_BF16: put(out, i, __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(raw)[i] << 16)); break;
      // int -> fp16: every |v| < 65520 converts to float exactly, and anything
      // larger rounds to a float >= 65520, which still overflows fp16 to inf,
      // so int -> float -> half equals the direct rounding numpy performs.
      case T_I8: put(out, i, (float)reinterpret_cast<const int8_t*>(raw)[i]); break;
      case T_I16: put(out, i, (float)reinterpret_cast<const int16_t*>(raw)[i]); break;
      case T_I32: put(out, i, (float)reinterpret_cast<const int32_t*>(raw)[i]); break;
      case T_I64: put(out, i, (float)reinterpret_cast<const int64_t*>(raw)[i]); break;
      default: break;
    }
  }
}

struct LaunchDequant {
  const uint8_t* raw;
  int64_t n_blocks;
  void* out;
  int out_dtype;
  cudaStream_t stream;
  template <int T>
  void operator()() {
    if (out_dtype == XM_DT_F16 && ((uintptr_t)raw & 15) == 0 && (n_blocks * QT<T>::QK) % 256 == 0) {
      const int64_t n_cols = n_blocks * QT<T>::QK / 256;
      const int64_t grid = (n_cols + kItemCols - 1) / kItemCols;
      if (grid == 0) return;
      k_dequant_items<T><<<(unsigned)grid, kThreads, 0, stream>>>(raw, n_cols, (__half*)out);
      return;
    }
    constexpr int BPC = DequantCfg<T>::BPC;
    const int64_t grid = (n_blocks + BPC - 1) / BPC;
    if (grid == 0) return;
    if (out_dtype == XM_DT_F16)
      k_dequant<T, __half><<<(unsigned)grid, kThreads, 0, stream>>>(raw, n_blocks, (__half*)out);
    else
      k_dequant<T, float><<<(unsigned)grid, kThreads, 0, stream>>>(raw, n_blocks, (float*)out);
  }
};

}  // namespace

extern "C" int xm_dequantize(int qtype, const void* d_raw, int64_t raw_bytes, int64_t n_elements, void* d_out,
                             int out_dtype, void* stream) {
  int qk = 0, rec = 0;
  if (!host_qtype_geometry(qtype, &qk, &rec))
    return xm_set_error(XM_ERR_UNSUPPORTED, "dequantize: type id %d is not implemented", qtype);
  if (out_dtype != XM_DT_F16 && out_dtype != XM_DT_F32)
    return xm_set_error(XM_ERR_INVALID, "dequantize: out_dtype must be F16 or F32");
  if (n_elements < 0 || raw_bytes < 0) return xm_set_error(XM_ERR_INVALID, "dequantize: negative size");
  if (n_elements % qk)
    return xm_set_error(XM_ERR_INVALID, "dequantize: %lld elements is not a multiple of the block size %d",
                        (long long)n_elements, qk);
  const int64_t n_blocks = n_elements / qk;
  if (n_blocks * (int64_t)rec > raw_bytes)
    return xm_set_error(XM_ERR_INVALID, "dequantize: need %lld bytes for %lld elements, got %lld",
                        (long long)(n_blocks * rec), (long long)n_elements, (long long)raw_bytes);
  if (n_elements == 0) return XM_OK;
  if (!d_raw || !d_out) return xm_set_error(XM_ERR_INVALID, "dequantize: null pointer");
  if (((uintptr_t)d_out & 15) != 0) return xm_set_error(XM_ERR_INVALID, "dequantize: output not 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  if (qk == 1) {
    if (((uintptr_t)d_raw % rec) != 0)
      return xm_set_error(XM_ERR_INVALID, "dequantize: plain input not aligned to its element size");
    int64_t grid = (n_elements + 255) / 256;
    if (grid > 148 * 32) grid = 148 * 32;
    if (out_dtype == XM_DT_F16)
      k_plain<__half><<<(unsigned)grid, 256, 0, st>>>(qtype, (const uint8_t*)d_raw, n_elements, (__half*)d_out);
    else
      k_plain<float><<<(unsigned)grid, 256, 0, st>>>(qtype, (const uint8_t*)d_raw, n_elements, (float*)d_out);
    return xm_check_launch("dequantize(plain)");
  }
  LaunchDequant l{(const uint8_t*)d_raw, n_blocks, d_out, out_dtype, st};
  dispatch_quant(qtype, l);
  return xm_check_launch("dequantize");
}
