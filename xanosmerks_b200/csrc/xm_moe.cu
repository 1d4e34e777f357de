// K5/K6: sparse mixture-of-experts block on quantized expert weights.
//
// Mirrors moe.py:54-115 (MoELayer.__call__):
//   router logits = x @ gate.T                     (moe.py:61)
//   top-k experts per token, softmax over the k selected logits
//                                                  (moe.py:75-81; dense softmax when k = E, moe.py:63-72)
//   stable sort of the (token, slot) pairs by expert (moe.py:83-93)
//   per expert: silu(x @ w1.T) * (x @ w3.T), then @ w2.T   (moe.py:97-113)
//   output[token] += expert_out * weight, experts in ascending order (moe.py:112)
//
// Device pipeline (one stream, no host round trip):
//   k_moe_router      one warp per token: E dot products (vector loads), top-k, softmax
//   k_moe_sort        one CTA: stable counting sort of the T*k pairs by expert
//   k_moe_gather_prep gathered rows of x -> fp16 with a power-of-two row scale
//   grouped GEMM      w1 and w3 over every expert's row range (tensor cores)
//   k_swiglu_prep     silu(g) * u -> fp16 with row scale (A of the next GEMM)
//   grouped GEMM      w2
//   k_moe_combine     weighted sum of each token's k expert rows, ascending expert
//                     (one block per token)
#include <algorithm>

#include "xm_internal.h"
#include "xm_qtypes.cuh"

namespace {

constexpr int kMaxExperts = 32;

// primitives.py:7-11 softmax (max-shifted, + 1e-12 in the denominator)
XM_DEV void softmax_small(float* v, int n) {
  float mx = v[0];
  for (int i = 1; i < n; ++i) mx = fmaxf(mx, v[i]);
  if (!(fabsf(mx) < INFINITY)) mx = 0.f;
  float s = 0.f;
  for (int i = 0; i < n; ++i) {
    v[i] = expf(v[i] - mx);
    s += v[i];
  }
  for (int i = 0; i < n; ++i) v[i] = v[i] / (s + 1e-12f);
}

// One warp per token.  Lane l covers elements 8l + 256i of the row (vector
// loads of x and of every expert's gate row); the E <= EC logits stay in
// registers (static indices only), go through shared memory after the warp
// reduction, and lane 0 selects the top k from there.
template <typename XT, int EC>
__global__ void __launch_bounds__(256) k_moe_router(const XT* __restrict__ x, const float* __restrict__ gate, int T,
                                                    int H, int E, int k, int* __restrict__ topk_e,
                                                    float* __restrict__ topk_w) {
  __shared__ float s_logit[8][EC];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  float acc[EC];
#pragma unroll
  for (int e = 0; e < EC; ++e) acc[e] = 0.f;
  const XT* xr = x + (int64_t)t * H;
  for (int h = lane * 8; h < H; h += 256) {
    float xv[8];
    ld4f<XT>(xr + h, *reinterpret_cast<float(*)[4]>(xv));
    ld4f<XT>(xr + h + 4, *reinterpret_cast<float(*)[4]>(xv + 4));
#pragma unroll
    for (int e = 0; e < EC; ++e) {
      if (e < E) {
        const float4 g0 = __ldg(reinterpret_cast<const float4*>(gate + (int64_t)e * H + h));
        const float4 g1 = __ldg(reinterpret_cast<const float4*>(gate + (int64_t)e * H + h + 4));
        float a = acc[e];
        a = fmaf(xv[0], g0.x, a); a = fmaf(xv[1], g0.y, a); a = fmaf(xv[2], g0.z, a); a = fmaf(xv[3], g0.w, a);
        a = fmaf(xv[4], g1.x, a); a = fmaf(xv[5], g1.y, a); a = fmaf(xv[6], g1.z, a); a = fmaf(xv[7], g1.w, a);
        acc[e] = a;
      }
    }
  }
#pragma unroll
  for (int e = 0; e < EC; ++e) {
    if (e < E) {
      const float v = warp_sum(acc[e]);
      if (lane == 0) s_logit[warp][e] = v;
    }
  }
  __syncwarp();
  if (lane != 0) return;
  const float* lg = s_logit[warp];
  int sel[EC];
  float val[EC];
  if (k == E) {
    for (int e = 0; e < E; ++e) { sel[e] = e; val[e] = lg[e]; }
  } else {
    unsigned used = 0;
    for (int j = 0; j < k; ++j) {       // the k largest logits (the set argpartition selects)
      int best = -1;
      for (int e = 0; e < E; ++e)
        if (!((used >> e) & 1u) && (best < 0 || lg[e] > lg[best])) best = e;
      used |= 1u << best;
      sel[j] = best;
      val[j] = lg[best];
    }
  }
  softmax_small(val, k);
  for (int j = 0; j < k; ++j) {
    topk_e[(int64_t)t * k + j] = sel[j];
    topk_w[(int64_t)t * k + j] = val[j];
  }
}

// Stable counting sort of P = T*k pairs by expert (one CTA of 1024 threads).
__global__ void __launch_bounds__(1024) k_moe_sort(const int* __restrict__ topk_e, const float* __restrict__ topk_w,
                                                   int P, int k, int E, int* __restrict__ sorted_tok,
                                                   float* __restrict__ sorted_w, int* __restrict__ pair_pos,
                                                   int* __restrict__ cnt, int* __restrict__ off) {
  __shared__ int s_cnt[kMaxExperts], s_base[kMaxExperts], s_tot[kMaxExperts];
  __shared__ int s_w[32][kMaxExperts];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < kMaxExperts) s_cnt[tid] = 0;
  __syncthreads();
  for (int i = tid; i < P; i += 1024) atomicAdd(&s_cnt[topk_e[i]], 1);
  __syncthreads();
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      cnt[e] = s_cnt[e];
      off[e] = run;
      s_base[e] = run;
      run += s_cnt[e];
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int c0 = 0; c0 < P; c0 += 1024) {
    const int i = c0 + tid;
    const int e = i < P ? topk_e[i] : -1;
    int rank = 0;
    for (int ex = 0; ex < E; ++ex) {
      const unsigned b = __ballot_sync(0xffffffffu, e == ex);
      if (lane == 0) s_w[warp][ex] = __popc(b);
      if (e == ex) rank = __popc(b & lt);
    }
    __syncthreads();
    if (tid < E) {                       // exclusive prefix over warps, per expert
      int run = 0;
      for (int w = 0; w < 32; ++w) {
        const int c = s_w[w][tid];
        s_w[w][tid] = run;
        run += c;
      }
      s_tot[tid] = run;
    }
    __syncthreads();
    if (i < P) {
      const int pos = s_base[e] + s_w[warp][e] + rank;
      sorted_tok[pos] = i / k;
      sorted_w[pos] = topk_w[i];
      pair_pos[i] = pos;
    }
    __syncthreads();
    if (tid < E) s_base[tid] += s_tot[tid];
    __syncthreads();
  }
}

// Rows (gathered in expert order) converted to fp16 with a power-of-two row
// scale (prep_row_fp16: the prefill GEMM's activation preparation).
template <typename XT>
__global__ void __launch_bounds__(kPrepThreads) k_moe_gather_prep(const XT* __restrict__ x,
                                                                  const int* __restrict__ sorted_tok, int P, int H,
                                                                  __half* __restrict__ a16,
                                                                  float* __restrict__ ascale) {
  __shared__ float red[32];
  const int p = blockIdx.x;
  const XT* xr = x + (int64_t)(sorted_tok ? sorted_tok[p] : p) * H;
  prep_row_fp16([&](int k, float (&v)[4]) { ld4f<XT>(xr + k, v); }, H, a16 + (int64_t)p * H, ascale + p, red);
}

// send[p] = x[sorted_tok[p]] (rows in expert order, x's element type kept)
template <typename XT>
__global__ void __launch_bounds__(256) k_moe_gather(const XT* __restrict__ x, const int* __restrict__ sorted_tok, int P,
                                                    int H, XT* __restrict__ send) {
  const int p = blockIdx.y;
  const XT* xr = x + (int64_t)sorted_tok[p] * H;
  XT* o = send + (int64_t)p * H;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < H; i += gridDim.x * blockDim.x) o[i] = xr[i];
}

// act(g) * u, then the fp16 row preparation of the down projection's
// activation.  act is the reference's apply_activation (primitives.py:37-62):
// silu x / (1 + exp(-x)), gelu (tanh form) 0.5 x (1 + tanh(0.7978845608 (x +
// 0.044715 x^3))), relu max(x, 0), identity.
template <int ACT>
XM_DEV float expert_act(float x) {
  return xm_act(ACT, x);
}

template <int ACT>
__global__ void __launch_bounds__(kPrepThreads) k_swiglu_prep(const float* __restrict__ g, const float* __restrict__ u,
                                                              int P, int F, __half* __restrict__ h16,
                                                              float* __restrict__ hscale) {
  __shared__ float red[32];
  const int p = blockIdx.x;
  const float* gr = g + (int64_t)p * F;
  const float* ur = u + (int64_t)p * F;
  prep_row_fp16(
      [&](int k, float (&v)[4]) {
        float uu[4];
        ld4f<float>(gr + k, v);
        ld4f<float>(ur + k, uu);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i] = expert_act<ACT>(v[i]) * uu[i];
      },
      F, h16 + (int64_t)p * F, hscale + p, red);
}

// fp32 rows (P x F) -> fp16 with a power-of-two row scale, one block per row,
// the row held in shared memory between the max and the conversion (one
// read of the row).  Dynamic shared memory: F floats.
__global__ void __launch_bounds__(kPrepThreads) k_rows_fp16(const float* __restrict__ h, int F, __half* __restrict__ h16,
                                                            float* __restrict__ hscale) {
  extern __shared__ float4 rowc[];
  __shared__ float red[32];
  const int p = blockIdx.x;
  const float4* hr = reinterpret_cast<const float4*>(h + (int64_t)p * F);
  const int F4 = F >> 2;
  float amax = 0.f;
  int k = threadIdx.x;
  for (; k + 3 * kPrepThreads < F4; k += 4 * kPrepThreads) {   // four independent loads in flight per thread
    float4 v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __ldcs(hr + k + i * kPrepThreads);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      rowc[k + i * kPrepThreads] = v[i];
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
    }
  }
  for (; k < F4; k += kPrepThreads) {
    const float4 v = __ldcs(hr + k);
    rowc[k] = v;
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  amax = block_max(amax, red);                    // (its barrier also orders the row cache)
  const int s = fp16_row_shift(amax);
  const float inv = ldexpf(1.0f, -s);
  __half* o = h16 + (int64_t)p * F;
  for (k = threadIdx.x; k < F4; k += kPrepThreads) {
    const float4 v = rowc[k];
    const __half2 a = __floats2half2_rn(v.x * inv, v.y * inv), b = __floats2half2_rn(v.z * inv, v.w * inv);
    *reinterpret_cast<uint2*>(o + 4 * k) = make_uint2(*reinterpret_cast<const uint32_t*>(&a),
                                                      *reinterpret_cast<const uint32_t*>(&b));
  }
  if (threadIdx.x == 0) hscale[p] = ldexpf(1.0f, s);
}

// out[t] = sum over the token's k expert rows, ascending expert order, of
// row * weight: products rounded, then added, as the numpy accumulation does
// (moe.py:110-113).  One block per token: the token's k (expert, row, weight)
// triples are ordered once in shared memory, then every thread sums 4
// consecutive columns (vector loads).
__global__ void __launch_bounds__(256) k_moe_combine(const float* __restrict__ d, const int* __restrict__ topk_e,
                                                     const float* __restrict__ topk_w, const int* __restrict__ pair_pos,
                                                     int T, int H, int k, float* __restrict__ out) {
  __shared__ int s_pos[kMaxExperts];
  __shared__ float s_w[kMaxExperts];
  const int t = blockIdx.x;
  if (threadIdx.x == 0) {
    int ord[kMaxExperts];
    for (int j = 0; j < k; ++j) ord[j] = j;
    for (int a = 1; a < k; ++a) {            // insertion sort of the k slots by expert id
      const int v = ord[a];
      int b = a - 1;
      while (b >= 0 && topk_e[(int64_t)t * k + ord[b]] > topk_e[(int64_t)t * k + v]) {
        ord[b + 1] = ord[b];
        --b;
      }
      ord[b + 1] = v;
    }
    for (int j = 0; j < k; ++j) {
      const int slot = (int)((int64_t)t * k + ord[j]);
      s_pos[j] = pair_pos[slot];
      s_w[j] = topk_w[slot];
    }
  }
  __syncthreads();
  for (int h = threadIdx.x * 4; h < H; h += 256 * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const float4 v = *reinterpret_cast<const float4*>(d + (int64_t)s_pos[j] * H + h);
      const float w = s_w[j];
      acc.x = __fadd_rn(acc.x, __fmul_rn(v.x, w));
      acc.y = __fadd_rn(acc.y, __fmul_rn(v.y, w));
      acc.z = __fadd_rn(acc.z, __fmul_rn(v.z, w));
      acc.w = __fadd_rn(acc.w, __fmul_rn(v.w, w));
    }
    *reinterpret_cast<float4*>(out + (int64_t)t * H + h) = acc;
  }
}

struct MoeWs {
  int *topk_e, *sorted_tok, *pair_pos, *cnt, *off;
  float *topk_w, *sorted_w, *ascale, *hscale, *g, *u, *d;
  __half *a16, *h16;
  int64_t bytes;
};

int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }

MoeWs carve(uint8_t* base, int64_t T, int64_t H, int64_t F, int E, int k) {
  MoeWs w{};
  const int64_t P = T * k;
  int64_t o = 0;
  auto take = [&](int64_t bytes) { uint8_t* p = base ? base + o : nullptr; o += align256(bytes); return p; };
  w.topk_e = (int*)take(P * 4);
  w.topk_w = (float*)take(P * 4);
  w.sorted_tok = (int*)take(P * 4);
  w.sorted_w = (float*)take(P * 4);
  w.pair_pos = (int*)take(P * 4);
  w.cnt = (int*)take(E * 4);
  w.off = (int*)take(E * 4);
  w.a16 = (__half*)take(P * H * 2);
  w.ascale = (float*)take(P * 4);
  w.g = (float*)take(P * F * 4);
  w.u = (float*)take(P * F * 4);
  w.h16 = (__half*)take(P * F * 2);
  w.hscale = (float*)take(P * 4);
  w.d = (float*)take(P * H * 4);
  w.bytes = o;
  return w;
}

}  // namespace

extern "C" int64_t xm_moe_workspace_size(int64_t T, int64_t H, int64_t F, int E, int k) {
  if (T < 1 || H < 1 || F < 1 || E < 1 || k < 1 || k > E) return 0;
  return carve(nullptr, T, H, F, E, k).bytes;
}

namespace {

int check_common(int E, int k, int64_t T, int64_t H, int x_dtype) {
  if (E < 1 || E > kMaxExperts) return xm_set_error(XM_ERR_INVALID, "moe: %d experts (1..%d supported)", E, kMaxExperts);
  if (k < 1 || k > E) return xm_set_error(XM_ERR_INVALID, "moe: num_experts_per_tok=%d outside 1..%d", k, E);
  if (T < 1 || H < 256 || H % 256) return xm_set_error(XM_ERR_INVALID, "moe: hidden size must be a positive multiple of 256");
  if (T * k > (1 << 30)) return xm_set_error(XM_ERR_INVALID, "moe: too many tokens");
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "moe: bad x dtype %d", x_dtype);
  return XM_OK;
}

template <typename XT>
void launch_router(const XT* x, const float* gate, int64_t T, int64_t H, int E, int k, int* topk_e, float* topk_w,
                   cudaStream_t st) {
  const unsigned grid = (unsigned)((T + 7) / 8);   // 8 tokens (warps) per block
  if (E <= 8)
    k_moe_router<XT, 8><<<grid, 256, 0, st>>>(x, gate, (int)T, (int)H, E, k, topk_e, topk_w);
  else if (E <= 16)
    k_moe_router<XT, 16><<<grid, 256, 0, st>>>(x, gate, (int)T, (int)H, E, k, topk_e, topk_w);
  else
    k_moe_router<XT, kMaxExperts><<<grid, 256, 0, st>>>(x, gate, (int)T, (int)H, E, k, topk_e, topk_w);
}

// router + stable sort: topk_e/topk_w/pair_pos/sorted_tok/cnt/off in the workspace
int route_and_sort(const void* d_x, int x_dtype, int64_t T, int64_t H, const float* d_gate, int E, int k,
                   const MoeWs& w, cudaStream_t st) {
  const int64_t P = T * k;
  if (x_dtype == XM_DT_F32)
    launch_router<float>((const float*)d_x, d_gate, T, H, E, k, w.topk_e, w.topk_w, st);
  else if (x_dtype == XM_DT_BF16)
    launch_router<__nv_bfloat16>((const __nv_bfloat16*)d_x, d_gate, T, H, E, k, w.topk_e, w.topk_w, st);
  else
    launch_router<__half>((const __half*)d_x, d_gate, T, H, E, k, w.topk_e, w.topk_w, st);
  int rc = xm_check_launch("moe router");
  if (rc) return rc;
  k_moe_sort<<<1, 1024, 0, st>>>(w.topk_e, w.topk_w, (int)P, k, E, w.sorted_tok, w.sorted_w, w.pair_pos, w.cnt, w.off);
  return xm_check_launch("moe sort");
}

// prepared fp16 rows a16 (P x H, already in expert order) -> d (P x H): the
// SwiGLU experts of G groups (rows [off[g], off[g] + cnt[g]) use weights tab[g],
// tab[G + g], tab[2G + g] for w1, w3, w2)
int run_experts(int qtype, int act, const __half* a16, const float* ascale, int64_t P, int64_t H, int64_t F,
                const uint8_t* const* tab, int G, const int* cnt, const int* off, int64_t max_rows, float* g,
                float* u, __half* h16, float* hscale, float* d, cudaStream_t st) {
  const int64_t expect = std::max<int64_t>(1, P / G);
  int rc;
  // w1 and w3 in one pass with act(gate) * up in the epilogue (g holds the
  // product), then one read of it for the fp16 conversion
  const int64_t rows_smem = F * (int64_t)sizeof(float);
  if (rows_smem <= 200 * 1024) {
    rc = qgemm_grouped_gate_up(qtype, act, a16, ascale, P, H, F, tab, tab + G, cnt, off, G, max_rows, expect, g, st);
    if (rc != 1) {
      if (rc) return rc;
      static bool attr_done[64] = {};
      int dev = 0;
      cudaGetDevice(&dev);
      if (rows_smem > 48 * 1024 && (dev < 0 || dev >= 64 || !attr_done[dev])) {
        cudaError_t e = cudaFuncSetAttribute(k_rows_fp16, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "moe: smem attribute: %s", cudaGetErrorString(e));
        if (dev >= 0 && dev < 64) attr_done[dev] = true;
      }
      k_rows_fp16<<<(unsigned)P, kPrepThreads, (size_t)rows_smem, st>>>(g, (int)F, h16, hscale);
      if ((rc = xm_check_launch("moe rows fp16"))) return rc;
      return qgemm_grouped(qtype, h16, hscale, P, F, H, tab + 2 * G, cnt, off, G, max_rows, expect, d, st);
    }
  }
  if ((rc = qgemm_grouped(qtype, a16, ascale, P, H, F, tab, cnt, off, G, max_rows, expect, g, st))) return rc;
  if ((rc = qgemm_grouped(qtype, a16, ascale, P, H, F, tab + G, cnt, off, G, max_rows, expect, u, st))) return rc;
  const unsigned pgrid = (unsigned)P;     // one block per row
  if (act == XM_ACT_SILU)
    k_swiglu_prep<XM_ACT_SILU><<<pgrid, kPrepThreads, 0, st>>>(g, u, (int)P, (int)F, h16, hscale);
  else if (act == XM_ACT_GELU)
    k_swiglu_prep<XM_ACT_GELU><<<pgrid, kPrepThreads, 0, st>>>(g, u, (int)P, (int)F, h16, hscale);
  else if (act == XM_ACT_RELU)
    k_swiglu_prep<XM_ACT_RELU><<<pgrid, kPrepThreads, 0, st>>>(g, u, (int)P, (int)F, h16, hscale);
  else
    k_swiglu_prep<XM_ACT_IDENTITY><<<pgrid, kPrepThreads, 0, st>>>(g, u, (int)P, (int)F, h16, hscale);
  if ((rc = xm_check_launch("moe swiglu"))) return rc;
  return qgemm_grouped(qtype, h16, hscale, P, F, H, tab + 2 * G, cnt, off, G, max_rows, expect, d, st);
}

// Expert weights of this type and shape have a tensor-core path, and the
// activation is one the reference knows.
int check_expert_type(const char* who, int qtype, int act, int64_t H, int64_t F) {
  if (act != XM_ACT_SILU && act != XM_ACT_GELU && act != XM_ACT_RELU && act != XM_ACT_IDENTITY)
    return xm_set_error(XM_ERR_INVALID, "%s: unknown activation %d", who, act);
  if (!qgemm_type_supported(qtype, H) || !qgemm_type_supported(qtype, F))
    return xm_set_error(XM_ERR_UNSUPPORTED,
                        "%s: expert type id %d with hidden %lld / intermediate %lld has no tensor-core path (block "
                        "type with rows of whole 16-byte units needed)",
                        who, qtype, (long long)H, (long long)F);
  return XM_OK;
}

struct ExpertWs {
  __half *a16, *h16;
  float *ascale, *hscale, *g, *u;
  int64_t bytes;
};

ExpertWs carve_experts(uint8_t* base, int64_t P, int64_t H, int64_t F) {
  ExpertWs w{};
  int64_t o = 0;
  auto take = [&](int64_t bytes) { uint8_t* p = base ? base + o : nullptr; o += align256(bytes); return p; };
  w.a16 = (__half*)take(P * H * 2);
  w.ascale = (float*)take(P * 4);
  w.g = (float*)take(P * F * 4);
  w.u = (float*)take(P * F * 4);
  w.h16 = (__half*)take(P * F * 2);
  w.hscale = (float*)take(P * 4);
  w.bytes = o;
  return w;
}

}  // namespace

extern "C" int xm_moe_forward(const void* d_x, int x_dtype, int64_t T, int64_t H, const float* d_gate, int E, int k,
                              int64_t F, const void* const* h_w1, const void* const* h_w3, const void* const* h_w2,
                              int qtype, int activation, float* d_out, void* d_ws, int64_t ws_bytes, void* stream) {
  if (int rc0 = check_common(E, k, T, H, x_dtype)) return rc0;
  if (F < 256 || F % 256)
    return xm_set_error(XM_ERR_INVALID, "moe: hidden and intermediate sizes must be positive multiples of 256");
  if (int rc0 = check_expert_type("moe", qtype, activation, H, F)) return rc0;
  if (!d_x || !d_gate || !d_out || !d_ws || !h_w1 || !h_w2 || !h_w3)
    return xm_set_error(XM_ERR_INVALID, "moe: null pointer");
  if (((uintptr_t)d_x | (uintptr_t)d_gate | (uintptr_t)d_out) & 15)
    return xm_set_error(XM_ERR_INVALID, "moe: x, gate and out must be 16-byte aligned");
  if (((uintptr_t)d_ws & 255) || ws_bytes < xm_moe_workspace_size(T, H, F, E, k))
    return xm_set_error(XM_ERR_INVALID, "moe: workspace too small or not 256-byte aligned");
  for (int e = 0; e < E; ++e)
    if (!h_w1[e] || !h_w2[e] || !h_w3[e] || ((uintptr_t)h_w1[e] & 15) || ((uintptr_t)h_w2[e] & 15) ||
        ((uintptr_t)h_w3[e] & 15))
      return xm_set_error(XM_ERR_INVALID, "moe: expert %d weight pointer null or not 16-byte aligned", e);
  cudaStream_t st = (cudaStream_t)stream;
  MoeWs w = carve((uint8_t*)d_ws, T, H, F, E, k);
  const int64_t P = T * k;

  // expert weight pointers (host array of device pointers, passed to the kernels by value)
  const uint8_t* tab[3 * kMaxExperts];
  for (int e = 0; e < E; ++e) {
    tab[e] = (const uint8_t*)h_w1[e];
    tab[E + e] = (const uint8_t*)h_w3[e];
    tab[2 * E + e] = (const uint8_t*)h_w2[e];
  }
  int rc = route_and_sort(d_x, x_dtype, T, H, d_gate, E, k, w, st);
  if (rc) return rc;
  const unsigned pgrid = (unsigned)P;     // one block per row
  if (x_dtype == XM_DT_F32)
    k_moe_gather_prep<float><<<pgrid, kPrepThreads, 0, st>>>((const float*)d_x, w.sorted_tok, (int)P, (int)H, w.a16, w.ascale);
  else if (x_dtype == XM_DT_BF16)
    k_moe_gather_prep<__nv_bfloat16><<<pgrid, kPrepThreads, 0, st>>>((const __nv_bfloat16*)d_x, w.sorted_tok, (int)P, (int)H,
                                                              w.a16, w.ascale);
  else
    k_moe_gather_prep<__half><<<pgrid, kPrepThreads, 0, st>>>((const __half*)d_x, w.sorted_tok, (int)P, (int)H, w.a16, w.ascale);
  if ((rc = xm_check_launch("moe gather"))) return rc;
  if ((rc = run_experts(qtype, activation, w.a16, w.ascale, P, H, F, tab, E, w.cnt, w.off, T, w.g, w.u, w.h16, w.hscale, w.d,
                       st)))
    return rc;
  k_moe_combine<<<(unsigned)T, 256, 0, st>>>(w.d, w.topk_e, w.topk_w, w.pair_pos, (int)T, (int)H, k, d_out);
  return xm_check_launch("moe combine");
}

// ---------------------------------------------------------------------------
// Expert parallelism: the block split at its two exchange points.
// ---------------------------------------------------------------------------
extern "C" int xm_moe_dispatch(const void* d_x, int x_dtype, int64_t T, int64_t H, const float* d_gate, int E, int k,
                               int64_t F, void* d_send, int* d_cnt, void* d_ws, int64_t ws_bytes, void* stream) {
  if (int rc = check_common(E, k, T, H, x_dtype)) return rc;
  if (!d_x || !d_gate || !d_send || !d_cnt || !d_ws) return xm_set_error(XM_ERR_INVALID, "moe_dispatch: null pointer");
  if (((uintptr_t)d_x | (uintptr_t)d_gate) & 15)
    return xm_set_error(XM_ERR_INVALID, "moe_dispatch: x and gate must be 16-byte aligned");
  if (((uintptr_t)d_ws & 255) || ws_bytes < xm_moe_workspace_size(T, H, F, E, k))
    return xm_set_error(XM_ERR_INVALID, "moe_dispatch: workspace too small or not 256-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  MoeWs w = carve((uint8_t*)d_ws, T, H, F, E, k);
  int rc = route_and_sort(d_x, x_dtype, T, H, d_gate, E, k, w, st);
  if (rc) return rc;
  const int64_t P = T * k;
  const dim3 grid((unsigned)std::min<int64_t>((H + 255) / 256, 8), (unsigned)P);
  if (x_dtype == XM_DT_F32)
    k_moe_gather<float><<<grid, 256, 0, st>>>((const float*)d_x, w.sorted_tok, (int)P, (int)H, (float*)d_send);
  else if (x_dtype == XM_DT_BF16)
    k_moe_gather<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)d_x, w.sorted_tok, (int)P, (int)H,
                                                       (__nv_bfloat16*)d_send);
  else
    k_moe_gather<__half><<<grid, 256, 0, st>>>((const __half*)d_x, w.sorted_tok, (int)P, (int)H, (__half*)d_send);
  if ((rc = xm_check_launch("moe gather"))) return rc;
  cudaError_t e = cudaMemcpyAsync(d_cnt, w.cnt, E * sizeof(int), cudaMemcpyDeviceToDevice, st);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "moe_dispatch: %s", cudaGetErrorString(e));
  return XM_OK;
}

extern "C" int64_t xm_moe_experts_workspace_size(int64_t P, int64_t H, int64_t F) {
  if (P < 1 || H < 1 || F < 1) return 0;
  return carve_experts(nullptr, P, H, F).bytes;
}

extern "C" int xm_moe_experts(const void* d_rows, int x_dtype, int64_t P, int64_t H, int64_t F, int G, const int* d_cnt,
                              const int* d_off, const void* const* h_w1, const void* const* h_w3,
                              const void* const* h_w2, int qtype, int activation, int64_t max_rows, float* d_out,
                              void* d_ws,
                              int64_t ws_bytes, void* stream) {
  if (G < 1 || G > kMaxExperts) return xm_set_error(XM_ERR_INVALID, "moe_experts: %d groups (1..%d)", G, kMaxExperts);
  if (P < 0 || H < 256 || H % 256 || F < 256 || F % 256 || max_rows < 0)
    return xm_set_error(XM_ERR_INVALID, "moe_experts: bad sizes");
  if (int rc0 = check_expert_type("moe_experts", qtype, activation, H, F)) return rc0;
  if (x_dtype != XM_DT_F32 && x_dtype != XM_DT_BF16 && x_dtype != XM_DT_F16)
    return xm_set_error(XM_ERR_INVALID, "moe_experts: bad x dtype %d", x_dtype);
  if (P == 0) return XM_OK;
  if (!d_rows || !d_cnt || !d_off || !d_out || !d_ws || !h_w1 || !h_w2 || !h_w3)
    return xm_set_error(XM_ERR_INVALID, "moe_experts: null pointer");
  if (((uintptr_t)d_rows | (uintptr_t)d_out) & 15)
    return xm_set_error(XM_ERR_INVALID, "moe_experts: rows and out must be 16-byte aligned");
  if (((uintptr_t)d_ws & 255) || ws_bytes < xm_moe_experts_workspace_size(P, H, F))
    return xm_set_error(XM_ERR_INVALID, "moe_experts: workspace too small or not 256-byte aligned");
  const uint8_t* tab[3 * kMaxExperts];
  for (int g = 0; g < G; ++g) {
    if (!h_w1[g] || !h_w2[g] || !h_w3[g] || ((uintptr_t)h_w1[g] & 15) || ((uintptr_t)h_w2[g] & 15) ||
        ((uintptr_t)h_w3[g] & 15))
      return xm_set_error(XM_ERR_INVALID, "moe_experts: group %d weight pointer null or not 16-byte aligned", g);
    tab[g] = (const uint8_t*)h_w1[g];
    tab[G + g] = (const uint8_t*)h_w3[g];
    tab[2 * G + g] = (const uint8_t*)h_w2[g];
  }
  cudaStream_t st = (cudaStream_t)stream;
  ExpertWs w = carve_experts((uint8_t*)d_ws, P, H, F);
  const unsigned pgrid = (unsigned)P;     // one block per row
  if (x_dtype == XM_DT_F32)
    k_moe_gather_prep<float><<<pgrid, kPrepThreads, 0, st>>>((const float*)d_rows, nullptr, (int)P, (int)H, w.a16, w.ascale);
  else if (x_dtype == XM_DT_BF16)
    k_moe_gather_prep<__nv_bfloat16><<<pgrid, kPrepThreads, 0, st>>>((const __nv_bfloat16*)d_rows, nullptr, (int)P, (int)H,
                                                              w.a16, w.ascale);
  else
    k_moe_gather_prep<__half><<<pgrid, kPrepThreads, 0, st>>>((const __half*)d_rows, nullptr, (int)P, (int)H, w.a16, w.ascale);
  int rc = xm_check_launch("moe_experts prep");
  if (rc) return rc;
  return run_experts(qtype, activation, w.a16, w.ascale, P, H, F, tab, G, d_cnt, d_off, std::max<int64_t>(1, max_rows), w.g, w.u,
                     w.h16, w.hscale, d_out, st);
}

extern "C" int xm_moe_combine(const float* d_rows, int64_t T, int64_t H, int E, int k, int64_t F, const void* d_ws,
                              float* d_out, void* stream) {
  if (int rc = check_common(E, k, T, H, XM_DT_F32)) return rc;
  if (!d_rows || !d_ws || !d_out) return xm_set_error(XM_ERR_INVALID, "moe_combine: null pointer");
  if (((uintptr_t)d_rows | (uintptr_t)d_out) & 15)
    return xm_set_error(XM_ERR_INVALID, "moe_combine: rows and out must be 16-byte aligned");
  MoeWs w = carve((uint8_t*)d_ws, T, H, F, E, k);
  k_moe_combine<<<(unsigned)T, 256, 0, (cudaStream_t)stream>>>(d_rows, w.topk_e, w.topk_w, w.pair_pos, (int)T, (int)H, k,
                                                          d_out);
  return xm_check_launch("moe combine");
}
