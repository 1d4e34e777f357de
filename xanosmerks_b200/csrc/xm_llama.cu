// Kernels around the quantized projections of a Llama-style decoder step:
// embedding gather from GGUF blocks, rotary embedding fused with the KV-cache
// append, grouped-query attention over the cache (split along the keys, the
// partial softmaxes merged by the last CTA of each head group), and greedy
// argmax.  RMSNorm, SwiGLU and the residual adds are fused into the GEMVs
// (xm_qgemv_ex).  These kernels move a few MB per step against the ~4.5 GB of
// weight blocks the projections stream, so they are written for latency
// (programmatic dependent launch, one wave) rather than bandwidth.
//
// Semantics: TransformerLayer.__call__ (forward.py:105-116) and
// TransformerModel._forward (forward.py:150-159); attention is causal
// scaled-dot-product with GQA sharing of KV heads (attention.py:59-115,
// :149-166), rotate-half rotary embedding (attention.py:66-70).
#include "xm_gemv_dot.cuh"

namespace {

constexpr int kHeadDim = 128;
constexpr int kAttnKeys = 64;    // keys per attention CTA
constexpr int kMaxGroup = 8;     // query heads per KV head
constexpr int kMaxLq = 8;        // new tokens per sequence in one call

// ---------------------------------------------------------------------------
// out[b][:] = fp16-rounded dequantized row ids[b] of a GGUF table (the
// reference dequantizes the table to fp16 and indexes it, forward.py:151).
// ---------------------------------------------------------------------------
template <int T>
__global__ void __launch_bounds__(256) k_embed(const uint8_t* __restrict__ table, int64_t row_bytes,
                                               const int* __restrict__ ids, int D, float* __restrict__ out) {
  using Q = QT<T>;
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.y;
  const int e0 = (blockIdx.x * 256 + threadIdx.x) * 8;
  if (e0 >= D) return;
  const uint8_t* row = table + (int64_t)ids[b] * row_bytes;
  float v[8];
  Q::decode8(row + (e0 / Q::QK) * Q::REC, e0 % Q::QK, v);
  float* o = out + (int64_t)b * D + e0;
#pragma unroll
  for (int t = 0; t < 8; ++t) o[t] = __half2float(__float2half_rn(v[t]));
}

struct EmbedLaunch {
  const uint8_t* table; int64_t row_bytes; const int* ids; int B, D; float* out; cudaStream_t st; cudaError_t err;
  template <int T>
  void operator()() {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((D / 8 + 255) / 256), (unsigned)B);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    err = cudaLaunchKernelEx(&cfg, k_embed<T>, table, row_bytes, ids, D, out);
  }
};

// ---------------------------------------------------------------------------
// Rotary embedding + KV append.  qkv row t = [q (Hq x 128) | k (Hk x 128) |
// v (Hk x 128)], fp32, token t of sequence seq[t] at position pos[t].  q and k
// are rotated in place (out[i] = x[i] cos - x[i+64] sin, out[i+64] = x[i+64]
// cos + x[i] sin, angle pos / theta^(2i/128)); k and v go to the fp16 caches
// [B][Hk][max_ctx][128] at that position.  Grid (T, Hq + 2 Hk), 64 threads.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(64) k_rope_append(float* __restrict__ qkv, int64_t qkv_stride,
                                                    const int* __restrict__ seq, const int* __restrict__ pos, int Hq,
                                                    int Hk, float theta, int max_ctx, __half* __restrict__ kc,
                                                    __half* __restrict__ vc) {
  grid_dep_wait();
  grid_dep_launch();
  const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  float* row = qkv + (int64_t)t * qkv_stride;
  const int p = pos[t];
  float* v = row + (int64_t)h * kHeadDim;
  float a = v[i], b = v[i + 64];
  if (h < Hq + Hk) {
    const float inv_freq = 1.0f / powf(theta, (float)(2 * i) / (float)kHeadDim);
    float sn, cs;
    sincosf((float)p * inv_freq, &sn, &cs);
    const float ra = a * cs - b * sn, rb = b * cs + a * sn;
    a = ra;
    b = rb;
    if (h < Hq) {
      v[i] = a;
      v[i + 64] = b;
      return;
    }
  }
  const int hk = h < Hq + Hk ? h - Hq : h - Hq - Hk;
  __half* cache = h < Hq + Hk ? kc : vc;
  const int64_t dst = (((int64_t)seq[t] * Hk + hk) * max_ctx + p) * kHeadDim;
  cache[dst + i] = __float2half_rn(a);
  cache[dst + i + 64] = __float2half_rn(b);
}

// ---------------------------------------------------------------------------
// Attention for Lq new tokens of each of B sequences.  CTA (b, hk, s) covers
// keys [64 s, 64 s + 64) of KV head hk of sequence b for all G = Hq/Hk query
// heads and all Lq tokens (token j sees keys 0 .. pos0[b] + j).  It writes
// its partial (max, sum, unnormalised output) per (j, g) to the workspace;
// the last CTA of (b, hk) to finish merges the partials in split order and
// writes out[b*Lq + j][hq][128].
// ---------------------------------------------------------------------------
struct AttnPart {
  float m, l;
};

__global__ void __launch_bounds__(256) k_attention(const float* __restrict__ qkv, int64_t qkv_stride,
                                                   const __half* __restrict__ kc, const __half* __restrict__ vc,
                                                   const int* __restrict__ pos0, int Lq, int Hq, int Hk, int max_ctx,
                                                   int nsplit, float* __restrict__ part_o,
                                                   AttnPart* __restrict__ part_ml, int* __restrict__ tickets,
                                                   float* __restrict__ out, int64_t out_stride) {
  __shared__ __align__(16) __half ks[kAttnKeys][kHeadDim + 8];
  __shared__ __align__(16) __half vs[kAttnKeys][kHeadDim + 8];
  __shared__ __align__(16) float qs[kMaxGroup][kHeadDim];
  __shared__ float sc[kMaxGroup][kAttnKeys];
  __shared__ int last;
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x / Hk, hk = blockIdx.x % Hk, s = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = Hq / Hk;
  const int p0 = pos0[b];
  const int k0 = s * kAttnKeys;
  const int kend = min(k0 + kAttnKeys, p0 + Lq);   // keys this CTA may need for its last token
  const float scale = rsqrtf((float)kHeadDim);
  const int64_t bh = (int64_t)b * Hk + hk;

  if (k0 < kend) {
    // stage the key and value tile (16-byte loads)
    const __half* K = kc + (bh * max_ctx + k0) * kHeadDim;
    const __half* V = vc + (bh * max_ctx + k0) * kHeadDim;
    const int nk = kend - k0;
    for (int i = tid; i < nk * (kHeadDim / 8); i += 256) {
      const int r = i / (kHeadDim / 8), c = (i % (kHeadDim / 8)) * 8;
      *reinterpret_cast<uint4*>(&ks[r][c]) = *reinterpret_cast<const uint4*>(K + (int64_t)r * kHeadDim + c);
      *reinterpret_cast<uint4*>(&vs[r][c]) = *reinterpret_cast<const uint4*>(V + (int64_t)r * kHeadDim + c);
    }
    for (int j = 0; j < Lq; ++j) {
      const int len = p0 + j + 1;                    // token j sees keys < len
      const int nkj = min(kend, len) - k0;           // keys of this tile it sees (may be <= 0)
      __syncthreads();                               // tiles staged / previous token done with qs, sc
      for (int i = tid; i < G * kHeadDim; i += 256) {
        const int g = i / kHeadDim, d = i % kHeadDim;
        qs[g][d] = qkv[((int64_t)b * Lq + j) * qkv_stride + (int64_t)(hk * G + g) * kHeadDim + d];
      }
      __syncthreads();
      // scores: warp w takes keys w*8 .. w*8+7; lanes over dims (4 each)
      for (int kk = 0; kk < 8; ++kk) {
        const int key = warp * 8 + kk;
        if (key >= nkj) break;
        const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&ks[key][4 * lane]));
        const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&ks[key][4 * lane + 2]));
        for (int g = 0; g < G; ++g) {
          const float4 q4 = *reinterpret_cast<const float4*>(&qs[g][4 * lane]);
          float d = q4.x * k01.x + q4.y * k01.y + q4.z * k23.x + q4.w * k23.y;
          d = warp_sum(d);
          if (lane == 0) sc[g][key] = d * scale;
        }
      }
      __syncthreads();
      // per head: max and exp over the tile (warp g handles head g; G <= 8)
      if (warp < G && nkj > 0) {
        const int g = warp;
        float mx = -INFINITY;
        for (int key = lane; key < nkj; key += 32) mx = fmaxf(mx, sc[g][key]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float sum = 0.f;
        for (int key = lane; key < nkj; key += 32) {
          const float e = expf(sc[g][key] - mx);
          sc[g][key] = e;
          sum += e;
        }
        sum = warp_sum(sum);
        if (lane == 0) {
          AttnPart pm;
          pm.m = mx;
          pm.l = sum;
          part_ml[((bh * nsplit + s) * kMaxLq + j) * kMaxGroup + g] = pm;
        }
      }
      __syncthreads();
      // unnormalised output: thread (g, 4 dims)
      if (nkj > 0) {
        for (int i = tid; i < G * (kHeadDim / 4); i += 256) {
          const int g = i / (kHeadDim / 4), d = (i % (kHeadDim / 4)) * 4;
          float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
          for (int key = 0; key < nkj; ++key) {
            const float pk = sc[g][key];
            const float2 v01 = __half22float2(*reinterpret_cast<const __half2*>(&vs[key][d]));
            const float2 v23 = __half22float2(*reinterpret_cast<const __half2*>(&vs[key][d + 2]));
            o0 = fmaf(pk, v01.x, o0);
            o1 = fmaf(pk, v01.y, o1);
            o2 = fmaf(pk, v23.x, o2);
            o3 = fmaf(pk, v23.y, o3);
          }
          *reinterpret_cast<float4*>(part_o + (((bh * nsplit + s) * kMaxLq + j) * kMaxGroup + g) * kHeadDim + d) =
              make_float4(o0, o1, o2, o3);
        }
      }
    }
  }
  // the last CTA of (b, hk) merges
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&tickets[bh], 1) == nsplit - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int i = tid; i < Lq * G * (kHeadDim / 4); i += 256) {
    const int j = i / (G * (kHeadDim / 4));
    const int rem = i % (G * (kHeadDim / 4));
    const int g = rem / (kHeadDim / 4), d = (rem % (kHeadDim / 4)) * 4;
    const int len = p0 + j + 1;
    const int ns = min(nsplit, (len + kAttnKeys - 1) / kAttnKeys);
    const float* mls = reinterpret_cast<const float*>(part_ml);
    float M = -INFINITY;
    for (int ss = 0; ss < ns; ++ss) M = fmaxf(M, __ldcg(&mls[2 * (((bh * nsplit + ss) * kMaxLq + j) * kMaxGroup + g)]));
    float L = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int ss = 0; ss < ns; ++ss) {
      const int64_t cell = ((bh * nsplit + ss) * kMaxLq + j) * kMaxGroup + g;
      const float w = expf(__ldcg(&mls[2 * cell]) - M);
      L = fmaf(__ldcg(&mls[2 * cell + 1]), w, L);
      const float4 o = __ldcg(reinterpret_cast<const float4*>(part_o + cell * kHeadDim + d));
      acc.x = fmaf(o.x, w, acc.x);
      acc.y = fmaf(o.y, w, acc.y);
      acc.z = fmaf(o.z, w, acc.z);
      acc.w = fmaf(o.w, w, acc.w);
    }
    const float inv = 1.0f / L;
    *reinterpret_cast<float4*>(out + ((int64_t)b * Lq + j) * out_stride + (int64_t)(hk * G + g) * kHeadDim + d) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
  if (tid == 0) tickets[bh] = 0;   // ready for the next call
}

// first index of the maximum of each row (np.argmax semantics; NaN-free input)
__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ logits, int V, int* __restrict__ out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x;
  const float* r = logits + (int64_t)b * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    const float v = r[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x + 31) / 32; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < idx)) {
        best = bv[w];
        idx = bi[w];
      }
    out[b] = idx == 0x7fffffff ? 0 : idx;
  }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

int launch_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return xm_check_launch(what);
}

}  // namespace

extern "C" {

int xm_embed(int qtype, const void* d_table, int64_t table_bytes, int64_t vocab, int64_t D, const int* d_ids,
             int64_t B, float* d_out, void* stream) {
  int qk = 0, rec = 0;
  if (!host_qtype_geometry(qtype, &qk, &rec) || qk == 1)
    return xm_set_error(XM_ERR_UNSUPPORTED, "embed: type id %d is not a block-quantized type", qtype);
  if (B < 1 || D < 8 || D % 8 || D % qk || vocab < 1 || !d_table || !d_ids || !d_out)
    return xm_set_error(XM_ERR_INVALID, "embed: bad arguments");
  const int64_t row_bytes = D / qk * rec;
  if (row_bytes * vocab > table_bytes) return xm_set_error(XM_ERR_INVALID, "embed: table too small");
  EmbedLaunch l{(const uint8_t*)d_table, row_bytes, d_ids, (int)B, (int)D, d_out, (cudaStream_t)stream, cudaSuccess};
  dispatch_quant(qtype, l);
  return launch_status(l.err, "embed");
}

int xm_rope_append(float* d_qkv, int64_t qkv_stride, const int* d_seq, const int* d_pos, int64_t T, int Hq, int Hk,
                   int head_dim, float theta, int64_t max_ctx, void* d_kcache, void* d_vcache, void* stream) {
  if (head_dim != kHeadDim) return xm_set_error(XM_ERR_UNSUPPORTED, "rope_append: head_dim %d (only 128)", head_dim);
  if (T < 1 || Hq < 1 || Hk < 1 || qkv_stride < (int64_t)(Hq + 2 * Hk) * kHeadDim || max_ctx < 1 ||
      max_ctx > (1 << 24) || !d_qkv || !d_seq || !d_pos || !d_kcache || !d_vcache)
    return xm_set_error(XM_ERR_INVALID, "rope_append: bad arguments");
  return launch_status(launch_pdl(k_rope_append, dim3((unsigned)T, (unsigned)(Hq + 2 * Hk)), dim3(64),
                                  (cudaStream_t)stream, d_qkv, qkv_stride, d_seq, d_pos, Hq, Hk, theta, (int)max_ctx,
                                  (__half*)d_kcache, (__half*)d_vcache),
                       "rope_append");
}

int64_t xm_attention_workspace_size(int64_t B, int Hk, int64_t max_ctx) {
  const int64_t nsplit = (max_ctx + kAttnKeys - 1) / kAttnKeys;
  const int64_t cells = B * Hk * nsplit * kMaxLq * kMaxGroup;
  return cells * kHeadDim * 4 + cells * (int64_t)sizeof(AttnPart) + B * Hk * 4 + 256;
}

int xm_attention(const float* d_qkv, int64_t qkv_stride, const void* d_kcache, const void* d_vcache,
                 const int* d_pos0, int64_t B, int Lq, int Hq, int Hk, int head_dim, int64_t max_ctx, float* d_out,
                 int64_t out_stride, void* d_workspace, int64_t workspace_bytes, void* stream) {
  if (head_dim != kHeadDim) return xm_set_error(XM_ERR_UNSUPPORTED, "attention: head_dim %d (only 128)", head_dim);
  if (B < 1 || Lq < 1 || Lq > kMaxLq || Hq < 1 || Hk < 1 || Hq % Hk || Hq / Hk > kMaxGroup)
    return xm_set_error(XM_ERR_INVALID, "attention: bad head counts (G <= 8) or more than 8 new tokens");
  if (max_ctx < 1 || out_stride < (int64_t)Hq * kHeadDim || !d_qkv || !d_kcache || !d_vcache || !d_pos0 || !d_out)
    return xm_set_error(XM_ERR_INVALID, "attention: bad arguments");
  if (!d_workspace || workspace_bytes < xm_attention_workspace_size(B, Hk, max_ctx) || ((uintptr_t)d_workspace & 15))
    return xm_set_error(XM_ERR_INVALID, "attention: workspace too small or unaligned");
  const int nsplit = (int)((max_ctx + kAttnKeys - 1) / kAttnKeys);
  const int64_t cells = B * Hk * nsplit * kMaxLq * kMaxGroup;
  float* part_o = (float*)d_workspace;
  AttnPart* part_ml = (AttnPart*)(part_o + cells * kHeadDim);
  int* tickets = (int*)(part_ml + cells);
  // tickets start at zero (the caller zeroes the workspace once) and every call leaves them at zero
  return launch_status(launch_pdl(k_attention, dim3((unsigned)(B * Hk), (unsigned)nsplit), dim3(256),
                                  (cudaStream_t)stream, d_qkv, qkv_stride, (const __half*)d_kcache,
                                  (const __half*)d_vcache, d_pos0, Lq, Hq, Hk, (int)max_ctx, nsplit, part_o, part_ml,
                                  tickets, d_out, out_stride),
                       "attention");
}

int xm_argmax(const float* d_logits, int64_t B, int64_t V, int* d_out, void* stream) {
  if (B < 1 || V < 1 || !d_logits || !d_out) return xm_set_error(XM_ERR_INVALID, "argmax: bad arguments");
  return launch_status(launch_pdl(k_argmax, dim3((unsigned)B), dim3(1024), (cudaStream_t)stream, d_logits, (int)V,
                                  d_out),
                       "argmax");
}

}  // extern "C"
