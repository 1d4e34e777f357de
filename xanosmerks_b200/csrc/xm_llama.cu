// Kernels around the quantized projections of a Llama-style decoder step:
// embedding gather from GGUF blocks, grouped-query attention over the KV
// cache with the rotary embedding and the cache append fused in (split along
// the keys, the partial softmaxes merged by the last CTA of each head group),
// and greedy argmax.  RMSNorm, SwiGLU and the residual adds are fused into the GEMVs
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
constexpr int kMaxLq = 64;       // new tokens per sequence in one call (a prefill chunk)
constexpr int kAttnTokensPerCta = 4;   // new tokens a CTA takes in turn (more tokens: more CTAs)

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
// Attention for Lq new tokens of each of B sequences, with the rotary
// embedding and the KV-cache append fused in.
//
// qkv row b*Lq + j = [q (Hq x 128) | k (Hk x 128) | v (Hk x 128)] of token j
// of sequence b, at position pos0[b] + j, as the QKV projection wrote it (not
// yet rotated).  Rotary embedding (rotate-half): out[i] = x[i] cos - x[i+64]
// sin, out[i+64] = x[i+64] cos + x[i] sin, angle = pos / theta^(2i/128).
//
// CTA (b, hk, s) covers keys [64 s, 64 s + 64) of KV head hk of sequence b,
// for the G = Hq/Hk query heads of that KV head and every new token (token j
// sees keys 0 .. pos0[b] + j).  Keys already in the cache come from it; the
// new tokens' keys and values that fall in the CTA's range are rotated,
// written to the cache and used from shared memory.  Each CTA rotates the
// query rows itself, writes its partial (max, sum, unnormalised output) per
// (token, head) to the workspace, and the last CTA of (b, hk) to finish merges
// the partials in split order into out[b*Lq + j][hq][128].  With many new
// tokens (a prefill chunk) the tokens are dealt over gridDim.z groups of CTAs
// (token j to group j % Z), each group with the same key tiles; group 0
// appends the new keys and values to the cache.
// ---------------------------------------------------------------------------
struct AttnPart {
  float m, l;
};

constexpr int kKvPitch = kHeadDim / 2 + 1;   // half2 words per cached row in shared memory (conflict-free)

XM_DEV void rope_pair(float& a, float& b, int pos, int i, float theta) {
  const float inv_freq = 1.0f / powf(theta, (float)(2 * i) / (float)kHeadDim);
  float sn, cs;
  sincosf((float)pos * inv_freq, &sn, &cs);
  const float ra = a * cs - b * sn, rb = b * cs + a * sn;
  a = ra;
  b = rb;
}

__global__ void __launch_bounds__(256) k_attention(const float* __restrict__ qkv, int64_t qkv_stride,
                                                   __half* __restrict__ kc, __half* __restrict__ vc,
                                                   const int* __restrict__ pos0, int Lq, int Hq, int Hk, int max_ctx,
                                                   int nsplit, float theta, float* __restrict__ part_o,
                                                   AttnPart* __restrict__ part_ml, int* __restrict__ tickets,
                                                   float* __restrict__ out, int64_t out_stride) {
  __shared__ __half2 ks[kAttnKeys][kKvPitch];
  __shared__ __half2 vs[kAttnKeys][kKvPitch];
  __shared__ __align__(16) float qs[kMaxGroup][kHeadDim];
  __shared__ float sc[kMaxGroup][kAttnKeys];
  __shared__ int last;
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x / Hk, hk = blockIdx.x % Hk, s = blockIdx.y;
  const int z = blockIdx.z, Z = gridDim.z;       // this CTA's tokens: j = z, z + Z, ...
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int G = Hq / Hk;
  const int p0 = pos0[b];
  const int k0 = s * kAttnKeys;
  const int kend = min(k0 + kAttnKeys, p0 + Lq);   // keys this CTA may need for its last token
  const float scale = rsqrtf((float)kHeadDim);
  const int64_t bh = (int64_t)b * Hk + hk;
  __half* K = kc + bh * max_ctx * kHeadDim;
  __half* V = vc + bh * max_ctx * kHeadDim;
  const int kv_off = Hq * kHeadDim;                // k heads follow the q heads in a qkv row

  if (k0 < kend) {
    const int nk = kend - k0;
    // old keys (positions < p0) from the cache, 16-byte loads
    const int nold = max(0, min(nk, p0 - k0));
    for (int i = tid; i < nold * (kHeadDim / 8); i += 256) {
      const int r = i / (kHeadDim / 8), c = (i % (kHeadDim / 8)) * 8;
      const uint4 kv = *reinterpret_cast<const uint4*>(K + (int64_t)(k0 + r) * kHeadDim + c);
      const uint4 vv = *reinterpret_cast<const uint4*>(V + (int64_t)(k0 + r) * kHeadDim + c);
      const __half2* k2 = reinterpret_cast<const __half2*>(&kv);
      const __half2* v2 = reinterpret_cast<const __half2*>(&vv);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        ks[r][c / 2 + e] = k2[e];
        vs[r][c / 2 + e] = v2[e];
      }
    }
    // new keys in range: rotate, append to the cache, keep in shared memory
    for (int i = tid; i < (nk - nold) * (kHeadDim / 2); i += 256) {
      const int r = nold + i / (kHeadDim / 2), d = i % (kHeadDim / 2);
      const int pos = k0 + r, j = pos - p0;
      const float* row = qkv + ((int64_t)b * Lq + j) * qkv_stride + kv_off;
      float ka = row[hk * kHeadDim + d], kb = row[hk * kHeadDim + d + 64];
      rope_pair(ka, kb, pos, d, theta);
      const float va = row[(Hk + hk) * kHeadDim + d], vb = row[(Hk + hk) * kHeadDim + d + 64];
      const __half hka = __float2half_rn(ka), hkb = __float2half_rn(kb);
      const __half hva = __float2half_rn(va), hvb = __float2half_rn(vb);
      if (z == 0) {                                  // one token group appends to the cache
        K[(int64_t)pos * kHeadDim + d] = hka;
        K[(int64_t)pos * kHeadDim + d + 64] = hkb;
        V[(int64_t)pos * kHeadDim + d] = hva;
        V[(int64_t)pos * kHeadDim + d + 64] = hvb;
      }
      reinterpret_cast<__half*>(&ks[r][0])[d] = hka;
      reinterpret_cast<__half*>(&ks[r][0])[d + 64] = hkb;
      reinterpret_cast<__half*>(&vs[r][0])[d] = hva;
      reinterpret_cast<__half*>(&vs[r][0])[d + 64] = hvb;
    }
    for (int j = z; j < Lq; j += Z) {
      const int len = p0 + j + 1;                    // token j sees keys < len
      const int nkj = min(kend, len) - k0;           // keys of this tile it sees (may be <= 0)
      __syncthreads();                               // tiles staged / previous token done with qs, sc
      // rotated query rows of the G heads
      for (int i = tid; i < G * (kHeadDim / 2); i += 256) {
        const int g = i / (kHeadDim / 2), d = i % (kHeadDim / 2);
        const float* qr = qkv + ((int64_t)b * Lq + j) * qkv_stride + (int64_t)(hk * G + g) * kHeadDim;
        float a = qr[d], c = qr[d + 64];
        rope_pair(a, c, p0 + j, d, theta);
        qs[g][d] = a * scale;
        qs[g][d + 64] = c * scale;
      }
      __syncthreads();
      if (nkj <= 0) continue;                        // uniform across the CTA
      // scores: thread (head group, key); lanes over keys, q broadcast
      {
        const int key = tid & (kAttnKeys - 1);
        for (int g = tid >> 6; g < G; g += 256 / kAttnKeys) {
          float acc = 0.f;
          if (key < nkj) {
            const float2* q2 = reinterpret_cast<const float2*>(qs[g]);
#pragma unroll 16
            for (int w = 0; w < kHeadDim / 2; ++w) {
              const float2 kf = __half22float2(ks[key][w]);
              const float2 qf = q2[w];
              acc = fmaf(qf.x, kf.x, acc);
              acc = fmaf(qf.y, kf.y, acc);
            }
          }
          sc[g][key] = key < nkj ? acc : -INFINITY;
        }
      }
      __syncthreads();
      // per head: max and exp over the tile (warp g handles head g)
      if (warp < G) {
        const int g = warp;
        const float s0 = sc[g][lane], s1 = sc[g][lane + 32];
        float mx = fmaxf(s0, s1);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float e0 = lane < nkj ? expf(s0 - mx) : 0.f, e1 = lane + 32 < nkj ? expf(s1 - mx) : 0.f;
        sc[g][lane] = e0;
        sc[g][lane + 32] = e1;
        const float sum = warp_sum(e0 + e1);
        if (lane == 0) {
          AttnPart pm;
          pm.m = mx;
          pm.l = sum;
          part_ml[((bh * nsplit + s) * kMaxLq + j) * kMaxGroup + g] = pm;
        }
      }
      __syncthreads();
      // unnormalised output: thread (head, 2 dims); lanes over dims
      for (int i = tid; i < G * (kHeadDim / 2); i += 256) {
        const int g = i / (kHeadDim / 2), d2 = i % (kHeadDim / 2);
        float o0 = 0.f, o1 = 0.f;
        for (int key = 0; key < nkj; ++key) {
          const float pk = sc[g][key];
          const float2 vf = __half22float2(vs[key][d2]);
          o0 = fmaf(pk, vf.x, o0);
          o1 = fmaf(pk, vf.y, o1);
        }
        *reinterpret_cast<float2*>(part_o + (((bh * nsplit + s) * kMaxLq + j) * kMaxGroup + g) * kHeadDim +
                                   2 * d2) = make_float2(o0, o1);
      }
    }
  }
  // the last CTA of (b, hk) merges
  __threadfence();
  __syncthreads();
  if (tid == 0) last = atomicAdd(&tickets[bh], 1) == nsplit * Z - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  const float* mls = reinterpret_cast<const float*>(part_ml);
  for (int i = tid; i < Lq * G * (kHeadDim / 4); i += 256) {
    const int j = i / (G * (kHeadDim / 4));
    const int rem = i % (G * (kHeadDim / 4));
    const int g = rem / (kHeadDim / 4), d = (rem % (kHeadDim / 4)) * 4;
    const int len = p0 + j + 1;
    const int ns = min(nsplit, (len + kAttnKeys - 1) / kAttnKeys);
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

// ---------------------------------------------------------------------------
// Prefill attention (16 or more new tokens per sequence): first the new
// tokens' keys and values are rotated and appended to the cache
// (k_kv_append, the same rotation and fp16 rounding as k_attention), then
// k_attn_chunk computes causal GQA attention from the cache on tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation, online softmax).
//
// CTA (b, hk, t): KV head hk of sequence b and new tokens 16t .. 16t + 15;
// warp g computes query head hk * G + g for those 16 tokens (the C fragment
// rows).  The CTA walks the keys 0 .. pos0 + last token in tiles of 64,
// staged in shared memory ([key][dim], 272-byte rows so that ldmatrix reads
// eight rows without bank conflicts) and shared by the G warps.  S = q k^T
// (q rotated and scaled by log2(e) / sqrt(128) in registers, fp16), the
// running max and sum per row, P (fp16) reuses the S fragments as the A
// operand of P V (ldmatrix.trans of the V rows), and O / l is written as fp32.
// Keys past the last written position read as zeros in shared memory and are
// masked, so no uninitialised cache entry enters a product.  The K / V tiles
// are double-buffered (dynamic shared memory, 2 x 2 x 64 x 272 bytes): the
// next tile's 16-byte cp.async copies are in flight while the warps compute
// on the current one.
// ---------------------------------------------------------------------------
constexpr int kChunkTok = 16;           // new tokens per CTA (the MMA's M)
constexpr int kKeyTile = 64;
constexpr int kRowH = kHeadDim + 8;     // halves per staged row (272 bytes)
constexpr int kAttnTileHalves = kKeyTile * kRowH;                      // one staged K or V tile
constexpr int kAttnSmem = 2 * 2 * kAttnTileHalves * (int)sizeof(__half);   // 2 buffers of K and V: 69,632 bytes

// 16-byte global -> shared copy; src_bytes = 0 writes zeros and reads nothing
XM_DEV void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
XM_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
XM_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(128) k_kv_append(const float* __restrict__ qkv, int64_t qkv_stride,
                                                   __half* __restrict__ kc, __half* __restrict__ vc,
                                                   const int* __restrict__ pos0, int Lq, int Hq, int Hk,
                                                   int max_ctx, float theta) {
  grid_dep_wait();
  grid_dep_launch();
  const int row = blockIdx.x, b = row / Lq, j = row % Lq;
  const int pos = pos0[b] + j;
  const float* r = qkv + (int64_t)row * qkv_stride + (int64_t)Hq * kHeadDim;
  for (int i = threadIdx.x; i < Hk * (kHeadDim / 2); i += blockDim.x) {
    const int hk = i / (kHeadDim / 2), d = i % (kHeadDim / 2);
    float ka = r[hk * kHeadDim + d], kb = r[hk * kHeadDim + d + 64];
    rope_pair(ka, kb, pos, d, theta);
    const float va = r[(Hk + hk) * kHeadDim + d], vb = r[(Hk + hk) * kHeadDim + d + 64];
    const int64_t at = (((int64_t)b * Hk + hk) * max_ctx + pos) * kHeadDim;
    kc[at + d] = __float2half_rn(ka);
    kc[at + d + 64] = __float2half_rn(kb);
    vc[at + d] = __float2half_rn(va);
    vc[at + d + 64] = __float2half_rn(vb);
  }
}

XM_DEV uint32_t pack_half2(float a, float b) {
  const __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<const uint32_t*>(&h);
}
XM_DEV void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
XM_DEV void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
XM_DEV void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__global__ void __launch_bounds__(32 * kMaxGroup) k_attn_chunk(const float* __restrict__ qkv, int64_t qkv_stride,
                                                               const __half* __restrict__ kc,
                                                               const __half* __restrict__ vc,
                                                               const int* __restrict__ pos0, int Lq, int Hq, int Hk,
                                                               int max_ctx, float theta, float* __restrict__ out,
                                                               int64_t out_stride) {
  extern __shared__ __align__(16) __half attn_sm[];   // [buffer][K, V][key][kRowH]
  grid_dep_wait();                                 // the appended keys come from the preceding kernel
  grid_dep_launch();
  const int b = blockIdx.x / Hk, hk = blockIdx.x % Hk;
  const int j0 = ((int)gridDim.y - 1 - (int)blockIdx.y) * kChunkTok;   // the longest (last) tiles start first
  const int G = Hq / Hk;
  const int tid = threadIdx.x, lane = tid & 31, g = tid >> 5;
  const int nthr = blockDim.x;
  const int p0 = pos0[b];
  const int jlast = min(j0 + kChunkTok, Lq) - 1;
  const int kend = p0 + jlast + 1;                 // keys this CTA's last token sees
  const int64_t bh = (int64_t)b * Hk + hk;
  const __half* K = kc + bh * max_ctx * kHeadDim;
  const __half* V = vc + bh * max_ctx * kHeadDim;
  const int r0 = lane >> 2, c2 = 2 * (lane & 3);   // fragment row (and row + 8), column pair
  // this lane's two tokens (rows r0, r0 + 8; rows past the last token repeat it and are not written)
  const int ja = min(j0 + r0, Lq - 1), jb = min(j0 + r0 + 8, Lq - 1);
  const int posa = p0 + ja, posb = p0 + jb;

  // q fragments: k-step s covers dims 16s .. 16s + 15; this lane holds dims 16s + c2 (+1) and
  // 16s + 8 + c2 (+1) of rows a and b, so dims d and d + 64 (steps s and s + 4) meet in one lane
  uint32_t qf[8][4];
  {
    const float qscale = 1.4426950408889634f * rsqrtf((float)kHeadDim);   // log2(e) / sqrt(d)
    const float* qa = qkv + ((int64_t)b * Lq + ja) * qkv_stride + (int64_t)(hk * G + g) * kHeadDim;
    const float* qb = qkv + ((int64_t)b * Lq + jb) * qkv_stride + (int64_t)(hk * G + g) * kHeadDim;
#pragma unroll
    for (int s4 = 0; s4 < 4; ++s4) {
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {            // dims 16 s4 + 8 hf + c2, +1
        const int d = 16 * s4 + 8 * hf + c2;
        float a0 = qa[d], a1 = qa[d + 1], a0h = qa[d + 64], a1h = qa[d + 65];
        float b0 = qb[d], b1 = qb[d + 1], b0h = qb[d + 64], b1h = qb[d + 65];
        rope_pair(a0, a0h, posa, d, theta);
        rope_pair(a1, a1h, posa, d + 1, theta);
        rope_pair(b0, b0h, posb, d, theta);
        rope_pair(b1, b1h, posb, d + 1, theta);
        qf[s4][2 * hf] = pack_half2(a0 * qscale, a1 * qscale);
        qf[s4][2 * hf + 1] = pack_half2(b0 * qscale, b1 * qscale);
        qf[s4 + 4][2 * hf] = pack_half2(a0h * qscale, a1h * qscale);
        qf[s4 + 4][2 * hf + 1] = pack_half2(b0h * qscale, b1h * qscale);
      }
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float ma = -INFINITY, mb = -INFINITY, la = 0.f, lb = 0.f;
  const uint32_t sm0 = (uint32_t)__cvta_generic_to_shared(attn_sm);
  const int mi = lane >> 3, mr = lane & 7;        // ldmatrix: this lane addresses row mr of matrix mi
  // tile kb -> buffer buf (K at buffer offset 0, V after it); keys >= kend are zero-filled
  auto stage = [&](int kb, int buf) {
    const uint32_t kdst = sm0 + (uint32_t)(buf * 2 * kAttnTileHalves) * 2u;
    const uint32_t vdst = kdst + (uint32_t)kAttnTileHalves * 2u;
    for (int i = tid; i < kKeyTile * (kHeadDim / 8); i += nthr) {
      const int r = i / (kHeadDim / 8), c = (i % (kHeadDim / 8)) * 8;
      const int key = kb + r;
      const bool ok = key < kend;
      const int64_t off = (int64_t)(ok ? key : 0) * kHeadDim + c;
      const uint32_t so = (uint32_t)(r * kRowH + c) * 2u;
      cp_async16(kdst + so, K + off, ok ? 16u : 0u);
      cp_async16(vdst + so, V + off, ok ? 16u : 0u);
    }
    cp_async_commit();
  };
  stage(0, 0);

  for (int kb = 0, t = 0; kb < kend; kb += kKeyTile, ++t) {
    __syncthreads();                               // every warp is done with the tile read two steps ago
    if (kb + kKeyTile < kend) {
      stage(kb + kKeyTile, (t + 1) & 1);           // the next tile loads while this one is used
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();                               // this tile's copies of every thread have landed
    const uint32_t ks0 = sm0 + (uint32_t)((t & 1) * 2 * kAttnTileHalves) * 2u;
    const uint32_t vs0 = ks0 + (uint32_t)kAttnTileHalves * 2u;
    // S = q k^T: 8 tiles of 8 keys
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.f;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {            // key tiles 2np, 2np + 1
        // matrices: (keys 16np..+7, dims 16s..+7), (same keys, dims +8), (keys +8, dims 16s), (keys +8, dims +8)
        const int key = 16 * np + mr + 8 * (mi >> 1), dim = 16 * s + 8 * (mi & 1);
        uint32_t k0, k1, k2, k3;
        ldsm_x4(ks0 + (uint32_t)(key * kRowH + dim) * 2u, k0, k1, k2, k3);
        mma_f16_16816(sc[2 * np], qf[s], k0, k1);
        mma_f16_16816(sc[2 * np + 1], qf[s], k2, k3);
      }
    }
    // mask (causal, and keys not yet written), online softmax
    float tma = -INFINITY, tmb = -INFINITY;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int key = kb + 8 * n + c2;
      if (key > posa) sc[n][0] = -INFINITY;
      if (key + 1 > posa) sc[n][1] = -INFINITY;
      if (key > posb) sc[n][2] = -INFINITY;
      if (key + 1 > posb) sc[n][3] = -INFINITY;
      tma = fmaxf(tma, fmaxf(sc[n][0], sc[n][1]));
      tmb = fmaxf(tmb, fmaxf(sc[n][2], sc[n][3]));
    }
    tma = fmaxf(tma, __shfl_xor_sync(~0u, tma, 1));
    tma = fmaxf(tma, __shfl_xor_sync(~0u, tma, 2));
    tmb = fmaxf(tmb, __shfl_xor_sync(~0u, tmb, 1));
    tmb = fmaxf(tmb, __shfl_xor_sync(~0u, tmb, 2));
    const float na = fmaxf(ma, tma), nb = fmaxf(mb, tmb);   // finite: key 0 is always visible
    const float aa = exp2f(ma - na), ab = exp2f(mb - nb);
    ma = na;
    mb = nb;
    float suma = 0.f, sumb = 0.f;
    uint32_t pf[4][4];                              // P as the A operand: k-step s = key tiles 2s, 2s + 1
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float e0 = exp2f(sc[n][0] - na), e1 = exp2f(sc[n][1] - na);
      const float e2 = exp2f(sc[n][2] - nb), e3 = exp2f(sc[n][3] - nb);
      suma += e0 + e1;
      sumb += e2 + e3;
      pf[n >> 1][2 * (n & 1)] = pack_half2(e0, e1);
      pf[n >> 1][2 * (n & 1) + 1] = pack_half2(e2, e3);
    }
    la = la * aa + suma;
    lb = lb * ab + sumb;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= aa;
      o[n][1] *= aa;
      o[n][2] *= ab;
      o[n][3] *= ab;
    }
    // O += P V: 4 k-steps of 16 keys, 16 tiles of 8 dims
#pragma unroll
    for (int s = 0; s < 4; ++s) {
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {            // dim tiles 2dp, 2dp + 1
        // matrices (transposed): (keys 16s..+7, dims 16dp..+7), (keys +8, same dims), (keys 16s, dims +8), (keys +8, dims +8)
        const int key = 16 * s + mr + 8 * (mi & 1), dim = 16 * dp + 8 * (mi >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(vs0 + (uint32_t)(key * kRowH + dim) * 2u, v0, v1, v2, v3);
        mma_f16_16816(o[2 * dp], pf[s], v0, v1);
        mma_f16_16816(o[2 * dp + 1], pf[s], v2, v3);
      }
    }
  }
  // row sums across the quad, then O / l
  la += __shfl_xor_sync(~0u, la, 1);
  la += __shfl_xor_sync(~0u, la, 2);
  lb += __shfl_xor_sync(~0u, lb, 1);
  lb += __shfl_xor_sync(~0u, lb, 2);
  const float ia = 1.0f / la, ib = 1.0f / lb;
  const bool wa = j0 + r0 < Lq, wb = j0 + r0 + 8 < Lq;
  float* oa = out + ((int64_t)b * Lq + ja) * out_stride + (int64_t)(hk * G + g) * kHeadDim;
  float* ob = out + ((int64_t)b * Lq + jb) * out_stride + (int64_t)(hk * G + g) * kHeadDim;
#pragma unroll
  for (int n = 0; n < 16; ++n) {
    if (wa) *reinterpret_cast<float2*>(oa + 8 * n + c2) = make_float2(o[n][0] * ia, o[n][1] * ia);
    if (wb) *reinterpret_cast<float2*>(ob + 8 * n + c2) = make_float2(o[n][2] * ib, o[n][3] * ib);
  }
}

// first index of the maximum of each row (np.argmax semantics; NaN-free
// input).  One CTA per row; 16-byte loads, eight in flight per thread.
XM_DEV void argmax_take(float v, int i, float& best, int& idx) {
  if (v > best || (v == best && i < idx)) {
    best = v;
    idx = i;
  }
}

__global__ void __launch_bounds__(1024) k_argmax(const float* __restrict__ logits, int V, int* __restrict__ out) {
  __shared__ float bv[32];
  __shared__ int bi[32];
  grid_dep_wait();
  grid_dep_launch();
  const int b = blockIdx.x;
  const float* r = logits + (int64_t)b * V;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  const bool vec = (((uintptr_t)r) & 15) == 0;
  const int V4 = vec ? V / 4 : 0;
  const float4* r4 = reinterpret_cast<const float4*>(r);
#pragma unroll 8
  for (int i = threadIdx.x; i < V4; i += blockDim.x) {
    const float4 v = __ldcs(r4 + i);
    argmax_take(v.x, 4 * i, best, idx);
    argmax_take(v.y, 4 * i + 1, best, idx);
    argmax_take(v.z, 4 * i + 2, best, idx);
    argmax_take(v.w, 4 * i + 3, best, idx);
  }
  for (int i = 4 * V4 + threadIdx.x; i < V; i += blockDim.x) argmax_take(r[i], i, best, idx);
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    argmax_take(ov, oi, best, idx);
  }
  if ((threadIdx.x & 31) == 0) {
    bv[threadIdx.x >> 5] = best;
    bi[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x + 31) / 32; ++w) argmax_take(bv[w], bi[w], best, idx);
    out[b] = idx == 0x7fffffff ? 0 : idx;
  }
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_smem(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, int smem,
                            Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, Args... args) {
  return launch_pdl_smem(kernel, grid, block, st, 0, args...);
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

int64_t xm_attention_workspace_size(int64_t B, int Hk, int64_t max_ctx) {
  const int64_t nsplit = (max_ctx + kAttnKeys - 1) / kAttnKeys;
  const int64_t cells = B * Hk * nsplit * kMaxLq * kMaxGroup;
  return cells * kHeadDim * 4 + cells * (int64_t)sizeof(AttnPart) + B * Hk * 4 + 256;
}

int xm_attention(const float* d_qkv, int64_t qkv_stride, void* d_kcache, void* d_vcache, const int* d_pos0, int64_t B,
                 int Lq, int Hq, int Hk, int head_dim, float theta, int64_t max_ctx, float* d_out,
                 int64_t out_stride, void* d_workspace, int64_t workspace_bytes, void* stream) {
  if (head_dim != kHeadDim) return xm_set_error(XM_ERR_UNSUPPORTED, "attention: head_dim %d (only 128)", head_dim);
  // 16 or more new tokens take the prefill path (any count); fewer, the split-key decode kernel (<= 64)
  const bool chunk = Lq >= kChunkTok && (out_stride % 2) == 0 && (qkv_stride % 2) == 0;
  if (B < 1 || Lq < 1 || (Lq > kMaxLq && !chunk) || Hq < 1 || Hk < 1 || Hq % Hk || Hq / Hk > kMaxGroup)
    return xm_set_error(XM_ERR_INVALID, "attention: bad head counts (G <= 8) or more than %d new tokens", kMaxLq);
  if (max_ctx < 1 || max_ctx > (1 << 24) || qkv_stride < (int64_t)(Hq + 2 * Hk) * kHeadDim ||
      out_stride < (int64_t)Hq * kHeadDim || !d_qkv || !d_kcache || !d_vcache || !d_pos0 || !d_out)
    return xm_set_error(XM_ERR_INVALID, "attention: bad arguments");
  if (!d_workspace || workspace_bytes < xm_attention_workspace_size(B, Hk, max_ctx) || ((uintptr_t)d_workspace & 15))
    return xm_set_error(XM_ERR_INVALID, "attention: workspace too small or unaligned");
  const int nsplit = (int)((max_ctx + kAttnKeys - 1) / kAttnKeys);
  const int64_t cells = B * Hk * nsplit * kMaxLq * kMaxGroup;
  float* part_o = (float*)d_workspace;
  AttnPart* part_ml = (AttnPart*)(part_o + cells * kHeadDim);
  int* tickets = (int*)(part_ml + cells);
  // tickets start at zero (the caller zeroes the workspace once) and every call leaves them at zero
  if (chunk) {
    // prefill chunk: append the new keys and values, then tensor-core attention from the cache
    const int G = Hq / Hk;
    int rc = launch_status(launch_pdl(k_kv_append, dim3((unsigned)(B * Lq)), dim3(128), (cudaStream_t)stream, d_qkv,
                                      qkv_stride, (__half*)d_kcache, (__half*)d_vcache, d_pos0, Lq, Hq, Hk,
                                      (int)max_ctx, theta),
                           "attention kv append");
    if (rc) return rc;
    static bool attn_attr[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64 || !attn_attr[dev]) {
      cudaError_t e = cudaFuncSetAttribute(k_attn_chunk, cudaFuncAttributeMaxDynamicSharedMemorySize, kAttnSmem);
      if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "attention: smem attribute: %s", cudaGetErrorString(e));
      if (dev >= 0 && dev < 64) attn_attr[dev] = true;
    }
    return launch_status(launch_pdl_smem(k_attn_chunk, dim3((unsigned)(B * Hk), (unsigned)((Lq + kChunkTok - 1) / kChunkTok)),
                                    dim3((unsigned)(32 * G)), (cudaStream_t)stream, kAttnSmem, d_qkv, qkv_stride,
                                    (const __half*)d_kcache, (const __half*)d_vcache, d_pos0, Lq, Hq, Hk,
                                    (int)max_ctx, theta, d_out, out_stride),
                         "attention chunk");
  }
  const unsigned Z = (unsigned)((Lq + kAttnTokensPerCta - 1) / kAttnTokensPerCta);
  return launch_status(launch_pdl(k_attention, dim3((unsigned)(B * Hk), (unsigned)nsplit, Z), dim3(256),
                                  (cudaStream_t)stream, d_qkv, qkv_stride, (__half*)d_kcache, (__half*)d_vcache,
                                  d_pos0, Lq, Hq, Hk, (int)max_ctx, nsplit, theta, part_o, part_ml, tickets, d_out,
                                  out_stride),
                       "attention");
}

int xm_argmax(const float* d_logits, int64_t B, int64_t V, int* d_out, void* stream) {
  if (B < 1 || V < 1 || !d_logits || !d_out) return xm_set_error(XM_ERR_INVALID, "argmax: bad arguments");
  return launch_status(launch_pdl(k_argmax, dim3((unsigned)B), dim3(1024), (cudaStream_t)stream, d_logits, (int)V,
                                  d_out),
                       "argmax");
}

}  // extern "C"
