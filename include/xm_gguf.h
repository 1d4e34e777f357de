/*
 * xm_gguf.h -- C ABI of the B200 (sm_100a) GGUF quantized-weight path.
 *
 * Every entry point takes plain device pointers, byte/element counts and a
 * CUDA stream (a cudaStream_t passed as void*, NULL = legacy default stream).
 * Nothing here allocates device memory unless stated; buffers belong to the
 * caller.  Calls are asynchronous on `stream`; argument errors are detected on
 * the host before any launch.
 *
 * Return value: XM_OK (0) or a negative XM_ERR_* status; xm_last_error()
 * gives the message of the last failure on the calling thread.
 *
 * Type ids (`qtype`) are the GGML numbers of the reference's GGUF reader
 * (dtype_map.py:33-65): F32=0 F16=1 Q4_0=2 Q4_1=3 Q5_0=6 Q5_1=7 Q8_0=8
 * Q8_1=9 Q2_K=10 Q3_K=11 Q4_K=12 Q5_K=13 Q6_K=14 Q8_K=15 I8=24 I16=25
 * I32=26 I64=27 BF16=30.  IQ and TQ types are rejected with
 * XM_ERR_UNSUPPORTED, as the reference raises NotImplementedError for them
 * (gguf_dequant.py:493-501).
 *
 * Weight layout: a 2-D weight W[n][k] is the GGUF byte stream of n rows, each
 * row k/QK consecutive block records (GGUF dims = [k, n]).  This is the byte
 * order the reference dequantizes (gguf_dequant.py:31-32, loaders.py:340-343).
 */
#ifndef XM_GGUF_H
#define XM_GGUF_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XM_OK 0
#define XM_ERR_INVALID (-1)     /* bad size / shape / pointer / alignment (numpy ValueError in the reference) */
#define XM_ERR_UNSUPPORTED (-2) /* type not implemented (NotImplementedError in the reference) */
#define XM_ERR_CUDA (-3)        /* CUDA runtime error */

/* element types of activations and outputs */
#define XM_DT_F32 0
#define XM_DT_F16 1
#define XM_DT_BF16 2

/* expert activations of the MoE entry points (primitives.py:37-62 apply_activation) */
#define XM_ACT_SILU 0     /* x / (1 + exp(-x)); also the reference's "swish" */
#define XM_ACT_GELU 1     /* 0.5 x (1 + tanh(0.7978845608 (x + 0.044715 x^3))) */
#define XM_ACT_RELU 2     /* max(x, 0) */
#define XM_ACT_IDENTITY 3 /* x */

/* activation prologues of xm_qgemv_ex */
#define XM_PRO_NONE 0    /* v = x */
#define XM_PRO_RMSNORM 1 /* v = (x / sqrt(mean(x^2) + eps)) * norm_w */
#define XM_PRO_SWIGLU 2  /* v = silu(x[:, :k]) * x[:, k:2k]  (x rows hold 2k values) */

/* ABI version of this header (bumped on any signature change). */
int xm_abi_version(void);

/* Message of the last failing call on this thread ("" if none). */
const char* xm_last_error(void);

/* Device error word of the current device: a non-zero bit means a bounded wait
 * inside a kernel gave up (XM_DEVERR_TIMEOUT = 1) instead of hanging.  With
 * clear != 0 the word is reset.  Returns the word (>= 0) or XM_ERR_CUDA. */
int xm_device_status(int clear);

/* Stream-ordered read of the same word: enqueues a copy of the current
 * device's error word into *h_word (pinned host memory) on `stream`, after the
 * work queued before it; read *h_word once the stream has been synchronised
 * (and clear a non-zero word with xm_device_status(1)). */
int xm_device_status_async(int* h_word, void* stream);

/* Block geometry of a type: elements per block and bytes per block record.
 * Replaces the lookup in GGUF_TYPE_BLOCK_SIZE (dtype_map.py:68-79). */
int xm_qtype_info(int qtype, int* qk, int* record_bytes);

/*
 * Dequantize `n_elements` values of GGUF type `qtype` from the raw block bytes
 * at `d_raw` (`raw_bytes` long; extra bytes are ignored) into `d_out`
 * (XM_DT_F16: the reference's fp16 result, bit for bit; XM_DT_F32: the fp32
 * value the reference holds before its final fp16 cast).  `d_out` must be
 * 16-byte aligned.
 *
 * Replaces gguf_dequant.py:477-523 `dequantize(raw_bytes, tensor_type, shape)`
 * and the per-type `dequant_<q>(raw_bytes, shape)` of gguf_dequant.py:25-455
 * (and meanflare convert.py:46 `dequantize_gguf_tensor`).  The shape only
 * fixes n_elements = prod(shape); the element order is the flat GGUF order.
 */
int xm_dequantize(int qtype, const void* d_raw, int64_t raw_bytes, int64_t n_elements,
                  void* d_out, int out_dtype, void* stream);

/*
 * Decode GEMV: y[m][n] = sum_k x[m][k] * W[n][k] (+ bias[n]) for 1 <= m <= 8,
 * W the GGUF blocks at `d_w` (`w_bytes` long, n rows of k elements), x
 * row-major [m][k] of x_dtype (16-byte aligned), y row-major [m][n] fp32,
 * bias fp32 [n] or NULL.  Fused: the blocks are unpacked in registers and
 * never written back.
 *
 * `d_workspace` (16-byte aligned, >= xm_qgemv_workspace_size(k, m) bytes)
 * holds the activation split of the integer-dot path.  With NULL, shapes whose
 * split needs the workspace take the exact path (each weight rounded to the
 * reference's fp16 value); Q4_K with m = 1 and k = 4096 splits inside its one
 * kernel and takes the integer-dot path either way.  Results of both paths
 * are within 1e-3 of the reference (max abs error / max |y|).
 *
 * Replaces the decode-time `x @ W.T` on dequantized weights: ops.py:62-67
 * `LinearOp.forward`, forward.py:93-101 (MLP), attention.py:47-51/:135
 * (projections), forward.py:158 (lm_head), all after gguf_dequant.dequantize.
 */
int64_t xm_qgemv_workspace_size(int64_t k, int64_t m);
int xm_qgemv(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
             const void* d_x, int x_dtype, int64_t m, const float* d_bias, float* d_y,
             void* d_workspace, int64_t workspace_bytes, void* stream);

/*
 * The two halves of the integer-dot GEMV, for callers that feed one activation
 * to several weights (Q/K/V, gate/up): xm_split_activation writes the split of
 * x into the workspace once; xm_qgemv_presplit runs the GEMV from it.  Types
 * without an integer-dot path return XM_ERR_UNSUPPORTED from the latter.
 */
int xm_split_activation(const void* d_x, int x_dtype, int64_t m, int64_t k,
                        void* d_workspace, int64_t workspace_bytes, void* stream);
int xm_qgemv_presplit(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                      int64_t m, const void* d_workspace, int64_t workspace_bytes,
                      const float* d_bias, float* d_y, void* stream);

/*
 * xm_qgemv with the decoder's neighbours fused in:
 *   y[m][n] (+)= sum_k pro(x)[m][k] * W[n][k] (+ bias[n])
 * `prologue` transforms each activation row before the product (XM_PRO_*:
 * RMSNorm with weight d_norm_w [k] and eps, or SwiGLU of a row holding gate
 * then up, 2k values); `x_stride` is the row pitch of x in elements (>= k, or
 * >= 2k for SwiGLU).  With `accumulate` the product is added to y instead of
 * overwriting it (the residual add).  Block types with an integer-dot path
 * (Q4_K, Q5_K, Q6_K, Q8_0) take any prologue; others only XM_PRO_NONE without
 * accumulate.  Workspace as for xm_qgemv (NULL allowed only where no split is
 * needed: Q4_K, m = 1, k = 4096 without SwiGLU).
 *
 * Replaces FusedRMSNormLinearOp.forward (ops.py:107-123), the MLP's
 * `swiglu(gate, up) @ W_down.T` (forward.py:97-101) and the residual adds
 * `x = residual + h` around them (forward.py:111, :116).
 */
int xm_qgemv_ex(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                const void* d_x, int x_dtype, int64_t m, int64_t x_stride, int prologue,
                const float* d_norm_w, float eps, const float* d_bias, float* d_y, int accumulate,
                void* d_workspace, int64_t workspace_bytes, void* stream);

/* The exact path alone, for every type and shape (every weight rounded to
 * the reference's fp16 value, fp32 products): the cross-check of the
 * integer-dot path.  Same arguments and limits as xm_qgemv, no workspace. */
int xm_qgemv_exact(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                   const void* d_x, int x_dtype, int64_t m, const float* d_bias, float* d_y,
                   void* stream);

/*
 * Prefill GEMM on 5th-generation tensor cores: y[m][n] = sum_k x[m][k] *
 * W[n][k] (+ bias[n]) for any m >= 1 (meant for m >= 64), x row-major [m][k]
 * of x_dtype (16-byte aligned), y row-major [m][n] fp32, W GGUF blocks of any
 * block-quantized type (Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1, Q2_K ... Q8_K)
 * with k a multiple of 256.  Each weight is decoded to the reference's fp16
 * value, x is converted to fp16 with an exact power-of-two scale per row,
 * tcgen05.mma accumulates in fp32: the result differs from the reference's
 * fp32 `x @ W.T` only in summation order.  A weight row must be a whole
 * number of 16-byte units (true for every type when k % 2048 == 0; Q6_K and
 * Q3_K rows of k = 1792, for example, are not): other shapes return
 * XM_ERR_UNSUPPORTED and callers use xm_qgemv on groups of 8 rows.
 * `d_workspace` (256-byte aligned, >= xm_qgemm_workspace_size(m, k) bytes)
 * holds the converted activations.  A workspace of
 * xm_qgemm_workspace_size_n(m, n, k) bytes also holds the partial sums of a
 * split-K launch, which the GEMM uses when its output tiles are too few to
 * occupy the device (n % 4 == 0, y and bias 16-byte aligned): each K part
 * writes its own plane and one kernel adds the planes in a fixed order, so the
 * result is the same on every run.
 *
 * Replaces the prefill `x @ W.T` of LinearOp.forward (ops.py:62-67) and of
 * the MLP / attention projections (forward.py:93-101, attention.py:47-51).
 */
int64_t xm_qgemm_workspace_size(int64_t m, int64_t k);
int64_t xm_qgemm_workspace_size_n(int64_t m, int64_t n, int64_t k);
int xm_qgemm(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
             const void* d_x, int x_dtype, int64_t m, const float* d_bias, float* d_y,
             void* d_workspace, int64_t workspace_bytes, void* stream);

/*
 * xm_qgemm with the prologues and the residual add of xm_qgemv_ex:
 *   y[m][n] (+)= sum_k pro(x)[m][k] * W[n][k] (+ bias[n])
 * `prologue` is XM_PRO_NONE, XM_PRO_RMSNORM (weight d_norm_w [k], eps) or
 * XM_PRO_SWIGLU (rows of x hold gate then up, 2k values); `x_stride` is the
 * row pitch of x in elements.  The prologue runs in fp32 before the fp16
 * conversion of the activation.
 *
 * Replaces FusedRMSNormLinearOp.forward (ops.py:107-123) for many rows, and
 * the prefill MLP `swiglu(gate, up) @ W_down.T` with its residual add
 * (forward.py:97-101, :116).
 */
int xm_qgemm_ex(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                const void* d_x, int x_dtype, int64_t m, int64_t x_stride, int prologue,
                const float* d_norm_w, float eps, const float* d_bias, float* d_y, int accumulate,
                void* d_workspace, int64_t workspace_bytes, void* stream);

/*
 * xm_qgemm_ex on weight rows stored `w_row_pitch` bytes apart (a multiple of
 * 16, at least the row's record bytes; w_bytes >= (n - 1) * pitch + row
 * bytes).  For K-slices whose rows are not whole 16-byte units (a Q6_K slice
 * of 7168 columns is 5880 bytes per row): the caller keeps a copy of the slice
 * with each row padded to the pitch, and the tensor-core GEMM reads that copy.
 * The padding bytes are never decoded.  Same replacement as xm_qgemm_ex, for
 * the row-parallel projections of a tensor-parallel model (the K-sliced
 * `x @ W.T` of forward.py:97-101 on one rank).
 */
int xm_qgemm_ex_pitched(int qtype, const void* d_w, int64_t w_row_pitch, int64_t w_bytes, int64_t n,
                        int64_t k, const void* d_x, int x_dtype, int64_t m, int64_t x_stride, int prologue,
                        const float* d_norm_w, float eps, const float* d_bias, float* d_y, int accumulate,
                        void* d_workspace, int64_t workspace_bytes, void* stream);

/*
 * RMSNorm of m rows of x (row pitch x_stride elements): out[m][k] fp32 =
 * (x / sqrt(mean(x^2) + eps)) * norm_w, in the reference's order
 * (primitives.py:20-23, ops.py:115-117).  The norm of FusedRMSNormLinearOp
 * for weights whose matmul has no fused prologue (dense weights, block types
 * without an integer-dot GEMV or tensor-core GEMM at that shape).
 */
int xm_rmsnorm(const void* d_x, int x_dtype, int64_t m, int64_t k, int64_t x_stride,
               const float* d_norm_w, float eps, float* d_out, void* stream);

/*
 * Sparse mixture-of-experts block (Mixtral-style gated experts):
 *   out[t] = sum over the k experts e chosen for token t (ascending e) of
 *            w[t][e] * ((act(x_t @ W1_e.T) * (x_t @ W3_e.T)) @ W2_e.T)
 * with act = XM_ACT_* (`activation`; silu for Mixtral)
 * with router logits x @ gate.T (gate fp32 [E][H]), the k largest logits per
 * token and a softmax over those k (over all E when k == E).  x row-major
 * [T][H] of x_dtype, out fp32 [T][H].  h_w1/h_w3 ([F][H]) and h_w2 ([H][F])
 * are HOST arrays of E device pointers to GGUF blocks of `qtype` (any type
 * that xm_qgemm takes at k = H and at k = F; others return
 * XM_ERR_UNSUPPORTED).  E <= 32; H and F multiples of 256.
 * `d_workspace` (256-byte aligned, xm_moe_workspace_size bytes) holds the
 * routing, the gathered activations and the expert intermediates.  The whole
 * block runs on `stream` without host synchronisation: routing, a stable
 * counting sort by expert, grouped tensor-core GEMMs, fused SwiGLU, combine.
 *
 * Replaces moe.py:54-115 `MoELayer.__call__` (sparse top-k path and the
 * dense k == E path).
 */
int64_t xm_moe_workspace_size(int64_t T, int64_t H, int64_t F, int E, int k);
int xm_moe_forward(const void* d_x, int x_dtype, int64_t T, int64_t H, const float* d_gate,
                   int E, int k, int64_t F, const void* const* h_w1, const void* const* h_w3,
                   const void* const* h_w2, int qtype, int activation, float* d_out, void* d_workspace,
                   int64_t workspace_bytes, void* stream);

/*
 * Expert parallelism: xm_moe_forward split at its two exchange points, for
 * experts sharded over ranks (rank r owns experts [r*E/R, (r+1)*E/R)).
 *
 * xm_moe_dispatch routes the T local tokens (router, top-k, softmax, stable
 * sort by expert: moe.py:61-93), writes the T*k selected rows of x in expert
 * order to d_send ([T*k][H], x's element type; the rows for rank r's experts
 * are therefore contiguous) and the per-expert row counts to d_cnt [E].  The
 * caller exchanges counts and rows (all-to-all) and runs
 * xm_moe_experts on the received rows: G groups of rows [off[g], off[g] +
 * cnt[g]) (device arrays; typically one group per (source rank, local
 * expert)) through the SwiGLU expert of group g (host pointer arrays h_w1,
 * h_w3, h_w2 of G entries; types as for xm_moe_forward), fp32 rows out;
 * max_rows bounds cnt[g].
 * After exchanging the result rows back into the send order, xm_moe_combine
 * forms out[t] = sum over the token's k rows, ascending expert, of row *
 * weight (moe.py:110-113), reading the routing from the dispatch workspace
 * (the same d_ws, xm_moe_workspace_size(T, H, F, E, k) bytes).  These entry
 * points have no C counterpart in the reference (its MoELayer is one process).
 */
int xm_moe_dispatch(const void* d_x, int x_dtype, int64_t T, int64_t H, const float* d_gate, int E, int k,
                    int64_t F, void* d_send, int* d_cnt, void* d_workspace, int64_t workspace_bytes, void* stream);
int64_t xm_moe_experts_workspace_size(int64_t P, int64_t H, int64_t F);
int xm_moe_experts(const void* d_rows, int x_dtype, int64_t P, int64_t H, int64_t F, int G, const int* d_cnt,
                   const int* d_off, const void* const* h_w1, const void* const* h_w3, const void* const* h_w2,
                   int qtype, int activation, int64_t max_rows, float* d_out, void* d_workspace,
                   int64_t workspace_bytes, void* stream);
int xm_moe_combine(const float* d_rows, int64_t T, int64_t H, int E, int k, int64_t F, const void* d_workspace,
                   float* d_out, void* stream);

/*
 * xm_qgemv without a workspace argument, for callers that cannot allocate
 * device memory (a host runtime that owns the allocator, a process that must
 * not allocate after start-up).  The activation split lives in a fixed array
 * built into this library, 320 KiB per GPU (limit: m <= 8 with k <= 16384;
 * larger requests return XM_ERR_INVALID).  The first call on each device
 * looks up that array's address (cudaGetSymbolAddress), so make it before any
 * stream capture; the address is kept for the life of the process, so a
 * device reset (cudaDeviceReset) between calls is not supported.  Calls share
 * the array: calls that overlap on the GPU race.  Nothing is allocated.  This
 * entry point has no counterpart in the reference.
 */
int xm_qgemv_noalloc(int qtype, const void* d_w, int64_t w_bytes, int64_t n, int64_t k,
                     const void* d_x, int x_dtype, int64_t m, const float* d_bias, float* d_y,
                     void* stream);

/*
 * Decoder-step kernels around the projections (Llama-style layer).  Head dim
 * 128 only; the caches are fp16 [B][Hk][max_ctx][128].  All of these launch
 * with programmatic dependent launch and run without host synchronisation.
 *
 * xm_embed: out[b][:] = fp16-rounded dequantized row ids[b] of a GGUF table
 * (vocab rows of D) -- the reference indexes its dequantized embedding
 * (forward.py:151).
 *
 * xm_attention: causal GQA attention of Lq new tokens per sequence (Lq <= 64, or
 * any Lq >= 16 when both row pitches are even: the prefill path, tensor cores).
 * qkv row b*Lq + j = [q | k | v] (Hq, Hk, Hk heads, fp32, row pitch
 * qkv_stride) of token j of sequence b at position pos0[b] + j, as the QKV
 * projection produced it.  Fused: rotate-half rotary embedding of q and k
 * (angle pos / theta^(2i/128), attention.py:66-70), append of the rotated k
 * and of v to the caches (attention.py:99-104), and out row b*Lq + j =
 * softmax(q k^T / sqrt(128) + causal mask) v per query head, Hq / Hk <= 8 query
 * heads per KV head (attention.py:105-115 with ninewas9's
 * scaled_dot_product_attention).  Keys are split 64 per CTA; the partial
 * softmaxes meet in `d_workspace` (xm_attention_workspace_size bytes, zeroed
 * once before the first call; every call leaves it ready for the next).
 *
 * xm_argmax: out[b] = first index of the maximum of logits row b (greedy
 * sampling, sampling.py:51-52 `sample_greedy`).
 *
 * These entry points have no C counterpart in the reference (it is numpy).
 */
int xm_embed(int qtype, const void* d_table, int64_t table_bytes, int64_t vocab, int64_t D, const int* d_ids,
             int64_t B, float* d_out, void* stream);
int64_t xm_attention_workspace_size(int64_t B, int Hk, int64_t max_ctx);
int xm_attention(const float* d_qkv, int64_t qkv_stride, void* d_kcache, void* d_vcache, const int* d_pos0, int64_t B,
                 int Lq, int Hq, int Hk, int head_dim, float theta, int64_t max_ctx, float* d_out,
                 int64_t out_stride, void* d_workspace, int64_t workspace_bytes, void* stream);
int xm_argmax(const float* d_logits, int64_t B, int64_t V, int* d_out, void* stream);

/*
 * Tensor-parallel exchange over NVLink peer memory (one process per GPU of a
 * node): the all-reduce of the row-parallel partial sums of the O and down
 * projections, added to the replicated residual stream (forward.py:111, :116
 * with those projections split over K).
 *
 * xm_comm_create allocates this rank's communication buffer for vectors of up
 * to max_elems fp32 values (xm_comm_buffer_size bytes) and returns an opaque
 * comm and a 64-byte CUDA IPC handle; the ranks exchange the handles (any
 * host channel) and each calls xm_comm_open_peer for every other rank.
 * xm_allreduce_add(comm, h, part, n): h[i] += sum over ranks r (in rank order,
 * identical on every rank) of part_r[i], for n <= max_elems (n % 4 == 0,
 * 16-byte aligned pointers).  One kernel of `nctas` CTAs per call; CTA j of
 * every rank exchanges the same slice with plain peer stores and per-(CTA,
 * rank) flags (no multicast), waits for the other ranks' flags for at most
 * 2 s (then sets XM_DEVERR_TIMEOUT in xm_device_status), and leaves the
 * buffer ready for the next call, so calls can be captured into CUDA graphs.
 * Every rank must make the same calls in the same order.  xm_comm_destroy
 * closes the peer mappings and frees the buffer; call it on every rank after
 * all ranks have finished their last xm_allreduce_add (host barrier + device
 * synchronisation).  These entry points have no counterpart in the reference.
 *
 * xm_comm_open_local: rank `peer_rank`'s buffer is the one of `peer_comm`,
 * created in this same process (one process driving several GPUs with peer
 * access enabled), instead of an IPC mapping.  xm_comm_set_wait_limit sets
 * the bounded wait of later xm_allreduce_add calls (1 us .. 60 s; default
 * 2 s).  A call whose wait gave up leaves the comm's epochs out of step with
 * the other ranks: destroy the comms of every rank and create new ones.
 */
int64_t xm_comm_buffer_size(int64_t max_elems);
int xm_comm_create(int world, int rank, int64_t max_elems, int nctas, void** out_comm, void* out_handle);
int xm_comm_open_peer(void* comm, int peer_rank, const void* handle);
int xm_comm_open_local(void* comm, int peer_rank, void* peer_comm);
int xm_comm_set_wait_limit(void* comm, int64_t limit_ns);
int xm_comm_destroy(void* comm);
int xm_allreduce_add(void* comm, float* d_h, const float* d_part, int64_t n_elems, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XM_GGUF_H */
