// One-shot all-reduce of the tensor-parallel decoder's row-parallel partial
// sums over NVLink peer memory (the exchange step of the O and down
// projections, forward.py:111 and :116 with the projection split over K).
//
// Every rank owns one communication buffer (cudaMalloc'd here, shared with the
// other ranks of the node through CUDA IPC handles):
//
//   [0, kHeaderBytes)   flags[kMaxCtas][kMaxRanks] (u32: epoch of the last push
//                       of CTA j's slice by rank src), epochs[kMaxCtas]
//   [kHeaderBytes, ...) recv[2][kMaxRanks][max_elems] fp32 (by epoch parity)
//
// CTA j of every rank handles the same slice of the [rows][dim] vector: it
// writes its rank's partial slice into recv[parity][my_rank] of every rank
// (plain peer stores, no multicast), fences, publishes its epoch in
// flags[j][my_rank] of every rank, waits (bounded) until flags[j][src] of its
// own buffer reach the epoch for every src, then adds the ranks' slices in rank
// order (so every rank computes bit-identical sums) to h.  The slices of one
// CTA never depend on another CTA, so there is no grid-wide synchronisation.
// Two receive buffers by epoch parity make reuse safe: a peer can only start
// push n+1 after it has consumed push n, which needed this rank's push n, and
// push n+2 needs this rank's push n+1, which comes after this rank's sum n.
#include <cstring>

#include "xm_gemv_dot.cuh"

namespace {

constexpr int kMaxRanks = 8;
constexpr int kMaxCtas = 32;
constexpr int kHeaderBytes = 4096;
static_assert(kMaxCtas * kMaxRanks * 4 + kMaxCtas * 4 <= kHeaderBytes, "header");
constexpr int kCommThreads = 256;

struct PeerTable {
  float* recv[kMaxRanks];        // each rank's recv base (parity 0, src 0)
  uint32_t* flags[kMaxRanks];    // each rank's flags[0][0]
};

constexpr uint64_t kDefaultWaitLimitNs = 2000000000ull;

XM_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

XM_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
XM_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(kCommThreads) k_allreduce_add(float* __restrict__ h,
                                                                const float* __restrict__ part, int64_t n_elems,
                                                                int64_t max_elems, int world, int rank,
                                                                PeerTable peers, uint32_t* __restrict__ my_flags,
                                                                uint32_t* __restrict__ my_epochs,
                                                                const float* __restrict__ my_recv,
                                                                uint64_t wait_limit_ns) {
  __shared__ uint32_t s_epoch;
  grid_dep_wait();
  const int j = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) s_epoch = my_epochs[j] + 1;
  __syncthreads();
  const uint32_t e = s_epoch;
  const int par = (int)(e & 1);
  // this CTA's slice, in float4 units (n_elems % 4 == 0)
  const int64_t n4 = n_elems / 4;
  const int64_t per = (n4 + gridDim.x - 1) / gridDim.x;
  const int64_t b4 = per * j, e4 = min(n4, b4 + per);
  const float4* src4 = reinterpret_cast<const float4*>(part);
  for (int r = 0; r < world; ++r) {
    float4* dst4 = reinterpret_cast<float4*>(peers.recv[r] + ((int64_t)par * kMaxRanks + rank) * max_elems);
    for (int64_t i = b4 + tid; i < e4; i += kCommThreads) dst4[i] = src4[i];
  }
  __syncthreads();
  if (tid < world) {
    __threadfence_system();   // this CTA's slice is visible on every rank before the flag
    st_release_sys(peers.flags[tid] + j * kMaxRanks + rank, e);
  }
  if (tid < world) {
    // bounded wait: a rank that never arrives costs the wait limit (2 s unless
    // set) and an error bit, not a hung GPU
    const uint32_t* f = my_flags + j * kMaxRanks + tid;
    const uint64_t t0 = globaltimer_ns();
    while ((int32_t)(ld_acquire_sys(f) - e) < 0) {
      if (globaltimer_ns() - t0 > wait_limit_ns) {
        atomicOr(&g_xm_device_error, XM_DEVERR_TIMEOUT);
        break;
      }
    }
  }
  __syncthreads();
  const float4* rv = reinterpret_cast<const float4*>(my_recv + (int64_t)par * kMaxRanks * max_elems);
  float4* h4 = reinterpret_cast<float4*>(h);
  for (int64_t i = b4 + tid; i < e4; i += kCommThreads) {
    float4 s = __ldcv(rv + i);
    for (int r = 1; r < world; ++r) {
      const float4 v = __ldcv(rv + (int64_t)r * (max_elems / 4) + i);
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
    float4 o = h4[i];
    o.x += s.x;
    o.y += s.y;
    o.z += s.z;
    o.w += s.w;
    h4[i] = o;
  }
  grid_dep_launch();
  if (tid == 0) my_epochs[j] = e;
}

struct Comm {
  int world = 0, rank = 0, nctas = 0;
  int64_t max_elems = 0;
  uint64_t wait_limit_ns = kDefaultWaitLimitNs;
  uint8_t* local = nullptr;            // this rank's buffer (owned)
  uint8_t* peer[kMaxRanks] = {};       // peer buffers: opened IPC mappings or in-process pointers
  bool ipc[kMaxRanks] = {};            // peer[r] is an IPC mapping (closed on destroy)
};

}  // namespace

extern "C" {

int64_t xm_comm_buffer_size(int64_t max_elems) {
  if (max_elems <= 0) return 0;
  const int64_t me = (max_elems + 3) / 4 * 4;
  return kHeaderBytes + 2LL * kMaxRanks * me * 4;
}

int xm_comm_create(int world, int rank, int64_t max_elems, int nctas, void** out_comm, void* out_handle) {
  if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || max_elems <= 0 || nctas < 1 ||
      nctas > kMaxCtas || !out_comm || !out_handle)
    return xm_set_error(XM_ERR_INVALID, "comm_create: bad arguments (world <= %d, ctas <= %d)", kMaxRanks, kMaxCtas);
  Comm* c = new Comm;
  c->world = world;
  c->rank = rank;
  c->nctas = nctas;
  c->max_elems = (max_elems + 3) / 4 * 4;
  const int64_t bytes = xm_comm_buffer_size(max_elems);
  cudaError_t e = cudaMalloc(&c->local, bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, bytes);
  cudaIpcMemHandle_t hd;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&hd, c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    return xm_set_error(XM_ERR_CUDA, "comm_create: %s", cudaGetErrorString(e));
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(out_handle, &hd, sizeof(hd));
  *out_comm = c;
  return XM_OK;
}

int xm_comm_open_peer(void* comm, int peer_rank, const void* handle) {
  Comm* c = (Comm*)comm;
  if (!c || peer_rank < 0 || peer_rank >= c->world || !handle)
    return xm_set_error(XM_ERR_INVALID, "comm_open_peer: bad arguments");
  if (peer_rank == c->rank) return XM_OK;
  cudaIpcMemHandle_t hd;
  memcpy(&hd, handle, sizeof(hd));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, hd, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "comm_open_peer(%d): %s", peer_rank, cudaGetErrorString(e));
  c->peer[peer_rank] = (uint8_t*)p;
  c->ipc[peer_rank] = true;
  return XM_OK;
}

int xm_comm_open_local(void* comm, int peer_rank, void* peer_comm) {
  Comm* c = (Comm*)comm;
  Comm* p = (Comm*)peer_comm;
  if (!c || !p || peer_rank < 0 || peer_rank >= c->world || p->world != c->world || p->rank != peer_rank ||
      p->max_elems != c->max_elems)
    return xm_set_error(XM_ERR_INVALID, "comm_open_local: the peer comm must be rank %d of the same shape", peer_rank);
  if (peer_rank == c->rank) return XM_OK;
  c->peer[peer_rank] = p->local;
  c->ipc[peer_rank] = false;
  return XM_OK;
}

int xm_comm_set_wait_limit(void* comm, int64_t limit_ns) {
  Comm* c = (Comm*)comm;
  if (!c || limit_ns < 1000 || limit_ns > 60000000000ll)
    return xm_set_error(XM_ERR_INVALID, "comm_set_wait_limit: limit outside 1 us .. 60 s");
  c->wait_limit_ns = (uint64_t)limit_ns;
  return XM_OK;
}

int xm_comm_destroy(void* comm) {
  Comm* c = (Comm*)comm;
  if (!c) return XM_OK;
  cudaError_t first = cudaSuccess;
  for (int r = 0; r < kMaxRanks; ++r)
    if (c->peer[r] && c->ipc[r]) {
      cudaError_t e = cudaIpcCloseMemHandle(c->peer[r]);
      if (first == cudaSuccess) first = e;
    }
  if (c->local) {
    cudaError_t e = cudaFree(c->local);
    if (first == cudaSuccess) first = e;
  }
  delete c;
  if (first != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "comm_destroy: %s", cudaGetErrorString(first));
  return XM_OK;
}

int xm_allreduce_add(void* comm, float* d_h, const float* d_part, int64_t n_elems, void* stream) {
  Comm* c = (Comm*)comm;
  if (!c || !d_h || !d_part) return xm_set_error(XM_ERR_INVALID, "allreduce_add: null argument");
  if (n_elems < 1 || n_elems > c->max_elems || n_elems % 4)
    return xm_set_error(XM_ERR_INVALID, "allreduce_add: %lld elements (multiple of 4, at most %lld)",
                        (long long)n_elems, (long long)c->max_elems);
  if (((uintptr_t)d_h & 15) || ((uintptr_t)d_part & 15))
    return xm_set_error(XM_ERR_INVALID, "allreduce_add: buffers must be 16-byte aligned");
  PeerTable t = {};
  for (int r = 0; r < c->world; ++r) {
    uint8_t* base = r == c->rank ? c->local : c->peer[r];
    if (!base) return xm_set_error(XM_ERR_INVALID, "allreduce_add: peer %d not opened", r);
    t.flags[r] = (uint32_t*)base;
    t.recv[r] = (float*)(base + kHeaderBytes);
  }
  uint32_t* flags = (uint32_t*)c->local;
  uint32_t* epochs = flags + kMaxCtas * kMaxRanks;
  const float* recv = (const float*)(c->local + kHeaderBytes);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)c->nctas);
  cfg.blockDim = dim3(kCommThreads);
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, k_allreduce_add, d_h, d_part, n_elems, c->max_elems, c->world, c->rank,
                                     t, flags, epochs, recv, c->wait_limit_ns);
  if (e != cudaSuccess) return xm_set_error(XM_ERR_CUDA, "allreduce_add launch: %s", cudaGetErrorString(e));
  return xm_check_launch("allreduce_add");
}

}  // extern "C"
