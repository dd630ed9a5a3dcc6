// Peer-memory exchange of finished parameter shards (sharded Muon step).
//
// After a rank has applied the updates of the matrices it owns, every other
// rank needs the new values. Instead of a library all-gather, each rank keeps
// a full replica of the flat, rank-major parameter buffer of every shape
// group in memory that the other ranks map through CUDA IPC, and stores its
// own shard straight into each peer's replica at the same byte offset:
//
//     peer q:  base_q + off  <-  base_self + off   for off in own shard
//
// The store kernel holds no shared memory and few registers per CTA, so its
// CTAs sit next to the persistent GEMM CTAs (one per SM, ~226 KB of shared
// memory each) and the transfer overlaps the next group's Newton–Schulz
// launches without taking SMs away from them. Each thread loads a 16-byte
// vector once from local HBM and issues one NVLink store per peer, in the
// order the caller lists the peers (rank + 1, rank + 2, ... modulo the world,
// so that at any moment the ranks' destinations form a permutation and no
// receiver is the target of every sender at once).
//
// No multicast object and no bulk-copy engine is involved: plain st.global to
// peer addresses opened with cudaIpcOpenMemHandle. Completion of the stores
// at the receivers is established by the caller with a barrier after the
// kernel (the stores are fenced system-wide before each thread exits).
#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int kPushThreads = 256;

int launch_status() { return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH; }

struct PeerDeltas {
  long long d[LSR_MAX_PEERS];  // byte distance from the local address to the peer's replica
};

__device__ __forceinline__ uint4 ld_stream16(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st16(void* p, const uint4& v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

// body: 16-byte aligned local address, n16 16-byte vectors; head / tail: the
// 2-byte elements before and after the aligned body (at most 7 each).
__global__ void __launch_bounds__(kPushThreads) peer_push_kernel(const uint8_t* body, long long n16,
                                                                 const uint16_t* head, int nhead,
                                                                 const uint16_t* tail, int ntail, PeerDeltas pd,
                                                                 int npeers) {
  constexpr int U = 4;  // vectors in flight per thread
  const long long tid = (long long)blockIdx.x * kPushThreads + threadIdx.x;
  const long long nthr = (long long)gridDim.x * kPushThreads;
  const uint4* src = reinterpret_cast<const uint4*>(body);
  uint8_t* self = const_cast<uint8_t*>(body);
  long long i = tid;
  for (; i + (U - 1) * nthr < n16; i += U * nthr) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) v[u] = ld_stream16(src + i + u * nthr);
#pragma unroll
    for (int k = 0; k < LSR_MAX_PEERS; ++k) {
      if (k >= npeers) break;
      const long long d = pd.d[k];
#pragma unroll
      for (int u = 0; u < U; ++u) st16(self + (i + u * nthr) * 16 + d, v[u]);
    }
  }
  for (; i < n16; i += nthr) {
    const uint4 v = ld_stream16(src + i);
#pragma unroll
    for (int k = 0; k < LSR_MAX_PEERS; ++k) {
      if (k >= npeers) break;
      st16(self + i * 16 + pd.d[k], v);
    }
  }
  if (blockIdx.x == 0 && threadIdx.x < 8) {
#pragma unroll
    for (int k = 0; k < LSR_MAX_PEERS; ++k) {
      if (k >= npeers) break;
      if ((int)threadIdx.x < nhead) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(const_cast<uint16_t*>(head)) + pd.d[k]);
        dst[threadIdx.x] = head[threadIdx.x];
      }
      if ((int)threadIdx.x < ntail) {
        uint16_t* dst = reinterpret_cast<uint16_t*>(reinterpret_cast<uint8_t*>(const_cast<uint16_t*>(tail)) + pd.d[k]);
        dst[threadIdx.x] = tail[threadIdx.x];
      }
    }
  }
  __threadfence_system();
}

}  // namespace
}  // namespace lsr

using namespace lsr;

extern "C" {

int lsr_ipc_alloc(size_t bytes, void** ptr, void* handle) {
  if (!ptr || !handle || bytes == 0) return LSR_ERR_ARG;
  *ptr = nullptr;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return LSR_ERR_PEER;
  }
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(p);
    return LSR_ERR_PEER;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == LSR_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *ptr = p;
  return LSR_OK;
}

int lsr_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return LSR_ERR_ARG;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
    cudaGetLastError();
    return LSR_ERR_PEER;
  }
  *ptr = p;
  return LSR_OK;
}

int lsr_ipc_close(void* ptr) {
  if (!ptr) return LSR_ERR_ARG;
  if (cudaIpcCloseMemHandle(ptr) != cudaSuccess) {
    cudaGetLastError();
    return LSR_ERR_PEER;
  }
  return LSR_OK;
}

int lsr_ipc_free(void* ptr) {
  if (!ptr) return LSR_ERR_ARG;
  if (cudaFree(ptr) != cudaSuccess) {
    cudaGetLastError();
    return LSR_ERR_PEER;
  }
  return LSR_OK;
}

int lsr_peer_push(const void* src, size_t bytes, const long long* peer_deltas, int npeers, int max_ctas,
                  lsr_stream_t stream) {
  if (npeers < 0 || npeers > LSR_MAX_PEERS || (npeers > 0 && !peer_deltas) || (bytes & 1)) return LSR_ERR_ARG;
  if (bytes == 0 || npeers == 0) return LSR_OK;
  if (!src || (reinterpret_cast<uintptr_t>(src) & 1)) return LSR_ERR_ARG;
  PeerDeltas pd{};
  for (int q = 0; q < npeers; ++q) {
    // a replica shares the local buffer's alignment (both are allocation bases plus the same offset)
    if (peer_deltas[q] & 15) return LSR_ERR_ARG;
    pd.d[q] = peer_deltas[q];
  }
  int rc = check_device();
  if (rc) return rc;
  const uintptr_t s = reinterpret_cast<uintptr_t>(src);
  const uintptr_t body = (s + 15) & ~uintptr_t(15);
  const uintptr_t end = s + bytes;
  int nhead = 0, ntail = 0;
  long long n16 = 0;
  uintptr_t tail = end;
  if (body >= end) {
    nhead = (int)((end - s) / 2);  // fewer than 16 bytes, none of them on an aligned vector
  } else {
    nhead = (int)((body - s) / 2);
    n16 = (long long)((end - body) / 16);
    tail = body + (uintptr_t)n16 * 16;
    ntail = (int)((end - tail) / 2);
  }
  const int sms = device_sm_count();
  int ctas = max_ctas > 0 ? max_ctas : sms;
  const long long need = (n16 + kPushThreads - 1) / kPushThreads;
  if (need < ctas) ctas = (int)(need > 0 ? need : 1);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ProfScope prof(PK_PEER_PUSH, st);
  peer_push_kernel<<<ctas, kPushThreads, 0, st>>>(reinterpret_cast<const uint8_t*>(body), n16,
                                                  reinterpret_cast<const uint16_t*>(s), nhead,
                                                  reinterpret_cast<const uint16_t*>(tail), ntail, pd, npeers);
  return launch_status();
}

}  // extern "C"
