// Multivariate Hawkes event update (hawkes_dense_kernel / hawkes_kron_kernel,
// hft.py:412-611): every stream n decays its excitation state and adds the
// column of the excitation matrix K that its event selects,
//   dense: out[n][j] = decay[n] state[n][j] + Kcol[event[n]][j]      (Kcol = K^T, [D][D])
//   kron : out[n][j] = decay[n] state[n][j] + KA[j / NE][ea[n]] KE[j % NE][et[n]]
//          (K = KA ⊗ KE, D = NA NE, never formed)
// HBM-bound: 8 bytes per state entry (read state, write out) plus the K column
// (dense: D floats per stream, mostly from L2; kron: the row's column of KA
// and of KE, NA + NE floats staged once per row in the warp's shared memory).
// One warp per stream row: the row moves as 16-byte vectors, 512 contiguous
// bytes per warp instruction; the stream's event and decay are loaded once per
// row. An event index outside [0, D) (dense) or [0, NA) x [0, NE) (kron) is
// not read: the row is written as NaN and ST_EVENT_INDEX is recorded in the
// device status word.
#include <atomic>

#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int HK_THREADS = 256;
constexpr int HK_WARPS = HK_THREADS / 32;
constexpr int ST_EVENT_INDEX = 110;

__device__ __forceinline__ bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Shared floats per warp for the staged Kronecker path (0: factors too large, gather instead).
__host__ __device__ __forceinline__ int hsm_floats_per_warp(int na, int ne) {
  return (long long)na + ne <= 2048 ? na + ne : 0;
}

template <bool KRON>
__global__ void __launch_bounds__(HK_THREADS) hawkes_kernel(const float* __restrict__ state,
                                                            const int* __restrict__ event,
                                                            const int* __restrict__ event_type,
                                                            const float* __restrict__ decay,
                                                            const float* __restrict__ K0,
                                                            const float* __restrict__ K1, float* __restrict__ out,
                                                            int n, int d, int na, int ne, int* status) {
  extern __shared__ float hsm[];  // kron: per warp, the row's KA column (na) and KE column (ne)
  const int lane = threadIdx.x & 31;
  const bool vec = (d % 4 == 0) && al16(state) && al16(out) && (KRON || al16(K0));
  const bool staged = KRON && hsm_floats_per_warp(na, ne) > 0;
  float* wa = staged ? hsm + (threadIdx.x >> 5) * (na + ne) : nullptr;
  float* we = staged ? wa + na : nullptr;
  for (long long row = (long long)blockIdx.x * HK_WARPS + (threadIdx.x >> 5); row < n;
       row += (long long)gridDim.x * HK_WARPS) {
    const float dec = __ldg(decay + row);
    const int e0 = __ldg(event + row);
    const int e1 = KRON ? __ldg(event_type + row) : 0;
    const bool ok = KRON ? (e0 >= 0 && e0 < na && e1 >= 0 && e1 < ne) : (e0 >= 0 && e0 < d);
    const float* s = state + row * d;
    float* o = out + row * d;
    if (!ok) {
      if (lane == 0) set_status(status, ST_EVENT_INDEX);
      for (int j = lane; j < d; j += 32) o[j] = __int_as_float(0x7fc00000);
      continue;
    }
    if (staged) {
      // column e0 of KA and column e1 of KE, once per row; then every entry is two shared reads.
      // The row's first 1024 state entries are requested before the columns are gathered, so
      // their DRAM latency overlaps the gather.
      constexpr int HK_PRE = 8;  // 16-byte vectors per lane issued ahead
      float4 svp[HK_PRE];
      if (vec) {
#pragma unroll
        for (int u = 0; u < HK_PRE; ++u) {
          const int j = 4 * lane + 128 * u;
          if (j < d) svp[u] = __ldcs(reinterpret_cast<const float4*>(s + j));
        }
      }
      __syncwarp();  // the previous row's reads of wa / we are done
      for (int a = lane; a < na; a += 32) wa[a] = __ldg(K0 + (long long)a * na + e0);
      for (int e = lane; e < ne; e += 32) we[e] = __ldg(K1 + (long long)e * ne + e1);
      __syncwarp();
      if (vec) {
        for (int j = 4 * lane, u = 0; j < d; j += 128, ++u) {
          float4 sv;
          if (u < HK_PRE) {
#pragma unroll
            for (int q = 0; q < HK_PRE; ++q)
              if (q == u) sv = svp[q];
          } else {
            sv = __ldcs(reinterpret_cast<const float4*>(s + j));
          }
          float k[4];
          int a = j / ne, e = j - a * ne;
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            k[t] = wa[a] * we[e];
            if (++e == ne) {
              e = 0;
              ++a;
            }
          }
          __stcs(reinterpret_cast<float4*>(o + j), make_float4(fmaf(dec, sv.x, k[0]), fmaf(dec, sv.y, k[1]),
                                                               fmaf(dec, sv.z, k[2]), fmaf(dec, sv.w, k[3])));
        }
      } else {
        for (int j = lane; j < d; j += 32) {
          const int a = j / ne, e = j - a * ne;
          o[j] = fmaf(dec, s[j], wa[a] * we[e]);
        }
      }
      continue;
    }
    if (!KRON && vec) {
      // dense: each 1024-entry segment of the row and of the K column is loaded in full before
      // any of it is stored (safe with out == state: every entry is read before it is written),
      // so eight 16-byte vectors of each are in flight per lane
      const float* kc = K0 + (long long)e0 * d;
      constexpr int HD = 8;
      for (int j0 = 0; j0 < d; j0 += 128 * HD) {
        float4 sv[HD], kv[HD];
#pragma unroll
        for (int u = 0; u < HD; ++u) {
          const int j = j0 + 4 * lane + 128 * u;
          if (j < d) {
            sv[u] = __ldcs(reinterpret_cast<const float4*>(s + j));
            kv[u] = __ldg(reinterpret_cast<const float4*>(kc + j));
          }
        }
#pragma unroll
        for (int u = 0; u < HD; ++u) {
          const int j = j0 + 4 * lane + 128 * u;
          if (j < d)
            __stcs(reinterpret_cast<float4*>(o + j),
                   make_float4(fmaf(dec, sv[u].x, kv[u].x), fmaf(dec, sv[u].y, kv[u].y),
                               fmaf(dec, sv[u].z, kv[u].z), fmaf(dec, sv[u].w, kv[u].w)));
        }
      }
    } else if (vec) {
      const float* kc = KRON ? nullptr : K0 + (long long)e0 * d;
      for (int j = 4 * lane; j < d; j += 128) {
        const float4 sv = __ldcs(reinterpret_cast<const float4*>(s + j));
        float4 kv;
        if constexpr (KRON) {
          // column j of KA ⊗ KE at event (e0, e1): KA[j / NE][e0] KE[j % NE][e1]
          float k[4];
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int jj = j + t, a = jj / ne, b = jj - a * ne;
            k[t] = __ldg(K0 + (long long)a * na + e0) * __ldg(K1 + (long long)b * ne + e1);
          }
          kv = make_float4(k[0], k[1], k[2], k[3]);
        } else {
          kv = __ldg(reinterpret_cast<const float4*>(kc + j));
        }
        __stcs(reinterpret_cast<float4*>(o + j), make_float4(fmaf(dec, sv.x, kv.x), fmaf(dec, sv.y, kv.y),
                                                             fmaf(dec, sv.z, kv.z), fmaf(dec, sv.w, kv.w)));
      }
    } else {
      for (int j = lane; j < d; j += 32) {
        float k;
        if constexpr (KRON) {
          const int a = j / ne, b = j - a * ne;
          k = __ldg(K0 + (long long)a * na + e0) * __ldg(K1 + (long long)b * ne + e1);
        } else {
          k = __ldg(K0 + (long long)e0 * d + j);
        }
        o[j] = fmaf(dec, s[j], k);
      }
    }
  }
}

template <bool KRON>
int launch_hawkes(const float* state, const int* event, const int* event_type, const float* decay, const float* K0,
                  const float* K1, float* out, int n, int d, int na, int ne, cudaStream_t st) {
  if (n == 0) return LSR_OK;
  int* status = status_ptr();
  if (!status) return LSR_ERR_LAUNCH;
  const long long rows_per_wave = (long long)HK_WARPS * 8 * device_sm_count();
  const int blocks = (int)std::min<long long>((n + HK_WARPS - 1) / HK_WARPS, rows_per_wave / HK_WARPS);
  const size_t smem = KRON ? (size_t)HK_WARPS * hsm_floats_per_warp(na, ne) * sizeof(float) : 0;
  if (smem > 48 * 1024) {
    static std::atomic<int> attr_set{0};
    if (!attr_set.load(std::memory_order_relaxed)) {
      if (cudaFuncSetAttribute(hawkes_kernel<KRON>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               HK_WARPS * 2048 * (int)sizeof(float)) != cudaSuccess)
        return LSR_ERR_LAUNCH;
      attr_set.store(1, std::memory_order_relaxed);
    }
  }
  ProfScope prof(PK_EW_OTHER, st);
  hawkes_kernel<KRON><<<blocks, HK_THREADS, smem, st>>>(state, event, event_type, decay, K0, K1, out, n, d, na, ne,
                                                        status);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

}  // namespace
}  // namespace lsr

extern "C" {

int lsr_hawkes_dense_f32(const float* state, const int* event, const float* decay, const float* kcol, float* out,
                         int n, int d, lsr_stream_t stream) {
  if (n < 0 || d <= 0) return LSR_ERR_ARG;
  if (n > 0 && (!state || !event || !decay || !kcol || !out)) return LSR_ERR_ARG;
  int rc = lsr::check_device();
  if (rc) return rc;
  return lsr::launch_hawkes<false>(state, event, nullptr, decay, kcol, nullptr, out, n, d, 0, 0,
                                   reinterpret_cast<cudaStream_t>(stream));
}

int lsr_hawkes_kron_f32(const float* state, const int* event_asset, const int* event_type, const float* decay,
                        const float* ka, const float* ke, float* out, int n, int na, int ne, lsr_stream_t stream) {
  if (n < 0 || na <= 0 || ne <= 0 || (long long)na * ne > (1LL << 30)) return LSR_ERR_ARG;
  if (n > 0 && (!state || !event_asset || !event_type || !decay || !ka || !ke || !out)) return LSR_ERR_ARG;
  int rc = lsr::check_device();
  if (rc) return rc;
  return lsr::launch_hawkes<true>(state, event_asset, event_type, decay, ka, ke, out, n, na * ne, na, ne,
                                  reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
