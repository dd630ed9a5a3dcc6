// Pauli-string Hamiltonian applied to a state vector (pauli_partial_kernel /
// pauli_reduce_kernel / native_apply, pauli.py:296-578), without forming H:
//   out[r] = sum_s coeff_s i^{ny_s} (-1)^{popcount((r ^ flip_s) & sign_s)} psi[r ^ flip_s]
// over N = 2^K amplitudes (complex, as separate real / imaginary fp32 arrays)
// and S strings encoded as bit masks (flip: X or Y on qubit k, sign: Y or Z,
// ny: number of Y factors mod 4; pauli.py:159-199).
//
// One thread computes one output amplitude over a slice of the strings; a
// block holds 256 / SPLIT consecutive outputs x SPLIT slices of the string
// list, and the slices are summed in a fixed order at the end (SPLIT grows for
// small N so that every SM has work; no partial arrays in global memory and a
// single launch). The strings are staged in shared memory in chunks, each with
// its phase folded into one complex weight w = coeff i^{ny}. The 32 lanes of a
// warp take 32 consecutive outputs of one slice: r ^ flip permutes each aligned
// 32-block, so every amplitude read of a warp is one coalesced 128-byte segment
// (the state, at most a few MB for the reference's sizes, stays in L2).
#include "runtime.cuh"

namespace lsr {
namespace {

constexpr int PA_THREADS = 256;
constexpr int PA_CHUNK = 1024;  // strings staged per pass

struct PauliTerm {
  unsigned flip, sign;
  float wr, wi;  // coeff i^{ny}
};

__global__ void __launch_bounds__(PA_THREADS) pauli_apply_kernel(const float* __restrict__ psi_r,
                                                                 const float* __restrict__ psi_i,
                                                                 const int* __restrict__ flip,
                                                                 const int* __restrict__ sign,
                                                                 const int* __restrict__ ny,
                                                                 const float* __restrict__ coeff,
                                                                 float* __restrict__ out_r, float* __restrict__ out_i,
                                                                 unsigned n, int S, int split) {
  __shared__ PauliTerm terms[PA_CHUNK];
  __shared__ float2 part[PA_THREADS];
  const int per = PA_THREADS / split;  // outputs per block
  const int o = threadIdx.x % per, q = threadIdx.x / per;
  const unsigned r = blockIdx.x * (unsigned)per + (unsigned)o;
  const bool live = r < n;
  const unsigned mask = n - 1;  // n is a power of two
  float ar = 0.f, ai = 0.f;
  for (int c0 = 0; c0 < S; c0 += PA_CHUNK) {
    const int cn = min(PA_CHUNK, S - c0);
    __syncthreads();  // the previous chunk's terms have been read
    for (int t = threadIdx.x; t < cn; t += PA_THREADS) {
      const float cf = __ldg(coeff + c0 + t);
      const int ph = __ldg(ny + c0 + t) & 3;  // i^0, i^1, i^2, i^3 = 1, i, -1, -i
      PauliTerm pt;
      pt.flip = (unsigned)__ldg(flip + c0 + t) & mask;
      pt.sign = (unsigned)__ldg(sign + c0 + t);
      pt.wr = ph == 0 ? cf : (ph == 2 ? -cf : 0.f);
      pt.wi = ph == 1 ? cf : (ph == 3 ? -cf : 0.f);
      terms[t] = pt;
    }
    __syncthreads();
    // this thread's slice of the chunk: [t0, t1)
    const int t0 = (int)((long long)cn * q / split), t1 = (int)((long long)cn * (q + 1) / split);
    if (live) {
      int t = t0;
      for (; t + 4 <= t1; t += 4) {
        float xr[4], xi[4];
        unsigned cc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          cc[u] = r ^ terms[t + u].flip;
          xr[u] = __ldg(psi_r + cc[u]);
          xi[u] = __ldg(psi_i + cc[u]);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const PauliTerm pt = terms[t + u];
          const float sg = (__popc(cc[u] & pt.sign) & 1) ? -1.f : 1.f;
          const float wr = sg * pt.wr, wi = sg * pt.wi;
          ar = fmaf(wr, xr[u], fmaf(-wi, xi[u], ar));
          ai = fmaf(wr, xi[u], fmaf(wi, xr[u], ai));
        }
      }
      for (; t < t1; ++t) {
        const PauliTerm pt = terms[t];
        const unsigned cc = r ^ pt.flip;
        const float xr = __ldg(psi_r + cc), xi = __ldg(psi_i + cc);
        const float sg = (__popc(cc & pt.sign) & 1) ? -1.f : 1.f;
        const float wr = sg * pt.wr, wi = sg * pt.wi;
        ar = fmaf(wr, xr, fmaf(-wi, xi, ar));
        ai = fmaf(wr, xi, fmaf(wi, xr, ai));
      }
    }
  }
  part[threadIdx.x] = make_float2(ar, ai);
  __syncthreads();
  if (q == 0 && live) {
    float sr = 0.f, si = 0.f;
    for (int k = 0; k < split; ++k) {
      const float2 v = part[k * per + o];
      sr += v.x;
      si += v.y;
    }
    out_r[r] = sr;
    out_i[r] = si;
  }
}

}  // namespace
}  // namespace lsr

extern "C" {

int lsr_pauli_apply_f32(const float* psi_r, const float* psi_i, const int* flip, const int* sign, const int* ny,
                        const float* coeff, float* out_r, float* out_i, int K, int S, lsr_stream_t stream) {
  if (K < 0 || K > 30 || S < 0) return LSR_ERR_ARG;
  if (!psi_r || !psi_i || !out_r || !out_i || (S > 0 && (!flip || !sign || !ny || !coeff))) return LSR_ERR_ARG;
  int rc = lsr::check_device();
  if (rc) return rc;
  const unsigned n = 1u << K;
  // slices of the string list per output: enough blocks for two per SM, each slice >= 16 strings
  int split = 1;
  const long long want = 2LL * lsr::device_sm_count();
  while (split < 32 && (long long)(n * (unsigned long long)split + lsr::PA_THREADS - 1) / lsr::PA_THREADS < want &&
         S / (2 * split) >= 16)
    split *= 2;
  const int per = lsr::PA_THREADS / split;
  const unsigned blocks = (n + per - 1) / per;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  lsr::ProfScope prof(lsr::PK_EW_OTHER, st);
  lsr::pauli_apply_kernel<<<blocks, lsr::PA_THREADS, 0, st>>>(psi_r, psi_i, flip, sign, ny, coeff, out_r, out_i, n, S,
                                                             split);
  return cudaGetLastError() == cudaSuccess ? LSR_OK : LSR_ERR_LAUNCH;
}

}  // extern "C"
