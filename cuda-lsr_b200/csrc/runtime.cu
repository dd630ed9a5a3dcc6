// Library runtime: version, error strings, device status word, TMA tensor-map
// encoding through the driver entry point (no link-time libcuda dependency).
#include <atomic>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "runtime.cuh"

namespace lsr {

// Device status word: 0 = no failure; otherwise the first failure code a
// kernel recorded (e.g. a bounded wait that timed out).
__device__ int g_status_word;

// Tile counters of the GEMM engine's dynamic scheduler: two words per launch
// slot, zero between launches (the last CTA of each launch resets its slot).
// Launches take slots round-robin, so launches running at the same time (on
// different streams) use different counters as long as fewer than
// kSchedSlots are in flight.
constexpr int kSchedSlots = 1024;
__device__ unsigned int g_tile_sched[2 * kSchedSlots];

namespace {
constexpr int kMaxDevices = 64;
// Per-device caches filled on first use. Atomic (relaxed): host threads that
// fill the same entry at once look up and store the same value.
std::atomic<int*> g_status_cache[kMaxDevices] = {};
std::atomic<unsigned int*> g_sched_cache[kMaxDevices] = {};
std::atomic<unsigned int> g_sched_next{0};
std::atomic<int> g_sm_cache[kMaxDevices] = {};
std::atomic<int> g_cc_cache[kMaxDevices] = {};

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
std::atomic<EncodeTiledFn> g_encode{nullptr};

int current_device() {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDevices) return -1;
  return d;
}
std::atomic<long long> g_launches{0};

struct ProfRec {
  int kind;
  cudaEvent_t a, b;
};
std::atomic<bool> g_prof_on{false};
std::mutex g_prof_mu;
std::vector<ProfRec> g_prof_open;   // begun, waiting for end (per kind, last one)
std::vector<ProfRec> g_prof_done;
std::vector<cudaEvent_t> g_prof_pool;

cudaEvent_t take_event() {
  if (!g_prof_pool.empty()) {
    cudaEvent_t e = g_prof_pool.back();
    g_prof_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}
}  // namespace

void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void prof_begin(int kind, cudaStream_t st) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  ProfRec r{kind, take_event(), nullptr};
  if (r.a) cudaEventRecord(r.a, st);
  g_prof_open.push_back(r);
}

void prof_end(int kind, cudaStream_t st) {
  if (!g_prof_on.load(std::memory_order_relaxed)) return;
  std::lock_guard<std::mutex> lk(g_prof_mu);
  for (size_t i = g_prof_open.size(); i-- > 0;) {
    if (g_prof_open[i].kind != kind) continue;
    ProfRec r = g_prof_open[i];
    g_prof_open.erase(g_prof_open.begin() + (long)i);
    r.b = take_event();
    if (r.b) cudaEventRecord(r.b, st);
    g_prof_done.push_back(r);
    return;
  }
}

int* status_ptr() {
  const int d = current_device();
  if (d < 0) return nullptr;
  int* s = g_status_cache[d].load(std::memory_order_relaxed);
  if (!s) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_status_word) != cudaSuccess) return nullptr;
    s = static_cast<int*>(p);
    g_status_cache[d].store(s, std::memory_order_relaxed);
  }
  return s;
}

unsigned int* sched_slot() {
  const int d = current_device();
  if (d < 0) return nullptr;
  unsigned int* base = g_sched_cache[d].load(std::memory_order_relaxed);
  if (!base) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tile_sched) != cudaSuccess) return nullptr;
    base = static_cast<unsigned int*>(p);
    g_sched_cache[d].store(base, std::memory_order_relaxed);
  }
  const unsigned int k = g_sched_next.fetch_add(1, std::memory_order_relaxed) % kSchedSlots;
  return base + 2 * k;
}

int device_sm_count() {
  const int d = current_device();
  if (d < 0) return 1;
  int n = g_sm_cache[d].load(std::memory_order_relaxed);
  if (!n) {
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
    n = n > 0 ? n : 1;
    g_sm_cache[d].store(n, std::memory_order_relaxed);
  }
  return n;
}

int check_device() {
  const int d = current_device();
  if (d < 0) return LSR_ERR_DEVICE;
  int major = g_cc_cache[d].load(std::memory_order_relaxed);
  if (!major) {
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d) != cudaSuccess) return LSR_ERR_DEVICE;
    g_cc_cache[d].store(major, std::memory_order_relaxed);
  }
  return major == 10 ? LSR_OK : LSR_ERR_DEVICE;
}

namespace {
EncodeTiledFn encode_fn() {
  EncodeTiledFn encode = g_encode.load(std::memory_order_relaxed);
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return nullptr;
    encode = reinterpret_cast<EncodeTiledFn>(fn);
    g_encode.store(encode, std::memory_order_relaxed);
  }
  return encode;
}
}  // namespace

int encode_tmap_k_blocks(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                         uint64_t block, uint64_t rows, uint64_t nblocks, uint64_t batch, uint64_t ld,
                         uint64_t bstride, uint32_t box_rows, uint32_t box_blocks) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return LSR_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * elem_bytes) & 15) || ((bstride * elem_bytes) & 15) ||
      ((block * elem_bytes) & 15))
    return LSR_ERR_SHAPE;
  // dims: element within a K block (contiguous), row, K block, batch
  cuuint64_t dims[4] = {block, rows, nblocks, batch};
  cuuint64_t strides[3] = {ld * elem_bytes, block * elem_bytes, bstride * elem_bytes};
  cuuint32_t box[4] = {(cuuint32_t)block, box_rows, box_blocks, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LSR_OK : LSR_ERR_DRIVER;
}

int encode_tmap_mn_chunks(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base,
                          uint64_t chunk, uint64_t krows, uint64_t nchunks, uint64_t batch, uint64_t ld,
                          uint64_t bstride, uint32_t box_chunks, uint32_t box_krows) {
  EncodeTiledFn encode = encode_fn();
  if (!encode) return LSR_ERR_DRIVER;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * elem_bytes) & 15) || ((bstride * elem_bytes) & 15) ||
      ((chunk * elem_bytes) & 15))
    return LSR_ERR_SHAPE;
  // dims: element within a chunk (contiguous), K row, chunk, batch
  cuuint64_t dims[4] = {chunk, krows, nchunks, batch};
  cuuint64_t strides[3] = {ld * elem_bytes, chunk * elem_bytes, bstride * elem_bytes};
  cuuint32_t box[4] = {(cuuint32_t)chunk, box_krows, box_chunks, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode(map, dtype, 4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LSR_OK : LSR_ERR_DRIVER;
}

int encode_tmap_3d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner,
                   uint64_t outer, uint64_t batch, uint64_t ld, uint64_t bstride, uint32_t box_inner,
                   uint32_t box_outer, CUtensorMapSwizzle swizzle) {
  EncodeTiledFn encode = g_encode.load(std::memory_order_relaxed);
  if (!encode) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
            cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return LSR_ERR_DRIVER;
    encode = reinterpret_cast<EncodeTiledFn>(fn);
    g_encode.store(encode, std::memory_order_relaxed);
  }
  // TMA requirements: 16-byte aligned base and strides.
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * elem_bytes) & 15) || ((bstride * elem_bytes) & 15))
    return LSR_ERR_SHAPE;
  cuuint64_t dims[3] = {inner, outer, batch};
  cuuint64_t strides[2] = {ld * elem_bytes, bstride * elem_bytes};
  cuuint32_t box[3] = {box_inner, box_outer, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode(map, dtype, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LSR_OK : LSR_ERR_DRIVER;
}

}  // namespace lsr

extern "C" {

const char* lsr_version(void) { return "lsr-b200 0.1.0 (sm_100a)"; }

const char* lsr_strerror(int code) {
  switch (code) {
    case LSR_OK: return "ok";
    case LSR_ERR_ARG: return "invalid argument";
    case LSR_ERR_SHAPE: return "unsupported shape, stride or alignment";
    case LSR_ERR_WORKSPACE: return "workspace missing or too small";
    case LSR_ERR_LAUNCH: return "kernel launch failed";
    case LSR_ERR_DRIVER: return "TMA tensor map encoding failed";
    case LSR_ERR_DEVICE: return "current device is not an sm_100 (B200-class) GPU";
    case LSR_ERR_TOO_LARGE: return "problem exceeds the fixed scratch capacity of the allocation-free entry point";
    case LSR_ERR_PEER: return "CUDA IPC / peer memory call failed";
    default: return "unknown liblsr error";
  }
}

long long lsr_launch_count(void) { return lsr::g_launches.load(); }

int lsr_profile_enable(int on) {
  lsr::g_prof_on.store(on != 0);
  return LSR_OK;
}

int lsr_profile_read(double* ms, long long* launches, int nkinds, int reset) {
  if (nkinds < 0 || (nkinds > 0 && (!ms || !launches))) return LSR_ERR_ARG;
  for (int k = 0; k < nkinds; ++k) {
    ms[k] = 0.0;
    launches[k] = 0;
  }
  std::lock_guard<std::mutex> lk(lsr::g_prof_mu);
  for (const auto& r : lsr::g_prof_done) {
    float t = 0.f;
    if (r.a && r.b && cudaEventSynchronize(r.b) == cudaSuccess && cudaEventElapsedTime(&t, r.a, r.b) == cudaSuccess &&
        r.kind < nkinds) {
      ms[r.kind] += t;
      launches[r.kind] += 1;
    }
  }
  if (reset) {
    for (auto& r : lsr::g_prof_done) {
      if (r.a) lsr::g_prof_pool.push_back(r.a);
      if (r.b) lsr::g_prof_pool.push_back(r.b);
    }
    lsr::g_prof_done.clear();
  }
  return LSR_OK;
}

int lsr_device_status(int* code, int clear) {
  if (!code) return LSR_ERR_ARG;
  int* p = lsr::status_ptr();
  if (!p) return LSR_ERR_DEVICE;
  if (cudaDeviceSynchronize() != cudaSuccess) return LSR_ERR_LAUNCH;
  if (cudaMemcpy(code, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return LSR_ERR_LAUNCH;
  if (clear && cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return LSR_ERR_LAUNCH;
  return LSR_OK;
}

}  // extern "C"
