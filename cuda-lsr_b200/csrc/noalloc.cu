// Allocation-free Newton–Schulz entry point.
//
// Some callers cannot call cudaMalloc: a host program that embeds the
// optimizer next to a framework whose caching allocator owns all device
// memory and offers no hook for foreign scratch requests, or a latency-bound
// caller that cannot afford the implicit device synchronisation cudaMalloc /
// cudaFree may perform in the middle of an asynchronous stream pipeline. For
// them lsr_ns_bf16_noalloc runs the same kernels as lsr_ns_bf16 with its
// scratch in the fixed device array below instead of a caller workspace.
//
// Properties of that array, by design:
//   * its size is fixed at LSR_NOALLOC_SCRATCH_BYTES (24 MiB) and every GPU
//     that loads this library holds it until the process exits;
//   * every call shares it and it keeps the last call's contents (the
//     Newton–Schulz stages overwrite everything they later read, so nothing
//     needs clearing between calls); calls whose work overlaps on the GPU
//     (different streams, or different host threads on the same device) race
//     on it — callers must order them;
//   * its device address is looked up once per device, on the first call made
//     with that device current; make that first call before any stream
//     capture.
#include <atomic>

#include "runtime.cuh"

#define LSR_NOALLOC_SCRATCH_BYTES (24u << 20)

namespace lsr {

int ns_bf16_fixed_scratch(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a,
                          float b, float c, float eps, uint8_t* scratch, cudaStream_t st);

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[LSR_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDev = 64;
// Per-device cache of the array's device address. Atomic so that host threads
// making their first call on one device at the same time do not race; both
// look the address up and store the same value.
std::atomic<uint8_t*> g_scratch_addr[kMaxDev] = {};

// Device address of the scratch array for the current device (nullptr on failure).
uint8_t* scratch_for_current_device() {
  int d = -1;
  if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= kMaxDev) return nullptr;
  uint8_t* addr = g_scratch_addr[d].load(std::memory_order_relaxed);
  if (!addr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || !ptr) return nullptr;
    addr = static_cast<uint8_t*>(ptr);
    g_scratch_addr[d].store(addr, std::memory_order_relaxed);
  }
  return addr;
}

}  // namespace
}  // namespace lsr

extern "C" {

size_t lsr_ns_noalloc_capacity(void) { return LSR_NOALLOC_SCRATCH_BYTES; }

int lsr_ns_bf16_noalloc(const void* in, void* out, int batch, int rows, int cols, int orient, int steps, float a,
                        float b, float c, float eps, lsr_stream_t stream) {
  if (batch < 0 || rows <= 0 || cols <= 0 || steps < 0 || batch > 65535) return LSR_ERR_ARG;
  if (batch == 0) return LSR_OK;
  if (!in || !out) return LSR_ERR_ARG;
  int rc = lsr::check_device();
  if (rc) return rc;
  if (lsr_ns_workspace_bytes(batch, rows, cols, orient) > LSR_NOALLOC_SCRATCH_BYTES) return LSR_ERR_TOO_LARGE;
  uint8_t* scratch = lsr::scratch_for_current_device();
  if (!scratch) return LSR_ERR_DEVICE;
  return lsr::ns_bf16_fixed_scratch(in, out, batch, rows, cols, orient, steps, a, b, c, eps, scratch,
                                    reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
