// Library-wide C entry points: ABI version, status strings, device queries.
#include <atomic>
#include <mutex>

#include "pi_common.cuh"

namespace pi {

int device_sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

namespace {
std::atomic<int> g_programmatic{0};
std::atomic<int> g_attn_ring{PI_ATTN_RING_AUTO};
}  // namespace

bool programmatic_launch() { return g_programmatic.load(std::memory_order_relaxed) != 0; }

int decode_attn_ring() { return g_attn_ring.load(std::memory_order_relaxed); }

}  // namespace pi

extern "C" int pi_abi_version(void) { return 3; }

extern "C" int pi_set_programmatic_launch(int enable) {
  pi::g_programmatic.store(enable ? 1 : 0, std::memory_order_relaxed);
  return PI_OK;
}

extern "C" int pi_set_decode_attn_ring(int mode) {
  if (mode != PI_ATTN_RING_AUTO && mode != PI_ATTN_RING_DEEP && mode != PI_ATTN_RING_SHALLOW)
    return PI_ERR_BAD_SHAPE;
  pi::g_attn_ring.store(mode, std::memory_order_relaxed);
  return PI_OK;
}

extern "C" const char* pi_error_string(int code) {
  switch (code) {
    case PI_OK: return "ok";
    case PI_ERR_NULL_POINTER: return "null pointer argument";
    case PI_ERR_BAD_SHAPE: return "invalid shape or size argument";
    case PI_ERR_MISALIGNED: return "pointer or stride not aligned as required";
    case PI_ERR_UNSUPPORTED: return "unsupported dtype or shape combination";
    case PI_ERR_CUDA: return "CUDA runtime error at launch";
    case PI_ERR_WORKSPACE: return "workspace missing or too small";
    case PI_ERR_SLOT_RANGE: return "slot index outside the page pool (write skipped)";
    case PI_ERR_PAGE_RANGE: return "page id outside the page pool (read skipped)";
    case PI_ERR_TIMEOUT: return "bounded device wait expired";
    case PI_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than the allocation-free entry point's built-in "
             "array (PI_NOALLOC_SCRATCH_BYTES); use pi_paged_decode_attn with a workspace";
    default: return "unknown status code";
  }
}
