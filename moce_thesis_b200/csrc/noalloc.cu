// moce_gate_route_noalloc: the gate-route forward for callers that cannot
// allocate device memory.
//
// Some hosts of this layer cannot call cudaMalloc at the point of the call.
// Examples are plugins inside an inference engine that gives them a fixed
// device-memory budget and no allocator, and latency-critical paths that
// cannot accept the device-wide synchronisation cudaMalloc may perform.
// moce_gate_route needs a caller-provided workspace (per-sample temperatures,
// pooled means, converted indices); this variant uses a fixed scratch array
// that lives in the library instead.
//
// Scratch: kNoAllocScratchBytes (4 MiB) in a file-scope __device__ array.
// Every GPU that loads the library holds this array until the process exits.
// Shapes whose workspace (moce_gate_route_workspace_bytes) exceeds it are
// rejected with MOCE_ERR_UNSUPPORTED.
//
// All calls share the one array and nothing in it needs to start at zero:
// each call writes every scratch byte it reads.  Calls that overlap on the
// GPU (two streams, or two host threads, at once) race on the array and must
// be serialised by the caller.
#include <mutex>

#include "common.cuh"

namespace moce {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

// In host code this name is only a host-side stand-in for the symbol, not a
// device address: a kernel given it would fault, or (where the GPU can reach
// host memory) silently use the wrong memory.  Host code must use the device
// address returned by cudaGetSymbolAddress (scratch_ptr below).  Device code
// in this file could name the array directly.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once
// per device with that device current.
int scratch_ptr(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return set_error(MOCE_ERR_CUDA, "moce_gate_route_noalloc: no current CUDA device");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    const cudaError_t err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (err != cudaSuccess || !p)
      return set_error(MOCE_ERR_CUDA, "moce_gate_route_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(err));
    g_ptr[dev] = p;
  }
  *out = g_ptr[dev];
  return MOCE_OK;
}

}  // namespace
}  // namespace moce

using namespace moce;

extern "C" size_t moce_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int moce_gate_route_noalloc(const void* x, int dtype, const float* pooled, const void* indices,
                                       int index_bits, const float* logits_norm, const float* gate_w,
                                       const float* gate_b, const int32_t* mask, float temp_min, float temp_max,
                                       float tau, void* y, int64_t B, int64_t C, int64_t HW, int64_t E_r,
                                       int64_t K, void* stream) {
  if (B == 0) return MOCE_OK;
  MOCE_REQUIRE(B > 0 && C >= 1 && E_r >= 1, MOCE_ERR_INVALID, "moce_gate_route_noalloc: invalid shape");
  const size_t need = moce_gate_route_workspace_bytes(B, C, E_r);
  MOCE_REQUIRE(need <= kNoAllocScratchBytes, MOCE_ERR_UNSUPPORTED,
               "moce_gate_route_noalloc: this shape needs %zu bytes of scratch, more than the %zu bytes the "
               "library reserves (B=%lld C=%lld E_r=%lld); use moce_gate_route with a caller workspace",
               need, kNoAllocScratchBytes, (long long)B, (long long)C, (long long)E_r);
  void* scratch = nullptr;
  const int rc = scratch_ptr(&scratch);
  if (rc) return rc;
  return moce_gate_route(x, dtype, pooled, indices, index_bits, logits_norm, gate_w, gate_b, mask, temp_min,
                         temp_max, tau, y, B, C, HW, E_r, K, scratch, kNoAllocScratchBytes, stream);
}
