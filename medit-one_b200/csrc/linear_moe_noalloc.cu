// one_linear_moe_noalloc: the LinearMoE operator for callers that cannot allocate device
// memory.
//
// one_linear_moe needs a device workspace (the clamped input copy, the gate logits and the
// combined inputs). Some callers have no way to provide one: a host program that binds this
// library through a foreign-function interface and only ever holds the device pointers it is
// handed (it owns no CUDA allocator), or a process whose device memory is entirely owned by
// another runtime's pool, where an extra cudaMalloc would fail or break that pool's
// accounting. For them this entry point runs the same operator on a fixed scratch array that
// is part of the library image: every GPU that loads the library holds
// ONE_NOALLOC_SCRATCH_BYTES of device memory for it until the process exits, and no call
// allocates or frees anything.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/one_b200.h"

extern "C" __attribute__((visibility("hidden"))) int one_set_error(int code, const char* msg);

namespace {

// The shared scratch. Host code must not use this symbol as an address: it names a host-side
// stand-in. The device address comes from cudaGetSymbolAddress, per device.
__device__ __align__(256) unsigned char g_noalloc_scratch[ONE_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
struct ScratchSlot {
  void* addr;
  unsigned long long ctx_id;  // the CUDA context the address belongs to (0 = unknown)
};
ScratchSlot g_scratch[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Unique id of the calling thread's current CUDA context (cuCtxGetId, never reused within the
// process), or 0 when it cannot be read. A cudaDeviceReset destroys the context that the cached
// address belongs to; the next context has a new id, so the address is looked up again.
unsigned long long current_context_id() {
  typedef CUresult (*GetCurrentFn)(CUcontext*);
  typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
  static GetCurrentFn get_current = nullptr;
  static GetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetIdFn>(p);
  });
  if (!get_current || !get_id) return 0;
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS) return 0;
  return id;
}

// Device address of the scratch on the current device. Looked up (cudaGetSymbolAddress) with
// that device current on the first call made there, and again whenever the device's context
// changed since (after a cudaDeviceReset); otherwise the cached address is returned.
int scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return one_set_error(ONE_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return one_set_error(ONE_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ScratchSlot& slot = g_scratch[dev];
  const unsigned long long ctx = slot.addr ? current_context_id() : 0;
  if (!slot.addr || ctx == 0 || ctx != slot.ctx_id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      char msg[256];
      snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
      return one_set_error(ONE_ERR_CUDA, msg);
    }
    slot.addr = p;
    slot.ctx_id = current_context_id();  // the lookup made the device's context current
  }
  *out = slot.addr;
  return ONE_OK;
}

}  // namespace

extern "C" int one_linear_moe_noalloc(const void* x, int32_t n, int32_t fin, int32_t fout, const void* weight,
                                      const void* bias, const void* gate_w, const void* experts, const void* bias2,
                                      int32_t num_experts, int32_t r, int32_t top_k, int32_t dtype, void* out,
                                      int32_t* idx_out, void* stream) {
  if (n < 1 || fin < 1 || r < 1) return one_set_error(ONE_ERR_INVALID, "one_linear_moe_noalloc: sizes must be positive");
  const size_t need = one_linear_moe_workspace_bytes(n, fin, r, dtype);
  if (need > (size_t)ONE_NOALLOC_SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "one_linear_moe_noalloc: %d tokens x %d inputs need %zu bytes of scratch, more than the %d-byte static "
             "scratch; split the call or use one_linear_moe with a workspace",
             (int)n, (int)fin, need, (int)ONE_NOALLOC_SCRATCH_BYTES);
    return one_set_error(ONE_ERR_INVALID, msg);
  }
  void* scratch = nullptr;
  const int rc = scratch_on_current_device(&scratch);
  if (rc != ONE_OK) return rc;
  // Nothing in the scratch has to start at zero: the operator writes every byte it reads
  // (clamped inputs, gate logits, combined inputs) before reading it.
  return one_linear_moe(x, n, fin, fout, weight, bias, gate_w, experts, bias2, num_experts, r, top_k, dtype, out,
                        idx_out, scratch, (size_t)ONE_NOALLOC_SCRATCH_BYTES, stream);
}
