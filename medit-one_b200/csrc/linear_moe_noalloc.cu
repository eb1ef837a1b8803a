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
void* g_scratch_addr[kMaxDevices] = {};
std::mutex g_scratch_mu;

// Device address of the scratch on the current device; looked up once per device, with that
// device current, on the first call made there.
int scratch_on_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return one_set_error(ONE_ERR_CUDA, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return one_set_error(ONE_ERR_UNSUPPORTED, "device index out of range");
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      char msg[256];
      snprintf(msg, sizeof(msg), "cudaGetSymbolAddress(scratch): %s", cudaGetErrorString(e));
      return one_set_error(ONE_ERR_CUDA, msg);
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
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
