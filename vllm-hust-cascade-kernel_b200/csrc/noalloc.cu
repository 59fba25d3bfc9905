// Allocation-free variant of the suffix decode entry point.
//
// cascade_suffix_decode() needs a device workspace for its split-KV partials,
// which the caller allocates. Some callers cannot allocate device memory at
// the point where they run the attention step: a C or Go host that binds the
// C ABI without any device allocator of its own, or a serving loop whose
// memory must be fixed before it starts replaying captured work. For them,
// cascade_suffix_decode_noalloc() takes only inputs and outputs and keeps the
// partials in a fixed scratch array compiled into this library
// (kScratchBytes, 16 MiB). Every GPU that loads the library reserves that
// array until the process exits.
//
// In host code `g_noalloc_scratch` names a host-side stand-in, not device
// memory, so its device address is resolved with cudaGetSymbolAddress on
// each device (with that device current) the first time the entry point runs
// there, and that address is what the kernels receive. Only a successful
// lookup is remembered: a failed one is reported to that caller and tried
// again on the next call.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/cascade_b200.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_addr[kMaxDevices];  // null until the lookup succeeded on that device

// Device address of the scratch array on the current device `dev`, or null
// with *err set when the lookup fails.
void* scratch_address(int dev, cudaError_t* err) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  *err = cudaSuccess;
  if (g_scratch_addr[dev] != nullptr) return g_scratch_addr[dev];
  void* ptr = nullptr;
  *err = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (*err != cudaSuccess || ptr == nullptr) {
    if (*err == cudaSuccess) *err = cudaErrorInvalidSymbol;
    cudaGetLastError();  // the failure is returned to this caller, not left for the next CUDA call
    return nullptr;
  }
  g_scratch_addr[dev] = ptr;
  return ptr;
}

}  // namespace

extern "C" int cascade_suffix_decode_noalloc(const cascade_paged_attn_t* p, void* out, float* lse,
                                             cascade_stream_t stream) {
  const char* op = "cascade_suffix_decode_noalloc";
  char msg[256];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    snprintf(msg, sizeof(msg), "%s: no usable current CUDA device", op);
    return cascade::set_error(CASCADE_ERR_CUDA, msg);
  }
  void* scratch = scratch_address(dev, &e);
  if (scratch == nullptr) {
    snprintf(msg, sizeof(msg), "%s: cudaGetSymbolAddress of the scratch array failed (%s)", op,
             cudaGetErrorString(e));
    return cascade::set_error(CASCADE_ERR_CUDA, msg);
  }
  if (p == nullptr) return cascade::set_error(CASCADE_ERR_INVALID, "cascade_suffix_decode_noalloc: null argument");
  if (p->q_seqlen_value <= 0) {
    // the per-request q-length path reads the seqlens back into host buffers
    return cascade::set_error(CASCADE_ERR_INVALID,
                              "cascade_suffix_decode_noalloc: needs q_seqlen_value > 0 (uniform q length)");
  }
  const size_t need = cascade_suffix_decode_workspace_size(p);
  if (need > kScratchBytes) {
    snprintf(msg, sizeof(msg),
             "%s: this call needs %zu bytes of split scratch, above the fixed %zu-byte maximum; "
             "use cascade_suffix_decode with a caller workspace",
             op, need, kScratchBytes);
    return cascade::set_error(CASCADE_ERR_UNSUPPORTED, msg);
  }
  return cascade_suffix_decode(p, out, lse, need ? scratch : nullptr, need ? kScratchBytes : 0, stream);
}
