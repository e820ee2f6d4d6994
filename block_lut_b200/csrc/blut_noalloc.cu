// blut_moe_forward_noalloc: the MoE layer forward for callers that cannot
// allocate device memory at the point of the call -- for example a plugin
// that a host framework calls with nothing but its input and output
// pointers (the framework owns every allocation), or a serving loop that
// must not call cudaMalloc because of its implicit device synchronisation.
//
// The scratch the forward needs lives in one file-scope device array of
// kNoAllocScratchBytes (16 MiB).  Each GPU holds that array from the
// library's first use there (from load time with eager module loading)
// until the process exits.  The launches are exactly those of
// blut_moe_forward; only the scratch comes from the array instead of a
// caller workspace.  The array's first word is the device status word, which
// blut_moe_check_status(NULL, stream) reads back.
#include <mutex>

#include "blut_common.cuh"
#include "blut_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

// Device scratch shared by every call of blut_moe_forward_noalloc on a GPU.
static __device__ __align__(256) unsigned char g_moe_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_moe_scratch on the current device.  In host code the
// symbol's name only stands in for the array, so the address is asked from
// the runtime, once per device, with that device current.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return BLUT_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_moe_scratch) != cudaSuccess || !p) return BLUT_ERR_CUDA;
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return BLUT_OK;
}

}  // namespace

namespace blut {
// Address of the current device's no-allocation scratch (its first word is
// the device status of the last blut_moe_forward_noalloc call there).
int noalloc_scratch(void** out) { return scratch_for_current_device(out); }
}  // namespace blut

extern "C" {

BLUT_API int blut_moe_forward_noalloc(const blut_moe_args* args, void* stream) {
  if (!args) return BLUT_ERR_INVALID;
  const int rc = blut::validate_moe(*args);
  if (rc != BLUT_OK) return rc;
  // the layer's scratch must fit the fixed array
  if (blut::moe_workspace(*args, nullptr, nullptr) > kNoAllocScratchBytes) return BLUT_ERR_WORKSPACE;
  void* scratch = nullptr;
  const int sc = scratch_for_current_device(&scratch);
  if (sc != BLUT_OK) return sc;
  // Everything the kernels read from the scratch is written earlier in the
  // same call; the one word that must start at zero, the device status, is
  // cleared by the plan kernel at the start of every call.
  return blut::moe_forward(*args, scratch, kNoAllocScratchBytes, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
