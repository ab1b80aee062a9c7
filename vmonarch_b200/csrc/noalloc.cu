// vmb_fea_bwd_noalloc: the FlashEntropyAttention backward for callers that cannot allocate device
// memory.
//
// vmb_fea_bwd needs a caller-provided scratch workspace (fp32 per-row statistics: three folded
// planes on the tcgen05 path; on the mma.sync path two constants and, when the gradients are
// written in bf16/fp16, an fp32 dQ accumulator). Some hosts cannot hand one over:
// an engine plugin whose enqueue hook must not allocate because the host framework owns every
// device buffer, a foreign-language binding that can only pass the tensors the user gave it, or a
// latency-critical pipeline where a cudaMalloc (and the device-wide synchronisation it can imply)
// is not acceptable inside the step. For them this entry point takes its scratch from a
// fixed-size array compiled into the library instead.
//
// Limits and contract:
//  - The scratch is kNoAllocScratchBytes (32 MiB) per device, a static __device__ array: every GPU
//    on which the library's module is loaded holds it until the process exits. Calls whose
//    minimal workspace (vmb_fea_bwd_min_workspace_bytes) exceeds it are rejected with
//    VMB_EINVAL; a call whose preferred workspace (with the dS^T buffer of the dQ-from-dS route)
//    also fits takes that route, otherwise the dQ kernel that recomputes S and dP.
//  - The first call on a device looks the array's device address up (cudaGetSymbolAddress) with
//    that device current; make that first call before any stream capture begins. The address is
//    cached per device ordinal for the life of the process, so the entry point must not be used
//    after cudaDeviceReset (which unloads the module and frees the array) or from a context other
//    than the device's primary context.
//  - All calls share the one array and it keeps the previous call's contents; the backward clears
//    what must start at zero (the dQ accumulator) on every call. Calls whose work overlaps on the
//    GPU (different streams, or different host threads on the same device) race on the array and
//    must be serialised by the caller.
//  - No cudaMalloc, cudaFree or allocating library routine is called.
#include <mutex>

#include "../../include/vmonarch_b200.h"
#include "launch.h"

namespace {

constexpr int64_t kNoAllocScratchBytes = int64_t(32) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return vmb::set_error(VMB_ECUDA, "vmb_fea_bwd_noalloc: cudaGetDevice failed");
  if (dev < 0 || dev >= kMaxDevices) return vmb::set_error(VMB_EINVAL, "vmb_fea_bwd_noalloc: device index out of range");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return vmb::set_error(VMB_ECUDA, "vmb_fea_bwd_noalloc: cudaGetSymbolAddress failed");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return VMB_OK;
}

}  // namespace

extern "C" int vmb_fea_bwd_noalloc(const vmb_fea_bwd_args* a, void* stream) {
  if (!a) return vmb::set_error(VMB_EINVAL, "vmb_fea_bwd_noalloc: null args");
  // the minimum; a call whose optional dS^T buffer also fits the scratch takes that route
  const int64_t need = vmb::fea_bwd_min_workspace_bytes(a);
  if (need < 0) return vmb::set_error(VMB_EINVAL, "vmb_fea_bwd_noalloc: bad sizes");
  if (need > kNoAllocScratchBytes)
    return vmb::set_error(VMB_EINVAL,
                          "vmb_fea_bwd_noalloc: this call needs %lld bytes of scratch but the built-in "
                          "scratch holds %lld; use vmb_fea_bwd with a caller-provided workspace",
                          (long long)need, (long long)kNoAllocScratchBytes);
  void* scratch = nullptr;
  const int rc = scratch_address(&scratch);
  if (rc != VMB_OK) return rc;
  vmb_fea_bwd_args b = *a;
  b.workspace = scratch;
  b.workspace_bytes = kNoAllocScratchBytes;
  return vmb_fea_bwd(&b, stream);
}
