// bsa_forward_noalloc: the forward pass with a built-in scratch area.
//
// Some callers cannot allocate device memory at the point where they run the
// attention: code that runs under a memory pool it does not own, a host
// runtime whose allocator is locked while it dispatches work, or embedded
// integrations that were handed fixed input and output buffers only.  For
// them this entry point takes the workspace from a file-scope device array
// instead of a caller-provided buffer, and calls no allocator at all.
//
// Limits and sharing:
//  * The array holds kNoAllocScratchBytes (64 MiB).  Problems are processed
//    (batch * head) unit by unit in passes that fit it; a problem whose single
//    unit needs more is rejected with BSA_ERR_WORKSPACE.
//  * Every call on a device uses the same array, and the array keeps the last
//    call's contents.  The forward clears what must start at zero (its
//    error word and work-item counter) at the start of every pass, so
//    back-to-back calls are independent -- but two calls whose GPU work
//    overlaps (different streams, no ordering between them) race on the
//    array and produce garbage.
//  * Every GPU that loads this file's device code holds the array until the
//    process exits (with CUDA's default lazy module loading, from this entry
//    point's first call on that GPU).
//  * The first call on a device resolves the array's device address there
//    (cudaGetSymbolAddress, host-side set-up); make that first call before
//    any stream capture.
#include <cstdio>
#include <mutex>

#include "common.cuh"

namespace bsa {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void set_last_error_message(const char* msg);  // api.cu

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_dev_ptr[kMaxDevices] = {};
}  // namespace

}  // namespace bsa

using namespace bsa;

extern "C" {

int bsa_forward_noalloc(const bsa_problem* p, const void* Q, const void* K, const void* V,
                        void* O, void* stream) {
  int st = bsa_check_problem(p);
  if (st != BSA_OK) return st;
  const size_t need_one_unit = bsa_workspace_bytes(p, 1);
  if (need_one_unit > kNoAllocScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "bsa_forward_noalloc: one (batch, head) unit needs %zu bytes of scratch; "
             "the built-in scratch holds %zu (use bsa_forward with a workspace)",
             need_one_unit, kNoAllocScratchBytes);
    set_last_error_message(msg);
    return BSA_ERR_WORKSPACE;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    set_last_error_message("bsa_forward_noalloc: no usable current CUDA device");
    return BSA_ERR_CUDA;
  }
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    ptr = g_scratch_dev_ptr[dev];
    if (ptr == nullptr) {
      // Host code must not pass g_noalloc_scratch itself to a kernel: in host
      // code the name refers to a host-side stand-in, not device memory.
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        char msg[256];
        snprintf(msg, sizeof(msg), "bsa_forward_noalloc: cudaGetSymbolAddress failed: %s",
                 cudaGetErrorString(e));
        set_last_error_message(msg);
        return BSA_ERR_CUDA;
      }
      g_scratch_dev_ptr[dev] = ptr;
    }
  }
  return bsa_forward(p, Q, K, V, O, ptr, kNoAllocScratchBytes, stream);
}

}  // extern "C"
