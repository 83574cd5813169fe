// Placeholder for the tensor-core kernels while they are being written.
#include "launchers.cuh"

namespace bsa {

bool select_tc_supported(const Shape&) { return false; }
cudaError_t launch_select_tc(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                             int32_t*, const Shape&, cudaStream_t) {
  return cudaErrorNotSupported;
}
bool fine_kv_supported(const Shape&) { return false; }
size_t fine_kv_workspace_bytes(const Shape&) { return 0; }
cudaError_t launch_fine_kv(const __nv_bfloat16*, const __nv_bfloat16*, const __nv_bfloat16*,
                           const int32_t*, __nv_bfloat16*, unsigned char*, const Shape&,
                           cudaStream_t, int*, void* const*, int) {
  return cudaErrorNotSupported;
}

}  // namespace bsa
