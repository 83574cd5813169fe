// Stage dispatch: the tensor-core kernels for the shapes they cover, the
// CUDA-core kernels for every other valid shape (or when a flag forces them).
#include "launchers.cuh"

namespace bsa {

bool select_uses_tensor_cores(const Shape& s, uint32_t flags) {
  return !(flags & BSA_FLAG_SIMT_SELECT) && select_tc_supported(s);
}

bool fine_uses_tensor_cores(const Shape& s, uint32_t flags) {
  return !(flags & BSA_FLAG_SIMT_FINE) && fine_kv_supported(s);
}

cudaError_t launch_select(const __nv_bfloat16* Q, const float* K_repr, const __nv_bfloat16* K_hi,
                          const __nv_bfloat16* K_lo, int32_t* idx, uint32_t* err, const Shape& s,
                          uint32_t flags, cudaStream_t st, int* n_launches) {
  *n_launches = 1;
  if (select_uses_tensor_cores(s, flags) && K_hi != nullptr)
    return launch_select_tc(Q, K_hi, K_lo, idx, err, s, st);
  return launch_select_simt(Q, K_repr, idx, s, st);
}

size_t fine_workspace_bytes(const Shape& s, uint32_t flags) {
  return fine_uses_tensor_cores(s, flags) ? fine_kv_workspace_bytes(s) : 0;
}

cudaError_t launch_fine(const __nv_bfloat16* Q, const __nv_bfloat16* K, const __nv_bfloat16* V,
                        const int32_t* idx, __nv_bfloat16* O, unsigned char* ws, size_t ws_bytes,
                        const Shape& s, uint32_t flags, cudaStream_t st, int* n_launches,
                        void* const* events, int n_events, bool pre_zeroed) {
  if (fine_uses_tensor_cores(s, flags) && ws_bytes >= fine_kv_workspace_bytes(s))
    return launch_fine_kv(Q, K, V, idx, O, ws, s, flags, st, n_launches, events, n_events,
                          pre_zeroed);
  // The CUDA-core path has no bucket or combine kernel: it is all "fine".
  *n_launches = 1;
  if (events != nullptr && n_events > 2 && events[2] != nullptr)
    cudaEventRecord((cudaEvent_t)events[2], st);
  cudaError_t e = launch_fine_simt(Q, K, V, idx, O, s, st);
  if (events != nullptr) {
    for (int i = 3; i < n_events && i < 5; ++i)
      if (events[i] != nullptr) cudaEventRecord((cudaEvent_t)events[i], st);
  }
  return e;
}

}  // namespace bsa
