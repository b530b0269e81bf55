// Chunked-prefill paged causal attention (placeholder until the tensor-core kernel lands).
#include "pkv_common.cuh"

extern "C" int pkv_paged_prefill(const void*, int64_t, int64_t, const int32_t*, int64_t, int64_t, const void*,
                                 const void*, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                 const void*, int64_t, int64_t, const void*, int, int64_t, int64_t, float, void*,
                                 int64_t, int64_t, int, int32_t*, void*) {
  pkv::set_error("paged_prefill: not implemented");
  return PKV_ERR_UNSUPPORTED;
}
