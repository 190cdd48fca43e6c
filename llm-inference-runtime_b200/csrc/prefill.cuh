// Ragged / chunked prefill attention over paged KV (sm_100a, tcgen05).
#pragma once

#include "pa_common.cuh"

namespace pa {

inline size_t prefill_workspace_bytes(int, int64_t, int, int, int) { return 0; }

inline int prefill_plan(const int32_t*, const int32_t*, const int32_t*, int, int64_t, int64_t, int,
                        int, int, int, void*, size_t, cudaStream_t) {
  return PA_ERR_UNSUPPORTED;
}

inline int prefill_run(const void*, int64_t, int64_t, const pa_kv_cache&, const int32_t*,
                       const int32_t*, const int32_t*, const int32_t*, int, int64_t, int, int,
                       float, void*, size_t, void*, float*, cudaStream_t) {
  return PA_ERR_UNSUPPORTED;
}

}  // namespace pa
