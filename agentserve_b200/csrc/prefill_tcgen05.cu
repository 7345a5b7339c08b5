// (4) Varlen prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
#include "common.cuh"
#include "host_util.h"
#include "prefill_tcgen05.h"

namespace asb {

bool prefill_tc_supported(int, int, int, int, const void*, int64_t, const void*, const void*,
                          const void*) {
  return false;
}

int prefill_tc_launch(void*, const void*, int64_t, const void*, const void*, const int32_t*,
                      int64_t, const int32_t*, const int32_t*, int, int, int, int, int, int, int,
                      int, float, int, cudaStream_t) {
  return fail(AS_ERR_UNSUPPORTED, "tcgen05 prefill not available");
}

}  // namespace asb
