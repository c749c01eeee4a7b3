// prefill_tc.cu -- placeholder until the tcgen05 prefill kernel lands.
#include "host_util.h"
#include "kernels.h"

namespace b200 {
bool prefill_tc_supported(const b200_prefill_args_t&) { return false; }
int launch_prefill_tc(const b200_prefill_args_t*, int64_t, cudaStream_t) {
  return fail(B200_ERR_UNSUPPORTED, "tensor-core prefill not built");
}
}  // namespace b200
