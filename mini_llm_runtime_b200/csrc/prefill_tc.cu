// tcgen05 causal chunk-prefill (BF16/F16, FP32 accumulation in TMEM).
#include "prefill_tc.cuh"

namespace pa {

bool prefill_tc_supported(const PrefillTcArgs&) { return false; }

int launch_prefill_tc(const PrefillTcArgs&, cudaStream_t) { return PA_ERR_UNSUPPORTED; }

}  // namespace pa
