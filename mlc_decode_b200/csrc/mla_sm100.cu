// tcgen05/TMA/TMEM split-KV decode kernel (sm_100a).
#include "mla_sm100.cuh"

namespace mla {

bool sm100_supports(int, int) { return false; }

SplitPlan sm100_plan(int, int, int seqlen_kv, const MlaCfg&, int* variant) {
  *variant = 0;
  return split_plan(seqlen_kv, 1, 128, false);
}

cudaError_t launch_sm100_decode(const DecodeArgs&, int) { return cudaErrorNotSupported; }

}  // namespace mla
