// prefill_tc.cu -- tcgen05/TMEM tensor-core chunked prefill (bf16 inputs, D = 64).
#include "prefill.cuh"

namespace pma {

bool tc_supported(int, int) { return false; }

cudaError_t launch_prefill_tc(const PrefillParams &, int, dim3, cudaStream_t) { return cudaErrorNotSupported; }

}  // namespace pma
