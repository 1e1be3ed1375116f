// Tensor-core (tcgen05/TMEM/TMA) DC-attention forward — placeholder until the
// kernel lands; AUTO dispatch uses the SIMT kernel meanwhile.
#include <cuda_runtime.h>

#include <string>

#include "common.cuh"

namespace dcattn {

bool tc_supports(const dc_attn_params &p, std::string *why) {
  (void)p;
  if (why) *why = "tensor-core kernel not built";
  return false;
}

cudaError_t launch_tc(const dc_attn_params &p, cudaStream_t st) {
  (void)p; (void)st;
  return cudaErrorNotSupported;
}

}  // namespace dcattn
