// Varlen causal prefill engine (placeholder until the tcgen05 engine lands).
#include "common.cuh"
#include "kernels.h"

namespace fp8attn {
cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t stream) {
  (void)p;
  (void)stream;
  return cudaErrorNotSupported;
}
}  // namespace fp8attn
