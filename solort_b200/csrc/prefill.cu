// Causal GQA prefill on tcgen05 (sm_100a). Status word of this translation unit.
#include "common.cuh"
#include "host_util.h"

namespace solort {

__device__ unsigned g_prefill_status;

int read_prefill_status(unsigned* flags) {
  unsigned v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_prefill_status, sizeof(v)) != cudaSuccess) return SOLORT_ERR_CUDA;
  if (v && cudaMemcpyToSymbol(g_prefill_status, &zero, sizeof(zero)) != cudaSuccess)
    return SOLORT_ERR_CUDA;
  *flags |= v;
  return SOLORT_OK;
}

}  // namespace solort
