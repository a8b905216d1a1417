// Split-TF32 GEMM on the sm_100a tensor cores (tcgen05 + TMEM + TMA).
// Placeholder until the tensor-core kernel lands: no shape is routed here.
#include "tl_common.cuh"

namespace tl {

bool gemm_tc_ok(int, int, int64_t, int64_t, int64_t, const float*, int64_t, const float*, int64_t,
                const float*, int64_t) {
  return false;
}

int gemm_tc(int, int, int64_t, int64_t, int64_t, const float*, int64_t, const float*, int64_t,
            float*, int64_t, const float*, int, int, cudaStream_t) {
  return TL_ERR_UNSUPPORTED;
}

}  // namespace tl
