// ssa_sm100_bwd.cu — SSA attention backward for sm_100a (tcgen05/TMA); not yet enabled.
#include "ssa_internal.h"

namespace ssa {

bool sm100_bwd_supports(int dtype, int D) {
  (void)dtype;
  (void)D;
  return false;
}

size_t sm100_bwd_workspace_bytes(const Problem& p) {
  (void)p;
  return 0;
}

int launch_bwd_sm100(int dtype, const Problem& p, TensorRef q, TensorRef k, TensorRef v,
                     TensorRef dout, const float* lse, const float* delta, TensorRef dq,
                     TensorRef dk, TensorRef dv, float* dn, float* db, void* ws, size_t ws_bytes,
                     cudaStream_t st) {
  return SSA_ERR_UNSUPPORTED;
}

}  // namespace ssa
