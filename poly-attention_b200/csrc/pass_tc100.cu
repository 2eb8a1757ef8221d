// tcgen05 / TMEM / TMA kernels for one poly-attention pass (sm_100a).
#include "common.cuh"

namespace poly {

bool pass_fwd_tc_eligible(const PolyPassArgs&) { return false; }
int launch_pass_fwd_tc(const PolyPassArgs&, cudaStream_t) { return POLY_EUNSUPPORTED; }
size_t pass_fwd_tc_workspace(const PolyPassArgs&) { return 0; }
bool pass_bwd_tc_eligible(const PolyPassBwdArgs&) { return false; }
int launch_pass_bwd_tc(const PolyPassBwdArgs&, cudaStream_t) { return POLY_EUNSUPPORTED; }
size_t pass_bwd_tc_workspace(const PolyPassBwdArgs&) { return 0; }

}  // namespace poly
