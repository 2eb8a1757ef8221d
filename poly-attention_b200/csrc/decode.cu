// KV-cache decode pass (few query rows against a long cache), HBM-bound.
#include "common.cuh"

namespace poly {

bool pass_decode_eligible(const PolyPassArgs&) { return false; }
int launch_pass_decode(const PolyPassArgs&, cudaStream_t) { return POLY_EUNSUPPORTED; }
size_t pass_decode_workspace(const PolyPassArgs&) { return 0; }

}  // namespace poly
