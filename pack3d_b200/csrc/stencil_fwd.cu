// Tensor-core fused forward on complete voxel stencils (placeholder until the
// tcgen05 kernel lands): reports "unsupported" so the indexed path runs.
#include "kernels.cuh"

namespace p3d {
bool stencil_fwd_supported(int, int, const int *, int) { return false; }
int launch_stencil_fwd(const StencilFwdArgs &, cudaStream_t) {
  return fail(P3D_ERR_UNSUPPORTED, "tensor-core stencil forward not built");
}
}  // namespace p3d
