// moe_h2.cu -- step kernel instantiations for H = 512 (moe_kernel.cuh).
#include "moe_kernel.cuh"

namespace bread {
template int step_launch_h<2>(StepArgs &a, cudaStream_t s, int nbi);
template int step_setup_h<2>(int nbi);
}  // namespace bread
