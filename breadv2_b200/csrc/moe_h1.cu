// moe_h1.cu -- step kernel instantiations for H = 256 (moe_kernel.cuh).
#include "moe_kernel.cuh"

namespace bread {
template int step_launch_h<1>(StepArgs &a, cudaStream_t s, int nbi);
template int step_setup_h<1>(int nbi);
}  // namespace bread
