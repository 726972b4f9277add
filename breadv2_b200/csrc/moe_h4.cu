// moe_h4.cu -- step kernel instantiations for H = 1024 (moe_kernel.cuh).
#include "moe_kernel.cuh"

namespace bread {
template int step_launch_h<4>(StepArgs &a, cudaStream_t s, int nbi);
template int step_setup_h<4>(int nbi);
}  // namespace bread
