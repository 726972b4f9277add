// moe_h16.cu -- step kernel instantiations for H = 4096 (moe_kernel.cuh).
#include "moe_kernel.cuh"

namespace bread {
template int step_launch_h<16>(StepArgs &a, cudaStream_t s, int nbi);
template int step_setup_h<16>(int nbi);
}  // namespace bread
