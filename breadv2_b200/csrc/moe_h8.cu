// moe_h8.cu -- step kernel instantiations for H = 2048 (moe_kernel.cuh).
#include "moe_kernel.cuh"

namespace bread {
template int step_launch_h<8>(StepArgs &a, cudaStream_t s, int nbi);
template int step_setup_h<8>(int nbi);
}  // namespace bread
