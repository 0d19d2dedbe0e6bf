// Instantiations of the decode GEMV whose input is computed inside the launch (the input prologue of
// exl3_gemv_kernel.cuh): the rotation of x (exl3_gemv_rot) and SwiGLU + rotation of [gate | up]
// (exl3_gemv_swiglu, and exl3_gemv_swiglu_peer with the push into the tensor-parallel peers). Separate
// from exl3_gemv.cu so they compile in parallel.
#include "exl3_gemv_kernel.cuh"

namespace exl3 {

template int launch_gemv_epi<0, kProRot>(int, int, const GemvParams&, int, cudaStream_t);
template int launch_gemv_epi<0, kProSwiglu>(int, int, const GemvParams&, int, cudaStream_t);
template int launch_gemv_epi<2, kProSwiglu>(int, int, const GemvParams&, int, cudaStream_t);

}  // namespace exl3
