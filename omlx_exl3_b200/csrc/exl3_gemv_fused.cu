// Instantiations of the decode GEMV with fused finishes: exl3_qkv_post's (1) and the LL push into the
// tensor-parallel peers' inboxes (2). Separate from exl3_gemv.cu so the two compile in parallel.
#include "exl3_gemv_kernel.cuh"

namespace exl3 {

template int launch_gemv_epi<1>(int, int, const GemvParams&, int, cudaStream_t);
template int launch_gemv_epi<2>(int, int, const GemvParams&, int, cudaStream_t);

}  // namespace exl3
