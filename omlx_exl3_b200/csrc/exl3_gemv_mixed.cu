// Instantiations of the mixed-bitrate decode GEMV (members of one group quantised at different bpw in
// one launch), plain and with exl3_qkv_post's finish. Separate from exl3_gemv.cu so they compile in
// parallel.
#include "exl3_gemv_kernel.cuh"

namespace exl3 {

template int launch_gemv_seg<0>(int, const GemvParams&, int, int, cudaStream_t);
template int launch_gemv_seg<1>(int, const GemvParams&, int, int, cudaStream_t);

}  // namespace exl3
