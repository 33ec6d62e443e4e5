// Instances of the norm-family kernels for __nv_bfloat16: spec.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__nv_bfloat16, NM_RMS_WROUND, 0)
B2K_NORM_INSTANTIATE(__nv_bfloat16, NM_RMS_1PW, 0)
B2K_NORM_INSTANTIATE(__nv_bfloat16, NM_L2, 0)
}  // namespace b2k
