// Instances of the norm-family kernels: __nv_bfloat16, epilogues 0..4.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__nv_bfloat16, 0)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 1)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 2)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 3)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 4)
}  // namespace b2k
