// Instances of the norm-family kernels: __nv_bfloat16, epilogues 10..14.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__nv_bfloat16, 10)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 11)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 12)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 13)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 14)
}  // namespace b2k
