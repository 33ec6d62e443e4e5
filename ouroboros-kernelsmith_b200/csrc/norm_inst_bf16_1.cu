// Instances of the norm-family kernels: __nv_bfloat16, epilogues 5..9.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__nv_bfloat16, 5)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 6)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 7)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 8)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 9)
}  // namespace b2k
