// Instances of the norm-family kernels: __nv_bfloat16, epilogues 15..19.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__nv_bfloat16, 15)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 16)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 17)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 18)
B2K_NORM_INSTANTIATE(__nv_bfloat16, 19)
}  // namespace b2k
