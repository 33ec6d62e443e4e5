// Instances of the norm-family kernels for __half: ln_b.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, NM_LN, 10)
B2K_NORM_INSTANTIATE(__half, NM_LN, 11)
B2K_NORM_INSTANTIATE(__half, NM_LN, 12)
B2K_NORM_INSTANTIATE(__half, NM_LN, 13)
B2K_NORM_INSTANTIATE(__half, NM_LN, 14)
B2K_NORM_INSTANTIATE(__half, NM_LN, 15)
B2K_NORM_INSTANTIATE(__half, NM_LN, 16)
B2K_NORM_INSTANTIATE(__half, NM_LN, 17)
B2K_NORM_INSTANTIATE(__half, NM_LN, 18)
B2K_NORM_INSTANTIATE(__half, NM_LN, 19)
}  // namespace b2k
