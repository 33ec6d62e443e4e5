// Instances of the norm-family kernels for __half: ln_a.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, NM_LN, 0)
B2K_NORM_INSTANTIATE(__half, NM_LN, 1)
B2K_NORM_INSTANTIATE(__half, NM_LN, 2)
B2K_NORM_INSTANTIATE(__half, NM_LN, 3)
B2K_NORM_INSTANTIATE(__half, NM_LN, 4)
B2K_NORM_INSTANTIATE(__half, NM_LN, 5)
B2K_NORM_INSTANTIATE(__half, NM_LN, 6)
B2K_NORM_INSTANTIATE(__half, NM_LN, 7)
B2K_NORM_INSTANTIATE(__half, NM_LN, 8)
B2K_NORM_INSTANTIATE(__half, NM_LN, 9)
}  // namespace b2k
