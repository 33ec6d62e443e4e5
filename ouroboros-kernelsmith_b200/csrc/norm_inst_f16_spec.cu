// Instances of the norm-family kernels for __half: spec.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, NM_RMS_WROUND, 0)
B2K_NORM_INSTANTIATE(__half, NM_RMS_1PW, 0)
B2K_NORM_INSTANTIATE(__half, NM_L2, 0)
}  // namespace b2k
