// Instances of the norm-family kernels for __half: rmsw_a.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 0)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 1)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 2)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 3)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 4)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 5)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 6)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 7)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 8)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 9)
}  // namespace b2k
