// Instances of the norm-family kernels for __half: rmsw_b.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 10)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 11)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 12)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 13)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 14)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 15)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 16)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 17)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 18)
B2K_NORM_INSTANTIATE(__half, NM_RMS_W, 19)
}  // namespace b2k
