// Instances of the norm-family kernels: __half, epilogues 0..4.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, 0)
B2K_NORM_INSTANTIATE(__half, 1)
B2K_NORM_INSTANTIATE(__half, 2)
B2K_NORM_INSTANTIATE(__half, 3)
B2K_NORM_INSTANTIATE(__half, 4)
}  // namespace b2k
