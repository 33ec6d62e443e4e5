// Instances of the norm-family kernels: __half, epilogues 5..9.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, 5)
B2K_NORM_INSTANTIATE(__half, 6)
B2K_NORM_INSTANTIATE(__half, 7)
B2K_NORM_INSTANTIATE(__half, 8)
B2K_NORM_INSTANTIATE(__half, 9)
}  // namespace b2k
