// Instances of the norm-family kernels: __half, epilogues 10..14.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, 10)
B2K_NORM_INSTANTIATE(__half, 11)
B2K_NORM_INSTANTIATE(__half, 12)
B2K_NORM_INSTANTIATE(__half, 13)
B2K_NORM_INSTANTIATE(__half, 14)
}  // namespace b2k
