// Instances of the norm-family kernels: __half, epilogues 15..19.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(__half, 15)
B2K_NORM_INSTANTIATE(__half, 16)
B2K_NORM_INSTANTIATE(__half, 17)
B2K_NORM_INSTANTIATE(__half, 18)
B2K_NORM_INSTANTIATE(__half, 19)
}  // namespace b2k
