// Instances of the norm-family kernels: float, epilogues 10..14.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(float, 10)
B2K_NORM_INSTANTIATE(float, 11)
B2K_NORM_INSTANTIATE(float, 12)
B2K_NORM_INSTANTIATE(float, 13)
B2K_NORM_INSTANTIATE(float, 14)
}  // namespace b2k
