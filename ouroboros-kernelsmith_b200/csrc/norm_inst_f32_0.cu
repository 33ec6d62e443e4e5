// Instances of the norm-family kernels: float, epilogues 0..4.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(float, 0)
B2K_NORM_INSTANTIATE(float, 1)
B2K_NORM_INSTANTIATE(float, 2)
B2K_NORM_INSTANTIATE(float, 3)
B2K_NORM_INSTANTIATE(float, 4)
}  // namespace b2k
