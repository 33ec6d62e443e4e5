// Instances of the norm-family kernels: float, epilogues 5..9.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(float, 5)
B2K_NORM_INSTANTIATE(float, 6)
B2K_NORM_INSTANTIATE(float, 7)
B2K_NORM_INSTANTIATE(float, 8)
B2K_NORM_INSTANTIATE(float, 9)
}  // namespace b2k
