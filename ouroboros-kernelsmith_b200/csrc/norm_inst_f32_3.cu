// Instances of the norm-family kernels: float, epilogues 15..19.
#define B2K_NORM_DEFINE_KERNELS
#include "norm_impl.cuh"

namespace b2k {
B2K_NORM_INSTANTIATE(float, 15)
B2K_NORM_INSTANTIATE(float, 16)
B2K_NORM_INSTANTIATE(float, 17)
B2K_NORM_INSTANTIATE(float, 18)
B2K_NORM_INSTANTIATE(float, 19)
}  // namespace b2k
