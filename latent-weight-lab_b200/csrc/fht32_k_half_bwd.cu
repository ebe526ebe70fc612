// fht32_k_half_bwd.cu -- instantiations of the fp32 whole-block transform kernels (half bwd);
// the kernel templates and their schedules are in fht32.cuh.
#include "fht32.cuh"

namespace lwl {
namespace f32k {

const void* kernel_half_bwd(int dtype, bool full, int n, int layers) {
  return dtype == LWL_BF16 ? pick<__nv_bfloat16, true>(full, n, layers, tile_bits(n))
                           : pick<__half, true>(full, n, layers, tile_bits(n));
}

}  // namespace f32k
}  // namespace lwl
