// fht32_k_half_fwd.cu -- instantiations of the fp32 whole-block transform kernels (half fwd);
// the kernel templates and their schedules are in fht32.cuh.
#include "fht32.cuh"

namespace lwl {
namespace f32k {

const void* kernel_half_fwd(int dtype, bool full, int n, int layers) {
  return dtype == LWL_BF16 ? pick<__nv_bfloat16, false>(full, n, layers, tile_bits(n))
                           : pick<__half, false>(full, n, layers, tile_bits(n));
}

}  // namespace f32k
}  // namespace lwl
