// fht32_k_f32_bwd.cu -- instantiations of the fp32 whole-block transform kernels (f32 bwd);
// the kernel templates and their schedules are in fht32.cuh.
#include "fht32.cuh"

namespace lwl {
namespace f32k {

const void* kernel_f32_bwd(bool full, int n, int layers) { return pick<float, true>(full, n, layers, tile_bits(n)); }

}  // namespace f32k
}  // namespace lwl
