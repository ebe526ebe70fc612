// fht32.cu -- host side of the fp32 whole-block transform (fht32.cuh):
// kernel choice, persistent grid, full/edge tile split, launches and the
// deterministic reduce of the backward's partial rows.
#include <algorithm>
#include <cmath>
#include <cstring>

#include "fht32.cuh"

namespace lwl {
namespace f32k {

int sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

const void* kernel_of(int dtype, bool bwd, bool full, int n, int layers) {
  if (dtype == LWL_F32) return bwd ? kernel_f32_bwd(full, n, layers) : kernel_f32_fwd(full, n, layers);
  return bwd ? kernel_half_bwd(dtype, full, n, layers) : kernel_half_fwd(dtype, full, n, layers);
}

size_t smem_of(int TB) {
  return TB == 13 ? Tile<13>::kSmem : (TB == 14 ? Tile<14>::kSmem : Tile<15>::kSmem);
}

// Persistent grid: every SM holds as many CTAs as fit, capped by the tiles.
int grid_for(const void* k, int TB, int64_t ntiles) {
  if (ntiles <= 0) return 0;
  if (!set_max_smem(k, (int)smem_of(TB))) return -1;
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, 1 << (TB - 6), smem_of(TB)) != cudaSuccess ||
      per_sm < 1)
    per_sm = 1;
  return (int)std::min<int64_t>(ntiles, (int64_t)sms() * per_sm);
}

// Tiles wholly inside the slice run unpredicated in one persistent launch;
// the (at most two) tiles that straddle the slice's ends run in a second,
// bounds-checked launch.  Backward: each CTA of either launch owns one
// partial row (edge rows follow the main rows).
struct Plan {
  Params main, edge;
  const void* kmain = nullptr;
  const void* kedge = nullptr;
  int gmain = 0, gedge = 0, TB = 13;
  int rows() const { return gmain + gedge; }
};

int make_plan(const FhtArgs& a, Plan& pl) {
  Params p;
  std::memset(&p, 0, sizeof(p));
  p.src = a.in;
  p.L = a.latent_size;
  p.n = ilog2(next_pow2(a.latent_size));
  p.layers = a.layers;
  p.seed32 = fold_seed(a.seed);
  p.scale = (float)std::pow((double)(int64_t(1) << p.n), -0.5 * a.layers);
  p.start = a.start;
  p.stop = a.stop;
  p.tile_step = 1;
  for (int s = 0; s <= a.layers; ++s) p.slot_layer[s] = a.backward ? a.layers - s : s;
  const int TB = tile_bits(p.n);
  const int64_t E = int64_t(1) << TB;
  pl.TB = TB;
  const int64_t t_first = a.start >> TB, t_last = (a.stop - 1) >> TB;  // stop > start
  const int64_t f0 = (a.start + E - 1) >> TB, f1 = a.stop >> TB;       // full tiles [f0, f1)
  pl.main = p;
  pl.main.first_tile = f0;
  pl.main.ntiles = std::max<int64_t>(f1 - f0, 0);
  int64_t edges[2];
  int ne = 0;
  if (f1 <= f0) {
    edges[ne++] = t_first;
    if (t_last != t_first) edges[ne++] = t_last;
  } else {
    if (t_first < f0) edges[ne++] = t_first;
    if (t_last >= f1) edges[ne++] = t_last;
  }
  pl.edge = p;
  pl.edge.ntiles = ne;
  pl.edge.first_tile = ne ? edges[0] : 0;
  pl.edge.tile_step = ne == 2 ? edges[1] - edges[0] : 1;
  pl.kmain = kernel_of(a.dtype, a.backward, true, p.n, a.layers);
  pl.kedge = kernel_of(a.dtype, a.backward, false, p.n, a.layers);
  pl.gmain = grid_for(pl.kmain, TB, pl.main.ntiles);
  pl.gedge = grid_for(pl.kedge, TB, pl.edge.ntiles);
  if (pl.gmain < 0 || pl.gedge < 0) return -1;
  pl.main.row0 = 0;
  pl.edge.row0 = pl.gmain;
  return 0;
}

}  // namespace f32k

bool fht32_supported(int dtype, int64_t L, bool backward, unsigned flags) {
  (void)backward;
  const int n = ilog2(next_pow2(L));
  if (n < 5 || n > 15) return false;
  return dtype == LWL_F32 || (flags & LWL_FLAG_EXACT);
}

int fht32_launches(const FhtArgs& a) {
  if (a.stop <= a.start) return 0;
  f32k::Plan pl;
  if (f32k::make_plan(a, pl) != 0) return -1;
  return (pl.gmain > 0) + (pl.gedge > 0) + (a.backward ? 1 : 0);
}

size_t fht32_workspace_bytes(const FhtArgs& a) {
  if (!a.backward || a.stop <= a.start) return 0;
  f32k::Plan pl;
  if (f32k::make_plan(a, pl) != 0) return 0;
  return size_t(pl.rows()) * size_t(a.latent_size) * 4;
}

template <typename T>
__global__ void fht32_reduce_kernel(const float* __restrict__ rows, int nrows, int64_t L, T* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < L; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // four loads in flight, fixed summation order
    int r = 0;
    for (; r + 4 <= nrows; r += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += rows[(int64_t)(r + u) * L + i];
    }
    for (; r < nrows; ++r) acc[0] += rows[(int64_t)r * L + i];
    out[i] = Cvt<T>::from_f((acc[0] + acc[1]) + (acc[2] + acc[3]));
  }
}

int fht32_run(const FhtArgs& a, cudaStream_t st) {
  using namespace f32k;
  if (a.stop <= a.start) {
    if (a.backward) LWL_CUDA_TRY(cudaMemsetAsync(a.out, 0, size_t(a.latent_size) * (a.dtype == LWL_F32 ? 4 : 2), st));
    return LWL_OK;
  }
  Plan pl;
  if (make_plan(a, pl) != 0) {
    set_error("fp32 whole-block transform: kernel setup failed: %s", cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  void* dst = a.out;
  if (a.backward) {
    const size_t need = size_t(pl.rows()) * size_t(a.latent_size) * 4;
    if (!a.workspace || a.workspace_bytes < need) {
      set_error("workspace of %zu bytes required, %zu given", need, a.workspace ? a.workspace_bytes : (size_t)0);
      return LWL_ERR_WORKSPACE;
    }
    dst = a.workspace;
  }
  pl.main.dst = pl.edge.dst = dst;
  const dim3 block(1 << (pl.TB - 6));
  const size_t smem = smem_of(pl.TB);
  if (pl.gmain > 0) {
    void* args[] = {&pl.main};
    if (cudaLaunchKernel(pl.kmain, dim3(pl.gmain), block, args, smem, st) != cudaSuccess) {
      set_error("fp32 whole-block transform launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
  }
  if (pl.gedge > 0) {
    void* args[] = {&pl.edge};
    if (cudaLaunchKernel(pl.kedge, dim3(pl.gedge), block, args, smem, st) != cudaSuccess) {
      set_error("fp32 whole-block transform (slice edges) launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
  }
  const int grid = pl.rows();
  if (a.backward) {
    const int threads = 256;
    const int blocks = (int)std::min<int64_t>((a.latent_size + threads - 1) / threads, 1024);
    const float* rows = reinterpret_cast<const float*>(a.workspace);
    if (a.dtype == LWL_BF16)
      fht32_reduce_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size,
                                                                      reinterpret_cast<__nv_bfloat16*>(a.out));
    else if (a.dtype == LWL_F16)
      fht32_reduce_kernel<__half><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size, reinterpret_cast<__half*>(a.out));
    else
      fht32_reduce_kernel<float><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size, reinterpret_cast<float*>(a.out));
    LWL_CUDA_TRY(cudaGetLastError());
  }
  return LWL_OK;
}

}  // namespace lwl
