// fht_mma.h -- tensor-core transform paths (16-bit dtypes) selected by the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "fht_tile.cuh"
#include "lwl_b200.h"

namespace lwl {

// True when lwl_fht_forward with these arguments runs on the tensor-core kernel.
bool mma_forward_supported(int dtype, int64_t latent_size, unsigned flags);
// Tensor-core forward for padded block size 2^15; returns 0 or -1 (launch failure).
int mma_forward(int dtype, const void* latent, int64_t latent_size, int layers, uint64_t seed, int64_t start,
                int64_t stop, void* out, cudaStream_t st);
// Many tensor-core forwards in as few launches as possible (up to 96 generators per launch).
int mma_forward_grouped(int dtype, int count, const lwl_fht_forward_desc* descs, cudaStream_t st);

// Tensor-core backward for padded block size 2^15 (fp32 partials in TMEM,
// one [L] row per CTA in the workspace, then a row reduction).
size_t mma_backward_grouped_workspace_bytes(int count, const lwl_fht_backward_desc* descs);
int mma_backward_grouped(int dtype, int count, const lwl_fht_backward_desc* descs, void* workspace, cudaStream_t st);
bool mma16_forward_supported(int dtype, int64_t latent_size, unsigned flags);
bool mma16_backward_supported(int dtype, int64_t latent_size, unsigned flags);
int mma16_forward(int dtype, const void* latent, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                  void* out, cudaStream_t st);
size_t mma16_backward_workspace_bytes(int64_t latent_size, int64_t start, int64_t stop);
int mma16_backward(int dtype, const void* grad, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                   void* grad_latent, void* workspace, cudaStream_t st);
bool mma_backward_supported(int dtype, int64_t latent_size, unsigned flags);
size_t mma_backward_workspace_bytes(int64_t latent_size, int64_t start, int64_t stop);
// test_stall != 0: the first bounded wait of every CTA gives up (LWL_FLAG_TEST_WAIT_TIMEOUT).
int mma_backward(int dtype, const void* grad, int64_t latent_size, int layers, uint64_t seed, int64_t start,
                 int64_t stop, void* grad_latent, void* workspace, cudaStream_t st, int test_stall = 0);

// Low-15-bit pass of large blocks (B = 2^16 .. 2^23, 16-bit dtypes) on the
// tensor-core tile kernel: one 2^15 tile per work item, input/output and signs
// described by a two-pass TileParams launch of the planner (p.lo = 1).
bool mma_lo_supported(int dtype, int n, unsigned flags);
int mma_lo_grid(const TileParams& p);
int mma_lo_launch(int dtype, const TileParams& p, int grid, cudaStream_t st);

// tcgen05 BlockFHTLinear forward (linear_tc.cu).
bool tc_linear_supported(int K, int N, int T);
// Optional terms of the fused linear (bf16 device vectors, an fp32 device
// scalar, a dense bf16 [N, K] base weight, or null):
//   y[:, n] = out_gain[n] * (x ((base + base_scale (W + offset)) * in_gain)^T)[:, n] + bias[n]
// (without base: base_scale = 1 and no base term).
struct LinExtras {
  const void* bias;
  const void* out_gain;
  const void* in_gain;
  const float* weight_offset;
  const void* base;
  float base_scale;
};
int tc_linear_launch(bool gen, const void* x, int T, int K, int N, const void* latent, int64_t L, int layers,
                     uint64_t seed, float wscale, const void* wdense, void* y, int* err, cudaStream_t st,
                     const LinExtras* extras = nullptr);

}  // namespace lwl
