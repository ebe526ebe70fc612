// fht_engine.h -- internal interface between the C ABI and the transform engines.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "fht_tile.cuh"

namespace lwl {

constexpr int kWholeBlockMaxLogFwd = 15;
constexpr int kWholeBlockMaxLogBwd = 14;
constexpr int kMaxLogB = 23;

struct FhtArgs {
  int dtype;
  bool backward;
  const void* in;       // forward: latent [L]; backward: grad_out [stop-start]
  void* out;            // forward: y [stop-start]; backward: grad_latent [L]
  int64_t latent_size;  // L
  int64_t size;
  int layers;
  uint64_t seed;
  int64_t start, stop;
  void* workspace;
  size_t workspace_bytes;
  unsigned flags;
};

struct TileLaunch {
  TileParams p;
  int threads;
  size_t smem;
  int grid;
};

struct FhtPlan {
  int nlaunch;
  TileLaunch launches[4];
  int64_t nblocks, B;
  int64_t partial_rows;  // backward: rows reduced into grad_latent
  size_t f32_off;        // bf16 backward plans: byte offset of the fp32 region the last launch writes
  size_t ws_bytes;
};

int plan_fht(const FhtArgs& a, FhtPlan& plan);
int run_fht(const FhtArgs& a, FhtPlan& plan, cudaStream_t st);

// Register-resident fp32 whole-block kernel (fht32.cu): fp32 dtype or
// LWL_FLAG_EXACT, padded block 2^5 .. 2^15, forward and backward.
bool fht32_supported(int dtype, int64_t latent_size, bool backward, unsigned flags);
size_t fht32_workspace_bytes(const FhtArgs& a);
int fht32_launches(const FhtArgs& a);  // kernels one call enqueues

// Small-block kernel (fhts.cu): padded block 2^5 .. 2^10, every dtype, fp32
// arithmetic, forward and backward.
bool fhts_supported(int dtype, int64_t latent_size, bool backward, int layers, unsigned flags);
size_t fhts_workspace_bytes(const FhtArgs& a);
int fhts_launches(const FhtArgs& a);
int fhts_run(const FhtArgs& a, cudaStream_t st);

// fp32 low pass of two-pass plans (fp32 and the exact mode, 2^16..2^23; fht32_lo.cu).
bool fht32_lo_supported(int dtype, int n, unsigned flags);
int fht32_lo_launch(int dtype, const TileParams& p, cudaStream_t st);
int fht32_lo_grid(const TileParams& p);  // the launch's grid (a multiple of the tiles per block with acc_rows)

// High-bit pass of two-pass plans with 15 low bits and 1..8 high bits (fht32_hi.cu).
bool fht_hi_eligible(int dtype, const TileParams& p);
int fht_hi_launch(int dtype, const TileParams& p, cudaStream_t st);
int fht32_run(const FhtArgs& a, cudaStream_t st);

}  // namespace lwl
