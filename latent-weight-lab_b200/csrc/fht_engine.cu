// fht_engine.cu -- host-side planning and launch of the generic tile engine.
//
// Two layouts, chosen by padded block size B = 2^n:
//  * whole-block: one tile holds entire blocks (2^m small blocks side by
//    side when n < 12); every layer is done in shared memory, one launch.
//    Forward for n <= 15, backward for n <= 14 (the backward also keeps an
//    fp32 accumulator over the latent positions in shared memory).
//  * two-pass: B = 2^a * 2^(n-a); pass P1 transforms the low a bits
//    (contiguous runs), pass P2 the high bits (8-element columns at stride
//    2^a).  Layers alternate P2,P1 / P1,P2 so neighbouring layers share a
//    pass: layers+1 launches over an fp32 workspace of #blocks * B.
// The backward runs the transposed chain (reversed sign layers) and reduces
// the per-block results over blocks deterministically (reduce_rows_kernel).
#include <cstdlib>
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>

#include "fht_engine.h"
#include "fht_tile.cuh"
#include "fht_mma.h"

namespace lwl {

namespace {

constexpr int kSmemLimit = 232448;  // 227 KB opt-in per CTA on sm_100

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Split `r` transform bits into ceil(r/5) balanced groups starting at tile bit `cb`.
int make_groups(int r, int cb, int8_t* glo, int8_t* gr) {
  int k = std::max(1, (r + 4) / 5);
  int base = r / k, rem = r % k, at = cb;
  for (int i = 0; i < k; ++i) {
    int s = base + (i < rem ? 1 : 0);
    glo[i] = (int8_t)at;
    gr[i] = (int8_t)s;
    at += s;
  }
  return k;
}

// Runs for `nseg` full transforms over the tile's transform bits, each
// followed by sign slot seg_slot[i] (-1 = none).  The last segment walks
// the groups upward so the final stores have consecutive lanes on
// consecutive positions; earlier segments alternate so that neighbours
// share a group (merged into one run).
void build_runs(TileParams& p, const int* seg_slot, int nseg) {
  int8_t glo[8], gr[8];
  int k = make_groups(p.r, p.cb, glo, gr);
  p.nruns = 0;
  for (int s = 0; s < nseg; ++s) {
    bool asc = ((nseg - 1 - s) % 2) == 0;
    for (int i = 0; i < k; ++i) {
      int g = asc ? i : k - 1 - i;
      int slot = (i == k - 1) ? seg_slot[s] : -1;
      RunDesc* last = p.nruns ? &p.runs[p.nruns - 1] : nullptr;
      if (last && last->glo == glo[g] && last->gr == gr[g] && last->nfht < 3) {
        last->slot[last->nfht] = (int8_t)slot;
        last->nfht++;
      } else {
        RunDesc rd;
        rd.glo = glo[g];
        rd.gr = gr[g];
        rd.nfht = 1;
        rd.slot[0] = (int8_t)slot;
        rd.slot[1] = rd.slot[2] = -1;
        p.runs[p.nruns++] = rd;
      }
    }
  }
}

size_t tile_smem(const TileParams& p) {
  size_t E = size_t(1) << p.e;
  size_t b = (E + E / 32) * 4 + size_t(p.nslots) * (E >> p.wshift) * 4;
  if (p.dst_kind == DST_ACC) b += size_t(p.L) * 4;
  return b;
}

int tile_threads(const TileParams& p) { return std::min(512, std::max(32, 1 << std::max(0, p.e - 5))); }

using TileKernel = void (*)(TileParams);

// The planner's (source, sink) combinations, each a separate instantiation.
template <typename T>
TileKernel tile_kernel_for(int src, int dst) {
  if (src == SRC_LATENT && dst == DST_SLICE) return fht_tile_kernel<T, SRC_LATENT, DST_SLICE>;
  if (src == SRC_LATENT && dst == DST_WS) return fht_tile_kernel<T, SRC_LATENT, DST_WS>;
  if (src == SRC_SLICE && dst == DST_ACC) return fht_tile_kernel<T, SRC_SLICE, DST_ACC>;
  if (src == SRC_SLICE && dst == DST_WS) return fht_tile_kernel<T, SRC_SLICE, DST_WS>;
  if (src == SRC_WS && dst == DST_SLICE) return fht_tile_kernel<T, SRC_WS, DST_SLICE>;
  return fht_tile_kernel<T, SRC_WS, DST_WS>;
}

template <typename T>
int occupancy(int src, int dst, int threads, size_t smem) {
  TileKernel k = tile_kernel_for<T>(src, dst);
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
  int blocks = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, k, threads, smem) != cudaSuccess) blocks = 1;
  return std::max(1, blocks);
}

int occupancy_for(int dtype, int src, int dst, int threads, size_t smem) {
  if (dtype == LWL_BF16) return occupancy<__nv_bfloat16>(src, dst, threads, smem);
  if (dtype == LWL_F16) return occupancy<__half>(src, dst, threads, smem);
  return occupancy<float>(src, dst, threads, smem);
}

void finish_launch(int dtype, TileLaunch& l) {
  l.threads = tile_threads(l.p);
  l.smem = tile_smem(l.p);
  int64_t cap = (int64_t)sm_count() * occupancy_for(dtype, l.p.src_kind, l.p.dst_kind, l.threads, l.smem);
  l.grid = (int)std::max<int64_t>(1, std::min<int64_t>(l.p.ntiles, cap));
}

void common_fields(TileParams& p, const FhtArgs& a, int n) {
  std::memset(&p, 0, sizeof(p));
  p.n = n;
  p.B = int64_t(1) << n;
  p.L = a.latent_size;
  p.seed32 = fold_seed(a.seed);
  p.scale = (float)(1.0 / std::sqrt((double)p.B));
  p.pre_slot = -1;
  p.start = a.start;
  p.stop = a.stop;
}

}  // namespace

int plan_fht(const FhtArgs& a, FhtPlan& plan) {
  std::memset(&plan, 0, sizeof(plan));
  const int n = ilog2(next_pow2(a.latent_size));
  const int64_t B = int64_t(1) << n;
  const int64_t first = a.start / B, last = (a.stop + B - 1) / B;
  const int64_t nblk = last - first;
  plan.nblocks = nblk;
  plan.B = B;
  if (nblk <= 0) return 0;
  const int L = a.layers;
  const bool bwd = a.backward;
  // sign layer applied before the first network, then after network i
  auto pre_layer = [&]() { return bwd ? L : 0; };
  auto post_layer = [&](int i) { return bwd ? L - 1 - i : i + 1; };

  const bool whole = bwd ? (n <= kWholeBlockMaxLogBwd) : (n <= kWholeBlockMaxLogFwd);
  if (whole) {
    TileLaunch& l = plan.launches[0];
    plan.nlaunch = 1;
    TileParams& p = l.p;
    common_fields(p, a, n);
    p.e = std::max(n, 12);
    p.cb = 0;
    p.tlo = 0;
    p.r = n;
    p.m = p.e - n;
    p.ulo = n;
    p.ublock = 1;
    p.rlo = 0;
    p.wshift = std::min(5, n);
    p.tiles_per_group = 1;
    p.first_block = first;
    p.nblocks = nblk;
    p.ntiles = (nblk + (int64_t(1) << p.m) - 1) >> p.m;
    p.nslots = L + 1;
    p.slot_layer[0] = pre_layer();
    int seg_slot[3];
    for (int i = 0; i < L; ++i) {
      p.slot_layer[i + 1] = post_layer(i);
      seg_slot[i] = i + 1;
    }
    p.pre_slot = 0;
    build_runs(p, seg_slot, L);
    p.src_kind = bwd ? SRC_SLICE : SRC_LATENT;
    p.dst_kind = bwd ? DST_ACC : DST_SLICE;
    finish_launch(a.dtype, l);
    if (bwd) {
      plan.partial_rows = l.grid;
      plan.ws_bytes = size_t(l.grid) * size_t(a.latent_size) * 4;
    }
    return 0;
  }

  // two-pass layout.  The low pass is exactly 15 bits: on the tensor-core
  // tile kernel for 16-bit dtypes (fht_lo_kernel), on the register-resident
  // fp32 kernel for fp32 and the exact mode (fht32_lo_kernel); the high n-15
  // bits run on fht_hi_kernel / fht_hi2_kernel where they qualify, else on
  // the tile engine.
  const bool use_lo = mma_lo_supported(a.dtype, n, a.flags);
  const bool use_lo32 = !use_lo && fht32_lo_supported(a.dtype, n, a.flags);
  const int abits = (use_lo || use_lo32) ? 15 : (n + 1) / 2;
  const int hbits = n - abits;
  // execution order of (part, post-layer) steps; part 1 = P1 (low bits), 2 = P2
  int step_part[6], step_sign[6], nsteps = 0;
  for (int i = 0; i < L; ++i) {
    bool p2_first = ((L - 1 - i) % 2) == 0;
    int first_part = p2_first ? 2 : 1, second_part = p2_first ? 1 : 2;
    step_part[nsteps] = first_part;
    step_sign[nsteps++] = -1;
    step_part[nsteps] = second_part;
    step_sign[nsteps++] = post_layer(i);
  }
  int s = 0;
  plan.nlaunch = 0;
  while (s < nsteps) {
    int e_ = s;
    while (e_ + 1 < nsteps && step_part[e_ + 1] == step_part[s]) ++e_;
    TileLaunch& l = plan.launches[plan.nlaunch];
    TileParams& p = l.p;
    common_fields(p, a, n);
    const bool is_first = (s == 0), is_last = (e_ == nsteps - 1);
    if (step_part[s] == 1) {
      p.cb = 0;
      p.tlo = 0;
      p.r = abits;
      p.m = std::min(hbits, std::max(0, 12 - abits));
      p.ulo = abits;
      p.rlo = abits + p.m;
      p.wshift = 5;
      p.tiles_per_group = int64_t(1) << (n - abits - p.m);
    } else {
      p.cb = 3;
      p.tlo = abits;
      p.r = hbits;
      p.m = std::min(abits - 3, std::max(0, 12 - 3 - hbits));
      p.ulo = 3;
      p.rlo = 3 + p.m;
      p.wshift = 3;
      p.tiles_per_group = int64_t(1) << (abits - 3 - p.m);
    }
    p.e = p.cb + p.r + p.m;
    p.ublock = 0;
    p.first_block = first;
    p.nblocks = nblk;
    p.ntiles = nblk * p.tiles_per_group;
    p.nslots = 0;
    if (is_first) {
      p.slot_layer[p.nslots] = pre_layer();
      p.pre_slot = p.nslots++;
    }
    int seg_slot[6], nseg = 0;
    for (int k = s; k <= e_; ++k) {
      if (step_sign[k] >= 0) {
        p.slot_layer[p.nslots] = step_sign[k];
        seg_slot[nseg++] = p.nslots++;
      } else {
        seg_slot[nseg++] = -1;
      }
    }
    build_runs(p, seg_slot, nseg);
    p.src_kind = is_first ? (bwd ? SRC_SLICE : SRC_LATENT) : SRC_WS;
    p.dst_kind = (is_last && !bwd) ? DST_SLICE : DST_WS;
    finish_launch(a.dtype, l);
    if ((use_lo || use_lo32) && step_part[s] == 1 && nseg <= 2) {
      p.lo = use_lo ? 1 : 2;
      p.lo_nseg = nseg;
      p.lo_seg_slot[0] = seg_slot[0];
      p.lo_seg_slot[1] = nseg > 1 ? seg_slot[1] : -1;
      if (use_lo) l.grid = mma_lo_grid(p);
    }
    plan.nlaunch++;
    s = e_ + 1;
  }
  plan.ws_bytes = size_t(nblk) * size_t(B) * 4;
  if (bwd) plan.partial_rows = nblk;
  // bf16 workspace: bf16 plans whose every launch is a tensor-core low pass or
  // a register-resident high pass (both read and write it).  The backward's
  // last launch (a low pass) writes fp32 into a second region, which the
  // block sum reads; fp16 keeps fp32 because its unnormalised intermediates
  // can leave the fp16 range.  One more bf16 rounding per launch: rel-L2
  // 3.4e-3 at 2^23 against 1.8e-3.  LWL_WS16=0 keeps fp32 (measurement only).
  static const bool ws16_env = [] {
    const char* e = std::getenv("LWL_WS16");
    return !(e && e[0] == '0');
  }();
  bool ws16 = ws16_env && use_lo && a.dtype == LWL_BF16 && (!bwd || plan.launches[plan.nlaunch - 1].p.lo == 1);
  for (int i = 0; ws16 && i < plan.nlaunch; ++i)
    if (!plan.launches[i].p.lo && !fht_hi_eligible(a.dtype, plan.launches[i].p)) ws16 = false;
  if (ws16) {
    for (int i = 0; i < plan.nlaunch; ++i) plan.launches[i].p.ws16 = 1;
    const size_t h = (size_t(nblk) * size_t(B) * 2 + 255) & ~size_t(255);
    plan.ws_bytes = h;
    if (bwd) {
      TileLaunch& last = plan.launches[plan.nlaunch - 1];
      plan.f32_off = h;
      if ((B >> 15) <= 256) {
        // the last low pass sums its tiles in tensor memory: partial rows of
        // [L] per group of tpb CTAs instead of an fp32 copy of every block
        last.p.acc_rows = 1;
        last.grid = mma_lo_grid(last.p);
        plan.partial_rows = last.grid >= (B >> 15) ? last.grid / (B >> 15) : 1;
        plan.ws_bytes = h + size_t(plan.partial_rows) * size_t(a.latent_size) * 4;
      } else {
        last.p.ws_out32 = 1;
        plan.ws_bytes = h + size_t(nblk) * size_t(B) * 4;
      }
    }
  } else if (bwd && plan.launches[plan.nlaunch - 1].p.lo != 0 && (B >> 15) <= 256) {
    // fp16 backward (fp32 workspace): the same tensor-memory sums in the last
    // low pass; fp32 and the exact mode (fht32_lo_kernel): per-CTA sums in an
    // L2-resident partial row segment
    TileLaunch& last = plan.launches[plan.nlaunch - 1];
    const size_t h = (size_t(nblk) * size_t(B) * 4 + 255) & ~size_t(255);
    last.p.acc_rows = 1;
    last.grid = last.p.lo == 1 ? mma_lo_grid(last.p) : fht32_lo_grid(last.p);
    plan.f32_off = h;
    plan.partial_rows = last.grid >= (B >> 15) ? last.grid / (B >> 15) : 1;
    plan.ws_bytes = h + size_t(plan.partial_rows) * size_t(a.latent_size) * 4;
  }
  return 0;
}

template <typename T>
__global__ void reduce_rows_kernel(const float* __restrict__ src, int64_t rows, int64_t row_stride,
                                   int64_t L, T* __restrict__ out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < L; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.0f;
#pragma unroll 8
    for (int64_t r = 0; r < rows; ++r) s += src[r * row_stride + i];
    out[i] = Cvt<T>::from_f(s);
  }
}

namespace {
template <typename T>
int run_plan_t(const FhtArgs& a, FhtPlan& plan, cudaStream_t st) {
  if (plan.nblocks <= 0) {
    if (a.backward) LWL_CUDA_TRY(cudaMemsetAsync(a.out, 0, size_t(a.latent_size) * sizeof(T), st));
    return LWL_OK;
  }
  if (plan.launches[0].p.ws16 && (reinterpret_cast<uintptr_t>(a.workspace) & 15) != 0) {
    set_error("the workspace of this call must be 16-byte aligned");
    return LWL_ERR_INVALID;
  }
  for (int i = 0; i < plan.nlaunch; ++i) {
    TileLaunch& l = plan.launches[i];
    TileParams& p = l.p;
    p.src = (p.src_kind == SRC_WS) ? a.workspace : a.in;
    if (p.dst_kind == DST_SLICE) p.dst = a.out;
    else if (p.dst_kind == DST_WS) p.dst = static_cast<char*>(a.workspace) + (p.ws_out32 ? plan.f32_off : 0);
    if (p.acc_rows) p.partial = reinterpret_cast<float*>(static_cast<char*>(a.workspace) + plan.f32_off);
    else p.partial = reinterpret_cast<float*>(a.workspace);
    if (p.lo == 2) {
      if (fht32_lo_launch(a.dtype, p, st) != 0) {
        set_error("fp32 low-pass launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return LWL_ERR_CUDA;
      }
      continue;
    }
    if (p.lo) {
      if (mma_lo_launch(a.dtype, p, l.grid, st) != 0) {
        set_error("tensor-core low-pass launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return LWL_ERR_CUDA;
      }
      continue;
    }
    if (fht_hi_eligible(a.dtype, p)) {
      if (fht_hi_launch(a.dtype, p, st) != 0) {
        set_error("high-bit pass launch failed: %s", cudaGetErrorString(cudaGetLastError()));
        return LWL_ERR_CUDA;
      }
      continue;
    }
    tile_kernel_for<T>(p.src_kind, p.dst_kind)<<<l.grid, l.threads, l.smem, st>>>(p);
    LWL_CUDA_TRY(cudaGetLastError());
  }
  if (a.backward) {
    const bool rows_of_L = plan.launches[0].p.dst_kind == DST_ACC || plan.launches[plan.nlaunch - 1].p.acc_rows;
    int64_t stride = rows_of_L ? a.latent_size : plan.B;
    int threads = 256;
    int64_t blocks = std::min<int64_t>((a.latent_size + threads - 1) / threads, 65535);
    reduce_rows_kernel<T><<<(int)blocks, threads, 0, st>>>(
        reinterpret_cast<const float*>(static_cast<const char*>(a.workspace) + plan.f32_off),
                                                            plan.partial_rows, stride, a.latent_size,
                                                            reinterpret_cast<T*>(a.out));
    LWL_CUDA_TRY(cudaGetLastError());
  }
  return LWL_OK;
}
}  // namespace

int run_fht(const FhtArgs& a, FhtPlan& plan, cudaStream_t st) {
  if (a.dtype == LWL_BF16) return run_plan_t<__nv_bfloat16>(a, plan, st);
  if (a.dtype == LWL_F16) return run_plan_t<__half>(a, plan, st);
  return run_plan_t<float>(a, plan, st);
}

}  // namespace lwl
