// fht_tile.cuh -- the generic BlockFHT tile engine (fp32 arithmetic).
//
// One CTA owns a "tile": 2^e elements of the generated-coordinate space held
// in shared memory (fp32, one pad word per 32 to spread banks).  Tile index
// bits map onto block positions / block numbers as
//   t = [ col : cb ][ transform : r ][ upper : m ]
//   pos = col | transform << tlo | (upper << ulo, unless upper selects blocks)
//         | tile-id bits << rlo
// so the same engine covers (a) a whole block (cb=0, tlo=0, r=n) with 2^m
// small blocks side by side, and (b) the two passes of large blocks
// (contiguous runs of the low bits; strided columns of the high bits).
//
// Inside a tile the transform is a list of "runs": a run loads the 2^gr
// elements of one radix group (gr <= 5 bits) per column into registers,
// applies 1..3 radix-2^gr butterfly networks with a sign/scale between them
// (adjacent layers share a group, so a layer boundary costs no extra shared
// memory round trip), and stores them back.  The first run reads straight
// from the source (latent, gradient slice or fp32 workspace) and the last run
// writes straight to the sink, so a tile costs (#runs - 1) shared round trips.
#pragma once
#include "lwl_common.cuh"

namespace lwl {

constexpr int kMaxRuns = 12;
constexpr int kMaxSlots = 4;

enum SrcKind : int { SRC_LATENT = 0, SRC_SLICE = 1, SRC_WS = 2 };
enum DstKind : int { DST_SLICE = 0, DST_WS = 1, DST_ACC = 2 };

struct RunDesc {
  int8_t glo;      // lowest tile bit of the group
  int8_t gr;       // group bits (1..5)
  int8_t nfht;     // butterfly networks applied in this run (1..3)
  int8_t slot[3];  // sign slot after each network, -1 = none
};

struct TileParams {
  int n;           // log2(B)
  int64_t B, L;
  int e, cb, tlo, r, m, ulo;
  int ublock;      // upper tile bits select blocks (whole-block config)
  int rlo;         // position of the tile-id bits inside pos
  int wshift;      // sign-table index = t >> wshift
  int64_t tiles_per_group;  // tiles per (block, or 2^m blocks when ublock)
  int64_t first_block, nblocks, ntiles;
  int nslots;
  int slot_layer[kMaxSlots];
  int pre_slot;    // slot applied to source values, -1 none
  uint32_t seed32;
  float scale;     // multiplies every post-sign (1/sqrt(B))
  int nruns;
  RunDesc runs[kMaxRuns];
  int src_kind, dst_kind;
  const void* src;
  void* dst;
  int64_t start, stop;
  float* partial;  // DST_ACC: [gridDim.x][L]
  // launches of the low-15-bit pass on the tensor-core kernel (16-bit dtypes, B > 2^15)
  int lo;           // 1: run on fht_lo_kernel (16-bit), 2: on fht32_lo_kernel (fp32 math), instead of fht_tile_kernel
  int lo_nseg;      // 1 or 2 applications of the 2^15 transform
  int lo_seg_slot[2];  // sign slot after each application, -1 = none
  // bf16 forward plans whose launches all run on fht_lo_kernel / fht_hi_kernel:
  // the workspace holds bf16 instead of fp32 (2 bytes per coordinate each way)
  // and the low pass streams its workspace tiles by bulk copy, one tile ahead.
  int ws16;
  int ws_out32;  // bf16 backward plans: this (last) launch writes its workspace output in fp32
  int acc_rows;  // ... or, with a grid that is a multiple of the tiles per block, sums its tiles in
                 // tensor memory and writes one [L] partial row segment per CTA into `partial`
};

__device__ __forceinline__ int pad_idx(int t) { return t + (t >> 5); }

struct TileCtx {
  int64_t tile_blk;   // first block of the tile
  int64_t fixed_pos;  // tile-id bits of pos
};

__device__ __forceinline__ void tile_coords(const TileParams& p, const TileCtx& c, int t,
                                            int64_t& pos, int64_t& blk) {
  int col = t & ((1 << p.cb) - 1);
  int k = (t >> p.cb) & ((1 << p.r) - 1);
  int u = t >> (p.cb + p.r);
  pos = (int64_t)col | ((int64_t)k << p.tlo) | c.fixed_pos;
  blk = c.tile_blk;
  if (p.ublock) blk += u;
  else pos |= (int64_t)u << p.ulo;
}

template <int R>
__device__ __forceinline__ void butterflies(float (&v)[1 << R]) {
#pragma unroll
  for (int h = 1; h < (1 << R); h <<= 1) {
#pragma unroll
    for (int i = 0; i < (1 << R); i += 2 * h) {
#pragma unroll
      for (int j = i; j < i + h; ++j) {
        float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
    }
  }
}

// One run of radix group GR over the tile.  first/last select source/sink I/O
// (SRC/DST are compile-time).  A group's bits are transform bits, so within a
// column the block is fixed and the position of element k is pos0 + (k << kshift).
template <typename T, int SRC, int DST, int GR>
__device__ void do_run(const TileParams& p, const TileCtx& c, const RunDesc& rd, float* data,
                       const uint32_t* signs, int words_per_slot, bool first, bool last) {
  const int glo = rd.glo;
  const int ncols = 1 << (p.e - GR);
  const int lowmask = (1 << glo) - 1;
  const int kshift = glo - p.cb + p.tlo;
  for (int col = threadIdx.x; col < ncols; col += blockDim.x) {
    const int base = (col & lowmask) | ((col >> glo) << (glo + GR));
    int64_t pos0, blk;
    tile_coords(p, c, base, pos0, blk);
    float v[1 << GR];
    if (first) {
      const int64_t bb = blk * p.B;
      const int64_t wrow = (blk - p.first_block) * p.B;
      const bool brow_ok = (blk - p.first_block) < p.nblocks;
#pragma unroll
      for (int k = 0; k < (1 << GR); ++k) {
        const int64_t pos = pos0 + ((int64_t)k << kshift);
        float x;
        if (SRC == SRC_LATENT) {
          x = pos < p.L ? Cvt<T>::to_f(reinterpret_cast<const T*>(p.src)[pos]) : 0.0f;
        } else if (SRC == SRC_SLICE) {
          const int64_t g = bb + pos;
          x = (g >= p.start && g < p.stop) ? Cvt<T>::to_f(reinterpret_cast<const T*>(p.src)[g - p.start]) : 0.0f;
        } else {
          x = brow_ok ? reinterpret_cast<const float*>(p.src)[wrow + pos] : 0.0f;
        }
        if (p.pre_slot >= 0) {
          const int t = base + (k << glo);
          uint32_t w = signs[p.pre_slot * words_per_slot + (t >> p.wshift)];
          x = ((w >> (pos & 31)) & 1u) ? x : -x;
        }
        v[k] = x;
      }
    } else {
#pragma unroll
      for (int k = 0; k < (1 << GR); ++k) v[k] = data[pad_idx(base + (k << glo))];
    }
    for (int f = 0; f < rd.nfht; ++f) {
      butterflies<GR>(v);
      int s = rd.slot[f];
      if (s >= 0) {
        const float sc = p.scale;
        const uint32_t* sws = signs + s * words_per_slot;
#pragma unroll
        for (int k = 0; k < (1 << GR); ++k) {
          const int t = base + (k << glo);
          const int64_t pos = pos0 + ((int64_t)k << kshift);
          uint32_t w = sws[t >> p.wshift];
          v[k] *= ((w >> (pos & 31)) & 1u) ? sc : -sc;
        }
      }
    }
    if (last && DST != DST_ACC) {
      const int64_t bb = blk * p.B;
      const int64_t wrow = (blk - p.first_block) * p.B;
      const bool brow_ok = (blk - p.first_block) < p.nblocks;
#pragma unroll
      for (int k = 0; k < (1 << GR); ++k) {
        const int64_t pos = pos0 + ((int64_t)k << kshift);
        if (DST == DST_SLICE) {
          const int64_t g = bb + pos;
          if (g >= p.start && g < p.stop) reinterpret_cast<T*>(p.dst)[g - p.start] = Cvt<T>::from_f(v[k]);
        } else if (brow_ok) {
          reinterpret_cast<float*>(p.dst)[wrow + pos] = v[k];
        }
      }
    } else {
#pragma unroll
      for (int k = 0; k < (1 << GR); ++k) data[pad_idx(base + (k << glo))] = v[k];
    }
  }
}

// Single-run tiles (the run both reads the source and writes the sink) with
// the group above the two lowest tile bits and at least two column bits --
// the high-bit pass of large blocks: each thread takes 4 consecutive columns,
// i.e. 4 consecutive positions per row, so a row is one 16-byte workspace
// access (8 bytes for 16-bit types) and one sign word instead of four.  Four
// times the bytes in flight of the scalar loop, which is latency-bound there.
// Accesses that are unaligned or cross the slice/latent edge fall back to
// scalars.
template <typename T, int SRC, int DST, int GR>
__device__ void do_run_v4(const TileParams& p, const TileCtx& c, const RunDesc& rd, const uint32_t* signs,
                          int words_per_slot) {
  const int glo = rd.glo;
  const int ncols = 1 << (p.e - GR);
  const int lowmask = (1 << glo) - 1;
  const int kshift = glo - p.cb + p.tlo;
  for (int col = 4 * threadIdx.x; col < ncols; col += 4 * blockDim.x) {
    const int base = (col & lowmask) | ((col >> glo) << (glo + GR));
    int64_t pos0, blk;
    tile_coords(p, c, base, pos0, blk);
    const int64_t bb = blk * p.B;
    const int64_t wrow = (blk - p.first_block) * p.B;
    const bool brow_ok = (blk - p.first_block) < p.nblocks;
    float v[4][1 << GR];
#pragma unroll
    for (int k = 0; k < (1 << GR); ++k) {
      const int64_t pos = pos0 + ((int64_t)k << kshift);
      if (SRC == SRC_WS) {
        const float* src = reinterpret_cast<const float*>(p.src) + wrow + pos;
        if (brow_ok && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
          const float4 x = *reinterpret_cast<const float4*>(src);
          v[0][k] = x.x, v[1][k] = x.y, v[2][k] = x.z, v[3][k] = x.w;
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i][k] = brow_ok ? src[i] : 0.0f;
        }
      } else {
        // source elements idx .. idx+3, valid for idx+i in [0, hi) (slice: g in [start, stop))
        const int64_t idx = SRC == SRC_LATENT ? pos : bb + pos - p.start;
        const int64_t hi = SRC == SRC_LATENT ? p.L : p.stop - p.start;
        const T* src = reinterpret_cast<const T*>(p.src) + idx;
        if (idx >= 0 && idx + 4 <= hi && (reinterpret_cast<uintptr_t>(src) & (4 * sizeof(T) - 1)) == 0) {
          if (sizeof(T) == 2) {
            const uint2 x = *reinterpret_cast<const uint2*>(src);
            const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i][k] = Cvt<T>::to_f(e[i]);
          } else {
            const float4 x = *reinterpret_cast<const float4*>(src);
            v[0][k] = Cvt<T>::to_f(reinterpret_cast<const T*>(&x)[0]);
            v[1][k] = Cvt<T>::to_f(reinterpret_cast<const T*>(&x)[1]);
            v[2][k] = Cvt<T>::to_f(reinterpret_cast<const T*>(&x)[2]);
            v[3][k] = Cvt<T>::to_f(reinterpret_cast<const T*>(&x)[3]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i][k] = (idx + i >= 0 && idx + i < hi) ? Cvt<T>::to_f(src[i]) : 0.0f;
        }
      }
      if (p.pre_slot >= 0) {
        const int t = base + (k << glo);
        const uint32_t w = signs[p.pre_slot * words_per_slot + (t >> p.wshift)] >> (pos & 31);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[i][k] = ((w >> i) & 1u) ? v[i][k] : -v[i][k];
      }
    }
    for (int f = 0; f < rd.nfht; ++f) {
#pragma unroll
      for (int i = 0; i < 4; ++i) butterflies<GR>(v[i]);
      const int s = rd.slot[f];
      if (s >= 0) {
        const float sc = p.scale;
        const uint32_t* sws = signs + s * words_per_slot;
#pragma unroll
        for (int k = 0; k < (1 << GR); ++k) {
          const int t = base + (k << glo);
          const int64_t pos = pos0 + ((int64_t)k << kshift);
          const uint32_t w = sws[t >> p.wshift] >> (pos & 31);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[i][k] *= ((w >> i) & 1u) ? sc : -sc;
        }
      }
    }
#pragma unroll
    for (int k = 0; k < (1 << GR); ++k) {
      const int64_t pos = pos0 + ((int64_t)k << kshift);
      if (DST == DST_SLICE) {
        const int64_t idx = bb + pos - p.start, hi = p.stop - p.start;
        T* dst = reinterpret_cast<T*>(p.dst) + idx;
        if (idx >= 0 && idx + 4 <= hi && (reinterpret_cast<uintptr_t>(dst) & (4 * sizeof(T) - 1)) == 0) {
          if (sizeof(T) == 2) {
            uint2 x;
            T* e = reinterpret_cast<T*>(&x);
#pragma unroll
            for (int i = 0; i < 4; ++i) e[i] = Cvt<T>::from_f(v[i][k]);
            *reinterpret_cast<uint2*>(dst) = x;
          } else {
            *reinterpret_cast<float4*>(dst) = make_float4(v[0][k], v[1][k], v[2][k], v[3][k]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i)
            if (idx + i >= 0 && idx + i < hi) dst[i] = Cvt<T>::from_f(v[i][k]);
        }
      } else if (brow_ok) {
        float* dst = reinterpret_cast<float*>(p.dst) + wrow + pos;
        if ((reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
          *reinterpret_cast<float4*>(dst) = make_float4(v[0][k], v[1][k], v[2][k], v[3][k]);
        } else {
#pragma unroll
          for (int i = 0; i < 4; ++i) dst[i] = v[i][k];
        }
      }
    }
  }
}

template <typename T, int SRC, int DST>
__device__ __forceinline__ void dispatch_run(const TileParams& p, const TileCtx& c, const RunDesc& rd,
                                             float* data, const uint32_t* signs, int wps, bool first,
                                             bool last) {
  if (DST != DST_ACC && first && last && rd.glo >= 2 && p.cb >= 2 && p.wshift >= 2 && rd.gr >= 1 && rd.gr <= 3) {
    switch (rd.gr) {
      case 1: do_run_v4<T, SRC, DST, 1>(p, c, rd, signs, wps); return;
      case 2: do_run_v4<T, SRC, DST, 2>(p, c, rd, signs, wps); return;
      default: do_run_v4<T, SRC, DST, 3>(p, c, rd, signs, wps); return;
    }
  }
  switch (rd.gr) {
    case 0: do_run<T, SRC, DST, 0>(p, c, rd, data, signs, wps, first, last); break;
    case 1: do_run<T, SRC, DST, 1>(p, c, rd, data, signs, wps, first, last); break;
    case 2: do_run<T, SRC, DST, 2>(p, c, rd, data, signs, wps, first, last); break;
    case 3: do_run<T, SRC, DST, 3>(p, c, rd, data, signs, wps, first, last); break;
    case 4: do_run<T, SRC, DST, 4>(p, c, rd, data, signs, wps, first, last); break;
    default: do_run<T, SRC, DST, 5>(p, c, rd, data, signs, wps, first, last); break;
  }
}

// Persistent tile kernel.  Shared memory: data (2^e + 2^e/32 floats), sign
// tables (nslots * 2^(e-wshift) words), and for DST_ACC an fp32 accumulator
// over the latent positions [L].
template <typename T, int SRC, int DST>
__global__ void __launch_bounds__(512) fht_tile_kernel(const __grid_constant__ TileParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int E = 1 << p.e;
  float* data = reinterpret_cast<float*>(smem_raw);
  uint32_t* signs = reinterpret_cast<uint32_t*>(data + E + (E >> 5));
  const int wps = E >> p.wshift;
  float* acc = reinterpret_cast<float*>(signs + p.nslots * wps);

  if (DST == DST_ACC)
    for (int i = threadIdx.x; i < p.L; i += blockDim.x) acc[i] = 0.0f;

  for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    TileCtx c;
    int64_t grp = tile / p.tiles_per_group;
    int64_t tib = tile - grp * p.tiles_per_group;
    c.tile_blk = p.first_block + (p.ublock ? (grp << p.m) : grp);
    c.fixed_pos = tib << p.rlo;

    // sign words for every slot used by this tile
    for (int i = threadIdx.x; i < p.nslots * wps; i += blockDim.x) {
      int s = i / wps, j = i - s * wps;
      int64_t pos, blk;
      tile_coords(p, c, j << p.wshift, pos, blk);
      signs[i] = sign_word(block_layer_key(p.seed32, blk, p.slot_layer[s]), pos >> 5);
    }
    __syncthreads();
    for (int ri = 0; ri < p.nruns; ++ri) {
      dispatch_run<T, SRC, DST>(p, c, p.runs[ri], data, signs, wps, ri == 0, ri == p.nruns - 1);
      __syncthreads();
    }
    if (DST == DST_ACC) {
      // sum the tile's blocks into the per-CTA latent-gradient accumulator
      const int nb = 1 << p.m;
      for (int i = threadIdx.x; i < p.L; i += blockDim.x) {
        float s = 0.0f;
        for (int bl = 0; bl < nb; ++bl) {
          if (c.tile_blk + bl - p.first_block < p.nblocks) s += data[pad_idx((bl << p.n) + i)];
        }
        acc[i] += s;
      }
      __syncthreads();
    }
  }
  if (DST == DST_ACC)
    for (int i = threadIdx.x; i < p.L; i += blockDim.x) p.partial[(int64_t)blockIdx.x * p.L + i] = acc[i];
}

}  // namespace lwl
