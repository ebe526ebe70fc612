// fht32.cuh -- whole-block BlockFHT in fp32 arithmetic for padded block sizes
// 2^5 .. 2^15 (forward and latent-gradient backward).
//
// The generic tile engine (fht_tile.cuh) spends most of its time on
// per-element bookkeeping (64-bit position math, bounds tests, a sign-table
// read per element).  This kernel instead keeps the data in registers:
//
//  * A CTA owns a "tile" of 2^TB consecutive generated coordinates
//    (2^(TB-n) whole blocks of B = 2^n; TB = 13 for n <= 13, so that four
//    CTAs of 128 threads share an SM and overlap each other's phases, else
//    TB = n with 2^(TB-6) threads).  Every thread holds 64 values; the TB tile
//    bits t are split into 6 register bits, 5 lane bits and TB-11 warp bits.
//    Three fixed splits ("sets") are used (shown for TB = 15):
//        A: registers t0..t5,  lanes t6..t10, warps t11..t14
//        B: registers t6..t11, lanes t0..t4,  warps t5, t12..t14
//        C: registers t9..t14, lanes t0..t4,  warps t5..t8
//    (C holds the top six tile bits).  A butterfly over a register bit is
//    pure register arithmetic.
//  * Between sets the tile goes through shared memory (one fp32 buffer of
//    2^TB words plus one pad word per 64).  With that padding the lanes of A
//    (t6..t10) and of B/C (t0..t4) fall on distinct banks, so every warp
//    access of both the writer and the reader is conflict free.
//  * The layer order is scheduled so that neighbouring layers share a set:
//    3 layers at n = 13..15 take 7 residencies (6 exchanges), at n = 7..12
//    four (3 exchanges), and at n <= 6 the whole chain runs in registers
//    (one exchange to lay the output out for coalesced stores).
//  * Signs: per tile and sign layer, the tile's sign words sit in shared
//    memory (the reference's stateless hash, lwl_common.cuh); a clear bit
//    flips the float's sign bit.  The layers' 1/sqrt(B) factors are applied
//    together, once, to the results (exact for even n, one rounding for odd n).
//  * The forward ends in set B or C, whose lanes run along t0..t4, so each
//    warp store writes 32 consecutive outputs.  The backward ends the same
//    way, sums the tile's blocks through shared memory and adds the result to
//    this CTA's [L] partial row in global memory (one thread per address, in
//    tile order, so the sums are deterministic); fht32_reduce_kernel then
//    sums the rows in a fixed order.
//
// Arithmetic is the reference's (fp32 butterflies and signs;
// latent_weight_lab/block_fht.py:18-33, 84-109) up to the order of the
// additions and where the normalisation is applied; results agree with the
// reference to fp32 rounding.
#include <algorithm>
#include <cmath>
#include <cstring>

#pragma once
#include "fht_engine.h"
#include "lwl_common.cuh"

namespace lwl {
namespace f32k {

constexpr int kRegs = 64;  // values per thread (6 register bits)
constexpr int kMaxSlots = 4;

template <int TB>
struct Tile {
  static constexpr int kE = 1 << TB;
  static constexpr int kThreads = 1 << (TB - 6);
  static constexpr int kWords = kE / 32;
  static constexpr int kBufWords = kE + kE / 16;
  static constexpr size_t kSmem = size_t(kBufWords) * 4 + size_t(kMaxSlots) * kWords * 4;
  static constexpr int kMinBlocks = TB == 13 ? 4 : 1;
  // register bits of the sets, as tile-bit masks
  static constexpr int kA = 0x3F, kB = 0xFC0, kC = 0x3F << (TB - 6);
  static constexpr int kChi = ((1 << TB) - 1) & ~0xFFF;       // C bits above B
  static constexpr int kBsub = ((1 << (TB - 6)) - 1) & ~0x3F;  // B bits below C
};

// Two more splits for TB = 15 (fht32_lo.cu) hold four consecutive tile
// elements (t0, t1) per register group, so a thread stores 16 bytes at once
// and a warp 512 (SD) or 2 x 256 (SD2) consecutive bytes:
//   SD:  registers t0, t1, t11..t14; lanes t2..t6;      warps t7..t10
//   SD2: registers t0, t1, t6..t9;   lanes t2..t5, t10; warps t11..t14
enum Set : int { SA = 0, SB = 1, SC = 2, SD = 3, SD2 = 4 };

template <int TB>
__host__ __device__ constexpr int reg_bit(int set, int j) {
  return set == SA ? j
       : set == SB ? 6 + j
       : set == SC ? TB - 6 + j
       : j < 2     ? j
       : set == SD ? TB - 6 + j
                   : 4 + j;
}

// tile index of register rho of this thread = base | spread(rho) (disjoint bits)
template <int TB, int SET>
__device__ __forceinline__ int base_of(int lane, int warp) {
  if (SET == SA) return (lane << 6) | (warp << 11);
  if (SET == SB) return lane | ((warp & 1) << 5) | ((warp >> 1) << 12);
  if (SET == SD) return (lane << 2) | (warp << 7);
  if (SET == SD2) return ((lane & 15) << 2) | ((lane >> 4) << 10) | (warp << 11);
  return lane | (warp << 5);
}
template <int TB, int SET>
__host__ __device__ constexpr int spread(int rho) {
  return SET == SA ? rho
       : SET == SB ? rho << 6
       : SET == SC ? rho << (TB - 6)
       : SET == SD ? (rho & 3) | ((rho >> 2) << (TB - 4))
                   : (rho & 3) | ((rho >> 2) << 6);
}
template <int SET>
__host__ __device__ constexpr bool quads() { return SET == SA || SET == SD || SET == SD2; }

// Shared-memory word address of tile element t: four pad words per 64.  For
// every set the lanes of a warp then hit distinct banks (lanes on t6..t10
// give bank t0..t4 + 4*lane, so each quarter-warp's 16-byte accesses of four
// consecutive registers cover all 32 banks; lanes on t0..t4 give
// lane + const), and pad(base | spread) = pad(base) + pad(spread), so each
// register's address is the thread's base plus a compile-time offset.  Set A
// moves four consecutive registers per 16-byte access.
__host__ __device__ constexpr int pad(int t) { return t + 4 * (t >> 6); }

struct Params {
  const void* src;  // forward: latent [L]; backward: grad slice [stop - start]
  void* dst;        // forward: output slice; backward: partial rows [grid][L]
  int64_t L;
  int n;            // log2 B (5..15)
  int layers;
  uint32_t seed32;
  float scale;      // 1/sqrt(B)^layers, applied once to the results
  int64_t start, stop;
  int64_t first_tile, ntiles, tile_step;  // tiles first_tile + i * tile_step, i < ntiles
  int row0;                               // backward: first partial row of this launch
  int slot_layer[kMaxSlots];              // sign layer of slot s, in chain order
};

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p) {
  return Cvt<T>::to_f(p[0]);
}

// Butterflies over the register bits of SET whose tile bits are in `mask`
// and below n (tile bits from n up select blocks, not positions).
template <int TB, int SET>
__device__ __forceinline__ void xform(float (&v)[kRegs], int mask, int n) {
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const int tb = reg_bit<TB>(SET, j);
    if (((mask >> tb) & 1) && tb < n) {
      const int h = 1 << j;
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        if (r & h) continue;
        const float a = v[r], b = v[r | h];
        v[r] = a + b;
        v[r | h] = a - b;
      }
    }
  }
}

// Sign flips of one layer: a clear sign bit negates (XOR of the float sign
// bit).  The 1/sqrt(B) of each layer is applied once, at the output.
__device__ __forceinline__ float flip(float x, uint32_t m) { return __uint_as_float(__float_as_uint(x) ^ m); }

template <int TB, int SET>
__device__ __forceinline__ void apply_sign(float (&v)[kRegs], const uint32_t* sw, int base) {
  if (SET == SA) {
    // t0..t4 are register bits: two words per thread; bit r of ~w moved to bit 31
    const uint32_t w0 = ~sw[base >> 5], w1 = ~sw[(base >> 5) | 1];
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const uint32_t w = (r & 32) ? w1 : w0;
      v[r] = flip(v[r], (w << (31 - (r & 31))) & 0x80000000u);
    }
  } else if (SET == SD || SET == SD2) {
    // t0, t1 are register bits, t2..t4 lane bits: one word per group of four
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const int t = base + spread<TB, SET>(4 * q);
      const uint32_t w = ~sw[t >> 5] >> (t & 31);
#pragma unroll
      for (int e = 0; e < 4; ++e) v[4 * q + e] = flip(v[4 * q + e], (w << (31 - e)) & 0x80000000u);
    }
  } else {
    // t0..t4 are the lane: one bit of a (warp-uniform) word per register;
    // (base >> 5) and (spread >> 5) have disjoint bits
    const int sh = 31 - (base & 31);
    const uint32_t* swb = sw + (base >> 5);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = flip(v[r], (~swb[spread<TB, SET>(r) >> 5] << sh) & 0x80000000u);
  }
}

template <int TB, int SET>
__device__ __forceinline__ void smem_write(const float (&v)[kRegs], float* b) {
  if (quads<SET>()) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q)
      *reinterpret_cast<float4*>(b + pad(spread<TB, SET>(4 * q))) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  } else {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) b[pad(spread<TB, SET>(r))] = v[r];
  }
}
template <int TB, int SET>
__device__ __forceinline__ void smem_read(float (&v)[kRegs], const float* b) {
  if (quads<SET>()) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const float4 x = *reinterpret_cast<const float4*>(b + pad(spread<TB, SET>(4 * q)));
      v[4 * q] = x.x, v[4 * q + 1] = x.y, v[4 * q + 2] = x.z, v[4 * q + 3] = x.w;
    }
  } else {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = b[pad(spread<TB, SET>(r))];
  }
}

template <int TB, int X, int Y>
__device__ __forceinline__ void exchange(float (&v)[kRegs], float* buf, int lane, int warp) {
  __syncthreads();  // every thread has finished reading the buffer
  smem_write<TB, X>(v, buf + pad(base_of<TB, X>(lane, warp)));
  __syncthreads();
  smem_read<TB, Y>(v, buf + pad(base_of<TB, Y>(lane, warp)));
}

// First residency: the tile's source values in set SET, zero outside the
// latent (forward) or the slice (backward).
template <typename T, int TB, int SET, bool BWD, bool FULL>
__device__ __forceinline__ void load_first(float (&v)[kRegs], const Params& p, int64_t tile, int base) {
  constexpr int kE = Tile<TB>::kE;
  const T* src = reinterpret_cast<const T*>(p.src);
  const int Bm = (1 << p.n) - 1;
  if (SET == SA) {
    // 64 consecutive tile elements per thread: 4-element vector loads where possible
    const T* s;
    int lo, hi;  // valid register offsets [lo, hi) relative to s
    if (BWD) {
      const int64_t off = (tile << TB) + base - p.start;
      s = src + off;
      lo = (int)std::min<int64_t>(std::max<int64_t>(-off, 0), kRegs);
      hi = (int)std::min<int64_t>(std::max<int64_t>(p.stop - p.start - off, 0), kRegs);
    } else {
      // position = t mod B; (base & Bm) and the register offsets have disjoint bits
      const int pb = base & Bm;
      s = src + pb;
      lo = 0;
      hi = (int)std::min<int64_t>(std::max<int64_t>(p.L - pb, 0), kRegs);
    }
    // vector loads need 4-element alignment, which a slice start not divisible by 4 breaks
    const bool vec = (reinterpret_cast<uintptr_t>(s) & (4 * sizeof(T) - 1)) == 0 &&
                     ((BWD && FULL) || (lo == 0 && hi == kRegs));
    if (vec) {
#pragma unroll
      for (int q = 0; q < kRegs / 4; ++q) {
        const int o = BWD ? 4 * q : ((4 * q) & Bm);
        if (sizeof(T) == 4) {
          const float4 x = *reinterpret_cast<const float4*>(s + o);
          v[4 * q] = x.x, v[4 * q + 1] = x.y, v[4 * q + 2] = x.z, v[4 * q + 3] = x.w;
        } else {
          const uint2 x = *reinterpret_cast<const uint2*>(s + o);
          const T* e = reinterpret_cast<const T*>(&x);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[4 * q + i] = Cvt<T>::to_f(e[i]);
        }
      }
    } else {
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int o = BWD ? r : (r & Bm);
        v[r] = (o >= lo && o < hi) ? ld_elem(s + o) : 0.0f;
      }
    }
  } else if (BWD && FULL) {
    const T* s = src + ((tile << TB) + base - p.start);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = ld_elem(s + spread<TB, SET>(r));
  } else if (BWD) {
    const int64_t off = (tile << TB) + base - p.start;
    const T* s = src + off;
    const int lo = (int)std::min<int64_t>(std::max<int64_t>(-off, 0), kE);
    const int hi = (int)std::min<int64_t>(std::max<int64_t>(p.stop - p.start - off, 0), kE);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int o = spread<TB, SET>(r);
      v[r] = (o >= lo && o < hi) ? ld_elem(s + o) : 0.0f;
    }
  } else {
    // position = t mod B; (base & Bm) and (spread & Bm) have disjoint bits
    const int pb = base & Bm;
    const T* s = src + pb;
    if (p.L == Bm + 1) {
#pragma unroll
      for (int r = 0; r < kRegs; ++r) v[r] = ld_elem(s + (spread<TB, SET>(r) & Bm));
    } else {
      const int hi = (int)std::min<int64_t>(p.L - pb, kE);
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int q = spread<TB, SET>(r) & Bm;
        v[r] = q < hi ? ld_elem(s + q) : 0.0f;
      }
    }
  }
}

// First residency in set A.  The backward's gradient slice arrives in set SD
// (four consecutive elements per register group, lanes on t2..t6: each warp
// load covers 512 contiguous bytes of fp32) and moves to set A through shared
// memory; set A's own loads (one 16-byte load per lane at a 256-byte stride)
// keep the L1 request queue full.  The forward reads the latent the same way
// (it is L2-resident, but the L1 request cost is the same), except for blocks
// of <= 128, whose positions repeat across the lanes of a set-A load (the
// SD path measured 3-5% slower at 128).
template <typename T, int TB, bool BWD, bool FULL>
__device__ __forceinline__ void load_first_a(float (&v)[kRegs], const Params& p, int64_t tile, int bA, float* buf,
                                             int lane, int warp, int n) {
  if (!BWD && n <= 7) {  // blocks of <= 128: a warp's lanes read the same few latent lines
    load_first<T, TB, SA, BWD, FULL>(v, p, tile, bA);
    return;
  }
  if (!BWD) {
    // latent positions (t mod B) of set SD: four consecutive per register group
    const int bD = base_of<TB, SD>(lane, warp);
    const int Bm = (1 << n) - 1;
    const T* src = reinterpret_cast<const T*>(p.src);
    const bool vec = (reinterpret_cast<uintptr_t>(src) & (4 * sizeof(T) - 1)) == 0;
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const int pos = (bD | spread<TB, SD>(4 * q)) & Bm;
      if (vec && pos + 4 <= p.L) {
        if (sizeof(T) == 4) {
          const float4 a = *reinterpret_cast<const float4*>(src + pos);
          v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
        } else {
          const uint2 a = *reinterpret_cast<const uint2*>(src + pos);
          const T* h = reinterpret_cast<const T*>(&a);
#pragma unroll
          for (int i = 0; i < 4; ++i) v[4 * q + i] = Cvt<T>::to_f(h[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * q + i] = pos + i < p.L ? ld_elem(src + pos + i) : 0.0f;
      }
    }
    exchange<TB, SD, SA>(v, buf, lane, warp);
    return;
  }
  const int bD = base_of<TB, SD>(lane, warp);
  const T* src = reinterpret_cast<const T*>(p.src);
  const int64_t off = (tile << TB) + bD - p.start;
  const T* s = src + off;
  if (FULL && (reinterpret_cast<uintptr_t>(s) & (4 * sizeof(T) - 1)) == 0) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const T* e = s + spread<TB, SD>(4 * q);
      if (sizeof(T) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(e);
        v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
      } else {
        const uint2 a = *reinterpret_cast<const uint2*>(e);
        const T* h = reinterpret_cast<const T*>(&a);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * q + i] = Cvt<T>::to_f(h[i]);
      }
    }
  } else {
    constexpr int kE = Tile<TB>::kE;
    const int lo = (int)std::min<int64_t>(std::max<int64_t>(-off, 0), kE);
    const int hi = (int)std::min<int64_t>(std::max<int64_t>(p.stop - p.start - off, 0), kE);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int o = spread<TB, SD>(r);
      v[r] = (o >= lo && o < hi) ? ld_elem(s + o) : 0.0f;
    }
  }
  exchange<TB, SD, SA>(v, buf, lane, warp);
}

// Forward output from set B or C (lanes along t0..t4: 32 consecutive outputs per warp store).
template <typename T, int TB, int SET, bool FULL>
__device__ __forceinline__ void store_out(const float (&v)[kRegs], const Params& p, int64_t tile, int base) {
  constexpr int kE = Tile<TB>::kE;
  const int64_t off = (tile << TB) - p.start + base;
  T* dst = reinterpret_cast<T*>(p.dst) + off;
  if (FULL) {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) dst[spread<TB, SET>(r)] = Cvt<T>::from_f(v[r] * p.scale);
    return;
  }
  // valid offsets [lo, hi) relative to dst (the whole tile unless it straddles the slice)
  const int lo = (int)std::min<int64_t>(std::max<int64_t>(-off, 0), kE);
  const int hi = (int)std::min<int64_t>(std::max<int64_t>(p.stop - p.start - off, 0), kE);
#pragma unroll
  for (int r = 0; r < kRegs; ++r) {
    const int o = spread<TB, SET>(r);
    if (o >= lo && o < hi) dst[o] = Cvt<T>::from_f(v[r] * p.scale);
  }
}

// Backward: the tile's per-block results (set B or C) summed over its blocks
// into this CTA's partial row.  Register bits that select blocks (tile bits at
// or above n) are summed in registers first; the rest of the block bits are
// summed through shared memory.  Thread i owns positions i, i + threads, ...
// for the whole kernel, so each address sees its additions in tile order.
template <int TB, int SET>
__device__ __forceinline__ void accumulate(float (&v)[kRegs], float* buf, const Params& p, int base, int tid, int n) {
  int regmask = 0;  // tile bits of the register bits summed here
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const int tb = reg_bit<TB>(SET, j);
    if (tb >= n) {
      regmask |= 1 << tb;
      const int h = 1 << j;
#pragma unroll
      for (int r = 0; r < kRegs; ++r)
        if (!(r & h)) v[r] += v[r | h];
    }
  }
  __syncthreads();
  float* wb = buf + pad(base);
#pragma unroll
  for (int r = 0; r < kRegs; ++r)
    if (!(spread<TB, SET>(r) & regmask)) wb[pad(spread<TB, SET>(r))] = v[r];
  __syncthreads();
  float* row = reinterpret_cast<float*>(p.dst) + (int64_t)(p.row0 + blockIdx.x) * p.L;
  const int nb = 1 << (TB - n);
  for (int q = tid; q < p.L; q += Tile<TB>::kThreads) {
    float s = 0.0f;
    for (int k = 0; k < nb; ++k)
      if (!((k << n) & regmask)) s += buf[pad((k << n) | q)];
    atomicAdd(row + q, s * p.scale);  // one thread per address: program order, deterministic
  }
}

// Residency schedules.  KCLS 1: n <= 6 (one register set); 2: n = 7..12 (sets
// A and B); 3: n = 13..15 (A, B and C = the top six bits).  Slot 0 is the
// pre-sign (no scale); slot l+1 follows network l and carries 1/sqrt(B).
template <typename T, int TB, int LAYERS, bool BWD, int KCLS, bool FULL, int NB>
__global__ void __launch_bounds__(Tile<TB>::kThreads, Tile<TB>::kMinBlocks)
    fht32_kernel(const __grid_constant__ Params p) {
  using Tl = Tile<TB>;
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  uint32_t* sw = reinterpret_cast<uint32_t*>(buf + Tl::kBufWords);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // NB > 0: block size fixed at compile time, so the butterflies of the bits at
  // and above n (block-select bits) are dropped rather than predicated off
  const int n = NB > 0 ? NB : p.n;
  if (BWD) {
    float* row = reinterpret_cast<float*>(p.dst) + (int64_t)(p.row0 + blockIdx.x) * p.L;
    for (int q = tid; q < p.L; q += Tl::kThreads) row[q] = 0.0f;
  }
  const int bA = base_of<TB, SA>(lane, warp), bB = base_of<TB, SB>(lane, warp), bC = base_of<TB, SC>(lane, warp);
  float v[kRegs];
  for (int64_t it = blockIdx.x; it < p.ntiles; it += gridDim.x) {
    const int64_t tile = p.first_tile + it * p.tile_step;
    if (BWD && TB > 13 && tid == 0 && it + gridDim.x < p.ntiles) {
      // one CTA per SM at TB > 13: the next tile's gradient slice into L2 while this one runs
      const int64_t g0 = ((p.first_tile + (it + gridDim.x) * p.tile_step) << TB) - p.start, ns = p.stop - p.start;
      const int64_t lo = g0 > 0 ? g0 : 0, hi = g0 + (1 << TB) < ns ? g0 + (1 << TB) : ns;
      if (hi > lo) prefetch_l2(p.src, lo * (int64_t)sizeof(T), hi * (int64_t)sizeof(T));
    }
    __syncthreads();  // the previous tile is done with the sign table
    {
      const int wsh = n - 5;  // words per block = 2^(n-5)
      const int64_t blk0 = tile << (TB - n);
      for (int i = tid; i < (LAYERS + 1) * Tl::kWords; i += Tl::kThreads) {
        const int s = i / Tl::kWords, c = i - s * Tl::kWords;
        sw[i] = sign_word(block_layer_key(p.seed32, blk0 + (c >> wsh), p.slot_layer[s]), c & ((1 << wsh) - 1));
      }
    }
    __syncthreads();
    const uint32_t* s0 = sw;
    const uint32_t* s1 = sw + Tl::kWords;
    const uint32_t* s2 = sw + 2 * Tl::kWords;
    const uint32_t* s3 = sw + 3 * Tl::kWords;
    if constexpr (KCLS == 1) {
      load_first_a<T, TB, BWD, FULL>(v, p, tile, bA, buf, lane, warp, n);
      apply_sign<TB, SA>(v, s0, bA);
      xform<TB, SA>(v, Tl::kA, n);
      apply_sign<TB, SA>(v, s1, bA);
      if (LAYERS >= 2) {
        xform<TB, SA>(v, Tl::kA, n);
        apply_sign<TB, SA>(v, s2, bA);
      }
      if (LAYERS >= 3) {
        xform<TB, SA>(v, Tl::kA, n);
        apply_sign<TB, SA>(v, s3, bA);
      }
      // (outputs from set SD instead measured 10-15% slower at n = 5, 6)
      exchange<TB, SA, SB>(v, buf, lane, warp);
      if (BWD) accumulate<TB, SB>(v, buf, p, bB, tid, n);
      else store_out<T, TB, SB, FULL>(v, p, tile, bB);
    } else if constexpr (KCLS == 2) {
      if (LAYERS == 2) {
        load_first<T, TB, SB, BWD, FULL>(v, p, tile, bB);
        apply_sign<TB, SB>(v, s0, bB);
        xform<TB, SB>(v, Tl::kB, n);
        exchange<TB, SB, SA>(v, buf, lane, warp);
        xform<TB, SA>(v, Tl::kA, n);
        apply_sign<TB, SA>(v, s1, bA);
        xform<TB, SA>(v, Tl::kA, n);
        exchange<TB, SA, SB>(v, buf, lane, warp);
        xform<TB, SB>(v, Tl::kB, n);
        apply_sign<TB, SB>(v, s2, bB);
      } else {
        load_first_a<T, TB, BWD, FULL>(v, p, tile, bA, buf, lane, warp, n);
        apply_sign<TB, SA>(v, s0, bA);
        xform<TB, SA>(v, Tl::kA, n);
        exchange<TB, SA, SB>(v, buf, lane, warp);
        xform<TB, SB>(v, Tl::kB, n);
        apply_sign<TB, SB>(v, s1, bB);
        if (LAYERS == 3) {
          xform<TB, SB>(v, Tl::kB, n);
          exchange<TB, SB, SA>(v, buf, lane, warp);
          xform<TB, SA>(v, Tl::kA, n);
          apply_sign<TB, SA>(v, s2, bA);
          xform<TB, SA>(v, Tl::kA, n);
          exchange<TB, SA, SB>(v, buf, lane, warp);
          xform<TB, SB>(v, Tl::kB, n);
          apply_sign<TB, SB>(v, s3, bB);
        }
      }
      if (BWD) accumulate<TB, SB>(v, buf, p, bB, tid, n);
      else store_out<T, TB, SB, FULL>(v, p, tile, bB);
    } else {
      if (LAYERS == 2) {
        load_first<T, TB, SC, BWD, FULL>(v, p, tile, bC);
        apply_sign<TB, SC>(v, s0, bC);
        xform<TB, SC>(v, Tl::kC, n);
        exchange<TB, SC, SA>(v, buf, lane, warp);
        xform<TB, SA>(v, Tl::kA, n);
        exchange<TB, SA, SB>(v, buf, lane, warp);
        xform<TB, SB>(v, Tl::kBsub, n);
        apply_sign<TB, SB>(v, s1, bB);
        xform<TB, SB>(v, Tl::kB, n);
        exchange<TB, SB, SA>(v, buf, lane, warp);
        xform<TB, SA>(v, Tl::kA, n);
        exchange<TB, SA, SC>(v, buf, lane, warp);
        xform<TB, SC>(v, Tl::kChi, n);
        apply_sign<TB, SC>(v, s2, bC);
      } else {
        load_first_a<T, TB, BWD, FULL>(v, p, tile, bA, buf, lane, warp, n);
        apply_sign<TB, SA>(v, s0, bA);
        xform<TB, SA>(v, Tl::kA, n);
        exchange<TB, SA, SB>(v, buf, lane, warp);
        xform<TB, SB>(v, Tl::kB, n);
        exchange<TB, SB, SC>(v, buf, lane, warp);
        xform<TB, SC>(v, Tl::kChi, n);
        apply_sign<TB, SC>(v, s1, bC);
        if (LAYERS == 3) {
          xform<TB, SC>(v, Tl::kC, n);
          exchange<TB, SC, SA>(v, buf, lane, warp);
          xform<TB, SA>(v, Tl::kA, n);
          exchange<TB, SA, SB>(v, buf, lane, warp);
          xform<TB, SB>(v, Tl::kBsub, n);
          apply_sign<TB, SB>(v, s2, bB);
          xform<TB, SB>(v, Tl::kB, n);
          exchange<TB, SB, SA>(v, buf, lane, warp);
          xform<TB, SA>(v, Tl::kA, n);
          exchange<TB, SA, SC>(v, buf, lane, warp);
          xform<TB, SC>(v, Tl::kChi, n);
          apply_sign<TB, SC>(v, s3, bC);
        }
      }
      // (outputs from set SD, one 16-byte store per register group, measured
      // 1-10% slower here than set C's 4-byte stores of 32 consecutive outputs)
      if (BWD) accumulate<TB, SC>(v, buf, p, bC, tid, n);
      else store_out<T, TB, SC, FULL>(v, p, tile, bC);
    }
  }
}

inline int tile_bits(int n) { return n <= 13 ? 13 : n; }

// Kernel of one (dtype, tile size, layer count, direction, full tiles), chosen
// by n.  fp32 full tiles get a kernel per block size (NB = n); slice edges and
// the 16-bit exact mode share one kernel per size class (NB = 0).
template <typename T, int TB, int LAYERS, bool BWD, bool FULL, int KCLS>
const void* by_n(int n) {
  if constexpr (FULL && sizeof(T) == 4) {
    if constexpr (KCLS == 1) {
      return n == 5 ? (const void*)fht32_kernel<T, TB, LAYERS, BWD, 1, FULL, 5>
                    : (const void*)fht32_kernel<T, TB, LAYERS, BWD, 1, FULL, 6>;
    } else if constexpr (KCLS == 2) {
      switch (n) {
        case 7: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 7>;
        case 8: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 8>;
        case 9: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 9>;
        case 10: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 10>;
        case 11: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 11>;
        default: return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 2, FULL, 12>;
      }
    } else {
      return (const void*)fht32_kernel<T, TB, LAYERS, BWD, 3, FULL, TB>;  // class 3: n == TB
    }
  } else {
    return (const void*)fht32_kernel<T, TB, LAYERS, BWD, KCLS, FULL, 0>;
  }
}

template <typename T, int TB, int LAYERS, bool BWD, bool FULL>
const void* kernel_for(int n) {
  if constexpr (TB > 13) {
    return by_n<T, TB, LAYERS, BWD, FULL, 3>(n);
  } else {
    if (n <= 6) return by_n<T, TB, LAYERS, BWD, FULL, 1>(n);
    if (n <= 12) return by_n<T, TB, LAYERS, BWD, FULL, 2>(n);
    return by_n<T, TB, LAYERS, BWD, FULL, 3>(n);
  }
}

template <typename T, bool BWD, bool FULL>
const void* pick_tb(int n, int layers, int TB) {
  if (TB == 13)
    return layers == 1 ? kernel_for<T, 13, 1, BWD, FULL>(n)
                       : (layers == 2 ? kernel_for<T, 13, 2, BWD, FULL>(n) : kernel_for<T, 13, 3, BWD, FULL>(n));
  if (TB == 14)
    return layers == 1 ? kernel_for<T, 14, 1, BWD, FULL>(n)
                       : (layers == 2 ? kernel_for<T, 14, 2, BWD, FULL>(n) : kernel_for<T, 14, 3, BWD, FULL>(n));
  return layers == 1 ? kernel_for<T, 15, 1, BWD, FULL>(n)
                     : (layers == 2 ? kernel_for<T, 15, 2, BWD, FULL>(n) : kernel_for<T, 15, 3, BWD, FULL>(n));
}

template <typename T, bool BWD>
const void* pick(bool full, int n, int layers, int TB) {
  return full ? pick_tb<T, BWD, true>(n, layers, TB) : pick_tb<T, BWD, false>(n, layers, TB);
}

// Kernel entry points of the four translation units that instantiate the
// kernels (fp32 / 16-bit exact mode x forward / backward), split so that they
// compile in parallel.
const void* kernel_f32_fwd(bool full, int n, int layers);
const void* kernel_f32_bwd(bool full, int n, int layers);
const void* kernel_half_fwd(int dtype, bool full, int n, int layers);
const void* kernel_half_bwd(int dtype, bool full, int n, int layers);

}  // namespace f32k
}  // namespace lwl
