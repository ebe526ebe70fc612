// fhts.cu -- small blocks (padded block size B = 2^5 .. 2^10), every dtype,
// fp32 arithmetic, forward and backward.
//
// The work unit is a warp tile of 1024 consecutive coordinates (2^(10-n)
// whole blocks).  Lane l holds the 32 coordinates 32 l .. 32 l + 31 of the
// tile in fp32 registers, so
//   * position bits 0..4 are register bits: those butterflies are register
//     arithmetic (one add per value per bit);
//   * position bits 5..n-1 are the low lane bits: one shfl.bfly + one FMA per
//     value per bit;
//   * the lane's 32 positions are exactly one sign word of the stateless hash
//     (latent_weight_lab/block_fht.py:46-81): one hash per lane per layer,
//     and the flip is a select of v or -v per bit.
// The chain is the reference's (block_fht.py:84-109): y_b = S_L H .. S_1 H S_0
// pad(z) with the layers' 1/sqrt(B) applied once at the end (the backward is
// the transposed chain, S_0 last, summed over blocks).
//
// Global memory moves in whole 16-byte chunks through a per-warp shared
// buffer: lane l owns chunks 4l..4l+3 (16-bit) or 8l..8l+7 (fp32) of the tile,
// the warp's global accesses are chunks l, l + 32, ... (512 contiguous bytes
// per instruction).  swz() XORs the chunk index with bits 3..5 so both the
// owner's and the streaming side's accesses are bank-conflict free.  Tiles
// that straddle the slice's ends, or slices not aligned to a chunk, go element
// by element (still lane-contiguous) with bounds tests.
//
// The forward's input is the same padded latent for every block, so each lane
// loads its 32 latent values once per launch (with the layers' 1/sqrt(B)
// folded in).  The backward streams its gradient tiles into two buffers per
// warp by cp.async, one tile ahead of the transform, and keeps the lane's
// 32 partial sums of the latent gradient in registers across its tiles; at
// the end lanes and warps holding the same positions are summed in a fixed
// order and each CTA writes one [L] row, which fhts_reduce_kernel adds up in a
// fixed order (deterministic, like every backward in this library).
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "fht_engine.h"
#include "lwl_common.cuh"

namespace lwl {
namespace smallk {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kTileLog = 10;
constexpr int kMinLog = 5, kMaxLog = 10;
constexpr int kXp = 10;                  // blocks of 2^10: lane bits by shared-memory transpose
constexpr int kBufBytes = 32 * 33 * 4;   // per warp: one tile in fp32 (16-bit tiles use less), or the
                                         // padded 32 x 33 transpose buffer

struct SParams {
  const void* src;  // forward: latent [L]; backward: gradient slice [stop - start]
  void* dst;        // forward: output slice [stop - start]; backward: fp32 rows [gridDim.x][L]
  int64_t L, start, stop;
  int64_t t_first, ntiles;  // warp tiles (1024 coordinates) touched by [start, stop)
  int layers;
  uint32_t seed32;
  float scale;  // B^(-layers/2): the forward multiplies the latent by it, the backward its sums
  int vec_ok;   // data pointer and slice start aligned to a 16-byte chunk
};

__device__ __forceinline__ int swz(int c) { return c ^ ((c >> 3) & 7); }

// Sign layer: bit r of w set -> +1, clear -> -1 (block_fht.py:55-81).  A
// select of v or -v per bit measured 2-8% faster than XOR-ing the shifted bit
// into the float's sign bit (same result bit for bit).
__device__ __forceinline__ void apply_sign(float (&v)[32], uint32_t w) {
#pragma unroll
  for (int r = 0; r < 32; ++r) v[r] = (w & (1u << r)) ? v[r] : -v[r];
}

// Unnormalised H over register bits 0 .. NB-1.
template <int NB = 5>
__device__ __forceinline__ void fht_regs(float (&v)[32]) {
#pragma unroll
  for (int h = 1; h < (1 << NB); h <<= 1) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      if (!(i & h)) {
        const float a = v[i], b = v[i + h];
        v[i] = a + b;
        v[i + h] = a - b;
      }
    }
  }
}

// Unnormalised butterflies over lane bits 0 .. N-6 (position bits 5 .. N-1):
// the lane with the bit clear keeps a + b, the other b' = a - b.
template <int N>
__device__ __forceinline__ void fht_lanes(float (&v)[32], int lane) {
#pragma unroll
  for (int j = 0; j < N - 5; ++j) {
    const int m = 1 << j;
    const float s = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const float o = __shfl_xor_sync(0xffffffffu, v[r], m);
      v[r] = fmaf(s, v[r], o);
    }
  }
}

// Blocks of 2^10 hold position bits 5..9 on all 5 lane bits, where a shuffle
// per value per bit costs more than moving the tile once per layer (measured:
// +8-17% at 2^10, and no gain at 2^9, whose 4 lane bits the shuffles keep):
// the warp's 32 x 32 tile M (row = lane, 32 consecutive positions per row:
// "orientation A") is transposed through a padded shared buffer, so that
// lane b holds column b ("orientation B": v[r] = M[r][b], register bits =
// position bits 5..9).  Both accesses of the buffer are bank-conflict free
// ((lane + r) mod 32 distinct).  The transpose is its own inverse.
__device__ __forceinline__ void xpose(float (&v)[32], float* tb, int lane) {
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 32; ++r) tb[lane * 33 + r] = v[r];
  __syncwarp();
#pragma unroll
  for (int r = 0; r < 32; ++r) v[r] = tb[r * 33 + lane];
}

// 32 x 32 bit-matrix transpose across the warp: lane a holds word w_a on
// entry; on exit lane b holds the word whose bit a is bit b of w_a (the sign
// bits of column b in orientation B).  Recursive block swap, five shuffles.
__device__ __forceinline__ uint32_t bit_xpose(uint32_t x, int lane) {
  constexpr uint32_t lo[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int s = 0; s < 5; ++s) {
    const int j = 16 >> s;
    const uint32_t y = __shfl_xor_sync(0xffffffffu, x, j);
    x = (lane & j) ? ((x & ~lo[s]) | ((y & ~lo[s]) >> j)) : ((x & lo[s]) | ((y & lo[s]) << j));
  }
  return x;
}

// One unnormalised H_B of a block of 2^N in the transpose scheme: the
// register bits of the current orientation, the transpose, the register bits
// of the other; returns the new orientation.
template <int N>
__device__ __forceinline__ int fht_xp(float (&v)[32], float* tb, int lane, int ori) {
  if (ori == 0) {
    fht_regs<5>(v);
    xpose(v, tb, lane);
    fht_regs<N - 5>(v);
  } else {
    fht_regs<N - 5>(v);
    xpose(v, tb, lane);
    fht_regs<5>(v);
  }
  return ori ^ 1;
}

template <typename T> struct Chunk;
template <> struct Chunk<float> {
  static constexpr int E = 4;  // elements per 16-byte chunk
  static __device__ __forceinline__ uint4 pack(const float* v) {
    return make_uint4(__float_as_uint(v[0]), __float_as_uint(v[1]), __float_as_uint(v[2]), __float_as_uint(v[3]));
  }
  static __device__ __forceinline__ void unpack(uint4 c, float* v) {
    v[0] = __uint_as_float(c.x);
    v[1] = __uint_as_float(c.y);
    v[2] = __uint_as_float(c.z);
    v[3] = __uint_as_float(c.w);
  }
};
template <typename H> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t w) {
    return __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&w));
  }
};
template <> struct Pair<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack(uint32_t w) { return __half22float2(*reinterpret_cast<__half2*>(&w)); }
};
template <typename H> struct Chunk16 {
  static constexpr int E = 8;
  static __device__ __forceinline__ uint4 pack(const float* v) {
    return make_uint4(Pair<H>::pack(v[0], v[1]), Pair<H>::pack(v[2], v[3]), Pair<H>::pack(v[4], v[5]),
                      Pair<H>::pack(v[6], v[7]));
  }
  static __device__ __forceinline__ void unpack(uint4 c, float* v) {
    const uint32_t w[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = Pair<H>::unpack(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
};
template <> struct Chunk<__nv_bfloat16> : Chunk16<__nv_bfloat16> {};
template <> struct Chunk<__half> : Chunk16<__half> {};

template <typename T, int N>
__global__ void __launch_bounds__(kThreads) fhts_forward_kernel(const __grid_constant__ SParams P) {
  __shared__ __align__(16) unsigned char sbuf[kWarps][kBufBytes];
  constexpr int E = Chunk<T>::E, CPT = 32 / E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lp = lane & ((1 << (N - 5)) - 1);  // position bits 5 .. N-1
  unsigned char* wb = sbuf[warp];
  constexpr bool XP = N >= kXp;
  // transpose scheme: start in orientation B for odd layer counts, so that the
  // last layer ends in A, whose rows of 32 consecutive positions are stored
  const int ori0 = XP ? (P.layers & 1) : 0;
  float zin[32];
  {
    const T* z = reinterpret_cast<const T*>(P.src);
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const int p = ori0 ? ((32 * r + lane) & ((1 << N) - 1)) : 32 * lp + r;
      zin[r] = p < P.L ? Cvt<T>::to_f(z[p]) * P.scale : 0.0f;  // the layers' 1/sqrt(B), once
    }
  }
  T* out = reinterpret_cast<T*>(P.dst);
  const int64_t nw = (int64_t)gridDim.x * kWarps;
  for (int64_t t = (int64_t)blockIdx.x * kWarps + warp; t < P.ntiles; t += nw) {
    const int64_t base = (P.t_first + t) << kTileLog;
    const int64_t blk = (base + 32 * lane) >> N;
    float v[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) v[r] = zin[r];
    if (XP) {
      float* tb = reinterpret_cast<float*>(wb);
      int ori = ori0;
      uint32_t w = sign_word(block_layer_key(P.seed32, blk, 0), lp);  // row `lane`'s word
      apply_sign(v, ori ? bit_xpose(w, lane) : w);
      for (int l = 1; l <= P.layers; ++l) {
        ori = fht_xp<N>(v, tb, lane, ori);
        w = sign_word(block_layer_key(P.seed32, blk, l), lp);
        apply_sign(v, ori ? bit_xpose(w, lane) : w);
      }
    } else {
      apply_sign(v, sign_word(block_layer_key(P.seed32, blk, 0), lp));
      for (int l = 1; l <= P.layers; ++l) {
        fht_regs(v);
        fht_lanes<N>(v, lane);
        apply_sign(v, sign_word(block_layer_key(P.seed32, blk, l), lp));
      }
    }
    __syncwarp();  // the previous tile's reads of the buffer are done
#pragma unroll
    for (int q = 0; q < CPT; ++q)
      *reinterpret_cast<uint4*>(wb + 16 * swz(CPT * lane + q)) = Chunk<T>::pack(v + E * q);
    __syncwarp();
    if (P.vec_ok && base >= P.start && base + (1 << kTileLog) <= P.stop) {
      uint4* dst = reinterpret_cast<uint4*>(out + (base - P.start));
#pragma unroll
      for (int k = 0; k < CPT; ++k) {
        const int c = lane + 32 * k;
        dst[c] = *reinterpret_cast<const uint4*>(wb + 16 * swz(c));
      }
    } else {
      const T* tb = reinterpret_cast<const T*>(wb);
      for (int k = 0; k < 32; ++k) {
        const int e = lane + 32 * k;
        const int64_t gi = base + e;
        if (gi >= P.start && gi < P.stop) out[gi - P.start] = tb[E * swz(e / E) + (e % E)];
      }
    }
  }
}

// Shared memory of the backward: two tile buffers per warp (the next tile's
// chunks arrive by cp.async while the current one is transformed); the same
// bytes serve the final cross-warp sums.
template <typename T, int N>
constexpr int bwd_tile_bytes() {  // one per-warp buffer: a tile, or the transpose buffer
  return N >= kXp && kBufBytes > 32 * 32 * (int)sizeof(T) ? kBufBytes : 32 * 32 * (int)sizeof(T);
}
template <typename T, int N>
constexpr int bwd_smem() {
  return 2 * kWarps * bwd_tile_bytes<T, N>() > kWarps * (1 << N) * 4 ? 2 * kWarps * bwd_tile_bytes<T, N>()
                                                                     : kWarps * (1 << N) * 4;
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
               "l"(gmem)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;\n" ::: "memory"); }

template <typename T, int N>
__global__ void __launch_bounds__(kThreads) fhts_backward_kernel(const __grid_constant__ SParams P) {
  constexpr int B = 1 << N;
  constexpr int TileBytes = bwd_tile_bytes<T, N>();  // a multiple of 16
  constexpr bool XP = N >= kXp;
  extern __shared__ __align__(16) unsigned char sbuf[];
  constexpr int E = Chunk<T>::E, CPT = 32 / E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int lp = lane & ((1 << (N - 5)) - 1);
  unsigned char* wb0 = sbuf + warp * 2 * TileBytes;
  const T* g = reinterpret_cast<const T*>(P.src);
  auto fast = [&](int64_t base) { return P.vec_ok && base >= P.start && base + (1 << kTileLog) <= P.stop; };
  // whole tiles inside the slice: 16-byte chunks straight into the buffer
  auto issue = [&](int64_t t, unsigned char* wb) {
    const int64_t base = (P.t_first + t) << kTileLog;
    if (t < P.ntiles && fast(base)) {
      const uint4* src = reinterpret_cast<const uint4*>(g + (base - P.start));
#pragma unroll
      for (int k = 0; k < CPT; ++k) cp_async16(wb + 16 * swz(lane + 32 * k), src + lane + 32 * k);
    }
    cp_async_commit();
  };
  float acc[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) acc[r] = 0.0f;
  const int64_t nw = (int64_t)gridDim.x * kWarps;
  int buf = 0;
  const int64_t t0 = (int64_t)blockIdx.x * kWarps + warp;
  issue(t0, wb0);
  for (int64_t t = t0; t < P.ntiles; t += nw, buf ^= 1) {
    const int64_t base = (P.t_first + t) << kTileLog;
    const int64_t blk = (base + 32 * lane) >> N;
    unsigned char* wb = wb0 + buf * TileBytes;
    issue(t + nw, wb0 + (buf ^ 1) * TileBytes);  // the other buffer was released at the end of the last tile
    cp_async_wait1();                            // this tile's chunks have landed
    if (!fast(base)) {
      T* tb = reinterpret_cast<T*>(wb);
      for (int k = 0; k < 32; ++k) {
        const int e = lane + 32 * k;
        const int64_t gi = base + e;
        tb[E * swz(e / E) + (e % E)] = (gi >= P.start && gi < P.stop) ? g[gi - P.start] : Cvt<T>::from_f(0.0f);
      }
    }
    __syncwarp();
    float v[32];
#pragma unroll
    for (int q = 0; q < CPT; ++q)
      Chunk<T>::unpack(*reinterpret_cast<const uint4*>(wb + 16 * swz(CPT * lane + q)), v + E * q);
    __syncwarp();  // every lane is done with this buffer
    if (XP) {
      // the buffer is free until the next tile's issue: it serves the transposes
      float* tb = reinterpret_cast<float*>(wb);
      int ori = 0;
      apply_sign(v, sign_word(block_layer_key(P.seed32, blk, P.layers), lp));
      for (int l = P.layers - 1; l >= 0; --l) {
        ori = fht_xp<N>(v, tb, lane, ori);
        const uint32_t w = sign_word(block_layer_key(P.seed32, blk, l), lp);
        apply_sign(v, ori ? bit_xpose(w, lane) : w);
      }
    } else {
      apply_sign(v, sign_word(block_layer_key(P.seed32, blk, P.layers), lp));
      for (int l = P.layers - 1; l >= 0; --l) {
        fht_regs(v);
        fht_lanes<N>(v, lane);
        apply_sign(v, sign_word(block_layer_key(P.seed32, blk, l), lp));
      }
    }
#pragma unroll
    for (int r = 0; r < 32; ++r) acc[r] += v[r];
  }
  asm volatile("cp.async.wait_all;\n" ::: "memory");  // nothing of this CTA may still be landing
  float* red = reinterpret_cast<float*>(sbuf);  // [kWarps][B]
  if (XP && (P.layers & 1)) {
    // odd layer counts end in orientation B: lane b, register r holds position
    // 32 (r mod B/32) + b; registers that differ in block-select bits are summed
#pragma unroll
    for (int m = B >> 5; m < 32; m <<= 1) {
#pragma unroll
      for (int r = 0; r < 32; ++r)
        if (!(r & m)) acc[r] += acc[r | m];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < (B >> 5); ++r) red[warp * B + 32 * r + lane] = acc[r];
  } else {
    // lanes that differ only in the block-select bits hold the same positions
#pragma unroll
    for (int m = 1 << (N - 5); m < 32; m <<= 1) {
#pragma unroll
      for (int r = 0; r < 32; ++r) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], m);
    }
    __syncthreads();
    if (lane < (B >> 5)) {
#pragma unroll
      for (int r = 0; r < 32; ++r) red[warp * B + 32 * lane + r] = acc[r];
    }
  }
  __syncthreads();
  float* row = reinterpret_cast<float*>(P.dst) + (int64_t)blockIdx.x * P.L;
  for (int p = threadIdx.x; p < P.L; p += kThreads) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) s += red[w * B + p];
    row[p] = s * P.scale;
  }
}

template <typename T>
__global__ void fhts_reduce_kernel(const float* __restrict__ rows, int nrows, int64_t L, T* __restrict__ out) {
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

template <typename T, bool BWD, int N>
const void* kernel_n() {
  return BWD ? (const void*)fhts_backward_kernel<T, N> : (const void*)fhts_forward_kernel<T, N>;
}
template <typename T>
int bwd_smem_t(int n) {
  switch (n) {
    case 5: return bwd_smem<T, 5>();
    case 6: return bwd_smem<T, 6>();
    case 7: return bwd_smem<T, 7>();
    case 8: return bwd_smem<T, 8>();
    case 9: return bwd_smem<T, 9>();
    default: return bwd_smem<T, 10>();
  }
}
int smem_of(int dtype, bool bwd, int n) {
  if (!bwd) return 0;
  return dtype == LWL_F32 ? bwd_smem_t<float>(n) : bwd_smem_t<__half>(n);
}
template <typename T, bool BWD>
const void* kernel_t(int n) {
  switch (n) {
    case 5: return kernel_n<T, BWD, 5>();
    case 6: return kernel_n<T, BWD, 6>();
    case 7: return kernel_n<T, BWD, 7>();
    case 8: return kernel_n<T, BWD, 8>();
    case 9: return kernel_n<T, BWD, 9>();
    default: return kernel_n<T, BWD, 10>();
  }
}
const void* kernel_of(int dtype, bool bwd, int n) {
  if (dtype == LWL_F32) return bwd ? kernel_t<float, true>(n) : kernel_t<float, false>(n);
  if (dtype == LWL_BF16) return bwd ? kernel_t<__nv_bfloat16, true>(n) : kernel_t<__nv_bfloat16, false>(n);
  return bwd ? kernel_t<__half, true>(n) : kernel_t<__half, false>(n);
}

int sm_count() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

// Persistent grid: every SM holds as many CTAs as fit, capped by the tiles.
int grid_of(const void* k, int smem, int64_t ntiles) {
  int per_sm = 1;
  if (smem > 0 && !set_max_smem(k, smem)) return -1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  const int64_t need = (ntiles + kWarps - 1) / kWarps;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, (int64_t)sm_count() * per_sm));
}

void make_params(const FhtArgs& a, SParams& p) {
  std::memset(&p, 0, sizeof(p));
  const int n = ilog2(next_pow2(a.latent_size));
  p.src = a.in;
  p.dst = a.out;
  p.L = a.latent_size;
  p.start = a.start;
  p.stop = a.stop;
  p.t_first = a.start >> kTileLog;
  p.ntiles = a.stop > a.start ? ((a.stop - 1) >> kTileLog) - p.t_first + 1 : 0;
  p.layers = a.layers;
  p.seed32 = fold_seed(a.seed);
  p.scale = (float)std::pow((double)(int64_t(1) << n), -0.5 * a.layers);
  const int64_t E = 16 / (int64_t)dtype_bytes(a.dtype);
  const void* data = a.backward ? a.in : a.out;
  p.vec_ok = (a.start % E == 0) && ((reinterpret_cast<uintptr_t>(data) & 15) == 0);
}

}  // namespace smallk

bool fhts_supported(int dtype, int64_t L, bool backward, int layers, unsigned flags) {
  // fp32 arithmetic throughout, so LWL_FLAG_EXACT is honoured as well.
  // LWL_SMALL_KERNEL=0 / =1 turns the kernel off / on for every size it
  // handles (measurement only).
  static const int mode = [] {
    const char* e = std::getenv("LWL_SMALL_KERNEL");
    return e ? std::atoi(e) : -1;
  }();
  if (mode == 0) return false;
  const int n = ilog2(next_pow2(L));
  if (n < smallk::kMinLog || n > smallk::kMaxLog) return false;
  if (mode == 1) return true;
  // fp32 (and the exact mode): faster than the fp32 whole-block kernel at every
  // size here.  16-bit: faster than the tensor-core tile kernel while the
  // lane-bit shuffles stay few (measured per size and layer count on B200).
  if (dtype == LWL_F32 || (flags & LWL_FLAG_EXACT)) return true;
  const int maxn = layers == 1 ? 10 : 8;
  return n <= maxn;
}

size_t fhts_workspace_bytes(const FhtArgs& a) {
  if (!a.backward || a.stop <= a.start) return 0;
  smallk::SParams p;
  smallk::make_params(a, p);
  const int n = ilog2(next_pow2(a.latent_size));
  const int grid = smallk::grid_of(smallk::kernel_of(a.dtype, true, n), smallk::smem_of(a.dtype, true, n), p.ntiles);
  return grid > 0 ? size_t(grid) * size_t(a.latent_size) * 4 : 0;
}

int fhts_launches(const FhtArgs& a) {
  if (a.stop <= a.start) return 0;
  return a.backward ? 2 : 1;
}

int fhts_run(const FhtArgs& a, cudaStream_t st) {
  using namespace smallk;
  if (a.stop <= a.start) {
    if (a.backward) LWL_CUDA_TRY(cudaMemsetAsync(a.out, 0, size_t(a.latent_size) * dtype_bytes(a.dtype), st));
    return LWL_OK;
  }
  SParams p;
  make_params(a, p);
  const int n = ilog2(next_pow2(a.latent_size));
  const void* k = kernel_of(a.dtype, a.backward, n);
  const int smem = smem_of(a.dtype, a.backward, n);
  const int grid = grid_of(k, smem, p.ntiles);
  if (grid < 0) {
    set_error("small-block transform: kernel setup failed: %s", cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  if (a.backward) {
    const size_t need = size_t(grid) * size_t(a.latent_size) * 4;
    if (!a.workspace || a.workspace_bytes < need) {
      set_error("workspace of %zu bytes required, %zu given", need, a.workspace ? a.workspace_bytes : (size_t)0);
      return LWL_ERR_WORKSPACE;
    }
    p.dst = a.workspace;
  }
  void* args[] = {&p};
  if (cudaLaunchKernel(k, dim3(grid), dim3(kThreads), args, (size_t)smem, st) != cudaSuccess) {
    set_error("small-block transform launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  if (a.backward) {
    const int threads = 256;
    const int blocks = (int)std::min<int64_t>((a.latent_size + threads - 1) / threads, 1024);
    const float* rows = reinterpret_cast<const float*>(a.workspace);
    if (a.dtype == LWL_BF16)
      fhts_reduce_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size,
                                                                     reinterpret_cast<__nv_bfloat16*>(a.out));
    else if (a.dtype == LWL_F16)
      fhts_reduce_kernel<__half><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size, reinterpret_cast<__half*>(a.out));
    else
      fhts_reduce_kernel<float><<<blocks, threads, 0, st>>>(rows, grid, a.latent_size, reinterpret_cast<float*>(a.out));
    LWL_CUDA_TRY(cudaGetLastError());
  }
  return LWL_OK;
}

}  // namespace lwl
