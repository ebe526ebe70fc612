// fht32_lo.cu -- the low-bit pass of the two-pass layout in fp32 arithmetic
// (fp32 generators and the exact mode, padded blocks 2^16 .. 2^23), on the
// register-resident scheme of fht32.cuh.
//
// H_B = H_hi (x) H_32768: this pass applies H_32768 to the 15 low position
// bits of every 2^15 chunk of a block, once or twice, with the plan's signs,
// and the high bits run in fht32_hi.cu.  A CTA of 512 threads owns one chunk
// (TB = 15, 64 values per thread).  One application is sets A, B and SD (three
// exchanges); two applications share set C between them:
//     one:  SD: [pre-sign] -> A: T(t0..5) -> B: T(t6..11) -> SD: T(t12..14) [sign]
//     two:  SD: [pre-sign] -> A: T(A) -> B: T(B) -> C: T(t12..14) [sign] T(t9..14)
//           -> A: T(A) -> SD2: T(t6..8) [sign]
// The first and last residencies (SD / SD2) hold four consecutive elements per
// register group, so the tile arrives and leaves with 16-byte accesses that
// are contiguous across the warp (set A's 16-byte loads, one per lane at a
// 256-byte stride, held the kernel on the L1 request queue).
// A sign that ends a layer carries the layer's 1/sqrt(B), exactly as the
// tile engine applies it; an application without one leaves the result
// unnormalised (the high pass of the same layer normalises it).
#include <algorithm>
#include <cmath>

#include "fht32.cuh"

namespace lwl {
namespace f32k {

// Source values of chunk j of block b in set SD (four consecutive elements per
// register group, lanes on t2..t6: each warp load covers 512 consecutive bytes
// of fp32), zero outside the latent / slice.
template <typename T, int SRC>
__device__ __forceinline__ void lo32_load(float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0,
                                          int base) {
  constexpr int TB = 15, SET = SD;
  if (SRC == SRC_WS) {
    const float* s = reinterpret_cast<const float*>(p.src) + (b - p.first_block) * p.B + pos0 + base;
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const float4 a = *reinterpret_cast<const float4*>(s + spread<TB, SET>(4 * q));
      v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
    }
    return;
  }
  const T* src = reinterpret_cast<const T*>(p.src);
  int64_t off, lo, hi;  // element base + r is src[off + offset(r)], valid for offsets in [lo, hi)
  if (SRC == SRC_LATENT) {
    off = pos0 + base;
    lo = -off;
    hi = p.L - off;
  } else {
    const int64_t g = b * p.B + pos0 + base;
    off = g - p.start;
    lo = p.start - g;
    hi = p.stop - g;
  }
  const T* s = src + off;
  const bool vec = (reinterpret_cast<uintptr_t>(s) & (4 * sizeof(T) - 1)) == 0;
  if (lo <= 0 && hi >= (int64_t(1) << TB) && vec) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const T* e = s + spread<TB, SET>(4 * q);
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
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int o = spread<TB, SET>(r);
      v[r] = (o >= lo && o < hi) ? Cvt<T>::to_f(s[o]) : 0.0f;
    }
  }
}

// Results of set SD / SD2 (four consecutive elements per register group): one
// 16-byte (fp32) or 8-byte (16-bit) store per group where aligned.
template <typename T, int SET, int DST>
__device__ __forceinline__ void lo32_store(const float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0,
                                           int base, bool first) {
  constexpr int TB = 15;
  static_assert(SET == SD || SET == SD2, "stores leave from the quad sets");
  if (DST == DST_WS && p.acc_rows) {
    // the backward's last launch: the grid is a multiple of the tiles per
    // block, so every tile of this CTA has the same index j and the CTA sums
    // them into its segment of partial row blockIdx.x / tpb (L2-resident):
    // the first tile stores, later ones add.  One thread owns each address,
    // so the sums keep program order (deterministic).
    // (with more tiles per block than CTAs, 2^23: grid = tpb / 2, row 0, the
    // CTA meets j = blockIdx.x and blockIdx.x + gridDim.x)
    const int tpb = (int)(p.B >> TB);
    float* row = p.partial + (tpb > (int)gridDim.x ? 0 : (int64_t)(blockIdx.x / tpb)) * p.L;
    const bool vec = (p.L & 3) == 0;
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      const int64_t pos = pos0 + base + spread<TB, SET>(4 * q);  // position inside the block
      float* d = row + pos;
      if (vec && pos + 4 <= p.L) {
        if (first) {
          *reinterpret_cast<float4*>(d) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        } else {
          asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(d), "f"(v[4 * q]),
                       "f"(v[4 * q + 1]), "f"(v[4 * q + 2]), "f"(v[4 * q + 3])
                       : "memory");
        }
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (pos + e < p.L) {
            if (first) d[e] = v[4 * q + e];
            else atomicAdd(d + e, v[4 * q + e]);
          }
        }
      }
    }
    return;
  }
  if (DST == DST_WS) {
    float* d = reinterpret_cast<float*>(p.dst) + (b - p.first_block) * p.B + pos0 + base;
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q)
      *reinterpret_cast<float4*>(d + spread<TB, SET>(4 * q)) =
          make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    return;
  }
  const int64_t g = b * p.B + pos0 + base;
  T* d = reinterpret_cast<T*>(p.dst) + (g - p.start);
  const int64_t lo = p.start - g, hi = p.stop - g;
  const int64_t t0 = b * p.B + pos0;  // the tile's range [t0, t0 + 2^TB) inside the slice?
  const bool full = t0 >= p.start && t0 + (int64_t(1) << TB) <= p.stop;
  const bool vec = ((p.start & 3) == 0) && (reinterpret_cast<uintptr_t>(p.dst) & (4 * sizeof(T) - 1)) == 0;
  if (full && vec) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      T* e = d + spread<TB, SET>(4 * q);
      if (sizeof(T) == 4) {
        *reinterpret_cast<float4*>(e) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      } else {
        T h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = Cvt<T>::from_f(v[4 * q + i]);
        *reinterpret_cast<uint2*>(e) = *reinterpret_cast<const uint2*>(h);
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int o = spread<TB, SET>(r);
      if (o >= lo && o < hi) d[o] = Cvt<T>::from_f(v[r]);
    }
  }
}

template <int TB, int SET>
__device__ __forceinline__ void sign_scaled(float (&v)[kRegs], const uint32_t* sw, int base, float scale) {
  apply_sign<TB, SET>(v, sw, base);
#pragma unroll
  for (int r = 0; r < kRegs; ++r) v[r] *= scale;
}

template <typename T, int SRC, int DST, int NSEG>
__global__ void __launch_bounds__(Tile<15>::kThreads, 1) fht32_lo_kernel(const __grid_constant__ TileParams p) {
  constexpr int TB = 15;
  using Tl = Tile<TB>;
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  uint32_t* sw = reinterpret_cast<uint32_t*>(buf + Tl::kBufWords);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bA = base_of<TB, SA>(lane, warp), bB = base_of<TB, SB>(lane, warp), bC = base_of<TB, SC>(lane, warp);
  const int bD = base_of<TB, SD>(lane, warp), bD2 = base_of<TB, SD2>(lane, warp);
  const int cpb = (int)(p.B >> TB);  // chunks per block
  const int64_t ntiles = p.nblocks * cpb;
  const int s1 = p.lo_seg_slot[0], s2 = NSEG == 2 ? p.lo_seg_slot[1] : -1;
  // acc_rows: the CTA's first tile of each tile index stores, later ones add
  const int64_t first_end = (int64_t)gridDim.x * (cpb > (int)gridDim.x ? 2 : 1);
  float v[kRegs];
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t b = p.first_block + tile / cpb;
    const int j = (int)(tile % cpb);
    const int64_t pos0 = (int64_t)j << TB;
    if (tid == 0 && tile + gridDim.x < ntiles) {  // the next tile's source into L2
      const int64_t nt = tile + gridDim.x, nb = p.first_block + nt / cpb, np = (nt % cpb) << TB;
      if (SRC == SRC_WS) {
        const int64_t e0 = (nb - p.first_block) * p.B + np;
        prefetch_l2(p.src, e0 * 4, (e0 + (1 << TB)) * 4);
      } else if (SRC == SRC_SLICE) {
        const int64_t g0 = nb * p.B + np - p.start, n = p.stop - p.start;
        const int64_t lo = g0 > 0 ? g0 : 0, hi = g0 + (1 << TB) < n ? g0 + (1 << TB) : n;
        if (hi > lo) prefetch_l2(p.src, lo * (int64_t)sizeof(T), hi * (int64_t)sizeof(T));
      }
    }
    __syncthreads();  // the previous tile is done with the sign table and the exchange buffer
    for (int i = tid; i < p.nslots * Tl::kWords; i += Tl::kThreads) {
      const int s = i / Tl::kWords, c = i - s * Tl::kWords;
      sw[i] = sign_word(block_layer_key(p.seed32, b, p.slot_layer[s]), ((int64_t)j << 10) + c);
    }
    __syncthreads();
    lo32_load<T, SRC>(v, p, b, pos0, bD);
    if (p.pre_slot >= 0) apply_sign<TB, SD>(v, sw + p.pre_slot * Tl::kWords, bD);
    exchange<TB, SD, SA>(v, buf, lane, warp);
    xform<TB, SA>(v, Tl::kA, TB);
    exchange<TB, SA, SB>(v, buf, lane, warp);
    xform<TB, SB>(v, Tl::kB, TB);
    if (NSEG == 1) {
      exchange<TB, SB, SD>(v, buf, lane, warp);
      xform<TB, SD>(v, Tl::kChi, TB);
      if (s1 >= 0) sign_scaled<TB, SD>(v, sw + s1 * Tl::kWords, bD, p.scale);
      lo32_store<T, SD, DST>(v, p, b, pos0, bD, tile < first_end);
    } else {
      exchange<TB, SB, SC>(v, buf, lane, warp);
      xform<TB, SC>(v, Tl::kChi, TB);
      if (s1 >= 0) sign_scaled<TB, SC>(v, sw + s1 * Tl::kWords, bC, p.scale);
      xform<TB, SC>(v, Tl::kC, TB);
      exchange<TB, SC, SA>(v, buf, lane, warp);
      xform<TB, SA>(v, Tl::kA, TB);
      exchange<TB, SA, SD2>(v, buf, lane, warp);
      xform<TB, SD2>(v, Tl::kBsub, TB);
      if (s2 >= 0) sign_scaled<TB, SD2>(v, sw + s2 * Tl::kWords, bD2, p.scale);
      lo32_store<T, SD2, DST>(v, p, b, pos0, bD2, tile < first_end);
    }
  }
}

template <typename T, int SRC, int DST>
const void* lo32_kernel_seg(int nseg) {
  return nseg == 1 ? (const void*)fht32_lo_kernel<T, SRC, DST, 1> : (const void*)fht32_lo_kernel<T, SRC, DST, 2>;
}

template <typename T>
const void* lo32_kernel(int src, int dst, int nseg) {
  if (dst == DST_WS) {
    if (src == SRC_WS) return lo32_kernel_seg<T, SRC_WS, DST_WS>(nseg);
    if (src == SRC_LATENT) return lo32_kernel_seg<T, SRC_LATENT, DST_WS>(nseg);
    return lo32_kernel_seg<T, SRC_SLICE, DST_WS>(nseg);
  }
  if (src == SRC_WS) return lo32_kernel_seg<T, SRC_WS, DST_SLICE>(nseg);
  return lo32_kernel_seg<T, SRC_LATENT, DST_SLICE>(nseg);
}

}  // namespace f32k

bool fht32_lo_supported(int dtype, int n, unsigned flags) {
  return n > 15 && n <= 23 && (dtype == LWL_F32 || (flags & LWL_FLAG_EXACT));
}

int fht32_lo_grid(const TileParams& p) {
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tpb = p.B >> 15, ntiles = p.nblocks * tpb;
  if (p.acc_rows && tpb > nsm) return (int)(tpb / 2);  // 2^23: each CTA meets two tile indices
  if (ntiles <= nsm) return (int)ntiles;
  return (int)(p.acc_rows ? (nsm / tpb) * tpb : nsm);  // acc_rows: a multiple of the tiles per block
}

int fht32_lo_launch(int dtype, const TileParams& p, cudaStream_t st) {
  using namespace f32k;
  const void* k = dtype == LWL_BF16 ? lo32_kernel<__nv_bfloat16>(p.src_kind, p.dst_kind, p.lo_nseg)
                : dtype == LWL_F16  ? lo32_kernel<__half>(p.src_kind, p.dst_kind, p.lo_nseg)
                                    : lo32_kernel<float>(p.src_kind, p.dst_kind, p.lo_nseg);
  const size_t smem = Tile<15>::kSmem;
  if (!set_max_smem(k, (int)smem)) return -1;
  const int grid = fht32_lo_grid(p);
  void* args[] = {const_cast<TileParams*>(&p)};
  return cudaLaunchKernel(k, dim3(grid), dim3(Tile<15>::kThreads), args, smem, st) == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
