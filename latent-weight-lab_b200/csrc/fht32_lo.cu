// fht32_lo.cu -- the low-bit pass of the two-pass layout in fp32 arithmetic
// (fp32 generators and the exact mode, padded blocks 2^16 .. 2^23), on the
// register-resident scheme of fht32.cuh.
//
// H_B = H_hi (x) H_32768: this pass applies H_32768 to the 15 low position
// bits of every 2^15 chunk of a block, once or twice, with the plan's signs,
// and the high bits run in fht32_hi.cu.  A CTA of 512 threads owns one chunk
// (TB = 15, 64 values per thread).  One application is sets A, B and C (two
// exchanges); two applications share set C between them:
//     one:  A: [pre-sign] T(t0..5) -> B: T(t6..11) -> C: T(t12..14) [sign]
//     two:  A: [pre-sign] T(A) -> B: T(B) -> C: T(t12..14) [sign] T(t9..14)
//           -> A: T(A) -> B: T(t6..8) [sign]
// A sign that ends a layer carries the layer's 1/sqrt(B), exactly as the
// tile engine applies it; an application without one leaves the result
// unnormalised (the high pass of the same layer normalises it).
#include <algorithm>
#include <cmath>

#include "fht32.cuh"

namespace lwl {
namespace f32k {

// Source values of chunk j of block b in set SET (zero outside the latent / slice).
template <typename T, int SET, int SRC>
__device__ __forceinline__ void lo32_load(float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0,
                                          int base) {
  constexpr int TB = 15;
  if (SRC == SRC_WS) {
    const float* s = reinterpret_cast<const float*>(p.src) + (b - p.first_block) * p.B + pos0 + base;
    if (SET == SA) {
#pragma unroll
      for (int q = 0; q < kRegs / 4; ++q) {
        const float4 a = *reinterpret_cast<const float4*>(s + 4 * q);
        v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
      }
    } else {
#pragma unroll
      for (int r = 0; r < kRegs; ++r) v[r] = s[spread<TB, SET>(r)];
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
  if (lo <= 0 && hi >= (int64_t(1) << TB)) {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = Cvt<T>::to_f(s[spread<TB, SET>(r)]);
  } else {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int o = spread<TB, SET>(r);
      v[r] = (o >= lo && o < hi) ? Cvt<T>::to_f(s[o]) : 0.0f;
    }
  }
}

template <typename T, int SET, int DST>
__device__ __forceinline__ void lo32_store(const float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0,
                                           int base) {
  constexpr int TB = 15;
  if (DST == DST_WS) {
    float* d = reinterpret_cast<float*>(p.dst) + (b - p.first_block) * p.B + pos0 + base;
#pragma unroll
    for (int r = 0; r < kRegs; ++r) d[spread<TB, SET>(r)] = v[r];
    return;
  }
  const int64_t g = b * p.B + pos0 + base;
  T* d = reinterpret_cast<T*>(p.dst) + (g - p.start);
  const int64_t lo = p.start - g, hi = p.stop - g;
  if (lo <= 0 && hi >= (int64_t(1) << TB)) {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) d[spread<TB, SET>(r)] = Cvt<T>::from_f(v[r]);
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
  const int cpb = (int)(p.B >> TB);  // chunks per block
  const int64_t ntiles = p.nblocks * cpb;
  const int s1 = p.lo_seg_slot[0], s2 = NSEG == 2 ? p.lo_seg_slot[1] : -1;
  float v[kRegs];
  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t b = p.first_block + tile / cpb;
    const int j = (int)(tile % cpb);
    const int64_t pos0 = (int64_t)j << TB;
    __syncthreads();  // the previous tile is done with the sign table and the exchange buffer
    for (int i = tid; i < p.nslots * Tl::kWords; i += Tl::kThreads) {
      const int s = i / Tl::kWords, c = i - s * Tl::kWords;
      sw[i] = sign_word(block_layer_key(p.seed32, b, p.slot_layer[s]), ((int64_t)j << 10) + c);
    }
    __syncthreads();
    lo32_load<T, SA, SRC>(v, p, b, pos0, bA);
    if (p.pre_slot >= 0) apply_sign<TB, SA>(v, sw + p.pre_slot * Tl::kWords, bA);
    xform<TB, SA>(v, Tl::kA, TB);
    exchange<TB, SA, SB>(v, buf, lane, warp);
    xform<TB, SB>(v, Tl::kB, TB);
    exchange<TB, SB, SC>(v, buf, lane, warp);
    xform<TB, SC>(v, Tl::kChi, TB);
    if (s1 >= 0) sign_scaled<TB, SC>(v, sw + s1 * Tl::kWords, bC, p.scale);
    if (NSEG == 1) {
      lo32_store<T, SC, DST>(v, p, b, pos0, bC);
    } else {
      xform<TB, SC>(v, Tl::kC, TB);
      exchange<TB, SC, SA>(v, buf, lane, warp);
      xform<TB, SA>(v, Tl::kA, TB);
      exchange<TB, SA, SB>(v, buf, lane, warp);
      xform<TB, SB>(v, Tl::kBsub, TB);
      if (s2 >= 0) sign_scaled<TB, SB>(v, sw + s2 * Tl::kWords, bB, p.scale);
      lo32_store<T, SB, DST>(v, p, b, pos0, bB);
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

int fht32_lo_launch(int dtype, const TileParams& p, cudaStream_t st) {
  using namespace f32k;
  const void* k = dtype == LWL_BF16 ? lo32_kernel<__nv_bfloat16>(p.src_kind, p.dst_kind, p.lo_nseg)
                : dtype == LWL_F16  ? lo32_kernel<__half>(p.src_kind, p.dst_kind, p.lo_nseg)
                                    : lo32_kernel<float>(p.src_kind, p.dst_kind, p.lo_nseg);
  const size_t smem = Tile<15>::kSmem;
  if (!set_max_smem(k, (int)smem)) return -1;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int64_t ntiles = p.nblocks * (p.B >> 15);
  const int grid = (int)std::min<int64_t>(ntiles, nsm);
  void* args[] = {const_cast<TileParams*>(&p)};
  return cudaLaunchKernel(k, dim3(grid), dim3(Tile<15>::kThreads), args, smem, st) == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
