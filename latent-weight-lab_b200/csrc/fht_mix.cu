// fht_mix.cu -- FixedFHTMix: y[r, :F] = (S * H_P/sqrt(P) * S * pad(x[r, :]))[:F]
// for every row r, P = next_pow2(F) <= 8192, S = diag(signs) (+-1 floats).
// Reference: examples/nanogpt/model.py:182-218 (normalized_fht_last_dim + FixedFHTMix.forward).
// The map is symmetric, so the same kernel computes the gradient.
//
// This kernel serves full rows of P = 256 .. 1024 and rows that are not
// 16-byte aligned up to P = 1024; the rest run on the tile kernels of
// fht32_mix.cu.  HBM-bound: one read and one write per element.  E = P / 32 values per lane
// (E <= 32, fp32 registers) in chunks of up to 16 bytes: lane l owns chunks
// l, l + 32, ... of the row's 1024-element slice of its warp, so every warp
// access is contiguous (P / 1024 warps per row when P > 1024).  Butterflies
// over the register bits run in registers, over the lane bits with shfl_xor,
// over the warp bits through a shared-memory exchange.  Signs are applied as
// sign-bit flips from a per-CTA bit table.  For P < 32 one warp holds 32 / P rows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdlib>

#include "lwl_common.cuh"

namespace lwl {
namespace mix {

constexpr int kThreads = 256;
constexpr int kMaxLog = 13;

__device__ __forceinline__ int swz(int p) { return p ^ ((p >> 5) & 31); }

template <typename T>
__device__ __forceinline__ float ld(const T* p) {
  return Cvt<T>::to_f(*p);
}
// element u of a 16-byte word group, and the inverse, without taking addresses
template <typename T> __device__ __forceinline__ float unpack(const uint32_t* wv, int u);
template <> __device__ __forceinline__ float unpack<float>(const uint32_t* wv, int u) { return __uint_as_float(wv[u]); }
template <> __device__ __forceinline__ float unpack<__nv_bfloat16>(const uint32_t* wv, int u) {
  return __uint_as_float((u & 1) ? (wv[u >> 1] & 0xffff0000u) : (wv[u >> 1] << 16));
}
template <> __device__ __forceinline__ float unpack<__half>(const uint32_t* wv, int u) {
  return __half2float(__ushort_as_half((unsigned short)((u & 1) ? (wv[u >> 1] >> 16) : (wv[u >> 1] & 0xffffu))));
}
template <typename T> __device__ __forceinline__ void pack(uint32_t* wv, const float* f);
template <> __device__ __forceinline__ void pack<float>(uint32_t* wv, const float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) wv[i] = __float_as_uint(f[i]);
}
template <> __device__ __forceinline__ void pack<__nv_bfloat16>(uint32_t* wv, const float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    wv[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}
template <> __device__ __forceinline__ void pack<__half>(uint32_t* wv, const float* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __half2 h = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    wv[i] = *reinterpret_cast<uint32_t*>(&h);
  }
}

template <typename T, int E>
__global__ void __launch_bounds__(kThreads) fht_mix_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                           const float* __restrict__ signs, int64_t rows, int F,
                                                           int logP, bool vec_ok) {
  __shared__ float buf[1 << kMaxLog];
  __shared__ uint32_t sbits[(1 << kMaxLog) / 32];  // bit p set: signs[p] < 0
  const int P = 1 << logP;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  for (int wd = w; wd < (P + 31) / 32; wd += kThreads / 32) {
    const int i = 32 * wd + lane;
    const uint32_t b = __ballot_sync(0xffffffffu, i < P && signs[i] < 0.0f);
    if (lane == 0) sbits[wd] = b;
  }
  __syncthreads();
  const int nw = P > 1024 ? P >> 10 : 1;       // warps per row
  const int rpw = P < 32 ? 32 / P : 1;         // rows per warp
  const int lanes = P < 32 ? P : 32;           // lanes per row
  const int rows_per_cta = (kThreads / 32) / nw * rpw;
  const int wr = w % nw, rg = w / nw;          // warp within its row, row group of the warp
  const int sub = lane / lanes, ln = lane % lanes;
  const float scale = rsqrtf((float)P);
  // Element e = c * CH + u of a lane sits at row position
  //   p(e) = wr * 1024 + CH * (ln + lanes * c) + u,
  // i.e. a lane owns chunks ln, ln + 32, ... of CH consecutive elements, so a
  // warp's 16-byte accesses are contiguous.  Register bits (u, c) and lane
  // bits each map to distinct position bits, so the butterflies below are the
  // natural-order transform whatever the assignment.
  constexpr int VEC = 16 / (int)sizeof(T);  // elements per 16-byte access
  constexpr int CH = E >= VEC ? VEC : E, NC = E / CH;
  auto pos = [&](int e) { return wr * 1024 + CH * (ln + lanes * (e / CH)) + e % CH; };
  uint32_t sbc[NC];  // sign bits of each chunk (CH <= 8 consecutive bits of one word)
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const int b0 = pos(c * CH);
    sbc[c] = sbits[b0 >> 5] >> (b0 & 31);
  }
  auto sgn = [&](float val, int e) {
    return __uint_as_float(__float_as_uint(val) ^ (((sbc[e / CH] >> (e % CH)) & 1u) << 31));
  };
  // the next row's full 16-byte chunks are loaded before the current row is
  // transformed, so each warp keeps one row of loads in flight
  const int64_t stride = (int64_t)gridDim.x * rows_per_cta;
  auto full = [&](int c, bool act) { return CH == VEC && vec_ok && act && pos(c * CH) + VEC <= F; };
  uint4 raw[NC];
  {
    const int64_t row0 = (int64_t)blockIdx.x * rows_per_cta + (int64_t)rg * rpw + sub;
#pragma unroll
    for (int c = 0; c < NC; ++c)
      if (full(c, row0 < rows)) raw[c] = __ldg(reinterpret_cast<const uint4*>(x + row0 * F + pos(c * CH)));
  }
  for (int64_t rb = (int64_t)blockIdx.x * rows_per_cta; rb < rows; rb += stride) {
    const int64_t row = rb + (int64_t)rg * rpw + sub;
    const bool active = row < rows;
    const T* xr = x + row * F;
    float v[E];
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int b0 = pos(c * CH);
      if (full(c, active)) {
        const uint32_t wv[4] = {raw[c].x, raw[c].y, raw[c].z, raw[c].w};
#pragma unroll
        for (int u = 0; u < CH; ++u) v[c * CH + u] = sgn(unpack<T>(wv, u), c * CH + u);
      } else {
#pragma unroll
        for (int u = 0; u < CH; ++u) v[c * CH + u] = (active && b0 + u < F) ? sgn(ld(xr + b0 + u), c * CH + u) : 0.0f;
      }
    }
    {
      const int64_t nrow = row + stride;
      const bool nact = nrow < rows;
#pragma unroll
      for (int c = 0; c < NC; ++c)
        if (full(c, nact)) raw[c] = __ldg(reinterpret_cast<const uint4*>(x + nrow * F + pos(c * CH)));
    }
    // bits of e
#pragma unroll
    for (int h = 1; h < E; h <<= 1) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((e & h) == 0) {
          const float a = v[e], b = v[e + h];
          v[e] = a + b;
          v[e + h] = a - b;
        }
      }
    }
    // bits of the lane
    for (int m = 1; m < lanes; m <<= 1) {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float o = __shfl_xor_sync(0xffffffffu, v[e], m);
        v[e] = (ln & m) ? o - v[e] : v[e] + o;
      }
    }
    if (nw > 1) {  // bits of the warp within the row, through shared memory; only the
                   // nw warps of the row group synchronise (named barrier 1 + rg)
      // row group rg owns buf[rg * P, (rg + 1) * P); element p at p ^ ((p >> 5) & 31),
      // conflict-free for the lane-strided writes and the consecutive gathers
      float* rbuf = buf + rg * P;
#pragma unroll
      for (int e = 0; e < E; ++e) rbuf[swz(pos(e))] = v[e];
      asm volatile("bar.sync %0, %1;\n" ::"r"(1 + rg), "r"(nw * 32) : "memory");
      for (int q = wr * 32 + lane; q < 1024; q += nw * 32) {
        float u[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) u[j] = j < nw ? rbuf[swz(q + 1024 * j)] : 0.0f;
#pragma unroll
        for (int h = 1; h < 8; h <<= 1)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            if ((j & h) == 0 && h < nw) {
              const float a = u[j], b = u[j + h];
              u[j] = a + b;
              u[j + h] = a - b;
            }
#pragma unroll
        for (int j = 0; j < 8; ++j)
          if (j < nw) rbuf[swz(q + 1024 * j)] = u[j];
      }
      asm volatile("bar.sync %0, %1;\n" ::"r"(1 + rg), "r"(nw * 32) : "memory");
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = rbuf[swz(pos(e))];
      asm volatile("bar.sync %0, %1;\n" ::"r"(1 + rg), "r"(nw * 32) : "memory");  // the next rows' exchange reuses the buffer
    }
    T* yr = y + row * F;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      const int b0 = pos(c * CH);
      if (CH == VEC && vec_ok && active && b0 + VEC <= F) {
        float f8[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) f8[u] = sgn(v[c * CH + u] * scale, c * CH + u);
        uint32_t wv[4];
        pack<T>(wv, f8);
        *reinterpret_cast<uint4*>(yr + b0) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      } else {
#pragma unroll
        for (int u = 0; u < CH; ++u)
          if (active && b0 + u < F) yr[b0 + u] = Cvt<T>::from_f(sgn(v[c * CH + u] * scale, c * CH + u));
      }
    }
  }
}

template <typename T, int E>
int launch_e(const void* x, void* y, const float* signs, int64_t rows, int F, int logP, cudaStream_t st) {
  const int P = 1 << logP;
  const int nw = P > 1024 ? P >> 10 : 1, rpw = P < 32 ? 32 / P : 1;
  const int rows_per_cta = (kThreads / 32) / nw * rpw;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t need = (rows + rows_per_cta - 1) / rows_per_cta;
  const int grid = (int)(need < (int64_t)sms * 8 ? need : (int64_t)sms * 8);
  const bool vec_ok = (F * (int)sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(y) & 15) == 0;
  fht_mix_kernel<T, E><<<grid, kThreads, 0, st>>>(reinterpret_cast<const T*>(x), reinterpret_cast<T*>(y), signs,
                                                   rows, F, logP, vec_ok);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <typename T>
int launch_t(const void* x, void* y, const float* signs, int64_t rows, int F, int logP, cudaStream_t st) {
  const int E = logP <= 5 ? 1 : (logP >= 10 ? 32 : 1 << (logP - 5));
  switch (E) {
    case 1: return launch_e<T, 1>(x, y, signs, rows, F, logP, st);
    case 2: return launch_e<T, 2>(x, y, signs, rows, F, logP, st);
    case 4: return launch_e<T, 4>(x, y, signs, rows, F, logP, st);
    case 8: return launch_e<T, 8>(x, y, signs, rows, F, logP, st);
    case 16: return launch_e<T, 16>(x, y, signs, rows, F, logP, st);
    default: return launch_e<T, 32>(x, y, signs, rows, F, logP, st);
  }
}

}  // namespace mix

bool fht_mix32_supported(int logP);
int fht_mix32_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                     cudaStream_t st);

bool fht_mix32p_supported(int dtype, const void* x, const void* y, int F, int logP);
int fht_mix32p_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                      cudaStream_t st);

// Kernel choice (LWL_MIX_KERNEL overrides for measurement: 1 = warp-per-row,
// 2 = tile, 3 = prefetching tile; each only where it applies).
static int mix_choice() {
  static const int v = [] {
    const char* s = std::getenv("LWL_MIX_KERNEL");
    return s ? std::atoi(s) : 0;
  }();
  return v;
}

int fht_mix_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                   cudaStream_t st) {
  const int c = mix_choice();
  // aligned rows: the prefetching register-resident tile kernel (fht32_mix.cu),
  // except for full rows of P = 256 .. 1024, where the warp-per-row kernel
  // below measured 3-8% faster
  const bool warp_rows = F == (1 << logP) && logP >= 8 && logP <= 10;
  if ((c == 3 || (c == 0 && !warp_rows)) && fht_mix32p_supported(dtype, x, y, F, logP))
    return fht_mix32p_launch(dtype, x, y, signs, rows, F, logP, st);
  // other P = 2048 .. 8192: the tile kernel without prefetch
  if (c != 1 && fht_mix32_supported(logP)) return fht_mix32_launch(dtype, x, y, signs, rows, F, logP, st);
  if (dtype == 0) return mix::launch_t<float>(x, y, signs, rows, F, logP, st);
  if (dtype == 1) return mix::launch_t<__nv_bfloat16>(x, y, signs, rows, F, logP, st);
  return mix::launch_t<__half>(x, y, signs, rows, F, logP, st);
}

}  // namespace lwl
