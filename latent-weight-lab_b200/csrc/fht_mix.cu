// fht_mix.cu -- FixedFHTMix: y[r, :F] = (S * H_P/sqrt(P) * S * pad(x[r, :]))[:F]
// for every row r, P = next_pow2(F) <= 8192, S = diag(signs) (+-1 floats).
// Reference: examples/nanogpt/model.py:182-218 (normalized_fht_last_dim + FixedFHTMix.forward).
// The map is symmetric, so the same kernel computes the gradient.
//
// HBM-bound: one read and one write per element.  Layout of a row in the
// threads that own it: position p = wr * 1024 + lane * E + e, with E = P / 32
// values per lane (E <= 32, fp32 registers), lane = 0..31, wr = warp of the
// row (P / 1024 warps when P > 1024).  Butterflies over the e bits run in
// registers, over the lane bits with shfl_xor, over the warp bits through a
// shared-memory exchange.  For P < 32 one warp holds 32 / P rows.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

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
  const int P = 1 << logP;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int nw = P > 1024 ? P >> 10 : 1;       // warps per row
  const int rpw = P < 32 ? 32 / P : 1;         // rows per warp
  const int lanes = P < 32 ? P : 32;           // lanes per row
  const int rows_per_cta = (kThreads / 32) / nw * rpw;
  const int wr = w % nw, rg = w / nw;          // warp within its row, row group of the warp
  const int sub = lane / lanes, ln = lane % lanes;
  const float scale = rsqrtf((float)P);
  for (int64_t rb = (int64_t)blockIdx.x * rows_per_cta; rb < rows; rb += (int64_t)gridDim.x * rows_per_cta) {
    const int64_t row = rb + (int64_t)rg * rpw + sub;
    const bool active = row < rows;
    float v[E];
    const int p0 = wr * 1024 + ln * E;
    constexpr int VEC = 16 / (int)sizeof(T);  // elements per 16-byte access
    const bool vec = (E % VEC == 0) && vec_ok && active && p0 + E <= F;
    if (vec) {
#pragma unroll
      for (int c = 0; c < E / VEC; ++c) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(x + row * F + p0) + c);
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int u = 0; u < VEC; ++u) v[c * VEC + u] = unpack<T>(wv, u) * signs[p0 + c * VEC + u];
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int p = p0 + e;
        v[e] = (active && p < F) ? ld(x + row * F + p) * signs[p] : 0.0f;
      }
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
    if (nw > 1) {  // bits of the warp within the row, through shared memory
      // row group rg owns buf[rg * P, (rg + 1) * P); element p at p ^ ((p >> 5) & 31),
      // conflict-free for the lane-strided writes and the consecutive gathers
      float* rbuf = buf + rg * P;
#pragma unroll
      for (int e = 0; e < E; ++e) rbuf[swz(p0 + e)] = v[e];
      __syncthreads();
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
      __syncthreads();
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = rbuf[swz(p0 + e)];
      __syncthreads();  // the next rows' exchange reuses the buffer
    }
    if (vec) {
#pragma unroll
      for (int c = 0; c < E / VEC; ++c) {
        float f8[VEC];
#pragma unroll
        for (int u = 0; u < VEC; ++u) f8[u] = v[c * VEC + u] * scale * signs[p0 + c * VEC + u];
        uint32_t wv[4];
        pack<T>(wv, f8);
        reinterpret_cast<uint4*>(y + row * F + p0)[c] = make_uint4(wv[0], wv[1], wv[2], wv[3]);
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int p = p0 + e;
        if (active && p < F) y[row * F + p] = Cvt<T>::from_f(v[e] * scale * signs[p]);
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

int fht_mix_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                   cudaStream_t st) {
  if (dtype == 0) return mix::launch_t<float>(x, y, signs, rows, F, logP, st);
  if (dtype == 1) return mix::launch_t<__nv_bfloat16>(x, y, signs, rows, F, logP, st);
  return mix::launch_t<__half>(x, y, signs, rows, F, logP, st);
}

}  // namespace lwl
