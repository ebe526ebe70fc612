// lwl_common.cuh -- shared device/host helpers for the BlockFHT sm_100a library.
//
// The sign hash is the reference's stateless generator restated
// (latent_weight_lab/block_fht.py:36-52, csrc/block_fht_ext_cuda.cu:27-48):
// one uint32 word per (seed, block, layer, word) covering 32 consecutive
// positions; bit (pos & 31) set means +1, clear means -1.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <utility>

#include "lwl_b200.h"

namespace lwl {

__host__ __device__ __forceinline__ uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

// Seed folding happens once on the host: seed32 = lo32(seed) ^ hi32(seed).
__host__ __device__ __forceinline__ uint32_t fold_seed(uint64_t seed) {
  return (uint32_t)seed ^ (uint32_t)(seed >> 32);
}

// Block/layer part of the mix, constant across a block's words.
__host__ __device__ __forceinline__ uint32_t block_layer_key(uint32_t seed32, int64_t block, int layer) {
  return seed32 ^ (0x9E3779B9u * (uint32_t)(block + 1)) ^ (0x85EBCA6Bu * (uint32_t)(layer + 1));
}

__host__ __device__ __forceinline__ uint32_t sign_word(uint32_t key, int64_t word) {
  return lowbias32(key ^ (0xC2B2AE35u * (uint32_t)(word + 1)));
}

// dtype <-> fp32
template <typename T> struct Cvt;
template <> struct Cvt<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

inline int ilog2(int64_t v) {
  int r = 0;
  while ((int64_t(1) << r) < v) ++r;
  return r;
}

inline int64_t next_pow2(int64_t v) {
  int64_t o = 1;
  while (o < v) o <<= 1;
  return o;
}

// Asks L2 to fetch bytes [lo, hi) of `base` (rounded inward to 16-byte
// boundaries, so nothing outside the range is touched), in 64 KB pieces.
// Issued by one thread for a tile that is loaded later, it lets the HBM fetch
// overlap the current tile's work; the later loads then hit L2.
__device__ __forceinline__ void prefetch_l2(const void* base, int64_t lo, int64_t hi) {
  uint64_t a = reinterpret_cast<uint64_t>(base) + (uint64_t)lo, e = reinterpret_cast<uint64_t>(base) + (uint64_t)hi;
  a = (a + 15) & ~uint64_t(15);
  e &= ~uint64_t(15);
  for (; a < e; a += 65536) {
    const uint32_t n = (uint32_t)((e - a) < 65536 ? (e - a) : 65536);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(a), "r"(n) : "memory");
  }
}

inline size_t dtype_bytes(int dtype) { return dtype == LWL_F32 ? 4 : 2; }

// Thread-local error text for lwl_last_error().
void set_error(const char* fmt, ...);
// Empties the calling thread's error text (every entry point starts with it).
void clear_error();

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device):
// the attribute belongs to the device, so a process that drives several GPUs
// sets it on each of them.
inline bool set_max_smem(const void* func, int bytes) {
  static std::mutex mu;
  static std::set<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  if (done.count({func, dev})) return true;
  if (cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess) return false;
  done.insert({func, dev});
  return true;
}

}  // namespace lwl

#define LWL_CUDA_TRY(expr)                                                        \
  do {                                                                            \
    cudaError_t _e = (expr);                                                      \
    if (_e != cudaSuccess) {                                                      \
      ::lwl::set_error("%s failed: %s", #expr, cudaGetErrorString(_e));           \
      return LWL_ERR_CUDA;                                                        \
    }                                                                             \
  } while (0)
