// fht32_mix.cu -- FixedFHTMix rows on the register-resident scheme of fht32.cuh.
//
// y[r, :F] = (S * H_P / sqrt(P) * S * pad(x[r, :]))[:F] for every row r, with
// P = next_pow2(F) and S = diag(signs) (reference examples/nanogpt/model.py:182-218).
// Two kernels: fht_mix32p_kernel (rows 16-byte aligned, P = 8 .. 8192)
// prefetches the next tile into shared memory with cp.async while the current
// one is transformed; fht_mix32_kernel (P = 2048 .. 8192, other rows) loads
// straight into registers.  The warp-per-row kernel of fht_mix.cu is held
// back by three CTA barriers per row group at the large widths.
//
// A CTA of 128 threads owns a tile of 2^13 elements = 2^(13-n) rows of P = 2^n
// and holds 64 fp32 values per thread.  Rows are loaded in set A (64
// consecutive columns per thread), the sign flip and the register bits t0..t5
// of the transform run there, one conflict-free shared-memory exchange moves
// the tile to set B (t6..t11, lanes along t0..t4) for the rest of the bits
// (bits t6..t(n-1); above n the tile bits select rows) (plus one more exchange to set C for bit 12 at P = 8192), and set B / C
// stores 32 consecutive columns per warp instruction.  The sign table is the
// fixed vector's sign bits, built once per CTA, and serves both flips.
#include <algorithm>
#include <cmath>

#include "fht32.cuh"

namespace lwl {
namespace f32k {

struct MixParams {
  const void* x;
  void* y;
  int64_t rows;
  int F;             // features per row (<= P)
  float scale;       // 1 / sqrt(P)
  int64_t ntiles;
  const float* signs;  // [P] +-1
};

// Source / sink element of tile index t: row (tile << (13 - n)) + (t >> n), column t mod P.
template <typename T, int N, int SET>
__device__ __forceinline__ void mix_load(float (&v)[kRegs], const MixParams& p, int64_t tile, int base) {
  constexpr int P = 1 << N;
  const T* x = reinterpret_cast<const T*>(p.x);
  const int64_t row0 = (tile << (13 - N)) + (base >> N);
  const int col0 = base & (P - 1);
  // SET A with N >= 6: the 64 registers are 64 consecutive columns of one row
  static_assert(SET == SA && N >= 6, "rows load in set A");
  const T* s = x + row0 * p.F + col0;
  const bool row_ok = row0 < p.rows;
  int hi = row_ok ? p.F - col0 : 0;  // valid columns [0, hi)
  if (hi > kRegs) hi = kRegs;
  if (hi == kRegs && (reinterpret_cast<uintptr_t>(s) & (4 * sizeof(T) - 1)) == 0) {
#pragma unroll
    for (int q = 0; q < kRegs / 4; ++q) {
      if (sizeof(T) == 4) {
        const float4 a = *reinterpret_cast<const float4*>(s + 4 * q);
        v[4 * q] = a.x, v[4 * q + 1] = a.y, v[4 * q + 2] = a.z, v[4 * q + 3] = a.w;
      } else {
        const uint2 a = *reinterpret_cast<const uint2*>(s + 4 * q);
        const T* e = reinterpret_cast<const T*>(&a);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * q + i] = Cvt<T>::to_f(e[i]);
      }
    }
  } else {
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = r < hi ? Cvt<T>::to_f(s[r]) : 0.0f;
  }
}

template <typename T, int N, int SET>
__device__ __forceinline__ void mix_store(const float (&v)[kRegs], const MixParams& p, int64_t tile, int base) {
  constexpr int P = 1 << N;
  T* y = reinterpret_cast<T*>(p.y);
  const int64_t row0 = (tile << (13 - N)) + (base >> N);
  const int col0 = base & (P - 1);
  T* d = y + row0 * p.F + col0;
#pragma unroll
  for (int r = 0; r < kRegs; ++r) {
    const int t = spread<13, SET>(r);  // register part of the tile index (disjoint from base)
    const int dr = t >> N, dc = t & (P - 1);
    if (col0 + dc < p.F && row0 + dr < p.rows) d[(int64_t)dr * p.F + dc] = Cvt<T>::from_f(v[r] * p.scale);
  }
}

template <typename T, int N>
__global__ void __launch_bounds__(Tile<13>::kThreads, Tile<13>::kMinBlocks)
    fht_mix32_kernel(const __grid_constant__ MixParams p) {
  using Tl = Tile<13>;
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  uint32_t* sw = reinterpret_cast<uint32_t*>(buf + Tl::kBufWords);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int P = 1 << N;
  // sign bits of the fixed vector (bit set = +1), repeated for every row of the tile
  for (int c = warp; c < Tl::kWords; c += Tl::kThreads / 32) {
    const int i = (32 * c + lane) & (P - 1);
    const uint32_t b = __ballot_sync(0xffffffffu, p.signs[i] > 0.0f);
    if (lane == 0) sw[c] = b;
  }
  __syncthreads();
  const int bA = base_of<13, SA>(lane, warp), bB = base_of<13, SB>(lane, warp), bC = base_of<13, SC>(lane, warp);
  float v[kRegs];
  for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    mix_load<T, N, SA>(v, p, tile, bA);
    apply_sign<13, SA>(v, sw, bA);
    xform<13, SA>(v, Tl::kA, N);
    exchange<13, SA, SB>(v, buf, lane, warp);
    xform<13, SB>(v, Tl::kB, N);
    if constexpr (N == 13) {
      exchange<13, SB, SC>(v, buf, lane, warp);
      xform<13, SC>(v, Tl::kChi, N);
      apply_sign<13, SC>(v, sw, bC);
      mix_store<T, N, SC>(v, p, tile, bC);
    } else {
      apply_sign<13, SB>(v, sw, bB);
      mix_store<T, N, SB>(v, p, tile, bB);
    }
  }
}

// ---------------------------------------------------------------------------
// Prefetching variant (x and y 16-byte aligned, F * sizeof(T) a multiple of
// 16).  The next tile's rows are copied into a shared-memory stage with
// 16-byte cp.async while this tile is transformed, so every CTA keeps one
// tile of loads in flight through its compute phase.  Stage layout: chunk c
// (64 consecutive tile elements) at c * (64 * sizeof(T) + 16) bytes, so the
// set-A reads (lanes one chunk apart, 16 bytes each) are bank-conflict free.
// The fixed sign vector is the same for every tile, so each thread gathers the
// 64 sign bits of its registers in a set once (bit r set = negate register r)
// and a flip is two integer ops per element.
template <int SET>
__device__ __forceinline__ uint64_t sign_mask(const uint32_t* sw, int base) {
  uint64_t m = 0;
#pragma unroll
  for (int r = 0; r < kRegs; ++r) {
    const int t = base | spread<13, SET>(r);
    m |= (uint64_t)((~sw[t >> 5] >> (t & 31)) & 1u) << r;
  }
  return m;
}
__device__ __forceinline__ void apply_mask(float (&v)[kRegs], uint64_t m) {
  // opaque copies: otherwise the compiler hoists 64 per-register flip words
  // out of the tile loop and runs out of registers
  uint32_t lo, hi;
  asm volatile("mov.b32 %0, %1;" : "=r"(lo) : "r"((uint32_t)m));
  asm volatile("mov.b32 %0, %1;" : "=r"(hi) : "r"((uint32_t)(m >> 32)));
#pragma unroll
  for (int r = 0; r < kRegs; ++r) v[r] = flip(v[r], ((r < 32 ? lo : hi) << (31 - (r & 31))) & 0x80000000u);
}

template <typename T>
struct Stage {
  static constexpr int kChunkBytes = 64 * (int)sizeof(T) + 16;
  static constexpr int kBytes = 128 * kChunkBytes;          // 2^13 elements
  static constexpr int kPieces = (1 << 13) * (int)sizeof(T) / 16;
  static constexpr int kPerChunk = 64 * (int)sizeof(T) / 16;  // 16-byte pieces per chunk
  static constexpr size_t kSmem = Tile<13>::kSmem + 2 * size_t(kBytes);
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}

// Issue the copies of tile `tile` into the stage at shared address `st` (zero-filled outside x).
template <typename T, int N>
__device__ __forceinline__ void mix_prefetch(const MixParams& p, int64_t tile, uint32_t st, int tid) {
  constexpr int PER = 16 / (int)sizeof(T);
  const T* x = reinterpret_cast<const T*>(p.x);
  if (tile < p.ntiles) {
#pragma unroll
    for (int j = 0; j < Stage<T>::kPieces / Tile<13>::kThreads; ++j) {
      const int k = tid + j * Tile<13>::kThreads;
      const int t = k * PER;  // first tile element of the piece
      const int64_t row = (tile << (13 - N)) + (t >> N);
      const int col = t & ((1 << N) - 1);
      const bool ok = row < p.rows && col < p.F;  // F is a multiple of PER
      const T* src = ok ? x + row * p.F + col : x;
      cp_async16(st + (k / Stage<T>::kPerChunk) * Stage<T>::kChunkBytes + (k % Stage<T>::kPerChunk) * 16, src,
                 ok ? 16 : 0);
    }
  }
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}

template <typename T, int N>
__global__ void __launch_bounds__(Tile<13>::kThreads)
    fht_mix32p_kernel(const __grid_constant__ MixParams p) {
  using Tl = Tile<13>;
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  uint32_t* sw = reinterpret_cast<uint32_t*>(buf + Tl::kBufWords);
  unsigned char* stage = smem + Tl::kSmem;
  const uint32_t st0 = (uint32_t)__cvta_generic_to_shared(stage);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int P = 1 << N;
  mix_prefetch<T, N>(p, blockIdx.x, st0, tid);
  for (int c = warp; c < Tl::kWords; c += Tl::kThreads / 32) {
    const int i = (32 * c + lane) & (P - 1);
    const uint32_t b = __ballot_sync(0xffffffffu, p.signs[i] > 0.0f);
    if (lane == 0) sw[c] = b;
  }
  const int bA = base_of<13, SA>(lane, warp), bB = base_of<13, SB>(lane, warp), bC = base_of<13, SC>(lane, warp);
  __syncthreads();  // the sign table is complete
  const uint64_t mA = sign_mask<SA>(sw, bA), mOut = N == 13 ? sign_mask<SC>(sw, bC) : sign_mask<SB>(sw, bB);
  float v[kRegs];
  int s = 0;
  for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x, s ^= 1) {
    // every thread is past the previous tile's first exchange barrier, so no
    // thread still reads the stage refilled here
    mix_prefetch<T, N>(p, tile + gridDim.x, st0 + (s ^ 1) * Stage<T>::kBytes, tid);
    asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    __syncthreads();  // this tile's stage (and, the first time, the sign table) is complete
    const unsigned char* ch = stage + s * Stage<T>::kBytes + (bA >> 6) * Stage<T>::kChunkBytes;
#pragma unroll
    for (int q = 0; q < Stage<T>::kPerChunk; ++q) {
      const uint4 raw = *reinterpret_cast<const uint4*>(ch + 16 * q);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
      constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
      for (int u = 0; u < PER; ++u) {
        float f;
        if (sizeof(T) == 4) f = __uint_as_float(wv[u]);
        else {
          const uint32_t h = (u & 1) ? (wv[u >> 1] >> 16) : (wv[u >> 1] & 0xffffu);
          f = Cvt<T>::to_f(*reinterpret_cast<const T*>(&h));
        }
        v[q * PER + u] = f;
      }
    }
    apply_mask(v, mA);
    xform<13, SA>(v, Tl::kA, N);
    exchange<13, SA, SB>(v, buf, lane, warp);
    xform<13, SB>(v, Tl::kB, N);
    if constexpr (N == 13) {
      exchange<13, SB, SC>(v, buf, lane, warp);
      xform<13, SC>(v, Tl::kChi, N);
      apply_mask(v, mOut);
      mix_store<T, N, SC>(v, p, tile, bC);
    } else {
      apply_mask(v, mOut);
      mix_store<T, N, SB>(v, p, tile, bB);
    }
  }
  asm volatile("cp.async.wait_group 0;\n" ::: "memory");
}

template <typename T>
const void* mix_p_kernel_for(int n) {
  switch (n) {
    case 3: return (const void*)fht_mix32p_kernel<T, 3>;
    case 4: return (const void*)fht_mix32p_kernel<T, 4>;
    case 5: return (const void*)fht_mix32p_kernel<T, 5>;
    case 6: return (const void*)fht_mix32p_kernel<T, 6>;
    case 7: return (const void*)fht_mix32p_kernel<T, 7>;
    case 8: return (const void*)fht_mix32p_kernel<T, 8>;
    case 9: return (const void*)fht_mix32p_kernel<T, 9>;
    case 10: return (const void*)fht_mix32p_kernel<T, 10>;
    case 11: return (const void*)fht_mix32p_kernel<T, 11>;
    case 12: return (const void*)fht_mix32p_kernel<T, 12>;
    default: return (const void*)fht_mix32p_kernel<T, 13>;
  }
}

template <typename T>
const void* mix_kernel_for(int n) {
  switch (n) {
    case 11: return (const void*)fht_mix32_kernel<T, 11>;
    case 12: return (const void*)fht_mix32_kernel<T, 12>;
    default: return (const void*)fht_mix32_kernel<T, 13>;
  }
}

}  // namespace f32k

bool fht_mix32_supported(int logP) { return logP >= 11 && logP <= 13; }

// The prefetching tile kernel: P = 2^3 .. 2^13 with aligned rows (F * sizeof(T)
// a multiple of 16 implies P >= 8).  For P <= 64 the whole transform runs in
// set A and one exchange lays the rows out for the stores in set B.
bool fht_mix32p_supported(int dtype, const void* x, const void* y, int F, int logP) {
  const int es = dtype == LWL_F32 ? 4 : 2;
  return logP >= 3 && logP <= 13 && (F * es) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(y) & 15) == 0;
}

int fht_mix32p_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                      cudaStream_t st) {
  using namespace f32k;
  MixParams p;
  p.x = x;
  p.y = y;
  p.rows = rows;
  p.F = F;
  p.scale = 1.0f / std::sqrt((float)(1 << logP));
  const int64_t rows_per_tile = int64_t(1) << (13 - logP);
  p.ntiles = (rows + rows_per_tile - 1) / rows_per_tile;
  p.signs = signs;
  const void* k;
  size_t smem;
  if (dtype == LWL_BF16) k = mix_p_kernel_for<__nv_bfloat16>(logP), smem = Stage<__nv_bfloat16>::kSmem;
  else if (dtype == LWL_F16) k = mix_p_kernel_for<__half>(logP), smem = Stage<__half>::kSmem;
  else k = mix_p_kernel_for<float>(logP), smem = Stage<float>::kSmem;
  if (!set_max_smem(k, (int)smem)) return -1;
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, Tile<13>::kThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>(p.ntiles, (int64_t)nsm * per_sm);
  void* args[] = {&p};
  return cudaLaunchKernel(k, dim3(grid), dim3(Tile<13>::kThreads), args, smem, st) == cudaSuccess ? 0 : -1;
}

int fht_mix32_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                     cudaStream_t st) {
  using namespace f32k;
  MixParams p;
  p.x = x;
  p.y = y;
  p.rows = rows;
  p.F = F;
  p.scale = 1.0f / std::sqrt((float)(1 << logP));
  const int64_t rows_per_tile = int64_t(1) << (13 - logP);
  p.ntiles = (rows + rows_per_tile - 1) / rows_per_tile;
  p.signs = signs;
  const void* k = dtype == LWL_BF16 ? mix_kernel_for<__nv_bfloat16>(logP)
                                    : (dtype == LWL_F16 ? mix_kernel_for<__half>(logP) : mix_kernel_for<float>(logP));
  const size_t smem = Tile<13>::kSmem;
  if (!set_max_smem(k, (int)smem)) return -1;
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, Tile<13>::kThreads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>(p.ntiles, (int64_t)nsm * per_sm);
  void* args[] = {&p};
  return cudaLaunchKernel(k, dim3(grid), dim3(Tile<13>::kThreads), args, smem, st) == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
