// fht32_hi.cu -- the high-bit pass of the two-pass layout (blocks of
// 2^16 .. 2^23 with a 15-bit low pass) on the register-resident scheme of
// fht32.cuh.
//
// The two-pass layout (fht_engine.cu) transforms a block of B = 2^n as
// H_B = H_hi (x) H_32768: the tensor-core low pass (fht_lo_kernel) takes the 15
// low position bits, and this pass the h = n - 15 high bits, which are
// strided by 2^15 in the block.  The generic tile engine ran the high pass
// with eight 4-byte loads in flight per thread, latency-bound at about
// 1.8 TB/s.  Here a CTA of 128 threads owns a tile of 2^13 elements: the
// 2^h high positions (tile bits 13-h .. 12) times 2^(13-h) consecutive low
// positions (tile bits 0 .. 12-h).  In set C of fht32.cuh (registers = tile
// bits 7..12, lanes = bits 0..4) the high bits are register bits, so the whole
// pass -- the optional pre-sign, the runs of butterflies and their signs --
// is one residency with no exchange, and every warp load and store covers 32
// consecutive positions.  Each thread holds 64 values in flight.
//
// Sources: the latent, the gradient slice or the workspace; sink: the
// workspace (16-bit plans always end with a low pass).  The workspace is fp32,
// or bf16 in the forward plans that keep a bf16 workspace (fht_engine.cu).  Blocks wholly
// inside the gradient slice load without bounds tests: with a 64-bit range
// test on every element this launch ran at half the speed of the tile engine.  Signs and the
// 1/sqrt(B) of each post-sign follow the plan's slots exactly as the tile
// engine applies them.
#include <algorithm>

#include "fht32.cuh"

namespace lwl {
namespace f32k {

// Four consecutive workspace elements (16-byte fp32 or 8-byte bf16 access).
__device__ __forceinline__ void ld4(const float* s, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(s);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = a.z;
  v[3] = a.w;
}
__device__ __forceinline__ void ld4(const __nv_bfloat16* s, float* v) {
  const uint2 a = *reinterpret_cast<const uint2*>(s);
  const float2 lo = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.x));
  const float2 hi = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&a.y));
  v[0] = lo.x;
  v[1] = lo.y;
  v[2] = hi.x;
  v[3] = hi.y;
}
__device__ __forceinline__ void st4(float* d, const float* v) {
  *reinterpret_cast<float4*>(d) = make_float4(v[0], v[1], v[2], v[3]);
}
__device__ __forceinline__ void st4(__nv_bfloat16* d, const float* v) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(d) = make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

template <typename T, int H, int SRC, typename W>
__global__ void __launch_bounds__(Tile<13>::kThreads, Tile<13>::kMinBlocks)
    fht_hi_kernel(const __grid_constant__ TileParams p) {
  using Tl = Tile<13>;
  constexpr int LOW = 13 - H;                   // consecutive low positions per tile
  constexpr int CHUNKS = 1 << (15 - LOW);       // tiles per block
  constexpr int HIMASK = ((1 << H) - 1) << LOW;  // tile bits of the high positions
  __shared__ uint32_t sw[kMaxSlots * Tl::kWords];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // bf16 workspace with up to 4 high bits (2^16 .. 2^19): the high bits are
  // register bits of set SD as well, whose threads hold four consecutive
  // positions, so every workspace access is 8 bytes and 256 contiguous bytes
  // per warp (+8-10% at 2^18 / 2^19) instead of 2-byte accesses.  The fp32
  // workspace keeps set C (16-byte SD accesses measured 2-5% slower), and so
  // does the gradient slice.
  constexpr int S = (H <= 4 && SRC != SRC_SLICE && sizeof(W) == 2) ? SD : SC;
  const int base = base_of<13, S>(lane, warp);
  const int nsw = p.nslots;
  float v[kRegs];
  for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    const int64_t b = p.first_block + tile / CHUNKS;  // block
    const int j = (int)(tile % CHUNKS);              // low chunk of the block
    const int64_t pos0 = (int64_t)j << LOW;          // position of tile element 0
    __syncthreads();  // the previous tile is done with the sign table
    // sign words of the tile: entry c covers high value c >> (8 - H), low word c & (2^(8-H) - 1)
    for (int i = tid; i < nsw * Tl::kWords; i += Tl::kThreads) {
      const int s = i / Tl::kWords, c = i - s * Tl::kWords;
      const int64_t word = ((int64_t)(c >> (8 - H)) << 10) + (pos0 >> 5) + (c & ((1 << (8 - H)) - 1));
      sw[i] = sign_word(block_layer_key(p.seed32, b, p.slot_layer[s]), word);
    }
    __syncthreads();
    // element t = base | spread(r): position pos0 + (t & low mask) + (t >> LOW) << 15
    const int lo_b = base & ((1 << LOW) - 1);
    const int64_t rowoff = (b - p.first_block) * p.B;
    if (SRC == SRC_WS) {
      const W* s = reinterpret_cast<const W*>(p.src) + rowoff + pos0 + lo_b;
      if (S == SD) {
#pragma unroll
        for (int q = 0; q < kRegs / 4; ++q) {
          const int t = spread<13, S>(4 * q);
          ld4(s + (t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15), v + 4 * q);
        }
      } else {
#pragma unroll
        for (int r = 0; r < kRegs; ++r) {
          const int t = spread<13, S>(r);
          v[r] = Cvt<W>::to_f(s[(t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15)]);
        }
      }
    } else if (SRC == SRC_LATENT) {
      const T* s = reinterpret_cast<const T*>(p.src);
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int t = spread<13, S>(r);
        const int64_t pos = pos0 + lo_b + (t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15);
        v[r] = pos < p.L ? Cvt<T>::to_f(s[pos]) : 0.0f;
      }
    } else if (b * p.B >= p.start && (b + 1) * p.B <= p.stop) {
      // the whole block lies inside the slice: unpredicated loads
      const T* s = reinterpret_cast<const T*>(p.src) + (b * p.B - p.start) + pos0 + lo_b;
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int t = spread<13, S>(r);
        v[r] = Cvt<T>::to_f(s[(t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15)]);
      }
    } else {
      const T* s = reinterpret_cast<const T*>(p.src);
      const int64_t g0 = b * p.B + pos0 + lo_b;
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int t = spread<13, S>(r);
        const int64_t g = g0 + (t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15);
        v[r] = (g >= p.start && g < p.stop) ? Cvt<T>::to_f(s[g - p.start]) : 0.0f;
      }
    }
    if (p.pre_slot >= 0) apply_sign<13, S>(v, sw + p.pre_slot * Tl::kWords, base);
    for (int ri = 0; ri < p.nruns; ++ri) {
      const RunDesc& rd = p.runs[ri];
      // the run's group: transform bits glo..glo+gr-1 of the engine's tile, whose
      // column bits (cb = 3) precede them, i.e. high bits glo-3 .. glo-3+gr-1
      const int mask = (((1 << rd.gr) - 1) << (rd.glo - 3 + LOW)) & HIMASK;
      for (int f = 0; f < rd.nfht; ++f) {
        xform<13, S>(v, mask, 13);
        const int sl = rd.slot[f];
        if (sl >= 0) {
          apply_sign<13, S>(v, sw + sl * Tl::kWords, base);
#pragma unroll
          for (int r = 0; r < kRegs; ++r) v[r] *= p.scale;
        }
      }
    }
    W* d = reinterpret_cast<W*>(p.dst) + rowoff + pos0 + lo_b;
    if (S == SD) {
#pragma unroll
      for (int q = 0; q < kRegs / 4; ++q) {
        const int t = spread<13, S>(4 * q);
        st4(d + (t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15), v + 4 * q);
      }
    } else {
#pragma unroll
      for (int r = 0; r < kRegs; ++r) {
        const int t = spread<13, S>(r);
        d[(t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15)] = Cvt<W>::from_f(v[r]);
      }
    }
  }
}

// 7 or 8 high bits (blocks of 2^22 / 2^23): a tile of 2^(7+h) elements = the
// 2^h high positions x 128 consecutive low positions (tile bits 0..6), so that
// every run's group of high bits lies in the registers of set B (tile bits
// 6..11) or set C (the top six); the runs execute in plan order and the tile
// moves between B and C through shared memory when the next group needs it.
template <typename T, int TB, int SET, int SRC, typename W>
__device__ __forceinline__ void hi2_load(float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0, int base) {
  constexpr int LOW = 7;
  auto off = [](int t) { return (int64_t)(t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15); };
  if (SRC == SRC_WS) {
    const W* s = reinterpret_cast<const W*>(p.src) + (b - p.first_block) * p.B + pos0 + off(base);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = Cvt<W>::to_f(s[off(spread<TB, SET>(r))]);
  } else if (SRC == SRC_LATENT) {
    const T* s = reinterpret_cast<const T*>(p.src);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int64_t pos = pos0 + off(base) + off(spread<TB, SET>(r));
      v[r] = pos < p.L ? Cvt<T>::to_f(s[pos]) : 0.0f;
    }
  } else if (b * p.B >= p.start && (b + 1) * p.B <= p.stop) {
    const T* s = reinterpret_cast<const T*>(p.src) + (b * p.B - p.start) + pos0 + off(base);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) v[r] = Cvt<T>::to_f(s[off(spread<TB, SET>(r))]);
  } else {
    const T* s = reinterpret_cast<const T*>(p.src);
    const int64_t g0 = b * p.B + pos0 + off(base);
#pragma unroll
    for (int r = 0; r < kRegs; ++r) {
      const int64_t g = g0 + off(spread<TB, SET>(r));
      v[r] = (g >= p.start && g < p.stop) ? Cvt<T>::to_f(s[g - p.start]) : 0.0f;
    }
  }
}

template <int TB, int SET, typename W>
__device__ __forceinline__ void hi2_store(const float (&v)[kRegs], const TileParams& p, int64_t b, int64_t pos0,
                                          int base) {
  constexpr int LOW = 7;
  auto off = [](int t) { return (int64_t)(t & ((1 << LOW) - 1)) + ((int64_t)(t >> LOW) << 15); };
  W* d = reinterpret_cast<W*>(p.dst) + (b - p.first_block) * p.B + pos0 + off(base);
#pragma unroll
  for (int r = 0; r < kRegs; ++r) d[off(spread<TB, SET>(r))] = Cvt<W>::from_f(v[r]);
}

template <typename T, int H, int SRC, typename W>
__global__ void __launch_bounds__(Tile<7 + H>::kThreads, 1) fht_hi2_kernel(const __grid_constant__ TileParams p) {
  constexpr int TB = 7 + H;
  using Tl = Tile<TB>;
  constexpr int LOW = 7;
  constexpr int CHUNKS = 1 << (15 - LOW);  // tiles per block
  constexpr int MASKC = Tl::kC;            // tile bits of set C's registers
  extern __shared__ __align__(16) unsigned char smem[];
  float* buf = reinterpret_cast<float*>(smem);
  uint32_t* sw = reinterpret_cast<uint32_t*>(buf + Tl::kBufWords);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bB = base_of<TB, SB>(lane, warp), bC = base_of<TB, SC>(lane, warp);
  // tile bits of run ri's group: high bits glo-3 .. glo-3+gr-1 (column bits cb = 3 precede them)
  auto group_mask = [&](int ri) { return ((1 << p.runs[ri].gr) - 1) << (p.runs[ri].glo - 3 + LOW); };
  float v[kRegs];
  for (int64_t tile = blockIdx.x; tile < p.ntiles; tile += gridDim.x) {
    const int64_t b = p.first_block + tile / CHUNKS;
    const int64_t pos0 = (int64_t)(tile % CHUNKS) << LOW;
    __syncthreads();  // the previous tile is done with the sign table and the exchange buffer
    for (int i = tid; i < p.nslots * Tl::kWords; i += Tl::kThreads) {
      const int s = i / Tl::kWords, c = i - s * Tl::kWords;
      const int64_t word = ((int64_t)(c >> (LOW - 5)) << 10) + (pos0 >> 5) + (c & ((1 << (LOW - 5)) - 1));
      sw[i] = sign_word(block_layer_key(p.seed32, b, p.slot_layer[s]), word);
    }
    __syncthreads();
    bool in_c = (group_mask(0) & ~MASKC) == 0;  // start in the set of the first run's group
    if (in_c) hi2_load<T, TB, SC, SRC, W>(v, p, b, pos0, bC);
    else hi2_load<T, TB, SB, SRC, W>(v, p, b, pos0, bB);
    if (p.pre_slot >= 0) {
      if (in_c) apply_sign<TB, SC>(v, sw + p.pre_slot * Tl::kWords, bC);
      else apply_sign<TB, SB>(v, sw + p.pre_slot * Tl::kWords, bB);
    }
    for (int ri = 0; ri < p.nruns; ++ri) {
      const int mask = group_mask(ri);
      const bool want_c = (mask & ~MASKC) == 0;
      if (want_c != in_c) {
        if (want_c) exchange<TB, SB, SC>(v, buf, lane, warp);
        else exchange<TB, SC, SB>(v, buf, lane, warp);
        in_c = want_c;
      }
      for (int f = 0; f < p.runs[ri].nfht; ++f) {
        const int sl = p.runs[ri].slot[f];
        if (in_c) {
          xform<TB, SC>(v, mask, TB);
          if (sl >= 0) apply_sign<TB, SC>(v, sw + sl * Tl::kWords, bC);
        } else {
          xform<TB, SB>(v, mask, TB);
          if (sl >= 0) apply_sign<TB, SB>(v, sw + sl * Tl::kWords, bB);
        }
        if (sl >= 0) {
#pragma unroll
          for (int r = 0; r < kRegs; ++r) v[r] *= p.scale;
        }
      }
    }
    if (in_c) hi2_store<TB, SC, W>(v, p, b, pos0, bC);
    else hi2_store<TB, SB, W>(v, p, b, pos0, bB);
  }
}

template <typename T, int SRC, typename W>
const void* hi_kernel_h(int h) {
  switch (h) {
    case 1: return (const void*)fht_hi_kernel<T, 1, SRC, W>;
    case 2: return (const void*)fht_hi_kernel<T, 2, SRC, W>;
    case 3: return (const void*)fht_hi_kernel<T, 3, SRC, W>;
    case 4: return (const void*)fht_hi_kernel<T, 4, SRC, W>;
    case 5: return (const void*)fht_hi_kernel<T, 5, SRC, W>;
    case 6: return (const void*)fht_hi_kernel<T, 6, SRC, W>;
    case 7: return (const void*)fht_hi2_kernel<T, 7, SRC, W>;
    default: return (const void*)fht_hi2_kernel<T, 8, SRC, W>;
  }
}

// W: the workspace element (fp32, or bf16 for the plans that keep a bf16
// workspace).
template <typename T>
const void* hi_kernel(int src, int h, bool ws16) {
  if (ws16) {
    if (src == SRC_WS) return hi_kernel_h<T, SRC_WS, __nv_bfloat16>(h);
    if (src == SRC_LATENT) return hi_kernel_h<T, SRC_LATENT, __nv_bfloat16>(h);
    return hi_kernel_h<T, SRC_SLICE, __nv_bfloat16>(h);
  }
  if (src == SRC_WS) return hi_kernel_h<T, SRC_WS, float>(h);
  if (src == SRC_LATENT) return hi_kernel_h<T, SRC_LATENT, float>(h);
  return hi_kernel_h<T, SRC_SLICE, float>(h);
}

}  // namespace f32k

// A planned tile-engine launch this pass can take: a two-pass plan's high-bit
// launch (column chunks of 8 below 15 low bits) of 1..8 high bits into the
// fp32 workspace, for any dtype (fp32 arithmetic throughout).
bool fht_hi_eligible(int dtype, const TileParams& p) {
  if (dtype != LWL_BF16 && dtype != LWL_F16 && dtype != LWL_F32) return false;
  if (p.lo || p.tlo != 15 || p.cb != 3 || p.dst_kind != DST_WS) return false;
  const int h = p.n - 15;
  if (h < 1 || h > 8 || p.r != h || p.nslots > f32k::kMaxSlots || p.nruns < 1) return false;
  for (int i = 0; i < p.nruns; ++i) {
    const RunDesc& rd = p.runs[i];
    if (rd.glo < 3 || rd.glo + rd.gr > 3 + h) return false;
    if (h > 6) {
      // every group must lie in the registers of set B (tile bits 6..11) or of
      // set C (the top six tile bits 1+h .. 6+h); high bit k is tile bit 7 + k
      const int lo = rd.glo + 4, hi = rd.glo + 4 + rd.gr;  // tile bits [lo, hi)
      if (!(lo >= 6 && hi <= 12) && !(lo >= 1 + h && hi <= 7 + h)) return false;
    }
  }
  return true;
}

int fht_hi_launch(int dtype, const TileParams& p_in, cudaStream_t st) {
  using namespace f32k;
  TileParams p = p_in;
  const int h = p.n - 15;
  // tiles of 2^13 (h <= 6: 2^(2+h) per block) or 2^(7+h) (h = 7, 8: 256 per block)
  const int tb = h <= 6 ? 13 : 7 + h;
  p.ntiles = p.nblocks << (h <= 6 ? h + 2 : 8);
  const int threads = 1 << (tb - 6);
  const size_t smem = h <= 6 ? 0 : (tb == 14 ? Tile<14>::kSmem : Tile<15>::kSmem);
  const bool ws16 = p.ws16 != 0 && dtype != LWL_F32;
  const void* k = dtype == LWL_BF16 ? hi_kernel<__nv_bfloat16>(p.src_kind, h, ws16)
                : dtype == LWL_F16  ? hi_kernel<__half>(p.src_kind, h, ws16)
                                    : hi_kernel<float>(p.src_kind, h, false);
  if (smem > 0 && !set_max_smem(k, (int)smem)) return -1;
  int per_sm = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int dev = 0, nsm = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
  const int grid = (int)std::min<int64_t>(p.ntiles, (int64_t)nsm * per_sm);
  void* args[] = {&p};
  return cudaLaunchKernel(k, dim3(grid), dim3(threads), args, smem, st) == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
