// fht_mma.cu -- tensor-core BlockFHT forward for 16-bit dtypes at block size 2^15.
//
// H_32768 is factored over the 15 position bits into 16x16 mma tiles.  A
// block lives in the registers of 16 warps (8 tiles of 256 elements per
// warp); two "passes" alternate:
//   pass A transforms position bits {5,6,7,3} (tile rows, H16) and
//          {4,9,10,11} (tile cols, H16);
//   pass B transforms bits {0,1,2,8} (rows, H16) and {12,13,14} (cols, H8;
//          col bit 0 = position bit 4 is carried through as an identity).
// Within a pass, H is applied to the tile rows as H*X (data in the
// B-operand slot) and to the columns as X*H (data in the A-operand slot);
// the f16 accumulator fragment of one mma is directly the A fragment of the
// next, so a pass needs no register shuffles.  Adjacent layers share a pass
// ([A s A], [B s B]), so three layers cost three shared-memory exchanges.
// Each exchange writes 16-byte chunks gathered across the 8 tiles a thread
// owns (st.shared.v4) and reads them back with ldmatrix; the XOR swizzles in
// lay_ab / lay_ba make both sides bank-conflict free.
//
// Arithmetic: fp16 operands and intermediates with orthonormal factors
// (H16/4, H8/2).  The input is pre-scaled by a power of two, taken from its
// largest magnitude, so that the block's L2 norm is below 2^12 -- every
// intermediate element is bounded by the block's norm, so nothing overflows,
// and typical elements stay far from subnormals (prescale_exponent).  The last column transform accumulates in fp32, is rescaled
// and rounded once to the output dtype.  Signs are XORed into packed pairs:
// positions p and p+16 share a register, so one shift + LOP3 flips both.
#include <cmath>
#include <cstdio>

#include "fht_mma_core.cuh"

namespace lwl {
namespace fmma {

// Forward kernel over a group of generators: work item = one 2^15-coordinate
// tile of one descriptor (a single call is a group of one).  The scaled fp16
// latent copy and the constant fragments are rebuilt only when a CTA moves to
// the next descriptor.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1) fht15_forward_kernel(const __grid_constant__ FwdGroup G) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* zbuf = reinterpret_cast<uint16_t*>(smem);   // scaled fp16 latent copy (64 KB)
  uint16_t* xbuf = zbuf + kB;                           // exchange buffers (64 KB each)
  uint16_t* ybuf = xbuf + kB;
  // two sign tables [layers+1][kWordsPad]: the next tile's words are written
  // during this tile, before its staging barrier, so a tile starts without one
  uint32_t* sw_buf = reinterpret_cast<uint32_t*>(ybuf + kB);
  __shared__ float red[kThreads / 32];
  __shared__ int k0_shared;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  __shared__ uint32_t tmem_base_shared;
  if (w == 0) {
    uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_shared);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 128;\n" ::"r"(dst));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  // this warp's 32 columns in its lane quadrant: the first run's input fragments
  const uint32_t tz = tmem_base_shared + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(32 * (w >> 2));
  const uint32_t zb = (uint32_t)__cvta_generic_to_shared(zbuf);
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xbuf);
  const uint32_t yb = (uint32_t)__cvta_generic_to_shared(ybuf);
  Frags f;
  int cur = -1, k0 = 0;
  // sign words of work item `it` (any descriptor) into dst
  auto gen_signs = [&](int64_t it, uint32_t* dst) {
    int dd = 0;
    while (dd + 1 < G.count && G.d[dd + 1].tile_prefix <= it) ++dd;
    const FwdDesc& E = G.d[dd];
    const int en = E.n, eBm = (1 << en) - 1;
    const int64_t eblk = E.first_tile + (it - E.tile_prefix);
    for (int i = tid; i < (E.layers + 1) * kWords; i += kThreads) {
      int l = i / kWords, wd = i - l * kWords;
      const int p = 32 * wd;
      dst[l * kWordsPad + spad(wd)] =
          sign_word(block_layer_key(E.seed32, (eblk << (kLog - en)) + (p >> en), l), (p & eBm) >> 5);
    }
  };
  if (blockIdx.x < G.total_tiles) gen_signs(blockIdx.x, sw_buf);
  __syncthreads();
  int parity = 0;

  for (int64_t item = blockIdx.x; item < G.total_tiles; item += gridDim.x) {
    uint32_t* sw = sw_buf + (parity ? 4 * kWordsPad : 0);
    uint32_t* sw_next = sw_buf + (parity ? 0 : 4 * kWordsPad);
    parity ^= 1;
    const bool has_next = item + gridDim.x < G.total_tiles;
    int di = 0;
    while (di + 1 < G.count && G.d[di + 1].tile_prefix <= item) ++di;
    const FwdDesc& D = G.d[di];
    const T* latent = reinterpret_cast<const T*>(D.latent);
    const int n = D.n, layers = D.layers, Bm = (1 << n) - 1;
    const int64_t L = D.L;
    // After the previous tile's staging barrier no warp reads the sign table,
    // the latent copy or red[] again; slower warps may still copy out of the
    // staging buffer (ybuf).  For 1 and 3 layers that buffer is next written
    // two barriers later, so no barrier is needed here; the first run of a
    // 2-layer tile writes ybuf, so it waits.
    if (layers == 2) __syncthreads();
    if (di != cur) {
      make_frags(f, g, t, n);
      // power-of-two prescale from the largest magnitude (block norm below 2^12)
      float mx = 0.0f;
      for (int64_t i = tid; i < L; i += kThreads) {
        float v = Cvt<T>::to_f(latent[i]);
        mx = fmaxf(mx, fabsf(v));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      if (lane == 0) red[w] = mx;
      __syncthreads();
      if (tid == 0) {
        float s = 0.0f;
        for (int i = 0; i < kThreads / 32; ++i) s = fmaxf(s, red[i]);
        int e = prescale_exponent(s, n);
        k0_shared = e;
      }
      __syncthreads();
      k0 = k0_shared;
      const float in_scale = ldexpf(1.0f, -k0);
      // the first run is pass B for layers 1 and 3, pass A for layers 2
      const bool first_is_b = (layers != 2);
      for (int c = tid; c < kB / 8; c += kThreads) {  // 8 consecutive positions per step
        float v[8];
        const int p0 = 8 * c, q0 = p0 & Bm;  // q0: position inside its block
        if (q0 + 8 <= L && (reinterpret_cast<uintptr_t>(latent) & 15) == 0) {
          uint4 raw = __ldg(reinterpret_cast<const uint4*>(latent + q0));
          const T* ev = reinterpret_cast<const T*>(&raw);
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = Cvt<T>::to_f(ev[e]) * in_scale;
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) v[e] = (q0 + e < L) ? Cvt<T>::to_f(latent[q0 + e]) * in_scale : 0.0f;
        }
        uint32_t hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) hv[e] = pack_h2(v[2 * e], v[2 * e + 1]);
        if (first_is_b) {
          *reinterpret_cast<uint4*>(zbuf + lay_ab(p0)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) zbuf[lay_ba(p0 + e)] = (uint16_t)(hv[e >> 1] >> (16 * (e & 1)));
        }
      }
      cur = di;
      __syncthreads();  // the latent copy is complete
      if (first_is_b)
        park_first_input<1>(zb, tz, w, lane);
      else
        park_first_input<0>(zb, tz, w, lane);
    }
    const float out_scale = ldexpf(1.0f, k0) * D.corr;
    T* out = reinterpret_cast<T*>(D.out);
    const bool vec_ok = ((D.start & 7) == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
    const int64_t blk = D.first_tile + (item - D.tile_prefix);
    // this tile's sign words were written before the previous tile's staging
    // barrier (or before the loop); the next tile's are written below, before
    // run_final's staging barrier, into the other table
    if (layers == 1) {
      run_first_tmem<1>(f, tz, xb, sw, w, lane, g, t);
      __syncthreads();
      if (has_next) gen_signs(item + gridDim.x, sw_next);
      run_final<T>(f, xb, yb, ybuf, sw + 1 * kWordsPad, out_scale, out, blk, D.start, D.stop, vec_ok, w, lane, g, t);
    } else if (layers == 2) {
      run_first_tmem<0>(f, tz, yb, sw, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      if (has_next) gen_signs(item + gridDim.x, sw_next);
      run_final<T>(f, xb, yb, ybuf, sw + 2 * kWordsPad, out_scale, out, blk, D.start, D.stop, vec_ok, w, lane, g, t);
    } else {
      run_first_tmem<1>(f, tz, xb, sw, w, lane, g, t);
      __syncthreads();
      run<0, true, false>(f, xb, yb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 2 * kWordsPad, w, lane, g, t);
      __syncthreads();
      if (has_next) gen_signs(item + gridDim.x, sw_next);
      run_final<T>(f, xb, yb, ybuf, sw + 3 * kWordsPad, out_scale, out, blk, D.start, D.stop, vec_ok, w, lane, g, t);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 128;\n" ::"r"(tmem_base_shared));
}

constexpr size_t kSmem = 3 * kB * 2 + 2 * 4 * kWordsPad * 4;  // two sign tables
static_assert(kSmem <= 232448, "shared memory per CTA");

template <typename T>
int launch_forward_t(const FwdGroup& G, cudaStream_t st) {
  if (!set_max_smem((const void*)fht15_forward_kernel<T>, (int)kSmem)) return -1;
  if (G.total_tiles <= 0) return 0;
  int sms = sm_count();
  int grid = (int)(G.total_tiles < sms ? G.total_tiles : sms);
  fht15_forward_kernel<T><<<grid, kThreads, kSmem, st>>>(G);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------
// Block size 2^16 forward (16-bit dtypes): one CTA per block holds both 2^15
// tiles in shared memory.  H_65536 = H_2 (position bit 15) (x) H_32768 (bits
// 0-14) and the factors commute, so each layer does the one-bit "hi"
// butterfly between the tiles first -- one pass over both tiles' fp16 buffers
// that also applies the layer's signs -- and then the tensor-core 2^15
// transform (pass B, pass A) of each tile.  The hi butterflies are
// unnormalised (the block norm grows by sqrt(2) per layer; the power-of-two
// prescale keeps every element inside fp16) and their 2^(-1/2) per layer is
// folded into the output scale.  Layer 0's hi pass reads the latent from
// global memory; the last layer ends with the staged copy-out of each tile.
// No HBM workspace and one launch, where the general large-block path needs
// an fp32 workspace pass per layer and per high-bit group.
constexpr size_t kSmem16 = 3 * kB * 2 + 2 * 4 * kWordsPad * 4;

// Two 16-bit values of type T packed in one word (low half first) -> float2.
template <typename T> __device__ __forceinline__ float2 w2f(uint32_t v);
template <> __device__ __forceinline__ float2 w2f<__half>(uint32_t v) {
  return __half22float2(*reinterpret_cast<const __half2*>(&v));
}
template <> __device__ __forceinline__ float2 w2f<__nv_bfloat16>(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

// Raw words of src[q0 .. q0+7] restricted to [0, n): the elements outside are
// zero.  For the chunks a caller's predicated 16-byte load did not cover.
__device__ __forceinline__ void gather8_words(const uint16_t* src, int64_t q0, int64_t n, uint32_t* r) {
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    const uint32_t bits = (q0 + e >= 0 && q0 + e < n) ? (uint32_t)src[q0 + e] : 0u;
    r[e >> 1] = (e & 1) ? (r[e >> 1] | (bits << 16)) : bits;
  }
}

// 1-bit hi butterfly of one chunk (8 values, 4 packed fp16 words) of tile 0
// and tile 1 at the same positions, in place: signs first (m0 / m1 = the
// inverted sign bits of the chunk from bit 0; sign bit set -> +1,
// block_fht.py:55-81) as one XOR per word, then sum and difference.  An fp16
// sum of two fp16 values rounds exactly like the fp32 sum rounded once.
__device__ __forceinline__ void hi2_chunk(uint32_t* x0, uint32_t* x1, uint32_t m0, uint32_t m1) {
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const uint32_t u0 = x0[e] ^ ((((m0 >> (2 * e)) & 3u) * 0x40008000u) & 0x80008000u);
    const uint32_t u1 = x1[e] ^ ((((m1 >> (2 * e)) & 3u) * 0x40008000u) & 0x80008000u);
    const __half2 a0 = *reinterpret_cast<const __half2*>(&u0), a1 = *reinterpret_cast<const __half2*>(&u1);
    const __half2 s = __hadd2(a0, a1), d = __hsub2(a0, a1);
    x0[e] = *reinterpret_cast<const uint32_t*>(&s);
    x1[e] = *reinterpret_cast<const uint32_t*>(&d);
  }
}

__device__ __forceinline__ void unpack_h8(const uint4 v, float* f) {
  const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
    f[2 * i] = h.x;
    f[2 * i + 1] = h.y;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    fht16_forward_kernel(const T* __restrict__ latent, int64_t L, int layers, uint32_t seed32, float scale_base,
                         int64_t first_block, int64_t nblocks, int64_t start, int64_t stop, T* __restrict__ out) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* z0 = reinterpret_cast<uint16_t*>(smem);  // tile 0 (positions 0..32767 of the block)
  uint16_t* z1 = z0 + kB;                           // tile 1 (positions 32768..65535)
  uint16_t* xs = z1 + kB;                           // exchange buffer
  uint32_t* sw = reinterpret_cast<uint32_t*>(xs + kB);  // [tile][layer][kWordsPad]
  __shared__ float red[kThreads / 32];
  __shared__ int k0_shared;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const uint32_t zb[2] = {(uint32_t)__cvta_generic_to_shared(z0), (uint32_t)__cvta_generic_to_shared(z1)};
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xs);
  Frags f;
  make_frags(f, g, t, kLog);
  // power-of-two prescale from the largest magnitude (block norm below 2^12)
  float mx = 0.0f;
  for (int64_t i = tid; i < L; i += kThreads) {
    const float v = Cvt<T>::to_f(latent[i]);
    mx = fmaxf(mx, fabsf(v));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) red[w] = mx;
  __syncthreads();
  if (tid == 0) {
    float s2 = 0.0f;
    for (int i = 0; i < kThreads / 32; ++i) s2 = fmaxf(s2, red[i]);
    int e = prescale_exponent(s2, 16);
    k0_shared = e;
  }
  __syncthreads();
  const int k0 = k0_shared;
  const float in_scale = ldexpf(1.0f, -k0), out_scale = ldexpf(1.0f, k0) * scale_base;
  const bool vec_ok = ((start & 7) == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  const bool lat_tail = (reinterpret_cast<uintptr_t>(latent) & 15) != 0 || (L & 7) != 0;

  for (int64_t bi = blockIdx.x; bi < nblocks; bi += gridDim.x) {
    const int64_t b = first_block + bi;
    __syncthreads();  // the previous block's copy-out is done with the buffers and sign tables
    // sign words of both tiles and all layers: tile j has words 1024 j .. of the block
    for (int i = tid; i < 2 * (layers + 1) * kWords; i += kThreads) {
      const int per = (layers + 1) * kWords, j = i / per, r = i - j * per, l = r / kWords, wd = r - l * kWords;
      sw[(4 * j + l) * kWordsPad + spad(wd)] = sign_word(block_layer_key(seed32, b, l), 1024 * j + wd);
    }
    __syncthreads();
    for (int l = 0; l < layers; ++l) {
      // hi butterfly of layer l (signs S_l first), written in the pass-B input layout
      const uint32_t* s0 = sw + (4 * 0 + l) * kWordsPad;
      const uint32_t* s1 = sw + (4 * 1 + l) * kWordsPad;
      // two halves of 4 chunks per thread; in layer 0 all 8 latent loads of a
      // half are in flight at once (predicated 16-byte loads when the latent
      // is aligned and a multiple of 8 long, else element by element)
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t raw[2][16];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
#pragma unroll
          for (int qq = 0; qq < 4; ++qq) {
            const int p0 = 8 * (tid + kThreads * (4 * h + qq));
            uint4 r = make_uint4(0u, 0u, 0u, 0u);
            if (l > 0) {
              r = *reinterpret_cast<const uint4*>((j ? z1 : z0) + lay_ab(p0));
            } else if (!lat_tail) {
              const int64_t q0 = (int64_t)kB * j + p0;
              if (q0 < L) r = __ldg(reinterpret_cast<const uint4*>(latent + q0));
            }
            raw[j][4 * qq] = r.x, raw[j][4 * qq + 1] = r.y, raw[j][4 * qq + 2] = r.z, raw[j][4 * qq + 3] = r.w;
          }
        }
        if (l == 0 && lat_tail) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
              gather8_words(reinterpret_cast<const uint16_t*>(latent),
                            (int64_t)kB * j + 8 * (tid + kThreads * (4 * h + qq)), L, &raw[j][4 * qq]);
          }
        }
        if (l == 0) {  // the input words, scaled, into packed fp16
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
              const float2 fv = w2f<T>(raw[j][r]);
              raw[j][r] = pack_h2(fv.x * in_scale, fv.y * in_scale);
            }
          }
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int p0 = 8 * (tid + kThreads * (4 * h + qq));
          uint32_t* o0 = &raw[0][4 * qq];
          uint32_t* o1 = &raw[1][4 * qq];
          hi2_chunk(o0, o1, ~(s0[spad(p0 >> 5)] >> (p0 & 31)), ~(s1[spad(p0 >> 5)] >> (p0 & 31)));
          *reinterpret_cast<uint4*>(z0 + lay_ab(p0)) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
          *reinterpret_cast<uint4*>(z1 + lay_ab(p0)) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
        }
      }
      __syncthreads();
      // 2^15 transform of each tile: pass B (z_j -> x), pass A (x -> z_j), or
      // in the last layer pass A with the last signs, staged through z_j
      // (consumed by pass B) and copied out
#pragma unroll 1
      for (int j = 0; j < 2; ++j) {
        run<1, false, false>(f, zb[j], xb, nullptr, nullptr, w, lane, g, t);
        __syncthreads();
        if (l + 1 < layers) {
          run<0, false, false>(f, xb, zb[j], nullptr, nullptr, w, lane, g, t);
        } else {
          run_final<T>(f, xb, zb[j], j ? z1 : z0, sw + (4 * j + layers) * kWordsPad, out_scale, out, 2 * b + j,
                       start, stop, vec_ok, w, lane, g, t);
        }
        __syncthreads();
      }
    }
  }
}

template <typename T>
int launch_forward16_t(const void* latent, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                       void* out, cudaStream_t st) {
  const int64_t B = 2 * kB;
  const int64_t first = start / B, last = (stop + B - 1) / B;
  if (last <= first) return 0;
  if (!set_max_smem((const void*)fht16_forward_kernel<T>, (int)kSmem16)) return -1;
  const int64_t nb = last - first, sms = sm_count();
  const int grid = (int)(nb < sms ? nb : sms);
  const float scale_base = (float)(std::pow(layer_correction(kLog), layers) * std::pow(2.0, -0.5 * layers));
  fht16_forward_kernel<T><<<grid, kThreads, kSmem16, st>>>(reinterpret_cast<const T*>(latent), L, layers,
                                                           fold_seed(seed), scale_base, first, nb, start, stop,
                                                           reinterpret_cast<T*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// fp32 partial-row staging of a 2^15 tile: the accumulator-layout writer varies
// position bits 5-7 and 9-10 across a warp (32-way bank conflicts on the
// plain index); XOR-ing them into bits 0-4 spreads them over all 32 banks,
// and the consecutive reader sees a warp-uniform XOR.
__device__ __forceinline__ int prow_swz(int p) { return p ^ (((p >> 5) & 7) | (((p >> 9) & 3) << 3)); }


// ---------------------------------------------------------------------------
// Backward: grad_z = sum_b [S0 Ĥ S1 ... Ĥ S_layers g_b][0:L].  Same runs as the
// forward with the sign layers reversed; the per-block result (fp32, from the
// last column transform) is accumulated across the blocks a CTA processes in
// tensor memory: 128 lanes x 256 columns hold the 32768 fp32 partial sums,
// each thread owning the 64 values of its final-run fragments.  At the end
// every CTA writes its partial [L] row; fht15_reduce_kernel sums the rows.

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float* v) {
  uint32_t r[8];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const float* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
               "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
               "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])));
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }


// Final backward run (pass A): transforms, scale, sign of layer 0, add into TMEM.
__device__ __forceinline__ void run_final_acc(const Frags& f, uint32_t in_base, const uint32_t* sw, float scale,
                                              uint32_t tbase, int w, int lane, int g, int t) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float c[8];
    final_tile(f, in_base, w, k, lane, c);
    float acc[8];
    tmem_ld8(tbase + 8 * k, acc);
    // c[i]: row g + 8((i>>1)&1), column 2t + (i&1) + 8(i>>2) of pass A, i.e.
    // position base + k + 8((i>>1)&1) + 16(i&1) + 2048(i>>2)
    const int wb = dep_a(w, 0, g, 2 * t) >> 5;
    const uint32_t u0 = ~sw[spad(wb)], u1 = ~sw[spad(wb + 64)];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int bit = k + 8 * ((i >> 1) & 1) + 16 * (i & 1);
      const uint32_t u = (i >> 2) ? u1 : u0;
      acc[i] += __uint_as_float(__float_as_uint(c[i] * scale) ^ ((u << (31 - bit)) & 0x80000000u));
    }
    tmem_st8(tbase + 8 * k, acc);
  }
  tmem_wait_st();
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    fht15_backward_kernel(const T* __restrict__ grad, int64_t L, int layers, int n, uint32_t seed32, float corr,
                          int64_t first_block,
                          int64_t nblocks, int64_t start, int64_t stop, float* __restrict__ partial,
                          int* __restrict__ err, int test_stall) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* xbuf = reinterpret_cast<uint16_t*>(smem);
  uint16_t* ybuf = xbuf + kB;
  uint16_t* stage = ybuf + kB;  // raw gradient of the next block (bulk copy target)
  // two sign tables: block i writes one while slower warps may still read
  // block i-1's in its last run, so the loop needs no barrier at its top
  uint32_t* sw_buf = reinterpret_cast<uint32_t*>(stage + kB);
  __shared__ float red[kThreads / 32];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __shared__ uint32_t tmem_base_shared;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  Frags f;
  make_frags(f, g, t, n);
  const int Bm = (1 << n) - 1;

  if (w == 0) {
    uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_shared);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;\n" ::"r"(dst));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  // warp w uses lanes 32*(w%4).. and columns 64*(w/4) .. +63
  const uint32_t tbase = tmem_base_shared + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(64 * (w >> 2));
  {
    float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) tmem_st8(tbase + 8 * k, z);
    tmem_wait_st();
  }

  const float layer_scale = corr;
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xbuf);
  const uint32_t yb = (uint32_t)__cvta_generic_to_shared(ybuf);
  const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
  const uint32_t mbar_s = (uint32_t)__cvta_generic_to_shared(&mbar);
  // landing buffer for the gradient: read by the first run (pass B via the
  // A->B layout for layers 1 and 3, pass A via the B->A layout for layers 2)
  const bool first_is_b = (layers != 2);
  uint16_t* land = first_is_b ? ybuf : xbuf;
  const bool vec_ok = ((start & 7) == 0) && ((reinterpret_cast<uintptr_t>(grad) & 15) == 0);
  // whole blocks inside the slice arrive by one 64 KB bulk copy into `stage`,
  // issued one block ahead; edge blocks are read with bounds checks instead
  auto bulk_ok = [&](int64_t blk) { return vec_ok && blk * kB >= start && (blk + 1) * kB <= stop; };
  auto issue = [&](int64_t blk) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar_s), "r"((uint32_t)(kB * 2)));
    const T* src = grad + (blk * kB - start);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(stage_s),
        "l"(src), "r"((uint32_t)(kB * 2)), "r"(mbar_s)
        : "memory");
  };
  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(mbar_s));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  uint32_t phase = 0;
  // Bounded waits: (1 << 22) polls normally.  test_stall (LWL_FLAG_TEST_WAIT_TIMEOUT)
  // leaves the first copy unissued and polls 256 times, so the first wait gives
  // up with no copy in flight and the call reports LWL_ERR_TIMEOUT.
  const int polls = test_stall ? 256 : (1 << 22);
  bool inflight = false;  // thread 0: a bulk copy was issued and has not been waited for
  if (tid == 0 && !test_stall && blockIdx.x < nblocks && bulk_ok(first_block + blockIdx.x)) {
    issue(first_block + blockIdx.x);
    inflight = true;
  }

  int parity = 0;
  for (int64_t bi = blockIdx.x; bi < nblocks; bi += gridDim.x) {
    const int64_t blk = first_block + bi;
    const int64_t bbase = blk * kB;
    uint32_t* sw = sw_buf + (parity ? 4 * kWordsPad : 0);
    parity ^= 1;
    // 2 layers land the gradient in xbuf, which the previous block's last run
    // still reads; 1 and 3 layers land it in ybuf, free since that run began
    if (layers == 2) __syncthreads();
    for (int i = tid; i < (layers + 1) * kWords; i += kThreads) {
      int l = i / kWords, wd = i - l * kWords;
      const int p = 32 * wd;
      sw[l * kWordsPad + spad(wd)] =
          sign_word(block_layer_key(seed32, (blk << (kLog - n)) + (p >> n), l), (p & Bm) >> 5);
    }
    // gradient chunks of this block into registers, with their largest magnitude
    uint4 raw[8];
    float mx = 0.0f;
    const bool bulk = bulk_ok(blk);
    if (bulk) {
      // bounded wait for the bulk copy; on time-out record the failure and stop
      uint32_t done = 0;
      for (int it = 0; it < polls && !done; ++it) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(mbar_s), "r"(phase)
            : "memory");
      }
      if (!done) {
        abort_flag = 1;
        atomicExch(err, 1);
      } else {
        inflight = false;
      }
      phase ^= 1u;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int c = tid + kThreads * i;
      int64_t gi = bbase + 8 * c;
      if (bulk) {
        raw[i] = reinterpret_cast<const uint4*>(stage)[c];
      } else {
        uint32_t vv[4] = {0, 0, 0, 0};
        for (int e = 0; e < 8; ++e) {
          int64_t gg = gi + e;
          if (gg >= start && gg < stop)
            vv[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t*>(grad)[gg - start] << (16 * (e & 1));
        }
        raw[i] = make_uint4(vv[0], vv[1], vv[2], vv[3]);
      }
      const T* ev = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = Cvt<T>::to_f(ev[e]);
        mx = fmaxf(mx, fabsf(v));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    if (abort_flag) break;  // uniform: set before the barrier above
    // the stage buffer is free again: fetch the next block while this one runs
    if (tid == 0) {
      int64_t nb = bi + gridDim.x;
      if (nb < nblocks && bulk_ok(first_block + nb)) {
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        issue(first_block + nb);
        inflight = true;
      }
    }
    // every thread forms the prescale exponent from the warp sums (same
    // summation order everywhere, so all threads agree; no second barrier)
    int k0 = 0;
    {
      float s = 0.0f;
      for (int i = 0; i < kThreads / 32; ++i) s = fmaxf(s, red[i]);
      k0 = prescale_exponent(s, n);
    }
    const float in_scale = ldexpf(1.0f, -k0);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int c = tid + kThreads * i;
      const T* ev = reinterpret_cast<const T*>(&raw[i]);
      uint32_t hv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        hv[e] = pack_h2(Cvt<T>::to_f(ev[2 * e]) * in_scale, Cvt<T>::to_f(ev[2 * e + 1]) * in_scale);
      if (first_is_b) {
        *reinterpret_cast<uint4*>(land + lay_ab(8 * c)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) land[lay_ba(8 * c + e)] = (uint16_t)(hv[e >> 1] >> (16 * (e & 1)));
      }
    }
    __syncthreads();
    const float scale = ldexpf(1.0f, k0) * layer_scale;
    if (layers == 1) {
      run<1, false, true>(f, yb, xb, sw + 1 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    } else if (layers == 2) {
      run<0, false, true>(f, xb, yb, sw + 2 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    } else {
      run<1, false, true>(f, yb, xb, sw + 3 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run<0, true, false>(f, xb, yb, nullptr, sw + 2 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    }
  }
  if (abort_flag && tid == 0 && inflight) {
    // let an outstanding copy land before the CTA exits (bounded)
    uint32_t done = 0;
    for (int it = 0; it < (1 << 22) && !done; ++it) {
      asm volatile(
          "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
          : "=r"(done)
          : "r"(mbar_s), "r"(phase ^ 1u)
          : "memory");
    }
  }
  // this CTA's partial gradient row, staged in natural order through the two
  // exchange buffers (128 KB = 32768 fp32) for coalesced stores
  __syncthreads();
  float* prow = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float acc[8];
    tmem_ld8(tbase + 8 * k, acc);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
      prow[prow_swz(dep_a(w, k, R, C))] = acc[i];
    }
  }
  __syncthreads();
  // fold the 2^(15-n) blocks of the tile onto the latent positions
  for (int64_t p = tid; p < L; p += kThreads) {
    float v = 0.0f;
    for (int j = 0; j < (kB >> n); ++j) v += prow[prow_swz((int)((j << n) + p))];
    partial[(int64_t)blockIdx.x * L + p] = v;
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem_base_shared));
}

// Sum of the per-CTA rows; a failed bulk-copy wait (err != 0) poisons the
// gradient with NaN so the failure cannot pass silently.
template <typename T>
__global__ void fht15_reduce_kernel(const float* __restrict__ partial, int rows, int64_t L, const int* __restrict__ err,
                                    T* __restrict__ out) {
  const bool bad = *err != 0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < L; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};  // eight loads in flight, fixed summation order
    int r = 0;
    for (; r + 8 <= rows; r += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += partial[(int64_t)(r + u) * L + i];
    }
    for (; r < rows; ++r) acc[0] += partial[(int64_t)r * L + i];
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    out[i] = Cvt<T>::from_f(bad ? __int_as_float(0x7fc00000) : s);
  }
}

constexpr size_t kSmemBwd = 3 * kB * 2 + 4 * kWordsPad * 4;
constexpr size_t kSmemBwd1 = 3 * kB * 2 + 2 * 4 * kWordsPad * 4;  // single backward: two sign tables
static_assert(kSmemBwd1 <= 232448, "shared memory per CTA");
constexpr size_t kBwdHeader = 256;  // workspace: [error word | pad] then the partial rows


template <typename T>
int launch_backward_t(const void* grad, int64_t L, int layers, int n, uint32_t seed32, int64_t first_block,
                      int64_t nblocks,
                      int64_t start, int64_t stop, void* grad_latent, void* workspace, cudaStream_t st,
                      int test_stall) {
  int* err = reinterpret_cast<int*>(workspace);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kBwdHeader);
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return -1;
  if (!set_max_smem((const void*)fht15_backward_kernel<T>, (int)kSmemBwd1)) return -1;
  int sms = sm_count();
  int grid = (int)(nblocks < sms ? nblocks : sms);
  const float corr = (float)std::pow(layer_correction(n), layers);
  fht15_backward_kernel<T><<<grid, kThreads, kSmemBwd1, st>>>(reinterpret_cast<const T*>(grad), L, layers, n, seed32,
                                                             corr,
                                                             first_block, nblocks, start, stop, partial, err,
                                                             test_stall);
  if (cudaGetLastError() != cudaSuccess) return -1;
  int rb = (int)((L + 255) / 256);
  fht15_reduce_kernel<T><<<rb, 256, 0, st>>>(partial, grid, L, err, reinterpret_cast<T*>(grad_latent));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}


// ---------------------------------------------------------------------------
// Block size 2^16 backward (16-bit dtypes): the transposed chain
// grad_z = sum_b [S0 H S1 ... H S_layers g_b][0:L] with the same building
// blocks as fht16_forward_kernel -- per step a hi pass (with that step's
// signs) and the 2^15 transform of each tile; the last pass A multiplies by
// S0 and accumulates into tensor memory (both tiles: 512 columns, 65536 fp32
// partial sums per CTA).  Each CTA writes one [L] partial row, tile by tile
// through shared memory; fht15_reduce_kernel sums the rows deterministically.
template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    fht16_backward_kernel(const T* __restrict__ grad, int64_t L, int layers, uint32_t seed32, float scale_base,
                          int64_t first_block, int64_t nblocks, int64_t start, int64_t stop,
                          float* __restrict__ partial) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* z0 = reinterpret_cast<uint16_t*>(smem);
  uint16_t* z1 = z0 + kB;
  uint16_t* xs = z1 + kB;
  uint32_t* sw = reinterpret_cast<uint32_t*>(xs + kB);  // [tile][layer][kWordsPad]
  __shared__ float red[kThreads / 32];
  __shared__ uint32_t tmem_base_shared;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const uint32_t zb[2] = {(uint32_t)__cvta_generic_to_shared(z0), (uint32_t)__cvta_generic_to_shared(z1)};
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xs);
  Frags f;
  make_frags(f, g, t, kLog);

  if (w == 0) {
    uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_shared);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;\n" ::"r"(dst));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  // warp w: lanes 32*(w%4).., columns 64*(w/4).. of tile 0 and 256 + 64*(w/4).. of tile 1
  const uint32_t tbase = tmem_base_shared + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(64 * (w >> 2));
  {
    float zf[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 16; ++k) tmem_st8(tbase + 8 * (k & 7) + 256 * (k >> 3), zf);
    tmem_wait_st();
  }
  const bool vec_ok = ((start & 7) == 0) && ((reinterpret_cast<uintptr_t>(grad) & 15) == 0);

  for (int64_t bi = blockIdx.x; bi < nblocks; bi += gridDim.x) {
    const int64_t b = first_block + bi;
    const int64_t bbase = b * 2 * kB;
    __syncthreads();  // the previous block's final runs are done with the buffers and sign tables
    for (int i = tid; i < 2 * (layers + 1) * kWords; i += kThreads) {
      const int per = (layers + 1) * kWords, j = i / per, r = i - j * per, l = r / kWords, wd = r - l * kWords;
      sw[(4 * j + l) * kWordsPad + spad(wd)] = sign_word(block_layer_key(seed32, b, l), 1024 * j + wd);
    }
    // Gradient chunks (8 values at block position p) as raw words: 16-byte
    // loads with no per-chunk test when the whole block lies inside
    // [start, stop) and the gradient is aligned, else element by element
    // with zeros outside the slice.
    const bool blk_full = vec_ok && bbase >= start && bbase + 2 * kB <= stop;
    const uint16_t* g16 = reinterpret_cast<const uint16_t*>(grad);
    // largest magnitude of the block's gradient (read again from L2 by the first hi pass)
    float mx = 0.0f;
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {
      uint32_t r[8][4];
      if (blk_full) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 x = __ldg(reinterpret_cast<const uint4*>(grad + (bbase - start) + 8 * (tid + kThreads * (8 * h + u))));
          r[u][0] = x.x, r[u][1] = x.y, r[u][2] = x.z, r[u][3] = x.w;
        }
      } else {
#pragma unroll
        for (int u = 0; u < 8; ++u)
          gather8_words(g16, bbase + 8 * (tid + kThreads * (8 * h + u)) - start, stop - start, r[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 fv = w2f<T>(r[u][e]);
          mx = fmaxf(mx, fmaxf(fabsf(fv.x), fabsf(fv.y)));
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    int k0 = 0;
    {
      float s2 = 0.0f;
      for (int i = 0; i < kThreads / 32; ++i) s2 = fmaxf(s2, red[i]);
      k0 = prescale_exponent(s2, 16);
    }
    const float in_scale = ldexpf(1.0f, -k0), scale = ldexpf(1.0f, k0) * scale_base;
    for (int st = 0; st < layers; ++st) {
      const int l = layers - st;  // signs S_l before this step's transform
      const uint32_t* s0 = sw + (4 * 0 + l) * kWordsPad;
      const uint32_t* s1 = sw + (4 * 1 + l) * kWordsPad;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t raw[2][16];
        if (st > 0) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const uint4 x = *reinterpret_cast<const uint4*>((j ? z1 : z0) + lay_ab(8 * (tid + kThreads * (4 * h + qq))));
              raw[j][4 * qq] = x.x, raw[j][4 * qq + 1] = x.y, raw[j][4 * qq + 2] = x.z, raw[j][4 * qq + 3] = x.w;
            }
          }
        } else if (blk_full) {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq) {
              const uint4 x = __ldg(reinterpret_cast<const uint4*>(grad + (bbase - start) + (int64_t)kB * j +
                                                                   8 * (tid + kThreads * (4 * h + qq))));
              raw[j][4 * qq] = x.x, raw[j][4 * qq + 1] = x.y, raw[j][4 * qq + 2] = x.z, raw[j][4 * qq + 3] = x.w;
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int qq = 0; qq < 4; ++qq)
              gather8_words(g16, bbase + (int64_t)kB * j + 8 * (tid + kThreads * (4 * h + qq)) - start, stop - start,
                            &raw[j][4 * qq]);
          }
        }
        if (st == 0) {  // the input words, scaled, into packed fp16
#pragma unroll
          for (int j = 0; j < 2; ++j) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
              const float2 fv = w2f<T>(raw[j][r]);
              raw[j][r] = pack_h2(fv.x * in_scale, fv.y * in_scale);
            }
          }
        }
#pragma unroll
        for (int qq = 0; qq < 4; ++qq) {
          const int p0 = 8 * (tid + kThreads * (4 * h + qq));
          uint32_t* o0 = &raw[0][4 * qq];
          uint32_t* o1 = &raw[1][4 * qq];
          hi2_chunk(o0, o1, ~(s0[spad(p0 >> 5)] >> (p0 & 31)), ~(s1[spad(p0 >> 5)] >> (p0 & 31)));
          *reinterpret_cast<uint4*>(z0 + lay_ab(p0)) = make_uint4(o0[0], o0[1], o0[2], o0[3]);
          *reinterpret_cast<uint4*>(z1 + lay_ab(p0)) = make_uint4(o1[0], o1[1], o1[2], o1[3]);
        }
      }
      __syncthreads();
#pragma unroll 1
      for (int j = 0; j < 2; ++j) {
        run<1, false, false>(f, zb[j], xb, nullptr, nullptr, w, lane, g, t);
        __syncthreads();
        if (st + 1 < layers)
          run<0, false, false>(f, xb, zb[j], nullptr, nullptr, w, lane, g, t);
        else
          run_final_acc(f, xb, sw + (4 * j + 0) * kWordsPad, scale, tbase + 256 * j, w, lane, g, t);
        __syncthreads();
      }
    }
  }
  // this CTA's partial row, one tile at a time through shared memory (fp32,
  // 128 KB over z0 | z1) for coalesced stores
  float* prow = reinterpret_cast<float*>(smem);
#pragma unroll 1
  for (int j = 0; j < 2; ++j) {
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float acc[8];
      tmem_ld8(tbase + 256 * j + 8 * k, acc);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
        prow[prow_swz(dep_a(w, k, R, C))] = acc[i];
      }
    }
    __syncthreads();
    for (int64_t pp = tid; pp < kB; pp += kThreads) {
      const int64_t q = (int64_t)kB * j + pp;
      if (q < L) partial[(int64_t)blockIdx.x * L + q] = prow[prow_swz((int)pp)];
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;\n" ::"r"(tmem_base_shared));
}

template <typename T>
int launch_backward16_t(const void* grad, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                        void* grad_latent, void* workspace, cudaStream_t st) {
  const int64_t B = 2 * kB;
  const int64_t first = start / B, last = (stop + B - 1) / B;
  if (last <= first) return cudaMemsetAsync(grad_latent, 0, size_t(L) * 2, st) == cudaSuccess ? 0 : -1;
  int* err = reinterpret_cast<int*>(workspace);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kBwdHeader);
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return -1;
  if (!set_max_smem((const void*)fht16_backward_kernel<T>, (int)kSmem16)) return -1;
  const int64_t nb = last - first, sms = sm_count();
  const int grid = (int)(nb < sms ? nb : sms);
  const float scale_base = (float)(std::pow(layer_correction(kLog), layers) * std::pow(2.0, -0.5 * layers));
  fht16_backward_kernel<T><<<grid, kThreads, kSmem16, st>>>(reinterpret_cast<const T*>(grad), L, layers,
                                                            fold_seed(seed), scale_base, first, nb, start, stop,
                                                            partial);
  if (cudaGetLastError() != cudaSuccess) return -1;
  const int rb = (int)((L + 255) / 256);
  fht15_reduce_kernel<T><<<rb, 256, 0, st>>>(partial, grid, L, err, reinterpret_cast<T*>(grad_latent));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

#include "fht_parked.cuh"

// ---------------------------------------------------------------------------
// Grouped backward: the latent gradients of many generators in one launch
// (the projection side of a model's weight cache).  The 2^15-coordinate
// tiles of all descriptors form one list; CTA c takes the contiguous range
// [c*T/G, (c+1)*T/G), so it meets few descriptors.  Per descriptor it
// accumulates in tensor memory exactly as the single-generator kernel does;
// when the descriptor changes it flushes the accumulator into its partial
// row of that descriptor (rows of descriptor d: the CTAs c_lo(d) ..) and
// starts from zero.  fht15_reduce_grouped_kernel sums each descriptor's rows.

struct BwdDesc {
  const void* grad;
  void* out;
  int64_t L, start, stop;
  int64_t first_block, nblocks, tile_prefix;  // tiles of this descriptor and their place in the list
  int64_t row_off;                            // float offset of its first partial row
  int c_lo, rows;                             // first CTA touching it, number of such CTAs
  uint32_t seed32;
  int n, layers;
  float corr;
};
struct BwdGroup {
  int count, grid;
  int64_t total_tiles;
  BwdDesc d[kMaxGroup];
};

template <typename T>
__global__ void __launch_bounds__(kThreads, 1)
    fht15_backward_grouped_kernel(const __grid_constant__ BwdGroup G, float* __restrict__ partial,
                                  int* __restrict__ err) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* xbuf = reinterpret_cast<uint16_t*>(smem);
  uint16_t* ybuf = xbuf + kB;
  uint16_t* stage = ybuf + kB;  // raw gradient of the next tile (bulk copy target)
  uint32_t* sw = reinterpret_cast<uint32_t*>(stage + kB);
  __shared__ float red[kThreads / 32];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ int abort_flag;
  __shared__ uint32_t tmem_base_shared;
  if (threadIdx.x == 0) abort_flag = 0;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  if (w == 0) {
    uint32_t dst = (uint32_t)__cvta_generic_to_shared(&tmem_base_shared);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 256;\n" ::"r"(dst));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  const uint32_t tbase = tmem_base_shared + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(64 * (w >> 2));
  auto zero_acc = [&]() {
    float z[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int k = 0; k < 8; ++k) tmem_st8(tbase + 8 * k, z);
    tmem_wait_st();
  };
  zero_acc();

  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xbuf);
  const uint32_t yb = (uint32_t)__cvta_generic_to_shared(ybuf);
  const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage);
  const uint32_t mbar_s = (uint32_t)__cvta_generic_to_shared(&mbar);
  const int64_t i0 = (int64_t)blockIdx.x * G.total_tiles / G.grid;
  const int64_t i1 = (int64_t)(blockIdx.x + 1) * G.total_tiles / G.grid;
  auto desc_of = [&](int64_t i, int from) {
    int d = from;
    while (d + 1 < G.count && G.d[d + 1].tile_prefix <= i) ++d;
    return d;
  };
  auto bulk_ok = [&](const BwdDesc& D, int64_t blk) {
    return ((D.start & 7) == 0) && ((reinterpret_cast<uintptr_t>(D.grad) & 15) == 0) && blk * kB >= D.start &&
           (blk + 1) * kB <= D.stop;
  };
  auto issue = [&](const BwdDesc& D, int64_t blk) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar_s), "r"((uint32_t)(kB * 2)));
    const T* src = reinterpret_cast<const T*>(D.grad) + (blk * kB - D.start);
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(stage_s),
        "l"(src), "r"((uint32_t)(kB * 2)), "r"(mbar_s)
        : "memory");
  };
  // partial row of descriptor D for this CTA, staged in natural order through
  // the exchange buffers; the accumulator restarts from zero
  auto flush = [&](const BwdDesc& D) {
    __syncthreads();
    float* prow = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      float acc[8];
      tmem_ld8(tbase + 8 * k, acc);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
        prow[prow_swz(dep_a(w, k, R, C))] = acc[i];
      }
    }
    __syncthreads();
    float* dst = partial + D.row_off + (int64_t)(blockIdx.x - D.c_lo) * D.L;
    for (int64_t p = tid; p < D.L; p += kThreads) {
      float v = 0.0f;
      for (int j = 0; j < (kB >> D.n); ++j) v += prow[prow_swz((int)((j << D.n) + p))];
      dst[p] = v;
    }
    zero_acc();
    __syncthreads();
  };

  if (tid == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(mbar_s));
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  uint32_t phase = 0;
  if (tid == 0 && i0 < i1) {
    const BwdDesc& D = G.d[desc_of(i0, 0)];
    const int64_t blk = D.first_block + (i0 - D.tile_prefix);
    if (bulk_ok(D, blk)) issue(D, blk);
  }
  Frags f;
  int cur = -1;
  for (int64_t i = i0; i < i1; ++i) {
    const int d = desc_of(i, cur < 0 ? 0 : cur);
    const BwdDesc& D = G.d[d];
    if (d != cur) {
      if (cur >= 0) flush(G.d[cur]);
      make_frags(f, g, t, D.n);
      cur = d;
    }
    const int n = D.n, layers = D.layers, Bm = (1 << n) - 1;
    const T* grad = reinterpret_cast<const T*>(D.grad);
    const int64_t blk = D.first_block + (i - D.tile_prefix);
    const int64_t bbase = blk * kB;
    const bool first_is_b = (layers != 2);
    uint16_t* land = first_is_b ? ybuf : xbuf;
    __syncthreads();
    for (int q = tid; q < (layers + 1) * kWords; q += kThreads) {
      int l = q / kWords, wd = q - l * kWords;
      const int p = 32 * wd;
      sw[l * kWordsPad + spad(wd)] =
          sign_word(block_layer_key(D.seed32, (blk << (kLog - n)) + (p >> n), l), (p & Bm) >> 5);
    }
    uint4 raw[8];
    float mx = 0.0f;
    const bool bulk = bulk_ok(D, blk);
    if (bulk) {
      uint32_t done = 0;
      for (int it = 0; it < (1 << 22) && !done; ++it) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(mbar_s), "r"(phase)
            : "memory");
      }
      if (!done) {
        abort_flag = 1;
        atomicExch(err, 1);
      }
      phase ^= 1u;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      int c = tid + kThreads * q;
      int64_t gi = bbase + 8 * c;
      if (bulk) {
        raw[q] = reinterpret_cast<const uint4*>(stage)[c];
      } else {
        uint32_t vv[4] = {0, 0, 0, 0};
        for (int e = 0; e < 8; ++e) {
          int64_t gg = gi + e;
          if (gg >= D.start && gg < D.stop)
            vv[e >> 1] |= (uint32_t)reinterpret_cast<const uint16_t*>(grad)[gg - D.start] << (16 * (e & 1));
        }
        raw[q] = make_uint4(vv[0], vv[1], vv[2], vv[3]);
      }
      const T* ev = reinterpret_cast<const T*>(&raw[q]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float v = Cvt<T>::to_f(ev[e]);
        mx = fmaxf(mx, fabsf(v));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    if (abort_flag) break;  // uniform: set before the barrier above
    if (tid == 0) {
      // the stage buffer is free again: fetch the next tile while this one runs
      if (i + 1 < i1) {
        const BwdDesc& N = G.d[desc_of(i + 1, d)];
        const int64_t nblk = N.first_block + (i + 1 - N.tile_prefix);
        if (bulk_ok(N, nblk)) {
          asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
          issue(N, nblk);
        }
      }
    }
    // every thread forms the prescale exponent from the warp sums (no second barrier)
    int k0 = 0;
    {
      float s2 = 0.0f;
      for (int q = 0; q < kThreads / 32; ++q) s2 = fmaxf(s2, red[q]);
      k0 = prescale_exponent(s2, n);
    }
    const float in_scale = ldexpf(1.0f, -k0);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      int c = tid + kThreads * q;
      const T* ev = reinterpret_cast<const T*>(&raw[q]);
      uint32_t hv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        hv[e] = pack_h2(Cvt<T>::to_f(ev[2 * e]) * in_scale, Cvt<T>::to_f(ev[2 * e + 1]) * in_scale);
      if (first_is_b) {
        *reinterpret_cast<uint4*>(land + lay_ab(8 * c)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) land[lay_ba(8 * c + e)] = (uint16_t)(hv[e >> 1] >> (16 * (e & 1)));
      }
    }
    __syncthreads();
    const float scale = ldexpf(1.0f, k0) * D.corr;
    if (layers == 1) {
      run<1, false, true>(f, yb, xb, sw + 1 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    } else if (layers == 2) {
      run<0, false, true>(f, xb, yb, sw + 2 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    } else {
      run<1, false, true>(f, yb, xb, sw + 3 * kWordsPad, nullptr, w, lane, g, t);
      __syncthreads();
      run<0, true, false>(f, xb, yb, nullptr, sw + 2 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
      __syncthreads();
      run_final_acc(f, xb, sw, scale, tbase, w, lane, g, t);
    }
  }
  if (abort_flag) {
    if (tid == 0) {
      // let an outstanding copy land before the CTA exits (bounded)
      uint32_t done = 0;
      for (int it = 0; it < (1 << 22) && !done; ++it) {
        asm volatile(
            "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(done)
            : "r"(mbar_s), "r"(phase ^ 1u)
            : "memory");
      }
    }
  } else if (cur >= 0) {
    flush(G.d[cur]);
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 256;\n" ::"r"(tmem_base_shared));
}

// Sum of each descriptor's partial rows (blockIdx.y = descriptor); a failed
// bulk-copy wait poisons every gradient of the group with NaN.
template <typename T>
__global__ void fht15_reduce_grouped_kernel(const __grid_constant__ BwdGroup G, const float* __restrict__ partial,
                                            const int* __restrict__ err) {
  const BwdDesc& D = G.d[blockIdx.y];
  const bool bad = *err != 0;
  const float* rows = partial + D.row_off;
  T* out = reinterpret_cast<T*>(D.out);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < D.L; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int r = 0;
    for (; r + 8 <= D.rows; r += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) acc[u] += rows[(int64_t)(r + u) * D.L + i];
    }
    for (; r < D.rows; ++r) acc[0] += rows[(int64_t)r * D.L + i];
    float s = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
    out[i] = Cvt<T>::from_f(bad ? __int_as_float(0x7fc00000) : s);
  }
}

// Host plan of one group: tiles, CTA ranges, partial-row layout.
inline int64_t cta_of_tile(int64_t i, int64_t total, int grid) {
  int64_t c = i * grid / total;
  while (c + 1 < grid && (c + 1) * total / grid <= i) ++c;
  while (c > 0 && c * total / grid > i) --c;
  return c;
}

inline size_t plan_backward_group(int count, const lwl_fht_backward_desc* q, BwdGroup& G) {
  G.count = count;
  int64_t prefix = 0;
  for (int i = 0; i < count; ++i) {
    BwdDesc& D = G.d[i];
    const int64_t first = q[i].start / kB, last = (q[i].stop + kB - 1) / kB;
    D.grad = q[i].grad_out;
    D.out = q[i].grad_latent;
    D.L = q[i].latent_size;
    D.start = q[i].start;
    D.stop = q[i].stop;
    D.first_block = first;
    D.nblocks = last > first ? last - first : 0;
    D.tile_prefix = prefix;
    prefix += D.nblocks;
    D.seed32 = fold_seed(q[i].seed);
    D.n = ilog2(next_pow2(q[i].latent_size));
    D.layers = q[i].layers;
    D.corr = (float)std::pow(layer_correction(D.n), D.layers);
  }
  G.total_tiles = prefix;
  const int sms = sm_count();
  G.grid = (int)(prefix < sms ? (prefix > 0 ? prefix : 1) : sms);
  int64_t off = 0;
  for (int i = 0; i < count; ++i) {
    BwdDesc& D = G.d[i];
    if (D.nblocks == 0) {
      D.c_lo = 0;
      D.rows = 0;
    } else {
      const int64_t lo = cta_of_tile(D.tile_prefix, prefix, G.grid);
      const int64_t hi = cta_of_tile(D.tile_prefix + D.nblocks - 1, prefix, G.grid);
      D.c_lo = (int)lo;
      D.rows = (int)(hi - lo + 1);
    }
    D.row_off = off;
    off += (int64_t)D.rows * D.L;
  }
  return kBwdHeader + size_t(off) * 4;
}

template <typename T>
int launch_backward_grouped_t(const BwdGroup& G, void* workspace, cudaStream_t st) {
  int* err = reinterpret_cast<int*>(workspace);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kBwdHeader);
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return -1;
  if (!set_max_smem((const void*)fht15_backward_grouped_kernel<T>, (int)kSmemBwd)) return -1;
  if (G.total_tiles > 0) {
    fht15_backward_grouped_kernel<T><<<G.grid, kThreads, kSmemBwd, st>>>(G, partial, err);
    if (cudaGetLastError() != cudaSuccess) return -1;
  }
  int64_t maxL = 1;
  for (int i = 0; i < G.count; ++i) maxL = G.d[i].L > maxL ? G.d[i].L : maxL;
  dim3 rgrid((unsigned)std::min<int64_t>((maxL + 255) / 256, 256), (unsigned)G.count);
  fht15_reduce_grouped_kernel<T><<<rgrid, 256, 0, st>>>(G, partial, err);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------
// Low pass of large blocks: one work item = one 2^15 tile (positions
// [j*2^15, (j+1)*2^15) of block b).  The planner's two-pass launch describes
// input (latent / gradient slice / fp32 workspace), signs and output (dtype
// slice / fp32 workspace); the transform is 1 or 2 applications of H_32768
// on the tile, exactly normalised on output (the high bits are done by the
// tile engine in fp32).

// fp32 staging of a whole tile in natural order (X and Y buffers, 128 KB);
// the XOR on bits 0-4 keeps both the scattered writer and the linear reader
// bank-conflict free.
__device__ __forceinline__ int lay_f32(int p) { return p ^ (((p >> 5) & 7) | (((p >> 9) & 3) << 3)); }

template <typename T>
__device__ __forceinline__ void lo_load8(const TileParams& p, int64_t b, int64_t pos0, float* v) {
  if (p.src_kind == SRC_WS) {
    const float* src = reinterpret_cast<const float*>(p.src) + (b - p.first_block) * p.B + pos0;
    float4 a = __ldg(reinterpret_cast<const float4*>(src));
    float4 c = __ldg(reinterpret_cast<const float4*>(src + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = c.x; v[5] = c.y; v[6] = c.z; v[7] = c.w;
    return;
  }
  const T* src = reinterpret_cast<const T*>(p.src);
  int64_t off;
  bool full;
  if (p.src_kind == SRC_LATENT) {
    off = pos0;
    full = pos0 + 8 <= p.L;
  } else {  // SRC_SLICE
    int64_t g0 = b * p.B + pos0;
    off = g0 - p.start;
    full = g0 >= p.start && g0 + 8 <= p.stop;
  }
  if (full && (((reinterpret_cast<uintptr_t>(src + off)) & 15) == 0)) {
    uint4 raw = __ldg(reinterpret_cast<const uint4*>(src + off));
    const T* ev = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = Cvt<T>::to_f(ev[e]);
  } else {
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      bool in;
      if (p.src_kind == SRC_LATENT) {
        in = pos0 + e < p.L;
      } else {
        int64_t g = b * p.B + pos0 + e;
        in = g >= p.start && g < p.stop;
      }
      v[e] = in ? Cvt<T>::to_f(src[off + e]) : 0.0f;
    }
  }
}

// L2 prefetch of the source of work item `tile` (the CTA's next one): its
// fp32 workspace tile or its part of the gradient slice (the latent is shared
// by all tiles and stays in L2).
template <typename T>
__device__ __forceinline__ void lo_prefetch_next(const TileParams& p, int64_t tile, int tpb) {
  const int64_t b = p.first_block + tile / tpb, pos0 = (tile % tpb) << kLog;
  if (p.src_kind == SRC_WS) {
    const int64_t e0 = (b - p.first_block) * p.B + pos0;
    prefetch_l2(p.src, e0 * 4, (e0 + kB) * 4);
  } else if (p.src_kind == SRC_SLICE) {
    const int64_t g0 = b * p.B + pos0 - p.start;
    const int64_t lo = g0 > 0 ? g0 : 0, hi = (g0 + kB < p.stop - p.start) ? g0 + kB : p.stop - p.start;
    if (hi > lo) prefetch_l2(p.src, lo * (int64_t)sizeof(T), hi * (int64_t)sizeof(T));
  }
}

constexpr size_t kSmemLo = 2 * kB * 2 + 4 * kWordsPad * 4;
constexpr size_t kSmemLo16 = kSmemLo + kB * 2;  // with the bulk-copy stage
static_assert(kSmemLo16 <= 232448, "shared memory per CTA");
static_assert(kSmemLo % 16 == 0, "bulk-copy stage alignment");

template <typename T>
__global__ void __launch_bounds__(kThreads, 1) fht_lo_kernel(const __grid_constant__ TileParams p, float corr1) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* xbuf = reinterpret_cast<uint16_t*>(smem);
  uint16_t* ybuf = xbuf + kB;
  uint32_t* sw = reinterpret_cast<uint32_t*>(ybuf + kB);  // [slot][kWordsPad]
  float* fstage = reinterpret_cast<float*>(smem);          // X+Y as 32768 fp32 (final fp32 output)
  __shared__ float red[kThreads / 32];

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  Frags f;
  make_frags(f, g, t, kLog);
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xbuf);
  const uint32_t yb = (uint32_t)__cvta_generic_to_shared(ybuf);
  const int tpb = (int)(p.B >> kLog);
  const int64_t ntiles = p.nblocks * tpb;
  const int nseg = p.lo_nseg;
  const int pre = p.pre_slot;
  const int post = p.lo_seg_slot[nseg - 1];
  const int mid = nseg == 2 ? p.lo_seg_slot[0] : -1;
  (void)corr1;  // the 2^-0.5 per application is folded into the exact 2^7 below

  // bf16 workspace source: each tile (64 KB, contiguous) arrives by one bulk
  // copy into `stage`, issued one tile ahead by thread 0; the waits are
  // bounded, and a wait that gives up turns every later tile of the CTA into
  // NaN (so the failure shows in the result) with no copy issued after it.
  const bool bulk = p.ws16 && p.src_kind == SRC_WS;
  uint16_t* stage16 = reinterpret_cast<uint16_t*>(smem + kSmemLo);
  __shared__ __align__(8) uint64_t lo_mbar;
  __shared__ int lo_abort;
  const uint32_t mbar_s = (uint32_t)__cvta_generic_to_shared(&lo_mbar);
  const uint32_t stage_s = (uint32_t)__cvta_generic_to_shared(stage16);
  auto issue = [&](int64_t tl) {
    const int64_t bb = p.first_block + tl / tpb;
    const __nv_bfloat16* src =
        reinterpret_cast<const __nv_bfloat16*>(p.src) + (bb - p.first_block) * p.B + ((tl % tpb) << kLog);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(mbar_s), "r"((uint32_t)(kB * 2)));
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(stage_s),
        "l"(src), "r"((uint32_t)(kB * 2)), "r"(mbar_s)
        : "memory");
  };
  if (tid == 0) {
    lo_abort = 0;
    if (bulk) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(mbar_s));
      asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    }
  }
  __syncthreads();
  // acc_rows: the CTA's tiles all share the tile index j = blockIdx.x mod tpb
  // (the grid is a multiple of tpb), so their final results are summed in
  // tensor memory, 128 lanes x 256 columns = the 32768 fp32 positions of tile
  // j, as in the 2^15 backward; one partial row segment per CTA at the end.
  // With 256 tiles per block (2^23) the grid is 128 and each CTA meets two
  // tile indices, j = blockIdx.x and blockIdx.x + 128: two 256-column slots.
  __shared__ uint32_t lo_tmem;
  uint32_t tacc = 0;
  const int slots = (p.acc_rows && tpb > (int)gridDim.x) ? 2 : 1;
  const uint32_t tcols = 256u * (uint32_t)slots;
  if (p.acc_rows) {
    if (w == 0) {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(
          (uint32_t)__cvta_generic_to_shared(&lo_tmem)), "r"(tcols));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n");
    tacc = lo_tmem + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(64 * (w >> 2));
    const float z8[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int s = 0; s < slots; ++s) {
#pragma unroll
      for (int k = 0; k < 8; ++k) tmem_st8(tacc + 256u * s + 8 * k, z8);
    }
    tmem_wait_st();
  }
  bool inflight = false;  // thread 0: a bulk copy was issued and not yet waited for
  uint32_t phase = 0;
  if (bulk && tid == 0 && blockIdx.x < ntiles) {
    issue(blockIdx.x);
    inflight = true;
  }

  for (int64_t tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
    const int64_t b = p.first_block + tile / tpb;
    const int j = (int)(tile % tpb);
    const int64_t tbase = (int64_t)j << kLog;  // first position of the tile in its block
    if (!bulk && tid == 0 && tile + gridDim.x < ntiles) lo_prefetch_next<T>(p, tile + gridDim.x, tpb);
    __syncthreads();
    for (int i = tid; i < p.nslots * kWords; i += kThreads) {
      int sl = i / kWords, wd = i - sl * kWords;
      sw[sl * kWordsPad + spad(wd)] = sign_word(block_layer_key(p.seed32, b, p.slot_layer[sl]), j * kWords + wd);
    }
    // the tile's 8 chunks of 8 per thread, all loads in flight at once, and
    // their largest magnitude; the values stay in registers for the landing
    float v[8][8];
    if (bulk) {
      uint32_t done = 0;
      if (!lo_abort) {
        for (int it = 0; it < (1 << 22) && !done; ++it) {
          asm volatile(
              "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}\n"
              : "=r"(done)
              : "r"(mbar_s), "r"(phase)
              : "memory");
        }
        if (!done) {
          lo_abort = 1;  // the copy of parity `phase` may still land: waited for at the end
        } else {
          if (tid == 0) inflight = false;
          phase ^= 1u;
        }
      }
      const float bad = __int_as_float(0x7fc00000);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint4 raw = reinterpret_cast<const uint4*>(stage16)[tid + kThreads * i];
        const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv[e]));
          v[i][2 * e] = done ? f2.x : bad;
          v[i][2 * e + 1] = done ? f2.y : bad;
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) lo_load8<T>(p, b, tbase + 8 * (tid + kThreads * i), v[i]);
    }
    float mx = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(v[i][e]));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    // the stage is consumed: fetch the CTA's next tile while this one runs
    if (bulk && tid == 0 && !lo_abort && tile + gridDim.x < ntiles) {
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      issue(tile + gridDim.x);
      inflight = true;
    }
    // every thread forms the prescale exponent from the warp maxima (same
    // order everywhere, so all agree; no second barrier).  red is rewritten
    // only after the next tile's loop-top barrier.
    int k0;
    {
      float s = 0.0f;
      for (int i = 0; i < kThreads / 32; ++i) s = fmaxf(s, red[i]);
      k0 = prescale_exponent(s, kLog);
    }
    const float in_scale = ldexpf(1.0f, -k0);
    uint16_t* land = nseg == 1 ? ybuf : xbuf;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = tid + kThreads * i;
      uint32_t hv[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) hv[e] = pack_h2(v[i][2 * e] * in_scale, v[i][2 * e + 1] * in_scale);
      if (nseg == 1) {
        *reinterpret_cast<uint4*>(land + lay_ab(8 * c)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) land[lay_ba(8 * c + e)] = (uint16_t)(hv[e >> 1] >> (16 * (e & 1)));
      }
    }
    __syncthreads();
    const uint32_t* pre_sw = pre >= 0 ? sw + pre * kWordsPad : nullptr;
    if (nseg == 1) {
      if (pre_sw) run<1, false, true>(f, yb, xb, pre_sw, nullptr, w, lane, g, t);
      else run<1, false, false>(f, yb, xb, nullptr, nullptr, w, lane, g, t);
    } else {
      if (pre_sw) run<0, false, true>(f, xb, yb, pre_sw, nullptr, w, lane, g, t);
      else run<0, false, false>(f, xb, yb, nullptr, nullptr, w, lane, g, t);
      __syncthreads();
      run<1, true, false>(f, yb, xb, nullptr, sw + mid * kWordsPad, w, lane, g, t);
    }
    __syncthreads();
    // The tile engine normalises once per layer (1/sqrt(B) with the sign that
    // ends the layer) and leaves the other part of the layer unnormalised, so
    // this pass outputs the unnormalised H_32768 result -- the fp16 internal
    // value times 2^(k0 + 7 per application), exactly -- times 1/sqrt(B) for
    // each application that ends a layer.
    float scale = ldexpf(1.0f, k0 + 7 * nseg);
    for (int sg = 0; sg < nseg; ++sg)
      if (p.lo_seg_slot[sg] >= 0) scale *= p.scale;
    if (p.acc_rows) {
      const uint32_t slot = (slots == 2 && j >= (int)gridDim.x) ? 256u : 0u;
      run_final_acc(f, xb, sw + post * kWordsPad, scale, tacc + slot, w, lane, g, t);
    } else if (p.dst_kind == DST_WS && p.ws16 && !p.ws_out32) {
      // bf16 workspace: the staged copy-out of the slice path, into the tile's
      // 64 KB of the workspace (tile index counted from the plan's first block)
      run_final<__nv_bfloat16>(f, xb, yb, ybuf, post >= 0 ? sw + post * kWordsPad : nullptr, scale,
                               reinterpret_cast<__nv_bfloat16*>(p.dst), (b - p.first_block) * tpb + j, 0,
                               p.nblocks * p.B, true, w, lane, g, t);
    } else if (p.dst_kind == DST_SLICE) {
      // the post sign is always present on the final launch of a forward
      run_final<T>(f, xb, yb, ybuf, sw + post * kWordsPad, scale, reinterpret_cast<T*>(p.dst), b * (p.B >> kLog) + j,
                   p.start, p.stop, ((p.start & 7) == 0) && ((reinterpret_cast<uintptr_t>(p.dst) & 15) == 0), w,
                   lane, g, t);
    } else {
      // fp32 workspace: inputs of all 8 tiles to registers, then the X/Y buffers become a natural-order fp32 stage
      uint32_t xin[8][4];
#pragma unroll
      for (int k = 0; k < 8; ++k) load_tile<0>(xb, w, k, lane, xin[k]);
      __syncthreads();
      const uint32_t* psw = post >= 0 ? sw + post * kWordsPad : nullptr;
      const int wb = dep_a(w, 0, g, 2 * t) >> 5;
      const uint32_t u0 = psw ? ~psw[spad(wb)] : 0u, u1 = psw ? ~psw[spad(wb + 64)] : 0u;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        uint32_t a[4];
        row_tf<0>(f, xin[k], a);
        float c[8];
        mma32(c, a[0], a[1], a[2], a[3], f.hc[0][0][0], f.hc[0][0][1]);
        mma32(c + 4, a[0], a[1], a[2], a[3], f.hc[0][1][0], f.hc[0][1][1]);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
          float v = c[i] * scale;
          if (psw) {
            const int bit = k + 8 * ((i >> 1) & 1) + 16 * (i & 1);
            const uint32_t u = (i >> 2) ? u1 : u0;
            v = __uint_as_float(__float_as_uint(v) ^ ((u << (31 - bit)) & 0x80000000u));
          }
          fstage[lay_f32(dep_a(w, k, R, C))] = v;
        }
      }
      __syncthreads();
      // lay_f32 XORs each aligned group of 4 positions with one mask, so a group
      // is one aligned 16-byte shared load, permuted back in registers
      float* dst = reinterpret_cast<float*>(p.dst) + (b - p.first_block) * p.B + tbase;
#pragma unroll 4
      for (int q = 4 * tid; q < kB; q += 4 * kThreads) {
        const int m = lay_f32(q) ^ q;  // the group's XOR mask
        const float4 a = *reinterpret_cast<const float4*>(fstage + (lay_f32(q) & ~3));
        // element i of the group sits in word i ^ m of the loaded 16 bytes
        const bool s0 = m & 1, s1 = m & 2;
        const float lo0 = s0 ? a.y : a.x, lo1 = s0 ? a.x : a.y, hi0 = s0 ? a.w : a.z, hi1 = s0 ? a.z : a.w;
        *reinterpret_cast<float4*>(dst + q) =
            s1 ? make_float4(hi0, hi1, lo0, lo1) : make_float4(lo0, lo1, hi0, hi1);
      }
    }
  }
  if (p.acc_rows) {
    // the CTA's sums of tile j in natural order through the exchange buffers,
    // then its segment [j 2^15, (j+1) 2^15) of partial row blockIdx.x / tpb
    // (two slots: segments blockIdx.x and blockIdx.x + 128 of row 0)
    float* prow = reinterpret_cast<float*>(smem);
    for (int s = 0; s < slots; ++s) {
      __syncthreads();
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        float acc[8];
        tmem_ld8(tacc + 256u * s + 8 * k, acc);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
          prow[prow_swz(dep_a(w, k, R, C))] = acc[i];
        }
      }
      __syncthreads();
      const int jj = slots == 2 ? (int)blockIdx.x + s * (int)gridDim.x : (int)blockIdx.x % tpb;
      const int64_t rix = slots == 2 ? 0 : blockIdx.x / tpb;
      float* row = p.partial + rix * p.L + ((int64_t)jj << kLog);
      const int64_t lim = p.L - ((int64_t)jj << kLog);  // positions of this segment inside [0, L)
      for (int q = tid; q < kB && q < lim; q += kThreads) row[q] = prow[prow_swz(q)];
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n");
    if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(lo_tmem), "r"(tcols));
  }
  if (bulk && tid == 0 && inflight) {
    // after a wait gave up: let the outstanding copy land before the CTA exits (bounded)
    uint32_t done = 0;
    for (int it = 0; it < (1 << 22) && !done; ++it) {
      asm volatile(
          "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n selp.u32 %0, 1, 0, q;\n}\n"
          : "=r"(done)
          : "r"(mbar_s), "r"(phase)
          : "memory");
    }
  }
}


}  // namespace fmma

bool mma_forward_supported(int dtype, int64_t latent_size, unsigned flags) {
  if (flags & LWL_FLAG_EXACT) return false;
  if (dtype != LWL_BF16 && dtype != LWL_F16) return false;
  // block sizes 2^5 .. 2^15; smaller blocks share a 2^15 tile
  const int64_t B = next_pow2(latent_size);
  return B >= 32 && B <= fmma::kB;
}

// Fill descriptor d of G for one generator call (tiles counted from G's running total).
static void add_forward_desc(fmma::FwdGroup& G, const void* latent, int64_t L, int layers, uint64_t seed,
                             int64_t start, int64_t stop, void* out) {
  const int64_t B = fmma::kB;
  int64_t first = start / B, last = (stop + B - 1) / B;
  fmma::FwdDesc& D = G.d[G.count++];
  D.latent = latent;
  D.out = out;
  D.L = L;
  D.start = start;
  D.stop = stop;
  D.first_tile = first;
  D.tile_prefix = G.total_tiles;
  D.seed32 = fold_seed(seed);
  D.n = ilog2(next_pow2(L));
  D.layers = layers;
  D.corr = (float)std::pow(fmma::layer_correction(D.n), layers);
  G.total_tiles += (last > first ? last - first : 0);
}

static int launch_group(int dtype, const fmma::FwdGroup& G, cudaStream_t st) {
  if (dtype == LWL_BF16) return fmma::launch_forward_t<__nv_bfloat16>(G, st);
  return fmma::launch_forward_t<__half>(G, st);
}

int mma_forward(int dtype, const void* latent, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                void* out, cudaStream_t st) {
  fmma::FwdGroup G;
  G.count = 0;
  G.total_tiles = 0;
  add_forward_desc(G, latent, L, layers, seed, start, stop, out);
  return launch_group(dtype, G, st);
}

int mma_forward_grouped(int dtype, int count, const lwl_fht_forward_desc* descs, cudaStream_t st) {
  fmma::FwdGroup G;
  G.count = 0;
  G.total_tiles = 0;
  for (int i = 0; i < count; ++i) {
    const lwl_fht_forward_desc& q = descs[i];
    if (q.stop <= q.start) continue;
    add_forward_desc(G, q.latent, q.latent_size, q.layers, q.seed, q.start, q.stop, q.out);
    if (G.count == fmma::kMaxGroup) {
      if (launch_group(dtype, G, st) != 0) return -1;
      G.count = 0;
      G.total_tiles = 0;
    }
  }
  return G.count ? launch_group(dtype, G, st) : 0;
}

}  // namespace lwl

namespace lwl {

bool mma16_forward_supported(int dtype, int64_t latent_size, unsigned flags) {
  if (flags & LWL_FLAG_EXACT) return false;
  if (dtype != LWL_BF16 && dtype != LWL_F16) return false;
  const int64_t P = next_pow2(latent_size);
  return P == 2 * fmma::kB || P == 4 * fmma::kB;
}

int mma16_forward(int dtype, const void* latent, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                  void* out, cudaStream_t st) {
  if (next_pow2(L) == 4 * fmma::kB) {
    if (dtype == LWL_BF16)
      return fmma::launch_forward_parked<__nv_bfloat16, 4>(latent, L, layers, seed, start, stop, out, st);
    return fmma::launch_forward_parked<__half, 4>(latent, L, layers, seed, start, stop, out, st);
  }
  if (dtype == LWL_BF16)
    return fmma::launch_forward16_t<__nv_bfloat16>(latent, L, layers, seed, start, stop, out, st);
  return fmma::launch_forward16_t<__half>(latent, L, layers, seed, start, stop, out, st);
}

bool mma16_backward_supported(int dtype, int64_t latent_size, unsigned flags) {
  return mma16_forward_supported(dtype, latent_size, flags);
}

size_t mma16_backward_workspace_bytes(int64_t latent_size, int64_t start, int64_t stop) {
  const int64_t B = next_pow2(latent_size);
  const int64_t nb = (stop + B - 1) / B - start / B;
  if (nb <= 0) return 0;
  const int64_t grid = nb < fmma::sm_count() ? nb : fmma::sm_count();
  return fmma::kBwdHeader + size_t(grid) * size_t(latent_size) * 4;
}

int mma16_backward(int dtype, const void* grad, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                   void* grad_latent, void* workspace, cudaStream_t st) {
  if (next_pow2(L) == 4 * fmma::kB) {
    if (dtype == LWL_BF16)
      return fmma::launch_backward_parked<__nv_bfloat16, 4>(grad, L, layers, seed, start, stop, grad_latent, workspace, st);
    return fmma::launch_backward_parked<__half, 4>(grad, L, layers, seed, start, stop, grad_latent, workspace, st);
  }
  if (dtype == LWL_BF16)
    return fmma::launch_backward16_t<__nv_bfloat16>(grad, L, layers, seed, start, stop, grad_latent, workspace, st);
  return fmma::launch_backward16_t<__half>(grad, L, layers, seed, start, stop, grad_latent, workspace, st);
}

bool mma_backward_supported(int dtype, int64_t latent_size, unsigned flags) {
  return mma_forward_supported(dtype, latent_size, flags);
}

size_t mma_backward_workspace_bytes(int64_t latent_size, int64_t start, int64_t stop) {
  const int64_t B = fmma::kB;
  int64_t nblk = (stop + B - 1) / B - start / B;
  if (nblk <= 0) return 0;
  int64_t grid = nblk < fmma::sm_count() ? nblk : fmma::sm_count();
  return fmma::kBwdHeader + size_t(grid) * size_t(latent_size) * 4;
}

int mma_backward(int dtype, const void* grad, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                 void* grad_latent, void* workspace, cudaStream_t st, int test_stall) {
  const int64_t B = fmma::kB;
  int64_t first = start / B, last = (stop + B - 1) / B;
  if (last <= first) {
    return cudaMemsetAsync(grad_latent, 0, size_t(L) * 2, st) == cudaSuccess ? 0 : -1;
  }
  uint32_t s32 = fold_seed(seed);
  if (dtype == LWL_BF16)
    return fmma::launch_backward_t<__nv_bfloat16>(grad, L, layers, ilog2(next_pow2(L)), s32, first, last - first, start, stop, grad_latent,
                                                  workspace, st, test_stall);
  return fmma::launch_backward_t<__half>(grad, L, layers, ilog2(next_pow2(L)), s32, first, last - first, start, stop, grad_latent,
                                         workspace, st, test_stall);
}

size_t mma_backward_grouped_workspace_bytes(int count, const lwl_fht_backward_desc* descs) {
  size_t need = 0;
  for (int g0 = 0; g0 < count; g0 += fmma::kMaxGroup) {
    fmma::BwdGroup G;
    const int c = count - g0 < fmma::kMaxGroup ? count - g0 : fmma::kMaxGroup;
    size_t b = fmma::plan_backward_group(c, descs + g0, G);
    need = b > need ? b : need;  // the groups run one after another on one stream
  }
  return need;
}

int mma_backward_grouped(int dtype, int count, const lwl_fht_backward_desc* descs, void* workspace,
                         cudaStream_t st) {
  for (int g0 = 0; g0 < count; g0 += fmma::kMaxGroup) {
    fmma::BwdGroup G;
    const int c = count - g0 < fmma::kMaxGroup ? count - g0 : fmma::kMaxGroup;
    fmma::plan_backward_group(c, descs + g0, G);
    int rc = dtype == LWL_BF16 ? fmma::launch_backward_grouped_t<__nv_bfloat16>(G, workspace, st)
                               : fmma::launch_backward_grouped_t<__half>(G, workspace, st);
    if (rc) return rc;
  }
  return 0;
}

}  // namespace lwl

namespace lwl {

bool mma_lo_supported(int dtype, int n, unsigned flags) {
  if (flags & LWL_FLAG_EXACT) return false;
  if (dtype != LWL_BF16 && dtype != LWL_F16) return false;
  return n > fmma::kLog && n <= fmma::kLog + 8;
}

int mma_lo_grid(const TileParams& p) {
  const int64_t tpb = p.B >> fmma::kLog, ntiles = p.nblocks * tpb;
  const int sms = fmma::sm_count();
  if (p.acc_rows) {  // a multiple of the tiles per block (ntiles is one), or half of them at 2^23
    if (tpb > sms) return (int)(tpb / 2);
    const int64_t g = ntiles < sms ? ntiles : (sms / tpb) * tpb;
    return (int)g;
  }
  return (int)(ntiles < sms ? ntiles : sms);
}

int mma_lo_launch(int dtype, const TileParams& p, int grid, cudaStream_t st) {
  const float corr1 = (float)fmma::layer_correction(fmma::kLog);
  // + the bulk-copy stage when the bf16 workspace is the source
  const size_t smem = fmma::kSmemLo + ((p.ws16 && p.src_kind == SRC_WS) ? size_t(fmma::kB) * 2 : 0);
  if (dtype == LWL_BF16) {
    if (!set_max_smem((const void*)fmma::fht_lo_kernel<__nv_bfloat16>, (int)fmma::kSmemLo16)) return -1;
    fmma::fht_lo_kernel<__nv_bfloat16><<<grid, fmma::kThreads, smem, st>>>(p, corr1);
  } else {
    if (!set_max_smem((const void*)fmma::fht_lo_kernel<__half>, (int)fmma::kSmemLo16)) return -1;
    fmma::fht_lo_kernel<__half><<<grid, fmma::kThreads, smem, st>>>(p, corr1);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
