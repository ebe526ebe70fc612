// fht_mma_core.cuh -- device building blocks of the tensor-core BlockFHT kernels
// (bit layouts, exchange layouts, mma/ldmatrix/movmatrix wrappers, sign
// application, run structure).  Included by fht_mma.cu and linear_tc.cu.
#pragma once
#include <cmath>
#include <cstdio>

#include "fht_mma.h"
#include "lwl_common.cuh"

namespace lwl {
namespace fmma {

constexpr int kLog = 15;
constexpr int kB = 1 << kLog;
constexpr int kThreads = 512;
constexpr int kWords = kB / 32;
// Sign words of one layer live at stride kWordsPad, word w at w + (w >> 7):
// the padding spreads the words that the lanes of pass B read (128 apart)
// over different banks.
constexpr int kWordsPad = kWords + kWords / 128 + 8;
__device__ __forceinline__ int spad(int w) { return w + (w >> 7); }

// One generator of a grouped forward launch (passed by value as a kernel parameter).
struct FwdDesc {
  const void* latent;
  void* out;
  int64_t L, start, stop;
  int64_t first_tile;   // first 2^15-coordinate tile touched by [start, stop)
  int64_t tile_prefix;  // work items of the descriptors before this one
  uint32_t seed32;
  int n, layers;
  float corr;  // exact-power-of-two factor scales -> 2^(-n/2) per layer
};
constexpr int kMaxGroup = 96;
struct FwdGroup {
  int count;
  int64_t total_tiles;
  FwdDesc d[kMaxGroup];
};

// position of element (warp w, tile k, tile row R, tile col C) in each pass
__device__ __forceinline__ int dep_a(int w, int k, int R, int C) {
  return k | ((R >> 3) & 1) << 3 | (C & 1) << 4 | (R & 7) << 5 | (w & 1) << 8 | ((C >> 1) & 3) << 9 |
         ((C >> 3) & 1) << 11 | (w >> 1) << 12;
}
__device__ __forceinline__ int dep_b(int w, int k, int R, int C) {
  return (R & 7) | (w & 1) << 3 | (C & 1) << 4 | k << 5 | ((R >> 3) & 1) << 8 | (w >> 1) << 9 | (C >> 1) << 12;
}
// shared-memory element offset of position p in the two exchange layouts
__device__ __forceinline__ int lay_ab(int p) {  // 8-element chunks along bits 0-2
  int c = p >> 3;
  int s = (((p >> 9) ^ (p >> 12)) & 1) | ((p >> 10) & 1) << 1 | ((p >> 13) & 1) << 2;
  return ((c ^ s) << 3) | (p & 7);
}
__device__ __forceinline__ int lay_ba(int p) {  // 8-element chunks along bits 5-7
  int c = (p & 31) | ((p >> 8) << 5);
  int s = ((p >> 4) & 1) | (((p >> 9) ^ (p >> 12)) & 1) << 1 | (((p >> 10) ^ (p >> 13)) & 1) << 2;
  return ((c ^ s) << 3) | ((p >> 5) & 7);
}

template <int PASS> struct Pass;
template <> struct Pass<0> {  // A: reads the B->A layout, writes the A->B layout
  static __device__ __forceinline__ int dep(int w, int k, int R, int C) { return dep_a(w, k, R, C); }
  static __device__ __forceinline__ int lay_in(int p) { return lay_ba(p); }
  static __device__ __forceinline__ int lay_out(int p) { return lay_ab(p); }
};
template <> struct Pass<1> {  // B
  static __device__ __forceinline__ int dep(int w, int k, int R, int C) { return dep_b(w, k, R, C); }
  static __device__ __forceinline__ int lay_in(int p) { return lay_ab(p); }
  static __device__ __forceinline__ int lay_out(int p) { return lay_ba(p); }
};

__device__ __forceinline__ void ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ uint32_t movt(uint32_t a) {
  uint32_t d;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;\n" : "=r"(d) : "r"(a));
  return d;
}
// Register-only operations are plain (non-volatile) asm so the compiler can
// interleave the independent tiles a warp owns.
// D(16x8, f16) = A(16x16, f16) * B(16x8, f16)
__device__ __forceinline__ void mma16(uint32_t& d0, uint32_t& d1, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                      uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 {%0,%1}, {%2,%3,%4,%5}, {%6,%7}, {%8,%8};\n"
      : "=r"(d0), "=r"(d1)
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0u));
}
// D(16x8, f32) = A * B
__device__ __forceinline__ void mma32(float* d, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                      uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%10,%10,%10};\n"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(0.0f));
}
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t d;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
  return d;
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
__device__ __forceinline__ int hsign(int i, int j) { return (__popc(i & j) & 1) ? -1 : 1; }

// Power-of-two prescale exponent k0 for an fp16 transform of 2^nbits-element
// blocks whose largest magnitude is `maxabs`.  After scaling by 2^-k0 the
// largest element is below 2^(12 - ceil(nbits/2)), so a block's L2 norm --
// which bounds every element of every orthonormal partial transform of it --
// stays below 2^12, far inside fp16.  Taken from the maximum rather than a
// sum of squares, the exponent is exact for every finite input: a float sum
// of squares overflows above |v| ~ 1.8e19 and flushes to zero below
// ~1e-19, both of which are legal bf16 values.  k0 is clamped to +-120 so
// that 2^-k0 and 2^k0 stay normal floats; blocks beyond that (all elements
// below 2^-108 or an infinity) keep the nearest representable scale.
__device__ __forceinline__ int prescale_exponent(float maxabs, int nbits) {
  if (!(maxabs > 0.0f) || isinf(maxabs)) return 0;
  int e = 0;
  frexpf(maxabs, &e);  // maxabs < 2^e
  const int k0 = e - (12 - ((nbits + 1) >> 1));
  return k0 < -120 ? -120 : (k0 > 120 ? 120 : k0);
}

template <typename T> __device__ __forceinline__ uint32_t pack_out(float lo, float hi);
template <> __device__ __forceinline__ uint32_t pack_out<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
template <> __device__ __forceinline__ uint32_t pack_out<__half>(float lo, float hi) { return pack_h2(lo, hi); }

// Tile axes and the position bits they carry (bit 0 first):
//   pass A rows {5,6,7,3}, pass A cols {4,9,10,11},
//   pass B rows {0,1,2,8}, pass B cols {4,12,13,14} (col bit 0 = position 4 is
//   an identity in pass B: pass A transforms it).
// For block size 2^n a 2^15 tile holds 2^(15-n) consecutive blocks and the
// position bits >= n select the block, so their factor is the identity.  An
// axis with m transformed bits applies (tensor product of H2 / I2) scaled by
// 2^-floor(m/2), which is exact in fp16 and grows norms by at most sqrt(2).
__host__ __device__ inline int axis_mask(int axis, int n) {
  const int pos[4][4] = {{5, 6, 7, 3}, {4, 9, 10, 11}, {0, 1, 2, 8}, {4, 12, 13, 14}};
  int m = 0;
  for (int b = 0; b < 4; ++b)
    if (pos[axis][b] < n && !(axis == 3 && b == 0)) m |= 1 << b;
  return m;
}
__host__ __device__ inline int popc4(int m) { return (m & 1) + ((m >> 1) & 1) + ((m >> 2) & 1) + ((m >> 3) & 1); }
__device__ __forceinline__ float axis_val(int i, int j, int mask) {
  float v = ldexpf(1.0f, -(popc4(mask) >> 1));
#pragma unroll
  for (int b = 0; b < 4; ++b) {
    int ib = (i >> b) & 1, jb = (j >> b) & 1;
    if ((mask >> b) & 1) {
      if (ib & jb) v = -v;
    } else if (ib != jb) {
      v = 0.0f;
    }
  }
  return v;
}

struct Frags {
  uint32_t hA[2][4];    // per pass: row-axis matrix as the A operand (row transform H*X)
  uint32_t hc[2][2][2]; // per pass: column-axis matrix as the B operand, per 8-column half
};

__device__ __forceinline__ void make_frags(Frags& f, int g, int t, int n) {
#pragma unroll
  for (int ps = 0; ps < 2; ++ps) {
    const int rm = axis_mask(ps == 0 ? 0 : 2, n), cm = axis_mask(ps == 0 ? 1 : 3, n);
    f.hA[ps][0] = pack_h2(axis_val(g, 2 * t, rm), axis_val(g, 2 * t + 1, rm));
    f.hA[ps][1] = pack_h2(axis_val(g + 8, 2 * t, rm), axis_val(g + 8, 2 * t + 1, rm));
    f.hA[ps][2] = pack_h2(axis_val(g, 2 * t + 8, rm), axis_val(g, 2 * t + 9, rm));
    f.hA[ps][3] = pack_h2(axis_val(g + 8, 2 * t + 8, rm), axis_val(g + 8, 2 * t + 9, rm));
#pragma unroll
    for (int nh = 0; nh < 2; ++nh) {
      int c = g + 8 * nh;
      f.hc[ps][nh][0] = pack_h2(axis_val(2 * t, c, cm), axis_val(2 * t + 1, c, cm));
      f.hc[ps][nh][1] = pack_h2(axis_val(2 * t + 8, c, cm), axis_val(2 * t + 9, c, cm));
    }
  }
}

// Product over the 2^n transform of the exact power-of-two axis scales,
// relative to the required 2^(-n/2) per layer.
inline double layer_correction(int n) {
  int applied = 0;
  for (int a = 0; a < 4; ++a) applied += popc4(axis_mask(a, n)) >> 1;
  return std::pow(2.0, applied - 0.5 * n);
}

// Row transform (H*X): X as B-operand fragments {x0,x1} (cols 0-7), {x2,x3}
// (cols 8-15); result in accumulator (= A operand) layout.
template <int PASS>
__device__ __forceinline__ void row_tf(const Frags& f, const uint32_t* x, uint32_t* a) {
  const uint32_t* h = f.hA[PASS];
  mma16(a[0], a[1], h[0], h[1], h[2], h[3], x[0], x[1]);
  mma16(a[2], a[3], h[0], h[1], h[2], h[3], x[2], x[3]);
}
// Column transform (X*Hc): A layout -> A layout.
template <int PASS>
__device__ __forceinline__ void col_tf(const Frags& f, uint32_t* a) {
  const uint32_t(*h)[2] = f.hc[PASS];
  uint32_t d0, d1, d2, d3;
  mma16(d0, d1, a[0], a[1], a[2], a[3], h[0][0], h[0][1]);
  mma16(d2, d3, a[0], a[1], a[2], a[3], h[1][0], h[1][1]);
  a[0] = d0;
  a[1] = d1;
  a[2] = d2;
  a[3] = d3;
}
// A layout -> B-operand layout of the same tile (8x8 transposes)
__device__ __forceinline__ void to_bop(const uint32_t* a, uint32_t* x) {
  x[0] = movt(a[0]);
  x[1] = movt(a[1]);
  x[2] = movt(a[2]);
  x[3] = movt(a[3]);
}

// XOR the signs of one layer into accumulator-layout registers of tile k.
// Register j holds (R = g + 8(j&1), C = 2t + 8(j>>1) + {0,1}); the pair sits
// at positions p and p+16 (C bit 0 is position bit 4), so one shifted copy of
// the inverted sign word gives both sign bits (bit 15 and bit 31).
//   pass A: p = base + k + 8(j&1) + 2048(j>>1), base bits 0-4 clear
//   pass B: p = base + 32k + 256(j&1) + 16384(j>>1), p & 15 = base & 15
template <int PASS>
__device__ __forceinline__ void sign_acc(uint32_t* a, const uint32_t* sw, int w, int k, int g, int t) {
  const int base = Pass<PASS>::dep(w, 0, g, 2 * t);
  const int wb = base >> 5;
  if (PASS == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t u = ~sw[spad(wb + 64 * (j >> 1))];
      a[j] ^= (u << (15 - k - 8 * (j & 1))) & 0x80008000u;
    }
  } else {
    const int sh = 15 - (base & 15);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t u = ~sw[spad(wb + k + 8 * (j & 1) + 512 * (j >> 1))];
      a[j] ^= (u << sh) & 0x80008000u;
    }
  }
}

// Signs applied to B-operand fragments (first run): register m holds
// (R = 2t + 8(m&1) + {0,1}, C = g + 8(m>>1)).  In pass B the pair is two
// neighbouring positions (p, p+1) of one word; the multiply moves bit 0 to
// bit 15 and bit 1 to bit 31 (no carries: the two partial products do not overlap).
template <int PASS>
__device__ __forceinline__ void sign_bop(uint32_t* x, const uint32_t* sw, int w, int k, int g, int t) {
  if (PASS == 1) {
    const int base = dep_b(w, 0, 2 * t, g);
    const int wb = base >> 5, q = base & 31;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      uint32_t u = ~sw[spad(wb + k + 8 * (m & 1) + 512 * (m >> 1))];
      x[m] ^= (((u >> q) & 3u) * 0x40008000u) & 0x80008000u;
    }
  } else {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      int R = 2 * t + 8 * (m & 1), C = g + 8 * (m >> 1);
      int p0 = dep_a(w, k, R, C);
      int p1 = dep_a(w, k, R + 1, C);
      uint32_t b0 = (sw[spad(p0 >> 5)] >> (p0 & 31)) & 1u;
      uint32_t b1 = (sw[spad(p1 >> 5)] >> (p1 & 31)) & 1u;
      x[m] ^= ((b0 ^ 1u) << 15) | ((b1 ^ 1u) << 31);
    }
  }
}

// Gather the thread's 8 tiles into 16-byte chunks in the next pass's layout.
template <int PASS>
__device__ __forceinline__ void write_exchange(uint32_t (*d)[4], uint32_t base, int w, int g, int t) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = h ? 0x7632u : 0x5410u;
      // dep and lay_out are XOR-linear over disjoint bit fields: the thread's
      // offset (formed once per run) XOR a compile-time constant per (j, h)
      const int off = Pass<PASS>::lay_out(Pass<PASS>::dep(w, 0, g, 2 * t)) ^
                      Pass<PASS>::lay_out(Pass<PASS>::dep(0, 0, 8 * (j & 1), h + 8 * (j >> 1)));
      uint32_t addr = base + 2u * (uint32_t)off;
      uint32_t v0 = prmt(d[0][j], d[1][j], sel), v1 = prmt(d[2][j], d[3][j], sel);
      uint32_t v2 = prmt(d[4][j], d[5][j], sel), v3 = prmt(d[6][j], d[7][j], sel);
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(v0), "r"(v1), "r"(v2), "r"(v3));
    }
  }
}

template <int PASS>
__device__ __forceinline__ void load_tile(uint32_t base, int w, int k, int lane, uint32_t* x) {
  int mm = lane >> 3, rr = lane & 7;
  // the thread's offset XOR a compile-time constant per sub-tile k (see write_exchange)
  const int off = Pass<PASS>::lay_in(Pass<PASS>::dep(w, 0, 8 * (mm & 1), rr + 8 * (mm >> 1))) ^
                  Pass<PASS>::lay_in(Pass<PASS>::dep(0, k, 0, 0));
  ldsm4(base + 2u * (uint32_t)off, x[0], x[1], x[2], x[3]);
}

// One run of pass PASS: read the input buffer, row + col transforms (and for
// DOUBLE runs sign + col + row of the next layer), write the output buffer.
template <int PASS, bool DOUBLE, bool PRESIGN>
__device__ __forceinline__ void run(const Frags& f, uint32_t in_base, uint32_t out_base, const uint32_t* pre_sw,
                                    const uint32_t* mid_sw, int w, int lane, int g, int t) {
  uint32_t d[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t x[4];
    load_tile<PASS>(in_base, w, k, lane, x);
    if (PRESIGN) sign_bop<PASS>(x, pre_sw, w, k, g, t);
    row_tf<PASS>(f, x, d[k]);
    col_tf<PASS>(f, d[k]);
    if (DOUBLE) {
      sign_acc<PASS>(d[k], mid_sw, w, k, g, t);
      col_tf<PASS>(f, d[k]);
      uint32_t y[4];
      to_bop(d[k], y);
      row_tf<PASS>(f, y, d[k]);
    }
  }
  write_exchange<PASS>(d, out_base, w, g, t);
}

// ---- the first run's input fragments kept in tensor memory --------------------
// Every tile of a forward descriptor starts from the same scaled latent copy,
// so each warp loads its 8 first-run B-operand fragments (32 registers) once
// per descriptor into its tensor-memory lanes (quadrant w % 4, 32 columns at
// 32 * (w / 4)) and each tile's first run reads them with one tcgen05.ld
// instead of eight ldmatrix from shared memory.
template <int PASS>
__device__ __forceinline__ void park_first_input(uint32_t in_base, uint32_t taddr, int w, int lane) {
  uint32_t x[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) load_tile<PASS>(in_base, w, k, lane, x[k]);
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(x[0][0]), "r"(x[0][1]), "r"(x[0][2]), "r"(x[0][3]), "r"(x[1][0]), "r"(x[1][1]), "r"(x[1][2]), "r"(x[1][3]),
      "r"(x[2][0]), "r"(x[2][1]), "r"(x[2][2]), "r"(x[2][3]), "r"(x[3][0]), "r"(x[3][1]), "r"(x[3][2]), "r"(x[3][3]),
      "r"(x[4][0]), "r"(x[4][1]), "r"(x[4][2]), "r"(x[4][3]), "r"(x[5][0]), "r"(x[5][1]), "r"(x[5][2]), "r"(x[5][3]),
      "r"(x[6][0]), "r"(x[6][1]), "r"(x[6][2]), "r"(x[6][3]), "r"(x[7][0]), "r"(x[7][1]), "r"(x[7][2]), "r"(x[7][3])
      : "memory");
  asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}

// First run (single pass, signs before the transform) with its input from tensor memory.
template <int PASS>
__device__ __forceinline__ void run_first_tmem(const Frags& f, uint32_t taddr, uint32_t out_base,
                                               const uint32_t* pre_sw, int w, int lane, int g, int t) {
  uint32_t d[8][4];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(d[0][0]), "=r"(d[0][1]), "=r"(d[0][2]), "=r"(d[0][3]), "=r"(d[1][0]), "=r"(d[1][1]), "=r"(d[1][2]),
        "=r"(d[1][3]), "=r"(d[2][0]), "=r"(d[2][1]), "=r"(d[2][2]), "=r"(d[2][3]), "=r"(d[3][0]), "=r"(d[3][1]),
        "=r"(d[3][2]), "=r"(d[3][3]), "=r"(d[4][0]), "=r"(d[4][1]), "=r"(d[4][2]), "=r"(d[4][3]), "=r"(d[5][0]),
        "=r"(d[5][1]), "=r"(d[5][2]), "=r"(d[5][3]), "=r"(d[6][0]), "=r"(d[6][1]), "=r"(d[6][2]), "=r"(d[6][3]),
        "=r"(d[7][0]), "=r"(d[7][1]), "=r"(d[7][2]), "=r"(d[7][3])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    uint32_t x[4] = {d[k][0], d[k][1], d[k][2], d[k][3]};
    sign_bop<PASS>(x, pre_sw, w, k, g, t);
    row_tf<PASS>(f, x, d[k]);
    col_tf<PASS>(f, d[k]);
  }
  write_exchange<PASS>(d, out_base, w, g, t);
}

// Natural-order staging layout for the output: chunk c = p >> 3 of 8
// consecutive positions, XOR-swizzled so both the gathering writer (varies
// chunk bits 2,6,7 within a phase) and the linear copy-out reader (bits 0-2)
// are bank-conflict free.
__device__ __forceinline__ int lay_nat_chunk(int c) { return c ^ ((c >> 6) & 3); }

// Last row transform + column transform of pass A accumulated in fp32 for
// tile k; f[0..3] / f[4..7] = column halves 0 / 1 in accumulator layout.
__device__ __forceinline__ void final_tile(const Frags& f, uint32_t in_base, int w, int k, int lane, float* c) {
  uint32_t x[4], a[4];
  load_tile<0>(in_base, w, k, lane, x);
  row_tf<0>(f, x, a);
  mma32(c, a[0], a[1], a[2], a[3], f.hc[0][0][0], f.hc[0][0][1]);
  mma32(c + 4, a[0], a[1], a[2], a[3], f.hc[0][1][0], f.hc[0][1][1]);
}

// Final run (pass A): transforms, rescale, round to the output dtype, last
// sign, then stage the block in natural order in shared memory and copy it
// out with full 16-byte-per-lane contiguous stores.
template <typename T>
__device__ __forceinline__ void run_final(const Frags& f, uint32_t in_base, uint32_t stage_base,
                                          const uint16_t* stage, const uint32_t* sw, float scale, T* out,
                                          int64_t blk, int64_t start, int64_t stop, bool vec_ok, int w, int lane,
                                          int g, int t) {
  uint32_t o[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float c[8];
    final_tile(f, in_base, w, k, lane, c);
    o[k][0] = pack_out<T>(c[0] * scale, c[1] * scale);
    o[k][1] = pack_out<T>(c[2] * scale, c[3] * scale);
    o[k][2] = pack_out<T>(c[4] * scale, c[5] * scale);
    o[k][3] = pack_out<T>(c[6] * scale, c[7] * scale);
    if (sw) sign_acc<0>(o[k], sw, w, k, g, t);  // sw == nullptr: no sign layer here
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = h ? 0x7632u : 0x5410u;
      // XOR-linear as in write_exchange; positions 8-aligned after >> 3 on both parts
      const int cidx = lay_nat_chunk(dep_a(w, 0, g, 2 * t) >> 3) ^
                       lay_nat_chunk(dep_a(0, 0, 8 * (j & 1), h + 8 * (j >> 1)) >> 3);
      uint32_t addr = stage_base + 16u * (uint32_t)cidx;
      uint32_t v0 = prmt(o[0][j], o[1][j], sel), v1 = prmt(o[2][j], o[3][j], sel);
      uint32_t v2 = prmt(o[4][j], o[5][j], sel), v3 = prmt(o[6][j], o[7][j], sel);
      asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"r"(addr), "r"(v0), "r"(v1), "r"(v2), "r"(v3));
    }
  }
  __syncthreads();
  const int64_t bbase = blk * kB;
  const uint4* st4 = reinterpret_cast<const uint4*>(stage);
  for (int c = threadIdx.x; c < kB / 8; c += kThreads) {
    uint4 v = st4[lay_nat_chunk(c)];
    int64_t gi = bbase + 8 * c;
    if (vec_ok && gi >= start && gi + 8 <= stop) {
      *reinterpret_cast<uint4*>(out + (gi - start)) = v;
    } else {
      uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int64_t gg = gi + e;
        if (gg >= start && gg < stop)
          reinterpret_cast<uint16_t*>(out)[gg - start] = (uint16_t)(vv[e >> 1] >> (16 * (e & 1)));
      }
    }
  }
}


inline int sm_count() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

}  // namespace fmma
}  // namespace lwl
