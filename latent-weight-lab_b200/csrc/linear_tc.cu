// linear_tc.cu -- BlockFHTLinear forward on tcgen05 with the weight generated on chip.
//
// y[T, N] = x[T, K] * (scale * W)^T, W = the BlockFHT generator's first N*K
// coordinates viewed as [N, K] (latent_weight_lab/block_fht.py:283-287, 306-311).
//
// One work item = a panel of 128 weight rows [n0, n0+128) x a range of
// 128-token tiles.  Per item the CTA
//   1. generates the 2^15-coordinate generator tiles that cover the panel with
//      the tensor-core FHT runs (fht_mma_core.cuh), stages each tile's part of
//      the panel in shared memory with a padded row pitch, and stores it into
//      tensor memory as the MMA A operand (128 lanes = weight rows, two bf16 per
//      32-bit column along K);
//   2. streams x tiles [128 tokens x 64] by TMA (128-byte swizzle, 8-stage
//      mbarrier ring over the latent copy and first exchange buffer, which the
//      next item rebuilds; no multicast) and issues tcgen05.mma (M=128 weight
//      rows, N=128 tokens, K=16) from one warp -- one elected lane issues,
//      the converged warp waits -- into tensor-memory accumulators;
//   3. drains an accumulator with eight epilogue warps (lane quadrant w % 4,
//      column half) into registers, releases it, and stages the bf16 output
//      tile in shared memory for a TMA store.
// The generated weight never leaves the SM.  Tensor memory: A uses K/2
// columns (K <= 768); two 128-column accumulators follow when K <= 512 (the
// next tile's MMAs overlap the previous drain), else one.
//
// The dense variant (GEN = false) loads a given bf16 W panel instead of
// generating it; it runs the same MMA pipeline and is used to validate it.
#include <cuda.h>

#include <cstring>
#include <mutex>

#include "fht_mma_core.cuh"
#include "tc_ptx.cuh"

namespace lwl {
namespace fmma {

constexpr int kLinThreads = 512;
constexpr int kStages = 8;
constexpr int kTT = 128;                    // tokens per MMA tile (N of the MMA)
constexpr int kStageBytes = kTT * 64 * 2;   // 128 tokens x 64 K bf16
constexpr int kYStageBytes = kTT * 128 * 2; // one output tile [128 tokens x 128 features] bf16
constexpr int kMaxK = 768;
constexpr int kEpiWarps = 8;                // warps 4..11: lane quadrant w % 4, column half (w - 4) / 4
constexpr int kStageOff = 0;                // TMA stages reuse the latent copy and the first exchange buffer
constexpr int kPanelStageOff = 2 * kB * 2; // padded panel staging (second exchange buffer, extended)
constexpr int kPanelStageBytes = 82944;    // >= rows-per-tile x (K + 8) x 2 (at most ~74 KB) for every supported K
constexpr int kSwOff = kPanelStageOff + kPanelStageBytes;
static_assert(kStages * kStageBytes <= 2 * kB * 2, "x stages must fit the latent copy + first exchange buffer");
static_assert(2 * kYStageBytes <= kPanelStageBytes, "two output tiles must fit the panel staging");
constexpr size_t kLinSmem = kSwOff + 4 * kWordsPad * 4 + 1024;  // + alignment slack

struct LinParams {
  const void* latent;
  const void* wdense;  // dense variant: bf16 [N, K]
  void* y;             // bf16 [T, N]
  int* err;
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* out_gain;  // [N] or null
  const __nv_bfloat16* in_gain;   // [K] or null
  const float* w_add;             // scalar added to every weight element (modulation), or null
  const __nv_bfloat16* base;      // dense residual base weight [N, K], or null
  float base_scale;               // the generated part's factor when base is set
  int64_t L;
  int n, layers;
  uint32_t seed32;
  float corr, wscale;
  int K, N, T;
  int panels, tsplit, tpt;  // items = panels * tsplit; token tiles per item
};

// Final run (pass A) of one generator tile, written into the padded panel
// staging: the panel rows this tile touches, starting at panel row
// `row_base`, at pitch K+8 elements (16-byte row offset so that threads
// reading different rows hit different bank groups).  A tile touches at most
// 32768/K + 1 rows, i.e. <= 73,872 bytes for every supported K.
__device__ __forceinline__ void final_to_panel(const Frags& f, uint32_t in_base, const uint32_t* sw, float scale,
                                               uint16_t* stage, int64_t tile_coord0, int64_t panel_lo,
                                               int64_t panel_hi, int row_base, int K, int w, int lane, int g,
                                               int t) {
  uint32_t o[8][4];
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float c[8];
    final_tile(f, in_base, w, k, lane, c);
    o[k][0] = pack_out<__nv_bfloat16>(c[0] * scale, c[1] * scale);
    o[k][1] = pack_out<__nv_bfloat16>(c[2] * scale, c[3] * scale);
    o[k][2] = pack_out<__nv_bfloat16>(c[4] * scale, c[5] * scale);
    o[k][3] = pack_out<__nv_bfloat16>(c[6] * scale, c[7] * scale);
    sign_acc<0>(o[k], sw, w, k, g, t);
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t sel = h ? 0x7632u : 0x5410u;
      const int p = dep_a(w, 0, g + 8 * (j & 1), 2 * t + h + 8 * (j >> 1));
      const int64_t f0 = tile_coord0 + p;  // 8 consecutive coordinates, never straddling a row (K % 8 == 0)
      if (f0 >= panel_lo && f0 < panel_hi) {
        const int64_t rel = f0 - panel_lo;
        const int row = (int)(rel / K), col = (int)(rel - (int64_t)row * K);
        const int srow = row - row_base;
        uint32_t v0 = prmt(o[0][j], o[1][j], sel), v1 = prmt(o[2][j], o[3][j], sel);
        uint32_t v2 = prmt(o[4][j], o[5][j], sel), v3 = prmt(o[6][j], o[7][j], sel);
        *reinterpret_cast<uint4*>(stage + (size_t)srow * (K + 8) + col) = make_uint4(v0, v1, v2, v3);
      }
    }
  }
}

template <bool GEN>
__global__ void __launch_bounds__(kLinThreads, 1)
    linear_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmy,
                     const __grid_constant__ LinParams P) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  // 1024-byte aligned base: the swizzled TMA stages and descriptors assume 1024-byte atoms
  unsigned char* smem = smem_raw + ((1024 - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023)) & 1023);
  uint16_t* zbuf = reinterpret_cast<uint16_t*>(smem);
  uint16_t* xbuf = reinterpret_cast<uint16_t*>(smem + kStageOff);
  uint16_t* pstage = reinterpret_cast<uint16_t*>(smem + kPanelStageOff);
  uint32_t* sw = reinterpret_cast<uint32_t*>(smem + kSwOff);
  __shared__ __align__(8) uint64_t bars[2 * kStages + 4];
  __shared__ uint32_t tmem_base_sh;
  __shared__ float red[kLinThreads / 32];
  __shared__ int k0_sh, abort_sh;

  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const uint32_t bar0 = (uint32_t)__cvta_generic_to_shared(&bars[0]);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto dfull = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto dempty = [&](int b) { return bar0 + 8u * (2 * kStages + 2 + b); };

  if (w == 0) tc::tmem_alloc((uint32_t)__cvta_generic_to_shared(&tmem_base_sh), 512);
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(full_bar(s), 1);
      tc::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(dfull(b), 1);
      tc::mbar_init(dempty(b), 32 * kEpiWarps);
    }
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = tmem_base_sh;
  const int K = P.K, KC = K / 64;

  // input scale exponent, once per CTA (every panel comes from the same generator)
  const int n = P.n, layers = P.layers, Bm = (1 << n) - 1;
  int k0 = 0;
  if (GEN) {
    const __nv_bfloat16* latent = reinterpret_cast<const __nv_bfloat16*>(P.latent);
    float mx = 0.0f;
    for (int64_t i = tid; i < P.L; i += kLinThreads) {
      float v = __bfloat162float(latent[i]);
      mx = fmaxf(mx, fabsf(v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[w] = mx;
    __syncthreads();
    if (tid == 0) {
      float s = 0.0f;
      for (int i = 0; i < kLinThreads / 32; ++i) s = fmaxf(s, red[i]);
      int e = prescale_exponent(s, n);
      k0_sh = e;
    }
    __syncthreads();
    k0 = k0_sh;
  }
  const uint32_t zb = (uint32_t)__cvta_generic_to_shared(zbuf);
  const uint32_t xb = (uint32_t)__cvta_generic_to_shared(xbuf);           // x stages
  const uint32_t eb = (uint32_t)__cvta_generic_to_shared(smem + kB * 2);  // first exchange buffer
  const uint32_t yb = (uint32_t)__cvta_generic_to_shared(smem + kPanelStageOff);
  const float out_scale = ldexpf(1.0f, k0) * P.corr * P.wscale;
  const int ntok_tiles = (P.T + kTT - 1) / kTT;
  const uint32_t idesc = tc::idesc_bf16(128, kTT);
  // accumulators after the K/2 columns of A: two when they fit, else one
  const int nd = (K / 2 <= 512 - 2 * kTT) ? 2 : 1;
  const uint32_t dbase = 512 - nd * kTT;
  // per-role pipeline state (each role is always the same thread / warps)
  uint32_t prod_it = 0, mma_it = 0, tcount = 0;

  for (int item = blockIdx.x; item < P.panels * P.tsplit; item += gridDim.x) {
    const int panel = item / P.tsplit, split = item - panel * P.tsplit;
    const int n0 = panel * 128;
    const int tt0 = split * P.tpt, tt1 = min(ntok_tiles, tt0 + P.tpt);
    __syncthreads();  // previous item fully drained (accumulator read, stages idle)

    if (GEN) {
      // scaled fp16 latent copy (the x stages of the previous item overwrote it)
      const __nv_bfloat16* latent = reinterpret_cast<const __nv_bfloat16*>(P.latent);
      const float in_scale = ldexpf(1.0f, -k0);
      const bool first_is_b = (layers != 2);
      for (int c = tid; c < kB / 8; c += kLinThreads) {
        const int p0 = 8 * c, q0 = p0 & Bm;
        uint32_t hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float a = (q0 + 2 * e < P.L) ? __bfloat162float(latent[q0 + 2 * e]) * in_scale : 0.0f;
          float b = (q0 + 2 * e + 1 < P.L) ? __bfloat162float(latent[q0 + 2 * e + 1]) * in_scale : 0.0f;
          hv[e] = pack_h2(a, b);
        }
        if (first_is_b) {
          *reinterpret_cast<uint4*>(zbuf + lay_ab(p0)) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) zbuf[lay_ba(p0 + e)] = (uint16_t)(hv[e >> 1] >> (16 * (e & 1)));
        }
      }
    }
    // ---- 1. weight panel -> tensor memory (A operand) ----
    const int q = w & 3, cgi = w >> 2;  // TMEM lane quadrant and column group of this warp
    const uint32_t a_lane = tmem + ((uint32_t)(32 * q) << 16);
    const int m = 32 * q + lane;        // panel row owned by this thread in the copy
    if (GEN) {
      const int64_t panel_lo = (int64_t)n0 * K, panel_hi = panel_lo + (int64_t)128 * K;
      const int64_t ct_first = panel_lo >> kLog, ct_last = (panel_hi - 1) >> kLog;
      for (int64_t ct = ct_first; ct <= ct_last; ++ct) {
        __syncthreads();
        for (int i = tid; i < (layers + 1) * kWords; i += kLinThreads) {
          int l = i / kWords, wd = i - l * kWords;
          const int p = 32 * wd;
          sw[l * kWordsPad + spad(wd)] =
              sign_word(block_layer_key(P.seed32, (ct << (kLog - n)) + (p >> n), l), (p & Bm) >> 5);
        }
        __syncthreads();
        Frags f;
        make_frags(f, g, t, n);
        const uint32_t* fsw = sw + layers * kWordsPad;
        if (layers == 1) {
          run<1, false, true>(f, zb, eb, sw, nullptr, w, lane, g, t);
        } else if (layers == 2) {
          run<0, false, true>(f, zb, yb, sw, nullptr, w, lane, g, t);
          __syncthreads();
          run<1, true, false>(f, yb, eb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
        } else {
          run<1, false, true>(f, zb, eb, sw, nullptr, w, lane, g, t);
          __syncthreads();
          run<0, true, false>(f, eb, yb, nullptr, sw + 1 * kWordsPad, w, lane, g, t);
          __syncthreads();
          run<1, true, false>(f, yb, eb, nullptr, sw + 2 * kWordsPad, w, lane, g, t);
        }
        __syncthreads();
        const int64_t tile_lo = ct << kLog;
        const int64_t seg_lo = max(tile_lo, panel_lo), seg_hi = min(tile_lo + kB, panel_hi);
        const int row_base = (int)((seg_lo - panel_lo) / K);  // first panel row this tile touches
        final_to_panel(f, eb, fsw, out_scale, pstage, tile_lo, panel_lo, panel_hi, row_base, K, w, lane, g, t);
        __syncthreads();
        // 64 coordinates (32 tensor-memory columns) of this lane's row per
        // step: eight independent 16-byte loads, one 32-column store.  A
        // 64-aligned chunk never straddles a generator tile (K % 64 == 0).
        const int64_t my_lo = panel_lo + (int64_t)m * K;  // this lane's row [my_lo, my_lo + K)
        for (int c64 = cgi; c64 < K / 64; c64 += 4) {
          const int64_t f0 = my_lo + 64 * c64;
          const bool mine = f0 >= seg_lo && f0 + 64 <= seg_hi;
          uint32_t v[32];
          if (!__all_sync(0xffffffffu, mine)) tc::tmem_ld32(a_lane + 32 * c64, v);  // keep other tiles' part
          if (mine) {
            const uint4* src = reinterpret_cast<const uint4*>(pstage + (m - row_base) * (K + 8) + 64 * c64);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const uint4 s4 = src[u];
              v[4 * u] = s4.x, v[4 * u + 1] = s4.y, v[4 * u + 2] = s4.z, v[4 * u + 3] = s4.w;
            }
            if (P.w_add) {  // the modulation offset, added to every element (block_fht.py:448-449)
              const float c = __ldg(P.w_add);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const __nv_bfloat162 r = __floats2bfloat162_rn(__uint_as_float(v[j] << 16) + c,
                                                               __uint_as_float(v[j] & 0xffff0000u) + c);
                v[j] = (uint32_t)__bfloat16_as_ushort(r.x) | ((uint32_t)__bfloat16_as_ushort(r.y) << 16);
              }
            }
            if (P.base) {  // residual base: base + base_scale * W (block_fht.py:451-452)
              const uint4* bsrc = reinterpret_cast<const uint4*>(P.base + (size_t)(n0 + m) * K + 64 * c64);
#pragma unroll
              for (int u = 0; u < 8; ++u) {
                const uint4 b4 = __ldg(bsrc + u);
                const uint32_t bw[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  const uint32_t vv = v[4 * u + e];
                  const __nv_bfloat162 r = __floats2bfloat162_rn(
                      __uint_as_float(bw[e] << 16) + P.base_scale * __uint_as_float(vv << 16),
                      __uint_as_float(bw[e] & 0xffff0000u) + P.base_scale * __uint_as_float(vv & 0xffff0000u));
                  v[4 * u + e] = (uint32_t)__bfloat16_as_ushort(r.x) | ((uint32_t)__bfloat16_as_ushort(r.y) << 16);
                }
              }
            }
            if (P.in_gain) {  // W[:, k] * in_gain[k]: columns 64*c64 .. +63 of this row
              const uint32_t* ig = reinterpret_cast<const uint32_t*>(P.in_gain + 64 * c64);
#pragma unroll
              for (int j = 0; j < 32; ++j) {
                const uint32_t gb = __ldg(ig + j);
                const __nv_bfloat162 r =
                    __floats2bfloat162_rn(__uint_as_float(v[j] << 16) * __uint_as_float(gb << 16),
                                          __uint_as_float(v[j] & 0xffff0000u) * __uint_as_float(gb & 0xffff0000u));
                v[j] = (uint32_t)__bfloat16_as_ushort(r.x) | ((uint32_t)__bfloat16_as_ushort(r.y) << 16);
              }
            }
          }
          tc::tmem_st32(a_lane + 32 * c64, v);
        }
        tc::tmem_wait_st();
      }
    } else {
      const __nv_bfloat16* W = reinterpret_cast<const __nv_bfloat16*>(P.wdense);
      for (int c64 = cgi; c64 < K / 64; c64 += 4) {
        uint32_t v[32];
        const uint4* src = reinterpret_cast<const uint4*>(W + (size_t)(n0 + m) * K + 64 * c64);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 s4 = n0 + m < P.N ? src[u] : make_uint4(0, 0, 0, 0);
          v[4 * u] = s4.x, v[4 * u + 1] = s4.y, v[4 * u + 2] = s4.z, v[4 * u + 3] = s4.w;
        }
        tc::tmem_st32(a_lane + 32 * c64, v);
      }
      tc::tmem_wait_st();
    }
    tc::tc_fence_before();
    __syncthreads();
    tc::tc_fence_after();

    // ---- 2./3. MMA pipeline over this item's token tiles ----
    if (tid == 0) {  // TMA producer
      // the stages reuse a buffer the transform wrote through the generic proxy
      asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
      for (int tt = tt0; tt < tt1 && !abort_sh; ++tt) {
        for (int c = 0; c < KC; ++c, ++prod_it) {
          const int s = prod_it % kStages;
          const uint32_t ph = (prod_it / kStages) & 1;
          if (!tc::mbar_wait(empty_bar(s), ph ^ 1)) {
            abort_sh = 1;
            atomicExch(P.err, 1);
            break;
          }
          tc::mbar_expect_tx(full_bar(s), kStageBytes);
          tc::tma_load_2d(xb + s * kStageBytes, &tmx, c * 64, tt * kTT, full_bar(s));
        }
      }
    } else if (w == 1) {  // MMA issuer: the whole warp runs the loop, one elected lane issues
      for (int tt = tt0; tt < tt1 && !__any_sync(0xffffffffu, abort_sh); ++tt, ++tcount) {
        const int b = nd == 2 ? (int)(tcount & 1) : 0;
        const uint32_t dph = (nd == 2 ? (tcount >> 1) : tcount) & 1;
        if (!__all_sync(0xffffffffu, tc::mbar_wait(dempty(b), dph ^ 1))) {
          abort_sh = 1;
          atomicExch(P.err, 1);
          break;
        }
        tc::tc_fence_after();
        const uint32_t dcol = tmem + dbase + kTT * b;
        for (int c = 0; c < KC; ++c, ++mma_it) {
          const int s = mma_it % kStages;
          const uint32_t ph = (mma_it / kStages) & 1;
          if (!__all_sync(0xffffffffu, tc::mbar_wait(full_bar(s), ph))) {
            abort_sh = 1;
            atomicExch(P.err, 1);
            break;
          }
          tc::tc_fence_after();
          const uint32_t sbase = xb + s * kStageBytes;
          if (tc::elect_one()) {
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              tc::mma_ts(dcol, tmem + (uint32_t)(c * 32 + kk * 8), tc::smem_desc_k128(sbase + 32 * kk), idesc,
                         (c > 0 || kk > 0) ? 1u : 0u);
            }
            tc::mma_commit(empty_bar(s));  // frees the stage when these MMAs finish
          }
          __syncwarp();
        }
        if (tc::elect_one()) tc::mma_commit(dfull(b));  // accumulator b complete
        __syncwarp();
      }
    } else if (w >= 4 && w < 4 + kEpiWarps) {
      // epilogue: warp w drains TMEM lanes 32*(w%4).. and accumulator columns 64*h..64*h+63
      const int qe = w & 3, h = (w - 4) >> 2, et = tid - 128;  // et: 0..255 within the epilogue
      const int frow = 32 * qe + lane;                           // feature (panel row) of this thread
      for (int tt = tt0; tt < tt1 && !abort_sh; ++tt, ++tcount) {
        const int b = nd == 2 ? (int)(tcount & 1) : 0;
        const uint32_t dph = (nd == 2 ? (tcount >> 1) : tcount) & 1;
        if (!tc::mbar_wait(dfull(b), dph)) {
          abort_sh = 1;
          atomicExch(P.err, 1);
          break;
        }
        tc::tc_fence_after();
        uint32_t r0[32], r1[32];
        const uint32_t dl = tmem + ((uint32_t)(32 * qe) << 16) + dbase + kTT * b + 64 * h;
        tc::tmem_ld32(dl, r0);
        tc::tmem_ld32(dl + 32, r1);
        tc::tc_fence_before();
        tc::mbar_arrive(dempty(b));  // the accumulator can be overwritten now
        // output tile in shared memory: [128 tokens][128 features], two buffers;
        // wait until the TMA store that last read this buffer is done
        const int yb_i = (int)(tcount & 1);
        if (et == 0) tc::tma_store_wait_read<1>();
        tc::named_bar(1, 32 * kEpiWarps);
        __nv_bfloat16* yst = reinterpret_cast<__nv_bfloat16*>(pstage) + yb_i * (kYStageBytes / 2) + 64 * h * 128;
        // per-feature output gain and bias (identity when absent)
        const float og = P.out_gain ? __bfloat162float(P.out_gain[n0 + frow]) : 1.0f;
        const float bs = P.bias ? __bfloat162float(P.bias[n0 + frow]) : 0.0f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          yst[i * 128 + frow] = __float2bfloat16_rn(fmaf(__uint_as_float(r0[i]), og, bs));
          yst[(i + 32) * 128 + frow] = __float2bfloat16_rn(fmaf(__uint_as_float(r1[i]), og, bs));
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
        tc::named_bar(1, 32 * kEpiWarps);
        if (et == 0)
          tc::tma_store_2d(&tmy, (uint32_t)__cvta_generic_to_shared(reinterpret_cast<__nv_bfloat16*>(pstage) +
                                                                     yb_i * (kYStageBytes / 2)),
                           n0, tt * kTT);
      }
      if (et == 0) tc::tma_store_wait_all();  // the next item's transform reuses these buffers
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  if (w == 0) tc::tmem_dealloc(tmem, 512);
}

}  // namespace fmma

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

bool tc_linear_supported(int K, int N, int T) {
  return K % 64 == 0 && K >= 64 && K <= fmma::kMaxK && N % 128 == 0 && N > 0 && T > 0;
}

int tc_linear_launch(bool gen, const void* x, int T, int K, int N, const void* latent, int64_t L, int layers,
                     uint64_t seed, float wscale, const void* wdense, void* y, int* err, cudaStream_t st,
                     const LinExtras* extras) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return -2;
  CUtensorMap map, ymap;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)T};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)fmma::kTT};
  cuuint32_t estr[2] = {1, 1};
  if (enc(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return -3;
  cuuint64_t ydims[2] = {(cuuint64_t)N, (cuuint64_t)T};
  cuuint64_t ystrides[1] = {(cuuint64_t)N * 2};
  cuuint32_t ybox[2] = {128, (cuuint32_t)fmma::kTT};
  if (enc(&ymap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, ydims, ystrides, ybox, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
          CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) !=
      CUDA_SUCCESS)
    return -3;
  fmma::LinParams P;
  std::memset(&P, 0, sizeof(P));
  P.latent = latent;
  P.wdense = wdense;
  P.y = y;
  P.err = err;
  if (extras) {
    P.bias = reinterpret_cast<const __nv_bfloat16*>(extras->bias);
    P.out_gain = reinterpret_cast<const __nv_bfloat16*>(extras->out_gain);
    P.in_gain = reinterpret_cast<const __nv_bfloat16*>(extras->in_gain);
    P.w_add = extras->weight_offset;
    P.base = reinterpret_cast<const __nv_bfloat16*>(extras->base);
    P.base_scale = extras->base_scale;
  }
  P.L = L;
  P.n = gen ? ilog2(next_pow2(L)) : 15;
  P.layers = layers;
  P.seed32 = fold_seed(seed);
  P.corr = gen ? (float)std::pow(fmma::layer_correction(P.n), layers) : 1.0f;
  P.wscale = wscale;
  P.K = K;
  P.N = N;
  P.T = T;
  P.panels = N / 128;
  const int ntok = (T + fmma::kTT - 1) / fmma::kTT;
  int sms = fmma::sm_count();
  P.tsplit = std::max(1, std::min(ntok, sms / std::max(1, P.panels)));
  P.tpt = (ntok + P.tsplit - 1) / P.tsplit;
  P.tsplit = (ntok + P.tpt - 1) / P.tpt;
  const int items = P.panels * P.tsplit;
  const int grid = std::min(items, sms);
  if (gen) {
    if (!set_max_smem((const void*)fmma::linear_tc_kernel<true>, (int)fmma::kLinSmem)) return -1;
    fmma::linear_tc_kernel<true><<<grid, fmma::kLinThreads, fmma::kLinSmem, st>>>(map, ymap, P);
  } else {
    if (!set_max_smem((const void*)fmma::linear_tc_kernel<false>, (int)fmma::kLinSmem)) return -1;
    fmma::linear_tc_kernel<false><<<grid, fmma::kLinThreads, fmma::kLinSmem, st>>>(map, ymap, P);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace lwl
