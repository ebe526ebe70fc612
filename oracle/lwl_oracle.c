/*
 * lwl_oracle.c -- CPU restatement of the reference BlockFHT algorithm.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * product path and the timed CPU baseline ("port") in bench.py.  Nothing in
 * the shipped package links, loads or calls it; only tests/, the smoke check
 * in __graft_entry__.py and bench.py's CPU-baseline / reference arm do.
 *
 * Parity is pinned: tests/test_oracle.py checks these functions against
 * golden vectors produced by the reference implementation itself
 * (tests/golden/make_golden.py imports latent_weight_lab from the reference
 * checkout and records its outputs).
 *
 * Every function restates the reference step by step, in the same floating
 * point operation order, so that the fp32 results are bit-identical to the
 * reference's pure-torch CPU path:
 *
 *   lowbias32 / sign_word_for   latent_weight_lab/block_fht.py:36-52
 *                               (device copy: csrc/block_fht_ext_cuda.cu:27-48)
 *   normalized_fht_last_dim     latent_weight_lab/block_fht.py:18-33
 *   block_fht_slice_torch       latent_weight_lab/block_fht.py:84-109
 *   backward (autograd through  latent_weight_lab/block_fht.py:179-196; the
 *   block_fht_slice_torch)      transposed chain of csrc/block_fht_ext_cuda.cu:185-223
 *
 * Blocks are independent, so the block loop is spread over OpenMP threads;
 * the backward keeps one partial gradient per thread and sums them in
 * thread order at the end.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* block_fht.py:36-43 */
static inline uint32_t lowbias32(uint32_t x) {
  x ^= x >> 16;
  x *= 0x7FEB352Du;
  x ^= x >> 15;
  x *= 0x846CA68Bu;
  x ^= x >> 16;
  return x;
}

/* block_fht.py:46-52: seed folded to 32 bits, then (block, layer, word)
 * mixed with three odd constants, all arithmetic mod 2^32. */
uint32_t lwl_oracle_sign_word(int64_t seed, int64_t block, int64_t layer, int64_t word) {
  uint64_t s = (uint64_t)seed;
  uint32_t x = (uint32_t)s ^ (uint32_t)(s >> 32);
  x ^= 0x9E3779B9u * (uint32_t)(block + 1);
  x ^= 0x85EBCA6Bu * (uint32_t)(layer + 1);
  x ^= 0xC2B2AE35u * (uint32_t)(word + 1);
  return lowbias32(x);
}

int64_t lwl_oracle_next_pow2(int64_t v) {
  int64_t o = 1;
  while (o < v) o <<= 1;
  return o;
}

/* values[pos] *= (bit pos&31 of word pos>>5) ? +1 : -1   (block_fht.py:79-81) */
static void apply_sign_f(float* v, int64_t n, int64_t seed, int64_t block, int layer) {
  for (int64_t w = 0; w < n / 32; ++w) {
    uint32_t bits = lwl_oracle_sign_word(seed, block, layer, w);
    for (int j = 0; j < 32; ++j)
      if (!((bits >> j) & 1u)) v[w * 32 + j] = -v[w * 32 + j];
  }
}

static void apply_sign_d(double* v, int64_t n, int64_t seed, int64_t block, int layer) {
  for (int64_t w = 0; w < n / 32; ++w) {
    uint32_t bits = lwl_oracle_sign_word(seed, block, layer, w);
    for (int j = 0; j < 32; ++j)
      if (!((bits >> j) & 1u)) v[w * 32 + j] = -v[w * 32 + j];
  }
}

/* Natural-order radix-2 WHT, stage widths 1, 2, 4, ... then divide by
 * sqrt(n) (block_fht.py:18-33).  torch divides a float tensor by the python
 * float math.sqrt(n), i.e. by that double rounded to float. */
static void fht_fwd_f(float* v, int64_t n) {
  for (int64_t h = 1; h < n; h <<= 1)
    for (int64_t i = 0; i < n; i += 2 * h)
      for (int64_t j = i; j < i + h; ++j) {
        float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
  float d = (float)sqrt((double)n);
  for (int64_t i = 0; i < n; ++i) v[i] = v[i] / d;
}

/* Autograd of fht_fwd_f: DivBackward (grad / d) first, then the stages in
 * reverse order; the butterfly is its own transpose. */
static void fht_bwd_f(float* v, int64_t n) {
  float d = (float)sqrt((double)n);
  for (int64_t i = 0; i < n; ++i) v[i] = v[i] / d;
  for (int64_t h = n >> 1; h >= 1; h >>= 1)
    for (int64_t i = 0; i < n; i += 2 * h)
      for (int64_t j = i; j < i + h; ++j) {
        float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
}

static void fht_d(double* v, int64_t n) {
  for (int64_t h = 1; h < n; h <<= 1)
    for (int64_t i = 0; i < n; i += 2 * h)
      for (int64_t j = i; j < i + h; ++j) {
        double a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
  double s = 1.0 / sqrt((double)n);
  for (int64_t i = 0; i < n; ++i) v[i] *= s;
}

/* block_fht.py:84-109.  latent [L] fp32 -> out [stop-start] fp32.
 * prec 0: fp32 in the reference's operation order; prec 1: fp64 math
 * (accuracy yardstick), rounded to fp32 once on output.
 * Returns 0, or -1 on an invalid slice / allocation failure. */
int lwl_oracle_fht_forward(const float* latent, int64_t L, int64_t size, int layers,
                           int64_t seed, int64_t start, int64_t stop, float* out,
                           int prec, int threads) {
  if (L <= 0 || size <= 0 || start < 0 || stop < start || stop > size) return -1;
  if (layers < 1 || layers > 3) return -1;
  int64_t B = lwl_oracle_next_pow2(L);
  int64_t first = start / B, last = (stop + B - 1) / B;
  int err = 0;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel
#endif
  {
    int64_t Bw = B < 32 ? 32 : B; /* scratch rounded up to a whole sign word */
    float* vf = prec == 0 ? (float*)malloc(sizeof(float) * Bw) : NULL;
    double* vd = prec == 1 ? (double*)malloc(sizeof(double) * Bw) : NULL;
    if ((prec == 0 && !vf) || (prec == 1 && !vd)) {
#ifdef _OPENMP
#pragma omp atomic write
#endif
      err = -1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
      for (int64_t b = first; b < last; ++b) {
        int64_t bs = b * B;
        int64_t lo = start > bs ? start - bs : 0;
        int64_t hi = stop - bs < B ? stop - bs : B;
        if (prec == 0) {
          memset(vf, 0, sizeof(float) * Bw);
          memcpy(vf, latent, sizeof(float) * L);
          apply_sign_f(vf, Bw, seed, b, 0);
          for (int l = 0; l < layers; ++l) {
            fht_fwd_f(vf, B);
            apply_sign_f(vf, Bw, seed, b, l + 1);
          }
          for (int64_t i = lo; i < hi; ++i) out[bs + i - start] = vf[i];
        } else {
          for (int64_t i = 0; i < Bw; ++i) vd[i] = i < L ? (double)latent[i] : 0.0;
          apply_sign_d(vd, Bw, seed, b, 0);
          for (int l = 0; l < layers; ++l) {
            fht_d(vd, B);
            apply_sign_d(vd, Bw, seed, b, l + 1);
          }
          for (int64_t i = lo; i < hi; ++i) out[bs + i - start] = (float)vd[i];
        }
      }
    }
    free(vf);
    free(vd);
  }
  return err;
}

/* Gradient of sum(out * grad_out) with respect to the latent, where out is
 * lwl_oracle_fht_forward's result: per block S0 Ĥ S1 ... Ĥ S_layers g_b,
 * truncated to the first L entries and summed over blocks
 * (block_fht.py:179-196 through autograd; csrc/block_fht_ext_cuda.cu:185-223). */
int lwl_oracle_fht_backward(const float* grad_out, int64_t L, int64_t size, int layers,
                            int64_t seed, int64_t start, int64_t stop, float* grad_latent,
                            int prec, int threads) {
  if (L <= 0 || size <= 0 || start < 0 || stop < start || stop > size) return -1;
  if (layers < 1 || layers > 3) return -1;
  int64_t B = lwl_oracle_next_pow2(L);
  int64_t Bw = B < 32 ? 32 : B;
  int64_t first = start / B, last = (stop + B - 1) / B;
  int nt = 1;
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
  nt = omp_get_max_threads();
#endif
  double* part = (double*)calloc((size_t)nt * (size_t)L, sizeof(double));
  float* partf = (float*)calloc((size_t)nt * (size_t)L, sizeof(float));
  if (!part || !partf) {
    free(part);
    free(partf);
    return -1;
  }
  int err = 0;
#ifdef _OPENMP
#pragma omp parallel
#endif
  {
    int tid = 0;
#ifdef _OPENMP
    tid = omp_get_thread_num();
#endif
    float* vf = (float*)malloc(sizeof(float) * Bw);
    double* vd = (double*)malloc(sizeof(double) * Bw);
    if (!vf || !vd) {
#ifdef _OPENMP
#pragma omp atomic write
#endif
      err = -1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
      for (int64_t b = first; b < last; ++b) {
        int64_t bs = b * B;
        int64_t lo = start > bs ? start - bs : 0;
        int64_t hi = stop - bs < B ? stop - bs : B;
        if (prec == 0) {
          memset(vf, 0, sizeof(float) * Bw);
          for (int64_t i = lo; i < hi; ++i) vf[i] = grad_out[bs + i - start];
          for (int l = layers - 1; l >= 0; --l) {
            apply_sign_f(vf, Bw, seed, b, l + 1);
            fht_bwd_f(vf, B);
          }
          apply_sign_f(vf, Bw, seed, b, 0);
          float* acc = partf + (size_t)tid * L;
          for (int64_t i = 0; i < L; ++i) acc[i] += vf[i];
        } else {
          memset(vd, 0, sizeof(double) * Bw);
          for (int64_t i = lo; i < hi; ++i) vd[i] = (double)grad_out[bs + i - start];
          for (int l = layers - 1; l >= 0; --l) {
            apply_sign_d(vd, Bw, seed, b, l + 1);
            fht_d(vd, B);
          }
          apply_sign_d(vd, Bw, seed, b, 0);
          double* acc = part + (size_t)tid * L;
          for (int64_t i = 0; i < L; ++i) acc[i] += vd[i];
        }
      }
    }
    free(vf);
    free(vd);
  }
  for (int64_t i = 0; i < L; ++i) {
    if (prec == 0) {
      float s = 0.0f;
      for (int t = 0; t < nt; ++t) s += partf[(size_t)t * L + i];
      grad_latent[i] = s;
    } else {
      double s = 0.0;
      for (int t = 0; t < nt; ++t) s += part[(size_t)t * L + i];
      grad_latent[i] = (float)s;
    }
  }
  free(part);
  free(partf);
  return err;
}

int lwl_oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
