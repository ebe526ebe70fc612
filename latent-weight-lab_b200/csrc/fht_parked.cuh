// Block sizes 2^16 and 2^17 (16-bit dtypes) with the block parked in tensor
// memory between layers.  Included by fht_mma.cu inside namespace lwl::fmma.
//
// A block of NT = 2 or 4 tiles of 2^15 coordinates is held in fp16 in tensor
// memory (NT x 64 KB: 256 or all 512 columns).  Thread (warp w, lane i) owns
// the 16-byte chunks c = tid + 512 q (q = 0..7) of every tile, in TMEM lane
// 32 (w mod 4) + i at columns NT*32 floor(w/4) + 32 j + 4 q (tile j); only the
// owner reads or writes them (tcgen05.ld/st 32x32b.x16 and their waits), so
// parking needs no barrier.  H_B = H_NT (x) H_32768 and the factors commute:
//   hi pass   -- the butterfly between the tiles (position bits 15 and, for
//                NT = 4, 16) on the parked chunks, in packed fp16 registers;
//   tile runs -- each tile unparked into shared memory, the tensor-core passes
//                of the 2^15 transform (run, run_final), parked again.
// Chunk slots: "by position" means chunk c holds positions 8c .. 8c+7 and sits
// at lay_ab(8c) of the pass-B input layout; "raw" means it is the 16-byte slot
// 8c of whatever exchange layout the last run wrote, which pairs the same
// positions in every tile, so unsigned hi passes work on raw slots.
//
// Schedules (the transposed chain of the backward uses the same ones with the
// sign layers reversed and S0 last):
//   layers 1, 2: per layer: hi pass with S_l by position; per tile pass B,
//                pass A (or the final pass A): 2 runs per tile per layer.
//   layers 3:    S0 + hi | B, A.S1.A (one DOUBLE run) | hi | B.S2.B | hi |
//                A final + S3: the sign layers between two layers fall inside
//                a DOUBLE run, so each tile runs 4 times instead of 6.
// Shared memory: two tile buffers and the NT tiles' sign tables.
// NT = 4: the hi butterfly carries its 1/2, so the block norm stays put;
// NT = 2: the 1-bit butterfly is unnormalised (x sqrt 2 per layer, folded into
// the output scale), as in the shared-memory 2^16 kernels.

template <int NT>
constexpr size_t parked_smem() { return 2 * kB * 2 + size_t(NT) * 4 * kWordsPad * 4; }

__device__ __forceinline__ void tm_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tm_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tm_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void tm_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

// The hi butterfly on half h of a thread's chunks (chunks tid + kThreads q,
// q = 4h .. 4h+3; v[j][4 (q - 4h) + e] holds elements 2e, 2e+1 of chunk q of
// tile j), in packed fp16.  With sgn (the sign table of tile 0 for one layer;
// tile j's at +4 j kWordsPad) the signs come first, looked up by position --
// sign bit set -> +1 (block_fht.py:55-81) -- as one XOR of the two fp16 sign
// bits per word: ((~bits) & 3) * 0x40008000 puts bit 0 at bit 15 and bit 1 at
// bit 31 (the partial products do not overlap).  A 1-bit butterfly rounds
// exactly as an fp32 sum rounded once; the 2-bit one (NT = 4) pre-scales by
// the exact 1/2 and rounds after each level.
template <int NT>
__device__ __forceinline__ void hi_butterfly(uint32_t (&v)[NT][16], const uint32_t* sgn, int h, int tid) {
  const __half2 half2_05 = __float2half2_rn(0.5f);
#pragma unroll
  for (int qq = 0; qq < 4; ++qq) {
    const int p0 = 8 * (tid + kThreads * (4 * h + qq));
    uint32_t m[NT];
#pragma unroll
    for (int j = 0; j < NT; ++j) m[j] = sgn ? ~(sgn[4 * j * kWordsPad + spad(p0 >> 5)] >> (p0 & 31)) : 0u;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = 4 * qq + e;
      __half2 a[NT];
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        const uint32_t x = v[j][r] ^ ((((m[j] >> (2 * e)) & 3u) * 0x40008000u) & 0x80008000u);
        a[j] = *reinterpret_cast<const __half2*>(&x);
        if (NT == 4) a[j] = __hmul2(a[j], half2_05);
      }
      __half2 o[NT];
      if (NT == 2) {
        o[0] = __hadd2(a[0], a[1]);
        o[1] = __hsub2(a[0], a[1]);
      } else {
        const __half2 b0 = __hadd2(a[0], a[1]), b1 = __hsub2(a[0], a[1]);
        const __half2 b2 = __hadd2(a[2], a[3]), b3 = __hsub2(a[2], a[3]);
        o[0] = __hadd2(b0, b2);
        o[1] = __hadd2(b1, b3);
        o[2] = __hsub2(b0, b2);
        o[3] = __hsub2(b1, b3);
      }
#pragma unroll
      for (int j = 0; j < NT; ++j) v[j][r] = *reinterpret_cast<const uint32_t*>(&o[j]);
    }
  }
}

// Tile j's parked chunks -> shared buffer, and back (see the slot modes above).
__device__ __forceinline__ void unpark_tile(uint32_t tcol, uint16_t* buf, bool by_pos, int tid) {
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t v[16];
    tm_ld16(tcol + 16 * h, v);
    tm_wait_ld();
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int c = tid + kThreads * (4 * h + qq);
      *reinterpret_cast<uint4*>(buf + (by_pos ? lay_ab(8 * c) : 8 * c)) =
          make_uint4(v[4 * qq], v[4 * qq + 1], v[4 * qq + 2], v[4 * qq + 3]);
    }
  }
}
__device__ __forceinline__ void park_tile(uint32_t tcol, const uint16_t* buf, bool by_pos, int tid) {
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t v[16];
#pragma unroll
    for (int qq = 0; qq < 4; ++qq) {
      const int c = tid + kThreads * (4 * h + qq);
      const uint4 u = *reinterpret_cast<const uint4*>(buf + (by_pos ? lay_ab(8 * c) : 8 * c));
      v[4 * qq] = u.x, v[4 * qq + 1] = u.y, v[4 * qq + 2] = u.z, v[4 * qq + 3] = u.w;
    }
    tm_st16(tcol + 16 * h, v);
  }
  tm_wait_st();
}

__device__ __forceinline__ uint32_t parked_alloc(uint32_t* slot, int cols, int w) {
  if (w == 0) {
    uint32_t dst = (uint32_t)__cvta_generic_to_shared(slot);
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(dst), "r"(cols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n");
  }
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  return *slot;
}
__device__ __forceinline__ void parked_free(uint32_t base, int cols, int w) {
  asm volatile("tcgen05.fence::before_thread_sync;\n");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;\n");
  if (w == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(cols));
}

// Sign tables of the block's NT tiles for layers 0..layers: [tile][layer][kWordsPad].
template <int NT>
__device__ __forceinline__ void parked_signs(uint32_t* sw, uint32_t seed32, int64_t b, int layers, int tid) {
  const int per = (layers + 1) * kWords;
  for (int i = tid; i < NT * per; i += kThreads) {
    const int j = i / per, r = i - j * per, l = r / kWords, wd = r - l * kWords;
    sw[(4 * j + l) * kWordsPad + spad(wd)] = sign_word(block_layer_key(seed32, b, l), 1024 * j + wd);
  }
}

template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    fhtp_forward_kernel(const T* __restrict__ latent, int64_t L, int layers, uint32_t seed32, float scale_base,
                        int64_t first_block, int64_t nblocks, int64_t start, int64_t stop, T* __restrict__ out) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* zs = reinterpret_cast<uint16_t*>(smem);
  uint16_t* xs = zs + kB;
  uint32_t* sw = reinterpret_cast<uint32_t*>(xs + kB);
  __shared__ float red[kThreads / 32];
  __shared__ int k0_shared;
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const uint32_t zb = (uint32_t)__cvta_generic_to_shared(zs), xb = (uint32_t)__cvta_generic_to_shared(xs);
  Frags f;
  make_frags(f, g, t, kLog);
  const uint32_t tbase = parked_alloc(&tmem_slot, NT * 128, w);
  const uint32_t tt0 = tbase + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(NT * 32 * (w >> 2));

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
    int e = prescale_exponent(s2, kLog + (NT == 4 ? 2 : 1));
    k0_shared = e;
  }
  __syncthreads();
  const int k0 = k0_shared;
  const float in_scale = ldexpf(1.0f, -k0), out_scale = ldexpf(1.0f, k0) * scale_base;
  const bool vec_ok = ((start & 7) == 0) && ((reinterpret_cast<uintptr_t>(out) & 15) == 0);
  const bool lat_tail = (reinterpret_cast<uintptr_t>(latent) & 15) != 0 || (L & 7) != 0;
  const bool fused = layers == 3;
  const int phases = fused ? 3 : layers;

  for (int64_t bi = blockIdx.x; bi < nblocks; bi += gridDim.x) {
    const int64_t b = first_block + bi;
    __syncthreads();  // the previous block's copy-out is done with the buffers and sign tables
    parked_signs<NT>(sw, seed32, b, layers, tid);
    __syncthreads();
    for (int ph = 0; ph < phases; ++ph) {
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t v[NT][16];
        if (ph == 0) {
          // the latent (the same for every block): all loads of the half in
          // flight at once when it is aligned and a multiple of 8 long
          if (!lat_tail) {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                const int64_t q0 = (int64_t)kB * j + 8 * (tid + kThreads * (4 * h + qq));
                uint4 r = make_uint4(0u, 0u, 0u, 0u);
                if (q0 < L) r = __ldg(reinterpret_cast<const uint4*>(latent + q0));
                v[j][4 * qq] = r.x, v[j][4 * qq + 1] = r.y, v[j][4 * qq + 2] = r.z, v[j][4 * qq + 3] = r.w;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq)
                gather8_words(reinterpret_cast<const uint16_t*>(latent),
                              (int64_t)kB * j + 8 * (tid + kThreads * (4 * h + qq)), L, &v[j][4 * qq]);
            }
          }
#pragma unroll
          for (int j = 0; j < NT; ++j) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
              const float2 fv = w2f<T>(v[j][r]);
              v[j][r] = pack_h2(fv.x * in_scale, fv.y * in_scale);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < NT; ++j) tm_ld16(tt0 + 32 * j + 16 * h, v[j]);
          tm_wait_ld();
        }
        hi_butterfly<NT>(v, (ph == 0 || !fused) ? sw + ph * kWordsPad : nullptr, h, tid);
#pragma unroll
        for (int j = 0; j < NT; ++j) tm_st16(tt0 + 32 * j + 16 * h, v[j]);
      }
      tm_wait_st();
#pragma unroll 1
      for (int j = 0; j < NT; ++j) {
        const uint32_t tcol = tt0 + 32 * j;
        const uint32_t* swj = sw + 4 * j * kWordsPad;
        if (!fused) {
          unpark_tile(tcol, zs, true, tid);
          __syncthreads();
          run<1, false, false>(f, zb, xb, nullptr, nullptr, w, lane, g, t);
          __syncthreads();
          if (ph + 1 < layers) {
            run<0, false, false>(f, xb, zb, nullptr, nullptr, w, lane, g, t);
            __syncthreads();
            park_tile(tcol, zs, true, tid);
          } else {
            run_final<T>(f, xb, zb, zs, swj + layers * kWordsPad, out_scale, out, NT * b + j, start, stop, vec_ok,
                         w, lane, g, t);
          }
        } else if (ph == 0) {
          unpark_tile(tcol, zs, true, tid);
          __syncthreads();
          run<1, false, false>(f, zb, xb, nullptr, nullptr, w, lane, g, t);
          __syncthreads();
          run<0, true, false>(f, xb, zb, nullptr, swj + 1 * kWordsPad, w, lane, g, t);
          __syncthreads();
          park_tile(tcol, zs, false, tid);
        } else if (ph == 1) {
          unpark_tile(tcol, zs, false, tid);
          __syncthreads();
          run<1, true, false>(f, zb, xb, nullptr, swj + 2 * kWordsPad, w, lane, g, t);
          __syncthreads();
          park_tile(tcol, xs, false, tid);
        } else {
          unpark_tile(tcol, xs, false, tid);
          __syncthreads();
          run_final<T>(f, xb, zb, zs, swj + 3 * kWordsPad, out_scale, out, NT * b + j, start, stop, vec_ok, w, lane,
                       g, t);
        }
        __syncthreads();
      }
    }
  }
  parked_free(tbase, NT * 128, w);
}

// Backward: grad_z = sum_b [S0 H S1 ... H S_layers g_b][0:L], the same
// schedules with the sign layers reversed.  The fp32 accumulator does not fit
// beside the parked block, so each tile's final pass A (scale, S0) is held in
// registers, staged as fp32 over both shared buffers and added, coalesced,
// into this CTA's [L] partial row (L2-resident): the CTA's first block stores,
// later ones use fire-and-forget red.global.add (one thread owns each
// address, so the sums keep program order and are deterministic).
// fht15_reduce_kernel sums the rows.
template <typename T, int NT>
__global__ void __launch_bounds__(kThreads, 1)
    fhtp_backward_kernel(const T* __restrict__ grad, int64_t L, int layers, uint32_t seed32, float scale_base,
                         int64_t first_block, int64_t nblocks, int64_t start, int64_t stop,
                         float* __restrict__ partial) {
  extern __shared__ __align__(128) unsigned char smem[];
  uint16_t* zs = reinterpret_cast<uint16_t*>(smem);
  uint16_t* xs = zs + kB;
  uint32_t* sw = reinterpret_cast<uint32_t*>(xs + kB);
  float* stg = reinterpret_cast<float*>(smem);  // fp32 staging of one tile over zs | xs
  __shared__ float red[kThreads / 32];
  __shared__ uint32_t tmem_slot;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, g = lane >> 2, t = lane & 3;
  const uint32_t zb = (uint32_t)__cvta_generic_to_shared(zs), xb = (uint32_t)__cvta_generic_to_shared(xs);
  Frags f;
  make_frags(f, g, t, kLog);
  const uint32_t tbase = parked_alloc(&tmem_slot, NT * 128, w);
  const uint32_t tt0 = tbase + ((uint32_t)(32 * (w & 3)) << 16) + (uint32_t)(NT * 32 * (w >> 2));
  const bool vec_ok = ((start & 7) == 0) && ((reinterpret_cast<uintptr_t>(grad) & 15) == 0);
  float* prow = partial + (int64_t)blockIdx.x * L;
  const bool row_vec = (L & 3) == 0 && (reinterpret_cast<uintptr_t>(partial) & 15) == 0;
  const uint16_t* g16 = reinterpret_cast<const uint16_t*>(grad);
  const bool fused = layers == 3;
  const int phases = fused ? 3 : layers;

  for (int64_t bi = blockIdx.x; bi < nblocks; bi += gridDim.x) {
    const int64_t b = first_block + bi;
    const int64_t bbase = b * NT * kB;
    const bool first = bi == blockIdx.x;
    __syncthreads();  // the previous block's row update is done with the buffers and sign tables
    parked_signs<NT>(sw, seed32, b, layers, tid);
    // gradient chunks as raw words: 16-byte loads with no per-chunk test when
    // the whole block lies inside [start, stop) and the gradient is aligned,
    // else element by element with zeros outside the slice
    const bool blk_full = vec_ok && bbase >= start && bbase + NT * kB <= stop;
    float mx = 0.0f;
#pragma unroll 1
    for (int h = 0; h < NT; ++h) {
      uint32_t r[8][4];
      if (blk_full) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const uint4 x =
              __ldg(reinterpret_cast<const uint4*>(grad + (bbase - start) + 8 * (tid + kThreads * (8 * h + u))));
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
      k0 = prescale_exponent(s2, kLog + (NT == 4 ? 2 : 1));
    }
    const float in_scale = ldexpf(1.0f, -k0), scale = ldexpf(1.0f, k0) * scale_base;

    // final pass A of tile j from the buffer at in_base: scale, signs S0,
    // fp32 staging, row update
    auto final_acc = [&](int j, uint32_t in_base) {
      const uint32_t* s0 = sw + 4 * j * kWordsPad;
      float c[8][8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        final_tile(f, in_base, w, k, lane, c[k]);
        // c[k][i]: row g + 8((i>>1)&1), column 2t + (i&1) + 8(i>>2) of pass A,
        // i.e. position base + k + 8((i>>1)&1) + 16(i&1) + 2048(i>>2)
        const int wb = dep_a(w, 0, g, 2 * t) >> 5;
        const uint32_t u0 = ~s0[spad(wb)], u1 = ~s0[spad(wb + 64)];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int bit = k + 8 * ((i >> 1) & 1) + 16 * (i & 1);
          const uint32_t u = (i >> 2) ? u1 : u0;
          c[k][i] = __uint_as_float(__float_as_uint(c[k][i] * scale) ^ ((u << (31 - bit)) & 0x80000000u));
        }
      }
      __syncthreads();  // every warp is done reading the input buffer
#pragma unroll
      for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int R = g + 8 * ((i >> 1) & 1), C = 2 * t + (i & 1) + 8 * (i >> 2);
          stg[prow_swz(dep_a(w, k, R, C))] = c[k][i];
        }
      }
      __syncthreads();
      const int64_t q0 = (int64_t)kB * j;
      if (first) {
        for (int pp = tid; pp < kB; pp += kThreads) {
          const int64_t q = q0 + pp;
          if (q < L) prow[q] = stg[prow_swz(pp)];
        }
      } else if (row_vec) {
        for (int pp = 4 * tid; pp < kB; pp += 4 * kThreads) {
          const int64_t q = q0 + pp;
          if (q < L)  // L % 4 == 0: all four are inside
            asm volatile("red.global.v4.f32.add [%0], {%1, %2, %3, %4};\n" ::"l"(prow + q),
                         "f"(stg[prow_swz(pp)]), "f"(stg[prow_swz(pp + 1)]), "f"(stg[prow_swz(pp + 2)]),
                         "f"(stg[prow_swz(pp + 3)])
                         : "memory");
        }
      } else {
        for (int pp = tid; pp < kB; pp += kThreads) {
          const int64_t q = q0 + pp;
          if (q < L) atomicAdd(prow + q, stg[prow_swz(pp)]);
        }
      }
    };

    for (int ph = 0; ph < phases; ++ph) {
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        uint32_t v[NT][16];
        if (ph == 0) {
          if (blk_full) {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq) {
                const uint4 x = __ldg(reinterpret_cast<const uint4*>(grad + (bbase - start) + (int64_t)kB * j +
                                                                     8 * (tid + kThreads * (4 * h + qq))));
                v[j][4 * qq] = x.x, v[j][4 * qq + 1] = x.y, v[j][4 * qq + 2] = x.z, v[j][4 * qq + 3] = x.w;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < NT; ++j) {
#pragma unroll
              for (int qq = 0; qq < 4; ++qq)
                gather8_words(g16, bbase + (int64_t)kB * j + 8 * (tid + kThreads * (4 * h + qq)) - start,
                              stop - start, &v[j][4 * qq]);
            }
          }
#pragma unroll
          for (int j = 0; j < NT; ++j) {
#pragma unroll
            for (int r = 0; r < 16; ++r) {
              const float2 fv = w2f<T>(v[j][r]);
              v[j][r] = pack_h2(fv.x * in_scale, fv.y * in_scale);
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < NT; ++j) tm_ld16(tt0 + 32 * j + 16 * h, v[j]);
          tm_wait_ld();
        }
        // step ph is preceded by S_(layers - ph)
        hi_butterfly<NT>(v, (ph == 0 || !fused) ? sw + (layers - ph) * kWordsPad : nullptr, h, tid);
#pragma unroll
        for (int j = 0; j < NT; ++j) tm_st16(tt0 + 32 * j + 16 * h, v[j]);
      }
      tm_wait_st();
#pragma unroll 1
      for (int j = 0; j < NT; ++j) {
        const uint32_t tcol = tt0 + 32 * j;
        const uint32_t* swj = sw + 4 * j * kWordsPad;
        if (!fused) {
          unpark_tile(tcol, zs, true, tid);
          __syncthreads();
          run<1, false, false>(f, zb, xb, nullptr, nullptr, w, lane, g, t);
          __syncthreads();
          if (ph + 1 < layers) {
            run<0, false, false>(f, xb, zb, nullptr, nullptr, w, lane, g, t);
            __syncthreads();
            park_tile(tcol, zs, true, tid);
          } else {
            final_acc(j, xb);
          }
        } else if (ph == 0) {
          unpark_tile(tcol, zs, true, tid);
          __syncthreads();
          run<1, false, false>(f, zb, xb, nullptr, nullptr, w, lane, g, t);
          __syncthreads();
          run<0, true, false>(f, xb, zb, nullptr, swj + 2 * kWordsPad, w, lane, g, t);
          __syncthreads();
          park_tile(tcol, zs, false, tid);
        } else if (ph == 1) {
          unpark_tile(tcol, zs, false, tid);
          __syncthreads();
          run<1, true, false>(f, zb, xb, nullptr, swj + 1 * kWordsPad, w, lane, g, t);
          __syncthreads();
          park_tile(tcol, xs, false, tid);
        } else {
          unpark_tile(tcol, xs, false, tid);
          __syncthreads();
          final_acc(j, xb);
        }
        __syncthreads();
      }
    }
  }
  parked_free(tbase, NT * 128, w);
}

// NT = 4: the hi butterflies carry their 1/2; NT = 2: 2^(-1/2) per layer here.
inline float parked_scale_base(int nt, int layers) {
  return (float)(std::pow(layer_correction(kLog), layers) * (nt == 2 ? std::pow(2.0, -0.5 * layers) : 1.0));
}

template <typename T, int NT>
int launch_forward_parked(const void* latent, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                          void* out, cudaStream_t st) {
  const int64_t B = NT * kB;
  const int64_t first = start / B, last = (stop + B - 1) / B;
  if (last <= first) return 0;
  if (!set_max_smem((const void*)fhtp_forward_kernel<T, NT>, (int)parked_smem<NT>())) return -1;
  const int64_t nb = last - first, sms = sm_count();
  const int grid = (int)(nb < sms ? nb : sms);
  fhtp_forward_kernel<T, NT><<<grid, kThreads, parked_smem<NT>(), st>>>(
      reinterpret_cast<const T*>(latent), L, layers, fold_seed(seed), parked_scale_base(NT, layers), first, nb,
      start, stop, reinterpret_cast<T*>(out));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

template <typename T, int NT>
int launch_backward_parked(const void* grad, int64_t L, int layers, uint64_t seed, int64_t start, int64_t stop,
                           void* grad_latent, void* workspace, cudaStream_t st) {
  const int64_t B = NT * kB;
  const int64_t first = start / B, last = (stop + B - 1) / B;
  if (last <= first) return cudaMemsetAsync(grad_latent, 0, size_t(L) * 2, st) == cudaSuccess ? 0 : -1;
  int* err = reinterpret_cast<int*>(workspace);
  float* partial = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + kBwdHeader);
  if (cudaMemsetAsync(err, 0, sizeof(int), st) != cudaSuccess) return -1;
  if (!set_max_smem((const void*)fhtp_backward_kernel<T, NT>, (int)parked_smem<NT>())) return -1;
  const int64_t nb = last - first, sms = sm_count();
  const int grid = (int)(nb < sms ? nb : sms);
  fhtp_backward_kernel<T, NT><<<grid, kThreads, parked_smem<NT>(), st>>>(
      reinterpret_cast<const T*>(grad), L, layers, fold_seed(seed), parked_scale_base(NT, layers), first, nb, start,
      stop, partial);
  if (cudaGetLastError() != cudaSuccess) return -1;
  const int rb = (int)((L + 255) / 256);
  fht15_reduce_kernel<T><<<rb, 256, 0, st>>>(partial, grid, L, err, reinterpret_cast<T*>(grad_latent));
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
