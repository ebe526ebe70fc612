/*
 * lwl_b200.h -- C ABI of the B200 (sm_100a) BlockFHT library (liblwl_b200.so).
 *
 * Every entry point takes plain device pointers, int64 sizes and a CUDA
 * stream (cudaStream_t passed as void*; NULL = legacy default stream).  The
 * library never allocates device memory: callers size scratch space with the
 * *_workspace_bytes queries and pass it in, 16-byte aligned (every cudaMalloc
 * or torch allocation is; the bf16 large-block plans require it).  Calls are stateless and
 * re-entrant; work is enqueued on the given stream and nothing synchronises
 * the host.  Every call returns an lwl_status; lwl_last_error() gives the
 * calling thread's message for the most recent failure.
 *
 * Index convention (shared with the reference): a generator with latent z of
 * length L and padded block size B = next_pow2(L) produces `size` coordinates;
 * coordinate i belongs to block i / B at position i % B, and block b is
 *   y_b = S_{b,layers} Ĥ ... S_{b,1} Ĥ S_{b,0} pad_B(z),   Ĥ = H_B / sqrt(B),
 * with H_B the natural-order Walsh-Hadamard matrix and S_{b,l} the +-1
 * diagonal from the stateless sign hash.
 */
#ifndef LWL_B200_H
#define LWL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lwl_status {
  LWL_OK = 0,
  LWL_ERR_INVALID = 1,      /* bad argument: the reference raises ValueError / TORCH_CHECK here */
  LWL_ERR_UNSUPPORTED = 2,  /* valid request outside what the kernels implement */
  LWL_ERR_WORKSPACE = 3,    /* workspace pointer missing or smaller than required */
  LWL_ERR_CUDA = 4,         /* a CUDA runtime call or launch failed */
  LWL_ERR_TIMEOUT = 5       /* a bounded device-side wait gave up */
} lwl_status;

typedef enum lwl_dtype { LWL_F32 = 0, LWL_BF16 = 1, LWL_F16 = 2 } lwl_dtype;

/* Flags for the transform entry points. */
#define LWL_FLAG_EXACT 1u /* bf16/fp16: force fp32 arithmetic end to end (no tensor-core factors) */
/* Testing only (lwl_fht_backward, tensor-core path): every CTA leaves its first
 * gradient copy unissued and polls its bounded wait only 256 times, so the wait
 * gives up with no copy in flight.  The result is NaN and
 * lwl_fht_backward_status reports LWL_ERR_TIMEOUT; the context stays usable. */
#define LWL_FLAG_TEST_WAIT_TIMEOUT 0x80000000u

/* Library version (major*10000 + minor*100 + patch). */
int lwl_version(void);

/* Human-readable name of a status code. */
const char* lwl_status_string(int status);

/* Message for the calling thread's most recent failure ("" if none). */
const char* lwl_last_error(void);

/* Writes `count` sign words for (seed, block, layer) starting at word
 * `first_word` into out[count] (device memory).
 * Replaces: sign_word_for, latent_weight_lab/block_fht.py:46-52 and the
 * device copy csrc/block_fht_ext_cuda.cu:36-43. */
int lwl_sign_words(uint64_t seed, int64_t block, int layer, int64_t first_word, int64_t count,
                   uint32_t* out, void* stream);

/* Workspace needed by lwl_fht_forward for these arguments (bytes; 0 if none). */
size_t lwl_fht_forward_workspace_bytes(int dtype, int64_t latent_size, int64_t size, int layers,
                                       int64_t start, int64_t stop, unsigned flags);

/* Generated coordinates [start, stop) of the BlockFHT with latent[latent_size]
 * (dtype) into out[stop - start] (dtype).  layers in {1,2,3}; padded block
 * size 2^5 .. 2^23.
 * Replaces: pybind `forward` (csrc/block_fht_ext.cpp:28-38) and
 * block_fht_forward_cuda (csrc/block_fht_ext_cuda.cu:516-566); dtype
 * coverage widened from fp32 to fp32/bf16/fp16. */
int lwl_fht_forward(int dtype, const void* latent, int64_t latent_size, int64_t size, int layers,
                    uint64_t seed, int64_t start, int64_t stop, void* out, void* workspace,
                    size_t workspace_bytes, unsigned flags, void* stream);

/* One generator call of a grouped forward. */
typedef struct lwl_fht_forward_desc {
  const void* latent;  /* [latent_size], the group's dtype */
  int64_t latent_size;
  int64_t size;
  int layers;
  uint64_t seed;
  int64_t start, stop;  /* coordinates [start, stop) */
  void* out;            /* [stop - start], the group's dtype */
} lwl_fht_forward_desc;

/* count lwl_fht_forward calls in as few kernel launches as possible (one
 * launch per 96 generators): the tiles of all generators share one persistent
 * grid, so many small weights (the linears of a model) fill the GPU.
 * 16-bit dtypes with padded block size <= 2^15 take the grouped path; other
 * descriptors are run one by one and must need no workspace (else
 * LWL_ERR_UNSUPPORTED).  No direct reference counterpart: replaces the
 * per-module generation loop of prepare_block_fht_weight_cache /
 * materialize_weight_cache (latent_weight_lab/block_fht.py:503-512, 560-563). */
int lwl_fht_forward_grouped(int dtype, int count, const lwl_fht_forward_desc* descs, unsigned flags,
                            void* stream);

/* Workspace needed by lwl_fht_backward (bytes). */
size_t lwl_fht_backward_workspace_bytes(int dtype, int64_t latent_size, int64_t size, int layers,
                                        int64_t start, int64_t stop, unsigned flags);

/* grad_latent[latent_size] (dtype, overwritten) = d/dz sum(y[start:stop] * grad_out),
 * grad_out[stop - start] (dtype).  Accumulates in fp32, deterministically.
 * Replaces: pybind `backward` (csrc/block_fht_ext.cpp:40-50) and
 * block_fht_backward_cuda (csrc/block_fht_ext_cuda.cu:568-622). */
int lwl_fht_backward(int dtype, const void* grad_out, int64_t latent_size, int64_t size,
                     int layers, uint64_t seed, int64_t start, int64_t stop, void* grad_latent,
                     void* workspace, size_t workspace_bytes, unsigned flags, void* stream);

/* One generator of a grouped backward: grad_latent[latent_size] (dtype) =
 * the latent gradient of grad_out[stop - start] (dtype), as lwl_fht_backward. */
typedef struct lwl_fht_backward_desc {
  const void* grad_out;
  int64_t latent_size;
  int64_t size;
  int layers;
  uint64_t seed;
  int64_t start, stop;
  void* grad_latent;
} lwl_fht_backward_desc;

/* Workspace for lwl_fht_backward_grouped with these descriptors. */
size_t lwl_fht_backward_grouped_workspace_bytes(int dtype, int count, const lwl_fht_backward_desc* descs,
                                                unsigned flags);

/* After a lwl_fht_backward call with these arguments and this workspace:
 * synchronises `stream`, then returns LWL_ERR_TIMEOUT (with a message) if a
 * bounded device-side wait of that call gave up, else LWL_OK.  Only the
 * tensor-core backward (16-bit, padded block <= 2^15) waits on the device; it
 * keeps the error word at the start of its workspace and poisons the gradient
 * with NaN on a time-out.  Other paths always report LWL_OK.  No reference
 * counterpart (the reference's kernels do not wait on the device). */
int lwl_fht_backward_status(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start,
                            int64_t stop, unsigned flags, const void* workspace, void* stream);

/* count lwl_fht_backward calls as one kernel + one reduce launch per 96
 * generators (16-bit dtypes, padded block size <= 2^15; other generators run
 * one by one inside the call): each CTA takes a contiguous range of all
 * generators' 2^15-coordinate tiles and writes one partial row per generator
 * it touches.  Deterministic.  Replaces: the per-module
 * block_fht_grad_latent calls of flush_block_fht_weight_cache
 * (latent_weight_lab/block_fht.py:514-557, 566-569). */
int lwl_fht_backward_grouped(int dtype, int count, const lwl_fht_backward_desc* descs, void* workspace,
                             size_t workspace_bytes, unsigned flags, void* stream);

/* Workspace for lwl_linear_forward: 16 bytes; its first int is a device
 * error word, 0 after a successful call (1 = a bounded pipeline wait gave up). */
size_t lwl_linear_forward_workspace_bytes(void);

/* y[tokens, out_features] (bf16) = x[tokens, in_features] (bf16) @ (weight_scale * W)^T,
 * W = the generator's first in*out coordinates viewed as [out, in], generated
 * on chip: each CTA regenerates its 128-row weight panel with the tensor-core
 * transform, keeps it in tensor memory as the tcgen05.mma A operand and
 * streams x tiles by TMA.  Supported: bf16, in_features % 64 == 0 and <= 768,
 * out_features % 128 == 0, padded block size <= 2^15; otherwise
 * LWL_ERR_UNSUPPORTED (callers then generate W and use a library GEMM).
 * Replaces: pybind `linear_forward` (csrc/block_fht_ext.cpp:52-67),
 * block_fht_linear_forward_cuda (csrc/block_fht_ext_cuda.cu:624-681), whose
 * kernel requires block % in_features == 0 and block <= 16384. */
int lwl_linear_forward(int dtype, const void* x, int64_t tokens, int64_t in_features, const void* latent,
                       int64_t latent_size, int64_t out_features, int layers, uint64_t seed, float weight_scale,
                       void* y, void* workspace, size_t workspace_bytes, void* stream);

/* After a lwl_linear_forward / lwl_linear_forward_ex / lwl_tc_linear_dense
 * call with this workspace: synchronises `stream` and returns
 * LWL_ERR_TIMEOUT if a bounded pipeline wait of that call gave up, else
 * LWL_OK.  No reference counterpart. */
int lwl_linear_forward_status(const void* workspace, void* stream);

/* Workspace for lwl_linear_backward: the generated W, grad_W (both [out, in]
 * in dtype), the transform workspace and 4 MiB for cuBLAS. */
size_t lwl_linear_backward_workspace_bytes(int dtype, int64_t tokens, int64_t in_features, int64_t out_features,
                                           int64_t latent_size, int layers, unsigned flags);

/* Backward of y = x @ (weight_scale * W)^T (fp32 / bf16 / fp16, all tensors of
 * one dtype, row-major, contiguous):
 *   grad_x[tokens, in]  = weight_scale * grad_y @ W          (skipped if grad_x is NULL)
 *   grad_latent[latent] = weight_scale * J^T (grad_y^T @ x)   (skipped if grad_latent is NULL)
 * W is regenerated into the workspace; the two products are plain cuBLAS
 * GEMMs (fp32 accumulation); J^T is lwl_fht_backward over all in*out
 * coordinates.  The bias gradient and the modulation terms stay with the
 * caller.  Replaces: _BlockFHTLinearFn.backward (latent_weight_lab/block_fht.py:322-356);
 * the reference's pybind module has no linear backward. */
int lwl_linear_backward(int dtype, const void* x, const void* grad_y, int64_t tokens, int64_t in_features,
                        int64_t out_features, const void* latent, int64_t latent_size, int layers, uint64_t seed,
                        float weight_scale, void* grad_x, void* grad_latent, void* workspace, size_t workspace_bytes,
                        unsigned flags, void* stream);

/* FixedFHTMix over the last dimension: for every row r,
 *   y[r, :features] = (S * H_P / sqrt(P) * S * pad(x[r, :]))[:features],
 * P = next_pow2(features) <= 8192, S = diag(signs), signs[P] fp32 (+-1) on the
 * device; x and y [rows, features] row-major in dtype, fp32 arithmetic.  The
 * map is its own adjoint, so the same call computes the input gradient.
 * Replaces: FixedFHTMix.forward / normalized_fht_last_dim
 * (examples/nanogpt/model.py:182-218), a pure-torch op in the reference. */
int lwl_fixed_fht_mix(int dtype, const void* x, int64_t rows, int64_t features, const float* signs, void* y,
                      void* stream);

/* lwl_linear_forward with the module's extra terms folded in (bias, out_gain,
 * in_gain: bf16 device vectors or NULL; weight_offset: one fp32 device
 * scalar or NULL; base: a dense bf16 [out_features, in_features] residual
 * base weight or NULL, with its factor base_scale):
 *   V = weight_scale * W + offset;  V = base + base_scale * V if base;
 *   y[:, n] = out_gain[n] * (x @ (V * in_gain[None, :])^T)[:, n] + bias[n].
 * The offset (the modulation term alpha * sum(z^2) [- expected]), the base
 * and the input gain are applied to the generated panel on chip, the output
 * gain and bias in the epilogue: one GEMM where the reference runs two.
 * Same shape limits as lwl_linear_forward; in_gain and weight_offset 4-byte
 * aligned, base 16-byte aligned.  Replaces: the materialised weight
 * (block_fht.py:444-462) and the torch modulation, residual-base and gain
 * terms of BlockFHTLinear.forward_fused (block_fht.py:482-501). */
int lwl_linear_forward_ex(int dtype, const void* x, int64_t tokens, int64_t in_features, const void* latent,
                          int64_t latent_size, int64_t out_features, int layers, uint64_t seed, float weight_scale,
                          const void* bias, const void* out_gain, const void* in_gain, const float* weight_offset,
                          const void* base, float base_scale, void* y, void* workspace, size_t workspace_bytes,
                          void* stream);

/* Dense-weight variant of the same tcgen05 pipeline: y = x @ w^T with a given
 * bf16 w[out_features, in_features] (same shape limits).  No reference
 * counterpart; it isolates the MMA pipeline from the generator for testing. */
int lwl_tc_linear_dense(const void* x, int64_t tokens, int64_t in_features, const void* w, int64_t out_features,
                        void* y, void* workspace, size_t workspace_bytes, void* stream);

/* Number of kernel launches one lwl_fht_forward (backward = 0) or
 * lwl_fht_backward (backward = 1) call with these arguments enqueues; -1 on
 * invalid arguments.  No reference counterpart (the reference launches
 * layers*(log2 B + 1) + 2 kernels for large blocks, csrc/block_fht_ext_cuda.cu:546-564);
 * used for launch accounting and graph-capture planning. */
int lwl_fht_launch_count(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start,
                         int64_t stop, int backward, unsigned flags);

/* The latent gradient of lwl_fht_backward, for callers that cannot allocate
 * device memory (no workspace argument).  No counterpart in the reference.
 * It always runs the fp32 tile engine, so fp32 results match
 * lwl_fht_backward's and bf16 / fp16 results match them up to rounding
 * (lwl_fht_backward may take the tensor-core path there).
 * Intended for code that has no device allocator at hand, e.g. a plugin
 * called from a host runtime that owns all device memory, or a callback whose
 * memory policy forbids allocating.  The per-CTA partial gradients live in a
 * fixed 8 MiB device array inside the library instead of a workspace:
 *  - padded block size at most 2^14, else LWL_ERR_UNSUPPORTED;
 *  - every GPU that loads the library holds the 8 MiB until the process exits;
 *  - the first call on a device looks up the array's device address
 *    (cudaGetSymbolAddress with that device current); make that first call
 *    before any stream capture;
 *  - all calls on a device share the array; calls that overlap on the GPU
 *    race on it and give wrong results: order them on one stream;
 *  - the looked-up address is kept for the life of the process, so it does
 *    not survive cudaDeviceReset (or another teardown of the device's primary
 *    context): do not call this entry point on a device after resetting it. */
int lwl_fht_backward_noalloc(int dtype, const void* grad_out, int64_t latent_size, int64_t size,
                             int layers, uint64_t seed, int64_t start, int64_t stop, void* grad_latent,
                             unsigned flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LWL_B200_H */
