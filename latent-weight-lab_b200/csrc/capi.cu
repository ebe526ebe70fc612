// capi.cu -- the extern "C" boundary of liblwl_b200.so (declared in include/lwl_b200.h).
//
// Argument validation mirrors the reference's checks so callers see the same
// failures: slice bounds and layer range (latent_weight_lab/block_fht.py:92-93,
// :609-610; csrc/block_fht_ext_cuda.cu:523-529), block-size range 2^5..2^23 is
// widened here down to 2^0 (the reference's CPU path accepts any size).
#include <cublas_v2.h>
#include <cstdarg>
#include <cstdio>
#include <cstdint>
#include <cstring>
#include <algorithm>
#include <vector>

#include "fht_engine.h"
#include "fht_mma.h"
#include "lwl_b200.h"
#include "lwl_common.cuh"

namespace lwl {
int fht_mix_launch(int dtype, const void* x, void* y, const float* signs, int64_t rows, int F, int logP,
                   cudaStream_t st);

static thread_local char g_err[512];

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}

void clear_error() { g_err[0] = 0; }

__global__ void sign_words_kernel(uint32_t key, int64_t first_word, int64_t count, uint32_t* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = sign_word(key, first_word + i);
}

static int validate_fht(int dtype, int64_t L, int64_t size, int layers, int64_t start, int64_t stop) {
  if (dtype != LWL_F32 && dtype != LWL_BF16 && dtype != LWL_F16) {
    set_error("unsupported dtype code %d (expected 0=fp32, 1=bf16, 2=fp16)", dtype);
    return LWL_ERR_INVALID;
  }
  if (L <= 0) {
    set_error("latent size must be positive");
    return LWL_ERR_INVALID;
  }
  if (size <= 0) {
    set_error("size must be positive");
    return LWL_ERR_INVALID;
  }
  if (layers < 1 || layers > 3) {
    set_error("layers must be 1, 2, or 3");
    return LWL_ERR_INVALID;
  }
  if (!(0 <= start && start <= stop && stop <= size)) {
    set_error("invalid slice [%lld, %lld) for size %lld", (long long)start, (long long)stop, (long long)size);
    return LWL_ERR_INVALID;
  }
  if (next_pow2(L) > (int64_t(1) << kMaxLogB)) {
    set_error("padded block size %lld exceeds the supported maximum 2^23", (long long)next_pow2(L));
    return LWL_ERR_UNSUPPORTED;
  }
  return LWL_OK;
}

static int fht_call(bool backward, int dtype, const void* in, void* out, int64_t L, int64_t size,
                    int layers, uint64_t seed, int64_t start, int64_t stop, void* ws, size_t ws_bytes,
                    unsigned flags, void* stream) {
  g_err[0] = 0;
  int st = validate_fht(dtype, L, size, layers, start, stop);
  if (st) return st;
  if ((stop > start && !in) || !out) {
    set_error("null data pointer");
    return LWL_ERR_INVALID;
  }
  FhtArgs a;
  a.dtype = dtype;
  a.backward = backward;
  a.in = in;
  a.out = out;
  a.latent_size = L;
  a.size = size;
  a.layers = layers;
  a.seed = seed;
  a.start = start;
  a.stop = stop;
  a.workspace = ws;
  a.workspace_bytes = ws_bytes;
  a.flags = flags;
  if (fhts_supported(dtype, L, backward, layers, flags)) return fhts_run(a, reinterpret_cast<cudaStream_t>(stream));
  if (!backward && mma_forward_supported(dtype, L, flags)) {
    if (mma_forward(dtype, in, L, layers, seed, start, stop, out, reinterpret_cast<cudaStream_t>(stream)) != 0) {
      set_error("tensor-core forward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
    return LWL_OK;
  }
  if (!backward && mma16_forward_supported(dtype, L, flags)) {
    if (mma16_forward(dtype, in, L, layers, seed, start, stop, out, reinterpret_cast<cudaStream_t>(stream)) != 0) {
      set_error("2^16 forward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
    return LWL_OK;
  }
  if (backward && mma_backward_supported(dtype, L, flags)) {
    size_t need = mma_backward_workspace_bytes(L, start, stop);
    if (need > 0 && (ws == nullptr || ws_bytes < need)) {
      set_error("workspace of %zu bytes required, %zu given", need, ws ? ws_bytes : (size_t)0);
      return LWL_ERR_WORKSPACE;
    }
    if (mma_backward(dtype, in, L, layers, seed, start, stop, out, ws, reinterpret_cast<cudaStream_t>(stream),
                     (flags & LWL_FLAG_TEST_WAIT_TIMEOUT) ? 1 : 0) != 0) {
      set_error("tensor-core backward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
    return LWL_OK;
  }
  if (backward && mma16_backward_supported(dtype, L, flags)) {
    const size_t need = mma16_backward_workspace_bytes(L, start, stop);
    if (need > 0 && (ws == nullptr || ws_bytes < need)) {
      set_error("workspace of %zu bytes required, %zu given", need, ws ? ws_bytes : (size_t)0);
      return LWL_ERR_WORKSPACE;
    }
    if (mma16_backward(dtype, in, L, layers, seed, start, stop, out, ws, reinterpret_cast<cudaStream_t>(stream)) !=
        0) {
      set_error("2^16 backward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
    return LWL_OK;
  }
  if (fht32_supported(dtype, L, backward, flags)) return fht32_run(a, reinterpret_cast<cudaStream_t>(stream));
  FhtPlan plan;
  plan_fht(a, plan);
  if (plan.ws_bytes > 0 && (ws == nullptr || ws_bytes < plan.ws_bytes)) {
    set_error("workspace of %zu bytes required, %zu given", plan.ws_bytes, ws ? ws_bytes : (size_t)0);
    return LWL_ERR_WORKSPACE;
  }
  return run_fht(a, plan, reinterpret_cast<cudaStream_t>(stream));
}

static size_t fht_ws(bool backward, int dtype, int64_t L, int64_t size, int layers, int64_t start,
                     int64_t stop, unsigned flags) {
  if (validate_fht(dtype, L, size, layers, start, stop) != LWL_OK) return 0;
  if (fhts_supported(dtype, L, backward, layers, flags)) {
    FhtArgs a;
    std::memset(&a, 0, sizeof(a));
    a.dtype = dtype;
    a.backward = backward;
    a.latent_size = L;
    a.size = size;
    a.layers = layers;
    a.start = start;
    a.stop = stop;
    a.flags = flags;
    return fhts_workspace_bytes(a);
  }
  if (!backward && mma_forward_supported(dtype, L, flags)) return 0;
  if (!backward && mma16_forward_supported(dtype, L, flags)) return 0;
  if (backward && mma_backward_supported(dtype, L, flags)) return mma_backward_workspace_bytes(L, start, stop);
  if (backward && mma16_backward_supported(dtype, L, flags)) return mma16_backward_workspace_bytes(L, start, stop);
  FhtArgs a;
  std::memset(&a, 0, sizeof(a));
  a.dtype = dtype;
  a.backward = backward;
  a.latent_size = L;
  a.size = size;
  a.layers = layers;
  a.start = start;
  a.stop = stop;
  a.flags = flags;
  if (fht32_supported(dtype, L, backward, flags)) return fht32_workspace_bytes(a);
  FhtPlan plan;
  plan_fht(a, plan);
  return plan.ws_bytes;
}

}  // namespace lwl

namespace {

// Linear backward workspace: [W (grad_x) | grad_W (grad_latent) | transform
// workspace | cuBLAS workspace], each 256-byte aligned.
constexpr size_t kCublasWs = size_t(4) << 20;
size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct LinBwdPlan {
  size_t w_off, gw_off, fht_off, cub_off, total;
};

LinBwdPlan plan_linear_backward(int dtype, int64_t K, int64_t N, int64_t L, int layers, unsigned flags) {
  const size_t es = dtype == LWL_F32 ? 4 : 2, wbytes = align256((size_t)(K * N) * es);
  const int64_t size = K * N;
  const size_t fws = std::max(lwl::fht_ws(false, dtype, L, size, layers, 0, size, flags),
                              lwl::fht_ws(true, dtype, L, size, layers, 0, size, flags));
  LinBwdPlan p;
  p.w_off = 0;
  p.gw_off = wbytes;
  p.fht_off = 2 * wbytes;
  p.cub_off = p.fht_off + align256(fws);
  p.total = p.cub_off + kCublasWs;
  return p;
}

cublasHandle_t cublas_handle() {
  static thread_local cublasHandle_t h[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return nullptr;
  if (!h[dev] && cublasCreate(&h[dev]) != CUBLAS_STATUS_SUCCESS) h[dev] = nullptr;
  return h[dev];
}

__global__ void scale_kernel(void* p, int dtype, int64_t n, float s) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    if (dtype == LWL_F32) {
      reinterpret_cast<float*>(p)[i] *= s;
    } else if (dtype == LWL_BF16) {
      __nv_bfloat16* q = reinterpret_cast<__nv_bfloat16*>(p) + i;
      *q = __float2bfloat16_rn(__bfloat162float(*q) * s);
    } else {
      __half* q = reinterpret_cast<__half*>(p) + i;
      *q = __float2half_rn(__half2float(*q) * s);
    }
  }
}

}  // namespace

extern "C" {

int lwl_version(void) { return 100; }

const char* lwl_status_string(int status) {
  switch (status) {
    case LWL_OK: return "ok";
    case LWL_ERR_INVALID: return "invalid argument";
    case LWL_ERR_UNSUPPORTED: return "unsupported";
    case LWL_ERR_WORKSPACE: return "workspace too small";
    case LWL_ERR_CUDA: return "CUDA error";
    case LWL_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

const char* lwl_last_error(void) { return lwl::g_err; }

int lwl_sign_words(uint64_t seed, int64_t block, int layer, int64_t first_word, int64_t count, uint32_t* out,
                   void* stream) {
  lwl::g_err[0] = 0;
  if (count < 0 || block < 0 || first_word < 0 || layer < 0) {
    lwl::set_error("block, layer, first_word and count must be non-negative");
    return LWL_ERR_INVALID;
  }
  if (count == 0) return LWL_OK;
  if (!out) {
    lwl::set_error("null output pointer");
    return LWL_ERR_INVALID;
  }
  uint32_t key = lwl::block_layer_key(lwl::fold_seed(seed), block, layer);
  int threads = 256;
  int64_t blocks = (count + threads - 1) / threads;
  if (blocks > 4096) blocks = 4096;
  lwl::sign_words_kernel<<<(int)blocks, threads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(key, first_word,
                                                                                               count, out);
  LWL_CUDA_TRY(cudaGetLastError());
  return LWL_OK;
}

size_t lwl_fht_forward_workspace_bytes(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start,
                                       int64_t stop, unsigned flags) {
  return lwl::fht_ws(false, dtype, latent_size, size, layers, start, stop, flags);
}

int lwl_fht_forward(int dtype, const void* latent, int64_t latent_size, int64_t size, int layers, uint64_t seed,
                    int64_t start, int64_t stop, void* out, void* workspace, size_t workspace_bytes,
                    unsigned flags, void* stream) {
  if (stop == start && lwl::validate_fht(dtype, latent_size, size, layers, start, stop) == LWL_OK) return LWL_OK;
  return lwl::fht_call(false, dtype, latent, out, latent_size, size, layers, seed, start, stop, workspace,
                       workspace_bytes, flags, stream);
}

size_t lwl_fht_backward_workspace_bytes(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start,
                                        int64_t stop, unsigned flags) {
  return lwl::fht_ws(true, dtype, latent_size, size, layers, start, stop, flags);
}

int lwl_fht_backward(int dtype, const void* grad_out, int64_t latent_size, int64_t size, int layers,
                     uint64_t seed, int64_t start, int64_t stop, void* grad_latent, void* workspace,
                     size_t workspace_bytes, unsigned flags, void* stream) {
  return lwl::fht_call(true, dtype, grad_out, grad_latent, latent_size, size, layers, seed, start, stop,
                       workspace, workspace_bytes, flags, stream);
}

// Reads a device error word written by a call's bounded waits (synchronises
// the stream first, so the call that wrote it has finished).
static int read_error_word(const void* word, void* stream, const char* what) {
  lwl::clear_error();
  int host = 0;
  LWL_CUDA_TRY(cudaStreamSynchronize(reinterpret_cast<cudaStream_t>(stream)));
  LWL_CUDA_TRY(cudaMemcpy(&host, word, sizeof(int), cudaMemcpyDeviceToHost));
  if (host != 0) {
    lwl::set_error("%s: a bounded device-side wait gave up (error word %d); the result was poisoned with NaN", what,
                   host);
    return LWL_ERR_TIMEOUT;
  }
  return LWL_OK;
}

int lwl_fht_backward_status(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start, int64_t stop,
                            unsigned flags, const void* workspace, void* stream) {
  lwl::clear_error();
  int st = lwl::validate_fht(dtype, latent_size, size, layers, start, stop);
  if (st) return st;
  // only the tensor-core backward waits on the device; it keeps its error word
  // at the start of a non-empty workspace
  if (lwl::fhts_supported(dtype, latent_size, true, layers, flags) ||
      !lwl::mma_backward_supported(dtype, latent_size, flags) ||
      lwl::mma_backward_workspace_bytes(latent_size, start, stop) == 0)
    return LWL_OK;
  if (!workspace) {
    lwl::set_error("null workspace");
    return LWL_ERR_INVALID;
  }
  return read_error_word(workspace, stream, "lwl_fht_backward");
}

int lwl_linear_forward_status(const void* workspace, void* stream) {
  if (!workspace) {
    lwl::clear_error();
    lwl::set_error("null workspace");
    return LWL_ERR_INVALID;
  }
  return read_error_word(workspace, stream, "lwl_linear_forward");
}

int lwl_fht_forward_grouped(int dtype, int count, const lwl_fht_forward_desc* descs, unsigned flags,
                            void* stream) {
  lwl::g_err[0] = 0;
  if (count < 0 || (count > 0 && !descs)) {
    lwl::set_error("invalid descriptor array");
    return LWL_ERR_INVALID;
  }
  bool all_fast = true;
  for (int i = 0; i < count; ++i) {
    const lwl_fht_forward_desc& q = descs[i];
    int st = lwl::validate_fht(dtype, q.latent_size, q.size, q.layers, q.start, q.stop);
    if (st) return st;
    if (q.stop > q.start && (!q.latent || !q.out)) {
      lwl::set_error("descriptor %d: null data pointer", i);
      return LWL_ERR_INVALID;
    }
    if (!lwl::mma_forward_supported(dtype, q.latent_size, flags)) all_fast = false;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  // Generators that a single call sends to the tensor-core tile kernel share
  // one grouped launch; the rest (the small-block kernel's sizes included)
  // run as single calls, so every output equals its single call bit for bit.
  std::vector<lwl_fht_forward_desc> grouped;
  std::vector<int> rest;
  for (int i = 0; i < count; ++i) {
    const lwl_fht_forward_desc& q = descs[i];
    if (all_fast && !lwl::fhts_supported(dtype, q.latent_size, false, q.layers, flags))
      grouped.push_back(q);
    else
      rest.push_back(i);
  }
  if (!grouped.empty()) {
    if (lwl::mma_forward_grouped(dtype, (int)grouped.size(), grouped.data(), st) != 0) {
      lwl::set_error("grouped forward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
      return LWL_ERR_CUDA;
    }
  }
  for (int i : rest) {
    const lwl_fht_forward_desc& q = descs[i];
    if (lwl::fht_ws(false, dtype, q.latent_size, q.size, q.layers, q.start, q.stop, flags) > 0) {
      lwl::set_error("descriptor %d needs a workspace; call lwl_fht_forward for it", i);
      return LWL_ERR_UNSUPPORTED;
    }
    int rc = lwl_fht_forward(dtype, q.latent, q.latent_size, q.size, q.layers, q.seed, q.start, q.stop, q.out,
                             nullptr, 0, flags, stream);
    if (rc) return rc;
  }
  return LWL_OK;
}

int lwl_fixed_fht_mix(int dtype, const void* x, int64_t rows, int64_t features, const float* signs, void* y,
                      void* stream) {
  lwl::g_err[0] = 0;
  if (dtype != LWL_F32 && dtype != LWL_BF16 && dtype != LWL_F16) {
    lwl::set_error("dtype must be fp32, bf16 or fp16");
    return LWL_ERR_INVALID;
  }
  if (rows < 0 || features <= 0) {
    lwl::set_error("rows must be >= 0 and features > 0");
    return LWL_ERR_INVALID;
  }
  const int logP = lwl::ilog2(features);
  if (logP > 13) {
    lwl::set_error("padded feature count %lld exceeds 8192", (long long)(int64_t(1) << logP));
    return LWL_ERR_UNSUPPORTED;
  }
  if (rows == 0) return LWL_OK;
  if (!x || !y || !signs) {
    lwl::set_error("null data pointer");
    return LWL_ERR_INVALID;
  }
  if (lwl::fht_mix_launch(dtype, x, y, signs, rows, (int)features, logP, reinterpret_cast<cudaStream_t>(stream))) {
    lwl::set_error("fixed FHT mix launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  return LWL_OK;
}

size_t lwl_linear_backward_workspace_bytes(int dtype, int64_t tokens, int64_t in_features, int64_t out_features,
                                           int64_t latent_size, int layers, unsigned flags) {
  (void)tokens;
  if (in_features <= 0 || out_features <= 0 || latent_size <= 0) return 0;
  return plan_linear_backward(dtype, in_features, out_features, latent_size, layers, flags).total;
}

int lwl_linear_backward(int dtype, const void* x, const void* grad_y, int64_t tokens, int64_t in_features,
                        int64_t out_features, const void* latent, int64_t latent_size, int layers, uint64_t seed,
                        float weight_scale, void* grad_x, void* grad_latent, void* workspace, size_t workspace_bytes,
                        unsigned flags, void* stream) {
  lwl::g_err[0] = 0;
  const int64_t T = tokens, K = in_features, N = out_features, size = K * N;
  if (T < 0 || K <= 0 || N <= 0) {
    lwl::set_error("tokens must be >= 0, in_features and out_features > 0");
    return LWL_ERR_INVALID;
  }
  int st = lwl::validate_fht(dtype, latent_size, size, layers, 0, size);
  if (st) return st;
  if (!grad_x && !grad_latent) return LWL_OK;
  if (!latent || (T > 0 && (!grad_y || (grad_latent && !x)))) {
    lwl::set_error("null data pointer");
    return LWL_ERR_INVALID;
  }
  const LinBwdPlan pl = plan_linear_backward(dtype, K, N, latent_size, layers, flags);
  if (!workspace || workspace_bytes < pl.total) {
    lwl::set_error("workspace of %zu bytes needed, %zu given", pl.total, workspace_bytes);
    return LWL_ERR_WORKSPACE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  char* ws = reinterpret_cast<char*>(workspace);
  const size_t fht_bytes = pl.cub_off - pl.fht_off;
  cublasHandle_t h = cublas_handle();
  if (!h) {
    lwl::set_error("cublasCreate failed");
    return LWL_ERR_CUDA;
  }
  if (cublasSetStream(h, s) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(h, ws + pl.cub_off, kCublasWs) != CUBLAS_STATUS_SUCCESS) {
    lwl::set_error("cuBLAS stream / workspace setup failed");
    return LWL_ERR_CUDA;
  }
  const cudaDataType_t dt = dtype == LWL_F32 ? CUDA_R_32F : dtype == LWL_BF16 ? CUDA_R_16BF : CUDA_R_16F;
  const float one = 1.0f, zero = 0.0f;
  // row-major [r, c] is column-major [c x r]
  if (grad_x) {
    if (T > 0) {
      // W = generator's first N*K coordinates, [N, K]
      st = lwl::fht_call(false, dtype, latent, ws + pl.w_off, latent_size, size, layers, seed, 0, size,
                         ws + pl.fht_off, fht_bytes, flags, stream);
      if (st) return st;
      // grad_x[T, K] = scale * grad_y[T, N] @ W[N, K]  (block_fht.py:330-337)
      if (cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_N, (int)K, (int)T, (int)N, &weight_scale, ws + pl.w_off, dt,
                       (int)K, grad_y, dt, (int)N, &zero, grad_x, dt, (int)K, CUBLAS_COMPUTE_32F,
                       CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS) {
        lwl::set_error("cublasGemmEx (grad_x) failed");
        return LWL_ERR_CUDA;
      }
    }
  }
  if (grad_latent) {
    if (T == 0) {
      LWL_CUDA_TRY(cudaMemsetAsync(grad_latent, 0, (size_t)latent_size * (dtype == LWL_F32 ? 4 : 2), s));
      return LWL_OK;
    }
    // grad_W[N, K] = grad_y^T[N, T] @ x[T, K]  (block_fht.py:339-341)
    if (cublasGemmEx(h, CUBLAS_OP_N, CUBLAS_OP_T, (int)K, (int)N, (int)T, &one, x, dt, (int)K, grad_y, dt, (int)N,
                     &zero, ws + pl.gw_off, dt, (int)K, CUBLAS_COMPUTE_32F,
                     CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS) {
      lwl::set_error("cublasGemmEx (grad_W) failed");
      return LWL_ERR_CUDA;
    }
    // grad_latent = scale * J^T grad_W  (block_fht.py:342-348)
    st = lwl::fht_call(true, dtype, ws + pl.gw_off, grad_latent, latent_size, size, layers, seed, 0, size,
                       ws + pl.fht_off, fht_bytes, flags, stream);
    if (st) return st;
    if (weight_scale != 1.0f) {
      scale_kernel<<<(int)std::min<int64_t>((latent_size + 255) / 256, 1024), 256, 0, s>>>(grad_latent, dtype,
                                                                                         latent_size, weight_scale);
      LWL_CUDA_TRY(cudaGetLastError());
    }
  }
  return LWL_OK;
}

// Generators that a single call sends to the tensor-core backward share the
// grouped launch; the small-block kernel's sizes run as single calls.
static bool grouped_bwd_fast(int dtype, const lwl_fht_backward_desc& q, unsigned flags) {
  return lwl::mma_backward_supported(dtype, q.latent_size, flags) &&
         !lwl::fhts_supported(dtype, q.latent_size, true, q.layers, flags);
}

size_t lwl_fht_backward_grouped_workspace_bytes(int dtype, int count, const lwl_fht_backward_desc* descs,
                                                unsigned flags) {
  if (count <= 0 || !descs) return 0;
  std::vector<lwl_fht_backward_desc> fast;
  size_t need = 0;
  for (int i = 0; i < count; ++i) {
    const lwl_fht_backward_desc& q = descs[i];
    if (grouped_bwd_fast(dtype, q, flags))
      fast.push_back(q);
    else
      need = std::max(need, lwl::fht_ws(true, dtype, q.latent_size, q.size, q.layers, q.start, q.stop, flags));
  }
  if (!fast.empty()) need = std::max(need, lwl::mma_backward_grouped_workspace_bytes((int)fast.size(), fast.data()));
  return need;
}

int lwl_fht_backward_grouped(int dtype, int count, const lwl_fht_backward_desc* descs, void* workspace,
                             size_t workspace_bytes, unsigned flags, void* stream) {
  lwl::g_err[0] = 0;
  if (count < 0 || (count > 0 && !descs)) {
    lwl::set_error("invalid descriptor array");
    return LWL_ERR_INVALID;
  }
  std::vector<lwl_fht_backward_desc> fast;
  for (int i = 0; i < count; ++i) {
    const lwl_fht_backward_desc& q = descs[i];
    int st = lwl::validate_fht(dtype, q.latent_size, q.size, q.layers, q.start, q.stop);
    if (st) return st;
    if (!q.grad_latent || (q.stop > q.start && !q.grad_out)) {
      lwl::set_error("descriptor %d: null data pointer", i);
      return LWL_ERR_INVALID;
    }
    if (grouped_bwd_fast(dtype, q, flags)) fast.push_back(q);
  }
  const size_t need = lwl_fht_backward_grouped_workspace_bytes(dtype, count, descs, flags);
  if (need > 0 && (!workspace || workspace_bytes < need)) {
    lwl::set_error("workspace of %zu bytes needed, %zu given", need, workspace_bytes);
    return LWL_ERR_WORKSPACE;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (!fast.empty() && lwl::mma_backward_grouped(dtype, (int)fast.size(), fast.data(), workspace, s) != 0) {
    lwl::set_error("grouped backward launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  for (int i = 0; i < count; ++i) {  // the rest, one by one, reusing the workspace in stream order
    const lwl_fht_backward_desc& q = descs[i];
    if (grouped_bwd_fast(dtype, q, flags)) continue;
    int rc = lwl_fht_backward(dtype, q.grad_out, q.latent_size, q.size, q.layers, q.seed, q.start, q.stop,
                              q.grad_latent, workspace, workspace_bytes, flags, stream);
    if (rc) return rc;
  }
  return LWL_OK;
}

size_t lwl_linear_forward_workspace_bytes(void) { return 16; }

static int linear_common(bool gen, int dtype, const void* x, int64_t T, int64_t K, int64_t N, const void* latent,
                         int64_t L, int layers, void* y, void* ws, size_t ws_bytes) {
  if (dtype != LWL_BF16) {
    lwl::set_error("the tcgen05 linear supports bf16 only");
    return LWL_ERR_UNSUPPORTED;
  }
  if (T <= 0 || K <= 0 || N <= 0 || T > INT32_MAX || K > INT32_MAX || N > INT32_MAX) {
    lwl::set_error("tokens, in_features and out_features must be positive");
    return LWL_ERR_INVALID;
  }
  if (gen) {
    int st = lwl::validate_fht(dtype, L, K * N, layers, 0, K * N);
    if (st) return st;
  }
  if (!x || !y || (gen && !latent)) {
    lwl::set_error("null data pointer");
    return LWL_ERR_INVALID;
  }
  if (!lwl::tc_linear_supported((int)K, (int)N, (int)T) || (gen && lwl::next_pow2(L) > 32768) ||
      (reinterpret_cast<uintptr_t>(x) & 15)) {
    lwl::set_error("shape outside the tcgen05 linear (in %% 64 == 0, in <= 768, out %% 128 == 0, block <= 2^15)");
    return LWL_ERR_UNSUPPORTED;
  }
  if (!ws || ws_bytes < 16) {
    lwl::set_error("workspace of 16 bytes required");
    return LWL_ERR_WORKSPACE;
  }
  return LWL_OK;
}

int lwl_linear_forward(int dtype, const void* x, int64_t tokens, int64_t in_features, const void* latent,
                       int64_t latent_size, int64_t out_features, int layers, uint64_t seed, float weight_scale,
                       void* y, void* workspace, size_t workspace_bytes, void* stream) {
  lwl::g_err[0] = 0;
  int st = linear_common(true, dtype, x, tokens, in_features, out_features, latent, latent_size, layers, y, workspace,
                         workspace_bytes);
  if (st) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LWL_CUDA_TRY(cudaMemsetAsync(workspace, 0, 16, s));
  int rc = lwl::tc_linear_launch(true, x, (int)tokens, (int)in_features, (int)out_features, latent, latent_size,
                                 layers, seed, weight_scale, nullptr, y, reinterpret_cast<int*>(workspace), s);
  if (rc) {
    lwl::set_error("tcgen05 linear launch failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  return LWL_OK;
}

int lwl_linear_forward_ex(int dtype, const void* x, int64_t tokens, int64_t in_features, const void* latent,
                          int64_t latent_size, int64_t out_features, int layers, uint64_t seed, float weight_scale,
                          const void* bias, const void* out_gain, const void* in_gain, const float* weight_offset,
                          const void* base, float base_scale, void* y, void* workspace, size_t workspace_bytes,
                          void* stream) {
  lwl::g_err[0] = 0;
  int st = linear_common(true, dtype, x, tokens, in_features, out_features, latent, latent_size, layers, y, workspace,
                         workspace_bytes);
  if (st) return st;
  if ((reinterpret_cast<uintptr_t>(in_gain) & 3) || (reinterpret_cast<uintptr_t>(out_gain) & 1) ||
      (reinterpret_cast<uintptr_t>(bias) & 1) || (reinterpret_cast<uintptr_t>(weight_offset) & 3) ||
      (reinterpret_cast<uintptr_t>(base) & 15)) {
    lwl::set_error("gain and bias vectors must be aligned bf16 arrays (in_gain: 4 bytes), weight_offset an fp32, "
                   "base 16-byte aligned");
    return LWL_ERR_UNSUPPORTED;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LWL_CUDA_TRY(cudaMemsetAsync(workspace, 0, 16, s));
  const lwl::LinExtras ex{bias, out_gain, in_gain, weight_offset, base, base ? base_scale : 1.0f};
  int rc = lwl::tc_linear_launch(true, x, (int)tokens, (int)in_features, (int)out_features, latent, latent_size,
                                 layers, seed, weight_scale, nullptr, y, reinterpret_cast<int*>(workspace), s, &ex);
  if (rc) {
    lwl::set_error("tcgen05 linear launch failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  return LWL_OK;
}

int lwl_tc_linear_dense(const void* x, int64_t tokens, int64_t in_features, const void* w, int64_t out_features,
                        void* y, void* workspace, size_t workspace_bytes, void* stream) {
  lwl::g_err[0] = 0;
  int st = linear_common(false, LWL_BF16, x, tokens, in_features, out_features, nullptr, 1, 1, y, workspace,
                         workspace_bytes);
  if (st) return st;
  if (!w) {
    lwl::set_error("null weight pointer");
    return LWL_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  LWL_CUDA_TRY(cudaMemsetAsync(workspace, 0, 16, s));
  int rc = lwl::tc_linear_launch(false, x, (int)tokens, (int)in_features, (int)out_features, nullptr, 1, 1, 0, 1.0f,
                                 w, y, reinterpret_cast<int*>(workspace), s);
  if (rc) {
    lwl::set_error("tcgen05 linear launch failed (%d): %s", rc, cudaGetErrorString(cudaGetLastError()));
    return LWL_ERR_CUDA;
  }
  return LWL_OK;
}

int lwl_fht_launch_count(int dtype, int64_t latent_size, int64_t size, int layers, int64_t start, int64_t stop,
                         int backward, unsigned flags) {
  if (lwl::validate_fht(dtype, latent_size, size, layers, start, stop) != LWL_OK) return -1;
  if (stop == start) return 0;
  if (lwl::fhts_supported(dtype, latent_size, backward != 0, layers, flags)) return backward ? 2 : 1;
  if (!backward && lwl::mma_forward_supported(dtype, latent_size, flags)) return 1;
  if (!backward && lwl::mma16_forward_supported(dtype, latent_size, flags)) return 1;
  if (backward && lwl::mma_backward_supported(dtype, latent_size, flags)) return 2;
  if (backward && lwl::mma16_backward_supported(dtype, latent_size, flags)) return 2;
  lwl::FhtArgs a;
  std::memset(&a, 0, sizeof(a));
  a.dtype = dtype;
  a.backward = backward != 0;
  a.latent_size = latent_size;
  a.size = size;
  a.layers = layers;
  a.start = start;
  a.stop = stop;
  a.flags = flags;
  if (lwl::fht32_supported(dtype, latent_size, backward != 0, flags)) return lwl::fht32_launches(a);
  lwl::FhtPlan plan;
  lwl::plan_fht(a, plan);
  return plan.nlaunch + (backward ? 1 : 0);
}

}  // extern "C"
