// noalloc.cu -- latent-gradient entry point that needs no caller-provided workspace.
//
// lwl_fht_backward normally asks the caller for a workspace holding one fp32
// partial gradient per CTA.  Some callers cannot hand one over: code that
// runs where no device allocator is reachable (a plugin invoked from a host
// runtime that owns all device memory, or a callback that must not allocate
// because allocation would synchronise or fail under its memory policy).
// lwl_fht_backward_noalloc serves them by keeping those partials in a fixed
// array that lives in the library's own device memory image.
//
// Limits and sharing rules (also stated in include/lwl_b200.h):
//  * padded block size up to 2^14 (the single-launch backward layout); the
//    partials use at most kScratchFloats floats (8 MiB), so the number of
//    CTAs is capped at kScratchFloats / latent_size;
//  * every GPU that loads the library holds the 8 MiB array until exit;
//  * all calls on a device share the one array and it keeps the last call's
//    contents; each call rewrites every partial it reads, so nothing needs
//    clearing, but calls whose executions overlap on the GPU (different
//    streams without ordering) race on it and give wrong results;
//  * the device address of the array is looked up once per device on that
//    device's first call (cudaGetSymbolAddress, with that device current) and
//    kept for the life of the process, so it is not valid across a
//    cudaDeviceReset (or any other teardown of the device's primary context):
//    a process that resets a device must not call this entry point on it
//    again;
//  * the partials are summed by the fp32 tile engine for every dtype, so for
//    bf16 / fp16 the result equals lwl_fht_backward's up to rounding (that
//    entry point may take the tensor-core path, which rounds differently).
#include <mutex>

#include "fht_engine.h"
#include "lwl_b200.h"
#include "lwl_common.cuh"

namespace lwl {
namespace {

constexpr int64_t kScratchFloats = int64_t(1) << 21;  // 8 MiB of fp32 partials
constexpr int kMaxDevices = 64;

static __device__ __align__(256) float g_backward_scratch[kScratchFloats];

std::mutex g_scratch_mutex;
float* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_backward_scratch on the current device (looked up once).
int scratch_for_current_device(float** out) {
  int dev = 0;
  LWL_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("device ordinal %d beyond the %d devices this entry point tracks", dev, kMaxDevices);
    return LWL_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_backward_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_error("cudaGetSymbolAddress for the backward scratch array failed: %s", cudaGetErrorString(e));
      return LWL_ERR_CUDA;
    }
    g_scratch_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_ptr[dev];
  return LWL_OK;
}

}  // namespace
}  // namespace lwl

extern "C" int lwl_fht_backward_noalloc(int dtype, const void* grad_out, int64_t latent_size, int64_t size,
                                        int layers, uint64_t seed, int64_t start, int64_t stop, void* grad_latent,
                                        unsigned flags, void* stream) {
  using namespace lwl;
  clear_error();
  // bad arguments are rejected before any device work
  if (dtype != LWL_F32 && dtype != LWL_BF16 && dtype != LWL_F16) {
    set_error("unsupported dtype code %d (expected 0=fp32, 1=bf16, 2=fp16)", dtype);
    return LWL_ERR_INVALID;
  }
  if (latent_size <= 0 || size <= 0 || layers < 1 || layers > 3 || !(0 <= start && start <= stop && stop <= size)) {
    set_error("invalid arguments: latent_size %lld, size %lld, layers %d, slice [%lld, %lld)",
              (long long)latent_size, (long long)size, layers, (long long)start, (long long)stop);
    return LWL_ERR_INVALID;
  }
  if (next_pow2(latent_size) > (int64_t(1) << kWholeBlockMaxLogBwd)) {
    set_error("lwl_fht_backward_noalloc supports padded block sizes up to 2^%d (got %lld); "
              "use lwl_fht_backward with a workspace",
              kWholeBlockMaxLogBwd, (long long)next_pow2(latent_size));
    return LWL_ERR_UNSUPPORTED;
  }
  if ((stop > start && !grad_out) || !grad_latent) {
    set_error("null data pointer");
    return LWL_ERR_INVALID;
  }
  float* scratch = nullptr;
  int st = scratch_for_current_device(&scratch);
  if (st != LWL_OK) return st;

  FhtArgs a;
  a.dtype = dtype;
  a.backward = true;
  a.in = grad_out;
  a.out = grad_latent;
  a.latent_size = latent_size;
  a.size = size;
  a.layers = layers;
  a.seed = seed;
  a.start = start;
  a.stop = stop;
  a.flags = flags;
  FhtPlan plan;
  plan_fht(a, plan);
  if (plan.nblocks > 0) {
    // one partial row of latent_size floats per CTA; cap the CTA count to the array
    int64_t max_rows = kScratchFloats / latent_size;
    if (plan.launches[0].grid > max_rows) plan.launches[0].grid = (int)max_rows;
    plan.partial_rows = plan.launches[0].grid;
    plan.ws_bytes = size_t(plan.partial_rows) * size_t(latent_size) * 4;
  }
  a.workspace = scratch;
  a.workspace_bytes = size_t(kScratchFloats) * 4;
  return run_fht(a, plan, reinterpret_cast<cudaStream_t>(stream));
}
