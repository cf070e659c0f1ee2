// lm_head + argmax for callers that cannot allocate device memory.
//
// q3_gemm_nt_group_argmax needs a little scratch: one packed 64-bit
// (value, index) key per row, which the per-tile row maxima are folded into
// with atomicMax before the result is merged into (best, bidx).  Normally the
// caller passes that scratch as a workspace.  Some callers cannot call
// cudaMalloc at all: a host that hands this library one fixed, pre-planned
// device buffer and owns no device allocator (the way the reference's guest
// program owns exactly one blob), or a serving loop that must not call
// cudaMalloc/cudaFree on its hot path because those calls can synchronize the
// whole device.  q3_gemm_nt_group_argmax_noalloc serves them: the scratch
// lives in a file-scope device array of this file instead.
//
// What a caller must know:
//  * at most Q3_NOALLOC_ARGMAX_MAX_ROWS rows per call (8 bytes of scratch per
//    row); more rows return Q3_ERR_CAPACITY before anything is launched;
//  * the array exists once per device for the life of the process and every
//    call uses it; each call zeroes the keys of its own rows first, but two
//    calls that overlap on the GPU (for example on two streams) race on it;
//  * the array's device address is looked up with cudaGetSymbolAddress on the
//    first call made on each device, with that device current, and cached
//    together with the identity of the device's context; a call that finds a
//    different context (after cudaDeviceReset, for example) looks it up again.
//    Make the first call on a device before any stream capture.
//  * nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda.h>
#include <mutex>
#include <stdio.h>

#include "q3_common.cuh"

static __device__ __align__(256) unsigned long long g_noalloc_argmax_keys[Q3_NOALLOC_ARGMAX_MAX_ROWS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
struct Cached {
  unsigned long long ctx_id;   // cuCtxGetId of the context the address belongs to
  void *ptr;
};
Cached g_scratch[kMaxDevices] = {};

// Unique id of the calling thread's current CUDA context (false if none).
// The driver functions are fetched through the runtime, so the library does
// not link libcuda directly and still loads on a host without a GPU driver.
bool current_context_id(unsigned long long *id) {
  using GetCurrent = CUresult (*)(CUcontext *);
  using GetId = CUresult (*)(CUcontext, unsigned long long *);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  if (!get_current || !get_id) {
    void *f = nullptr, *g = nullptr;
    cudaDriverEntryPointQueryResult q1, q2;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q1) != cudaSuccess ||
        q1 != cudaDriverEntryPointSuccess ||
        cudaGetDriverEntryPoint("cuCtxGetId", &g, cudaEnableDefault, &q2) != cudaSuccess ||
        q2 != cudaDriverEntryPointSuccess)
      return false;
    get_current = reinterpret_cast<GetCurrent>(f);
    get_id = reinterpret_cast<GetId>(g);
  }
  CUcontext ctx = nullptr;
  return get_current(&ctx) == CUDA_SUCCESS && ctx && get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of the scratch array in the current device's context.  The
// lookup is cached per device and redone when the context changed: a device
// reset unloads this module, and the array may come back at another address.
int scratch_on_current_device(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    char msg[128];
    snprintf(msg, sizeof msg,
             "q3_gemm_nt_group_argmax_noalloc: device %d is beyond the %d devices this entry "
             "point serves", dev, kMaxDevices);
    q3h::set_error_message(msg);
    return Q3_ERR_CAPACITY;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  Cached &c = g_scratch[dev];
  unsigned long long ctx_id = 0;
  if (c.ptr && current_context_id(&ctx_id) && c.ctx_id == ctx_id) {
    *out = c.ptr;
    return Q3_OK;
  }
  void *p = nullptr;
  e = cudaGetSymbolAddress(&p, g_noalloc_argmax_keys);   // initialises the context if needed
  if (e != cudaSuccess || !p) {
    q3h::set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    return Q3_ERR_CUDA;
  }
  if (!current_context_id(&ctx_id)) {
    q3h::set_error_message("q3_gemm_nt_group_argmax_noalloc: no current CUDA context");
    return Q3_ERR_CUDA;
  }
  c = Cached{ctx_id, p};
  *out = c.ptr;
  return Q3_OK;
}

}  // namespace

extern "C" int q3_gemm_nt_group_argmax_noalloc(const q3_view *a, const q3_view *a_scale,
                                               const q3_view *b, const q3_view *b_scale,
                                               float *best, int32_t *bidx, uint32_t group_k,
                                               void *stream) {
  if (!a) return Q3_ERR_NULL;
  if (a->rows > Q3_NOALLOC_ARGMAX_MAX_ROWS) {
    char msg[160];
    snprintf(msg, sizeof msg,
             "q3_gemm_nt_group_argmax_noalloc: %u rows exceed the built-in scratch of %d rows",
             a->rows, Q3_NOALLOC_ARGMAX_MAX_ROWS);
    q3h::set_error_message(msg);
    return Q3_ERR_CAPACITY;
  }
  void *scratch = nullptr;
  Q3_TRY(scratch_on_current_device(&scratch));
  return q3_gemm_nt_group_argmax(a, a_scale, b, b_scale, best, bidx, group_k, scratch,
                                 sizeof(g_noalloc_argmax_keys), stream);
}
