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
//    first call made on each device, with that device current, and cached;
//    make that first call before any stream capture.
//  * nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>
#include <stdio.h>

#include "q3_common.cuh"

static __device__ __align__(256) unsigned long long g_noalloc_argmax_keys[Q3_NOALLOC_ARGMAX_MAX_ROWS];

namespace {

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once).
int scratch_on_current_device(void **out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) return Q3_ERR_CAPACITY;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_scratch[dev]) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_argmax_keys);
    if (e != cudaSuccess || !p) {
      q3h::set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
      return Q3_ERR_CUDA;
    }
    g_scratch[dev] = p;
  }
  *out = g_scratch[dev];
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
