// Shared device numerics and host helpers for the Qwen3 w8a8 path.
//
// Every float32 step that the reference rounds (tools/ref_qwen3.py) is written
// with an explicit round-to-nearest intrinsic (__fmul_rn, __fadd_rn, ...), so
// no multiply-add is ever contracted; the library is also built with
// -fmad=false.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/q3_ops.h"
#include "exp2_hard_table.inc"

namespace q3 {

// tools/ref_qwen3.py:18-21, kernels/config.h:63-68
constexpr unsigned kLog2eBits = 0x3FB8AA3Bu;   // 1.4426950216293335f
constexpr float kInv127 = 1.0f / 127.0f;
constexpr float kEps = 1e-6f;
constexpr float kNegFltMax = -3.402823466e38f;
constexpr float kNegInf = -__builtin_huge_valf();

// Hard-case table of gen_exp2_table.py (one copy per translation unit).
static __device__ const unsigned int g_exp2_hard_x[Q3_EXP2_HARD_COUNT] = Q3_EXP2_HARD_X_INIT;
static __device__ const unsigned int g_exp2_hard_y[Q3_EXP2_HARD_COUNT] = Q3_EXP2_HARD_Y_INIT;

// Binary search of the table (sorted by float32 bit pattern).
static __device__ __noinline__ float exp2_hard_lookup(float x, float fallback) {
  const unsigned key = __float_as_uint(x);
  int lo = 0, hi = Q3_EXP2_HARD_COUNT - 1;
  while (lo <= hi) {
    const int mid = (lo + hi) >> 1;
    const unsigned v = g_exp2_hard_x[mid];
    if (v == key) return __uint_as_float(g_exp2_hard_y[mid]);
    if (v < key) lo = mid + 1; else hi = mid - 1;
  }
  return fallback;
}

// ---------------------------------------------------------------------------
// Correctly rounded float32 exp2.
// y = exp2 in double (CUDA libm, max 1 ulp); RN_f32(y) equals RN_f32(2^x)
// unless y lies within 2^-47*y of a midpoint between adjacent float32 values;
// those inputs are in the table made by gen_exp2_table.py (every float32 input
// whose 2^x is within 2^-46 of a midpoint, resolved at 200 bits).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp2_cr(float x) {
  const double y = exp2(static_cast<double>(x));
  const float r = __double2float_rn(y);
  const unsigned rb = __float_as_uint(r);
  if (rb >= 0x7f800000u) return r;                 // +inf (x >= 128)
  const double rd = static_cast<double>(r);
  const unsigned nb = (y >= rd) ? rb + 1u : (rb ? rb - 1u : rb);
  const double mid = (rd + static_cast<double>(__uint_as_float(nb))) * 0.5;
  if (fabs(y - mid) <= y * 7.105427357601002e-15 /* 2^-47 */ && y > 0.0)
    return exp2_hard_lookup(x, r);
  return r;
}

// exp as amulx(log2e) + aexp2 (ref_qwen3.py:27-29)
__device__ __forceinline__ float exp_ref(float x) {
  return exp2_cr(__fmul_rn(x, __uint_as_float(kLog2eBits)));
}

// rne(x / scale) saturated to +-127, NaN -> 0 (ref_qwen3.py:69-76)
__device__ __forceinline__ int quant1(float x, float scale) {
  const float q = __fdiv_rn(x, scale);
  if (q != q) return 0;
  int v = __float2int_rn(q);
  v = v > 127 ? 127 : v;
  v = v < -127 ? -127 : v;
  return v;
}

// 1/sqrt with two roundings (ref_qwen3.py:37-38)
__device__ __forceinline__ float rsqrt_ref(float x) {
  return __fdiv_rn(1.0f, __fsqrt_rn(x));
}

// max as np.where(b > a, b, a) (ref_qwen3.py:57-58)
__device__ __forceinline__ float max_ref(float a, float b) { return b > a ? b : a; }

// Warp adjacent-pair reduction trees (ref_qwen3.py:41-63): a butterfly over
// lanes 1,2,4,8,16 pairs exactly the reference's tree when absent lanes hold
// the identity (0 for sums, -inf for maxima); every lane gets the result.
__device__ __forceinline__ float warp_tree_sum(float v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_tree_max(float v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = fmaxf(v, w);
  }
  return v;
}

// Programmatic dependent launch: let the next kernel of the stream start its
// prologue (launch_dependents), and wait until every earlier kernel of the
// stream has finished and its writes are visible (wait).  Both are no-ops for a
// kernel launched without the programmatic-serialisation attribute.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// int32 -> float32 for |v| < 2^22 with two full-rate ops (exact).
__device__ __forceinline__ float i2f_small(int v) {
  return __fsub_rn(__int_as_float(v + 0x4B400000), 12582912.0f);
}

}  // namespace q3

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
namespace q3h {

const char *set_cuda_error(cudaError_t e);
void set_error_message(const char *msg);   // text returned by q3_last_cuda_error
int launch_argmax_row(const float *row, int n, int32_t *out_id, cudaStream_t s);
void count_launch();

// Every kernel launch of the library is followed by this check (it also
// counts the launch for q3_launch_count).
inline int launch_status() {
  count_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  return Q3_OK;
}

// Launch with programmatic stream serialisation when `pdl` is set: the kernel
// may start while the previous kernel of the stream is still running, so it
// must call pdl_wait() before it reads what earlier kernels wrote or writes
// anything they might still read.
template <typename... KArgs, typename... Args>
inline int launch_ex(bool pdl, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                     cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) {
    count_launch();
    cudaGetLastError();
    set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  return launch_status();
}

// Benchmark timing hook (q3_timer_attach): events around launches of a family.
enum TimerFamily { TIMER_NONE = 0, TIMER_ATTENTION = 1, TIMER_GEMM = 2 };
void timer_begin(int family, cudaStream_t s);
void timer_end(int family, cudaStream_t s);

inline int dt_size(uint8_t dt) { return (dt == Q3_DT_I8 || dt == Q3_DT_U8) ? 1 : 4; }

// A view usable by the kernels: non-null, dtype as expected, elements
// contiguous within a row (col_bytes == element size), aligned to `align`
// bytes at its base and in its row stride (when it has more than one row).
inline int check_view(const q3_view *v, uint8_t dtype, int align = 4) {
  if (!v || !v->data) return Q3_ERR_NULL;
  if (v->dtype != dtype) return Q3_ERR_DTYPE;
  if (v->col_bytes != dt_size(dtype)) return Q3_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(v->data) % align) return Q3_ERR_ALIGN;
  if (v->rows > 1 && (v->row_bytes <= 0 || v->row_bytes % align)) return Q3_ERR_ALIGN;
  return Q3_OK;
}

}  // namespace q3h

#define Q3_TRY(expr)                 \
  do {                               \
    int _st = (expr);                \
    if (_st != Q3_OK) return _st;    \
  } while (0)
