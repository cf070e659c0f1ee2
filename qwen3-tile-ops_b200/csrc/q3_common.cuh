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
#include "exp2_t256_table.inc"
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
//
// exp2_cr_libm: y = exp2 in double (CUDA libm, max 1 ulp); RN_f32(y) equals
// RN_f32(2^x) unless y lies within 2^-47*y of a midpoint between adjacent
// float32 values; those inputs are in the table made by gen_exp2_table.py
// (every float32 input whose 2^x is within 2^-46 of a midpoint, resolved at
// 200 bits).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float exp2_cr_libm(float x) {
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

// 2^(i/64), i = 0..63, correctly rounded to double (computed at 300 bits).
static __device__ const unsigned long long g_exp2_frac64[64] = {
    0x3ff0000000000000ull, 0x3ff02c9a3e778061ull, 0x3ff059b0d3158574ull, 0x3ff0874518759bc8ull,
    0x3ff0b5586cf9890full, 0x3ff0e3ec32d3d1a2ull, 0x3ff11301d0125b51ull, 0x3ff1429aaea92de0ull,
    0x3ff172b83c7d517bull, 0x3ff1a35beb6fcb75ull, 0x3ff1d4873168b9aaull, 0x3ff2063b88628cd6ull,
    0x3ff2387a6e756238ull, 0x3ff26b4565e27cddull, 0x3ff29e9df51fdee1ull, 0x3ff2d285a6e4030bull,
    0x3ff306fe0a31b715ull, 0x3ff33c08b26416ffull, 0x3ff371a7373aa9cbull, 0x3ff3a7db34e59ff7ull,
    0x3ff3dea64c123422ull, 0x3ff4160a21f72e2aull, 0x3ff44e086061892dull, 0x3ff486a2b5c13cd0ull,
    0x3ff4bfdad5362a27ull, 0x3ff4f9b2769d2ca7ull, 0x3ff5342b569d4f82ull, 0x3ff56f4736b527daull,
    0x3ff5ab07dd485429ull, 0x3ff5e76f15ad2148ull, 0x3ff6247eb03a5585ull, 0x3ff6623882552225ull,
    0x3ff6a09e667f3bcdull, 0x3ff6dfb23c651a2full, 0x3ff71f75e8ec5f74ull, 0x3ff75feb564267c9ull,
    0x3ff7a11473eb0187ull, 0x3ff7e2f336cf4e62ull, 0x3ff82589994cce13ull, 0x3ff868d99b4492edull,
    0x3ff8ace5422aa0dbull, 0x3ff8f1ae99157736ull, 0x3ff93737b0cdc5e5ull, 0x3ff97d829fde4e50ull,
    0x3ff9c49182a3f090ull, 0x3ffa0c667b5de565ull, 0x3ffa5503b23e255dull, 0x3ffa9e6b5579fdbfull,
    0x3ffae89f995ad3adull, 0x3ffb33a2b84f15fbull, 0x3ffb7f76f2fb5e47ull, 0x3ffbcc1e904bc1d2ull,
    0x3ffc199bdd85529cull, 0x3ffc67f12e57d14bull, 0x3ffcb720dcef9069ull, 0x3ffd072d4a07897cull,
    0x3ffd5818dcfba487ull, 0x3ffda9e603db3285ull, 0x3ffdfc97337b9b5full, 0x3ffe502ee78b3ff6ull,
    0x3ffea4afa2a490daull, 0x3ffefa1bee615a27ull, 0x3fff50765b6e4540ull, 0x3fffa7c1819e90d8ull};

// exp2_cr: the same correctly rounded result with a table-driven double
// evaluation (Tang's method for exp): x = k/64 + r with k = rint(64 x) and
// |r| <= 1/128 (both exact), 2^x = 2^(k >> 6) * 2^((k & 63)/64) * 2^r, and 2^r
// by its Taylor series in r ln2 to degree 5 (truncation < 2^-54).  The double
// result is within about 2^-51 (relative) of 2^x, so when its 29 bits below
// the float32 precision are more than 64 double ulps away from the midpoint
// pattern, rounding it to float32 rounds 2^x; otherwise the input is looked up
// in the hard-case table (every input within 2^-46 of a midpoint).  Results
// below 2^-125 (float32 subnormals) and non-finite inputs take exp2_cr_libm.
// `tab` is g_exp2_frac64 or a copy of it (kernels that evaluate many exps keep
// one in shared memory: the index varies per lane).
__device__ __forceinline__ float exp2_cr_t(float x, const unsigned long long *tab) {
  if (!(x >= -125.0f && x < 128.0f)) return x < -151.0f ? 0.0f : exp2_cr_libm(x);
  const float kf = rintf(__fmul_rn(x, 64.0f));                  // exact
  const int k = static_cast<int>(kf);
  const double r = __fma_rn(static_cast<double>(kf), -0.015625, static_cast<double>(x));  // exact
  double p = 0.0013333558146428443;                              // (ln2)^5 / 5!
  p = __fma_rn(p, r, 0.009618129107628477);                      // (ln2)^4 / 4!
  p = __fma_rn(p, r, 0.05550410866482158);                       // (ln2)^3 / 3!
  p = __fma_rn(p, r, 0.24022650695910072);                       // (ln2)^2 / 2!
  p = __fma_rn(p, r, 0.6931471805599453);                        // ln2
  p = __fma_rn(p, r, 1.0);
  const double t = __longlong_as_double(static_cast<long long>(tab[k & 63]));
  const long long yb =
      __double_as_longlong(__dmul_rn(t, p)) + (static_cast<long long>(k >> 6) << 52);
  const float res = __double2float_rn(__longlong_as_double(yb));
  const unsigned low = static_cast<unsigned>(yb) & 0x1FFFFFFFu;  // bits below float32 precision
  if (low - ((1u << 28) - 64u) <= 128u) return exp2_hard_lookup(x, res);
  return res;
}

// 2^(i/256), i = 0..255, correctly rounded to double (gen_exp2_t256_table.py).
static __device__ const unsigned long long g_exp2_t256[Q3_EXP2_T256_N] = Q3_EXP2_T256_INIT;

// exp2_cr_fast: the same correctly rounded result with fewer double operations
// (the prefill attention evaluates ~2e9 exps per layer; measured 10 % more
// exps per second than exp2_cr_t).  Callers evaluate it in batches through
// exp2_cr_fast_n where they can: a single evaluation is one long chain.  x = k/256 + r with k = rint(256 x) and
// |r| <= 2^-9, both exact in float32 (the rint by the 1.5 * 2^23 shifter);
// 2^x = 2^(k >> 8) * T * 2^r with T = 2^((k & 255)/256) from the table, and
// T * 2^r = T + (T r) * (ln2 + r (ln2^2/2 + r (ln2^3/6 + r ln2^4/24))) in
// double (truncation < 2^-54, the whole evaluation within a few double ulps).
// The rounding test on the double's 29 bits below float32 precision is
// exp2_cr_t's; flagged inputs and x outside [-125, 128) take exp2_cr_t.  The
// float32 result is scaled by 2^(k >> 8) through its exponent field (exact:
// the result is normal, or +inf when it rounds to 2^128).  Checked identical
// to exp2_cr_t on every float32 input (q3_exp2_selfcheck).
// `tab` is g_exp2_t256 or a copy of it in shared memory (the index varies per
// lane: a shared copy serves a warp's lookups without the L1 tag traffic).
// The shifter's bit pattern u = 0x4B400000 + k gives k's low 8 bits (the table
// index) as u & 255 and (k >> 8) << 23 (the exponent step, mod 2^32) as
// (u << 15) & 0xFF800000, since 0x4B400000 is a multiple of 2^22.
__device__ __forceinline__ unsigned exp2_step_bits(unsigned ub) { return (ub << 15) & 0xFF800000u; }

__device__ __forceinline__ float exp2_cr_fast_t(float x, const unsigned long long *tab) {
  if (!(x >= -125.0f && x < 128.0f)) return exp2_cr_t(x, g_exp2_frac64);
  const float u = __fadd_rn(__fmul_rn(x, 256.0f), 12582912.0f);
  const float kf = __fsub_rn(u, 12582912.0f);
  const unsigned ub = __float_as_uint(u);
  const double r = static_cast<double>(__fmaf_rn(kf, -0.00390625f, x));   // exact
  double p = __fma_rn(0.009618129107628477, r, 0.05550410866482158);      // ln2^4/4!, ln2^3/3!
  p = __fma_rn(p, r, 0.24022650695910072);                                 // ln2^2/2!
  p = __fma_rn(p, r, 0.6931471805599453);                                  // ln2
  const double t = __longlong_as_double(static_cast<long long>(tab[ub & 255u]));
  const double y = __fma_rn(__dmul_rn(t, r), p, t);
  const unsigned low = static_cast<unsigned>(__double_as_longlong(y)) & 0x1FFFFFFFu;
  if (low - ((1u << 28) - 64u) <= 128u) return exp2_cr_t(x, g_exp2_frac64);
  return __uint_as_float(__float_as_uint(__double2float_rn(y)) + exp2_step_bits(ub));
}

// exp2_cr_fast_t of N values at once: every value takes the common path without
// a branch (so the N evaluations interleave: one chain after another would
// leave the double pipes waiting), inputs below -151 give 0 there as well, and
// when any value is of the rare rest -- x in [-151, -125), x >= 128 or NaN, or
// a double result near a float32 rounding midpoint -- all N are redone by
// exp2_cr_t afterwards (one flag instead of a mask: the redo is rare and
// exp2_cr_t is exact for every input).  Same results as exp2_cr_fast_t value by
// value.  NONPOS: the caller's inputs are <= 0, -inf or NaN (a softmax's
// s - max), so the upper end of the range needs no test.
template <int N, bool NONPOS = false>
__device__ __forceinline__ void exp2_cr_fast_n(const float (&x)[N], float (&y)[N],
                                               const unsigned long long *tab) {
  bool redo = false;
#pragma unroll
  for (int i = 0; i < N; ++i) {
    const float xi = x[i];
    const bool in = NONPOS ? xi >= -125.0f : (xi >= -125.0f && xi < 128.0f);
    const float xc = in ? xi : 0.0f;                      // keeps the arithmetic finite
    const float u = __fadd_rn(__fmul_rn(xc, 256.0f), 12582912.0f);
    const float kf = __fsub_rn(u, 12582912.0f);
    const unsigned ub = __float_as_uint(u);
    const double r = static_cast<double>(__fmaf_rn(kf, -0.00390625f, xc));   // exact
    double p = __fma_rn(0.009618129107628477, r, 0.05550410866482158);
    p = __fma_rn(p, r, 0.24022650695910072);
    p = __fma_rn(p, r, 0.6931471805599453);
    const double t = __longlong_as_double(static_cast<long long>(tab[ub & 255u]));
    const double yd = __fma_rn(__dmul_rn(t, r), p, t);
    const unsigned low = static_cast<unsigned>(__double_as_longlong(yd)) & 0x1FFFFFFFu;
    const bool hard = low - ((1u << 28) - 64u) <= 128u;
    const float fy = __uint_as_float(__float_as_uint(__double2float_rn(yd)) + exp2_step_bits(ub));
    const bool zero = xi < -151.0f;
    y[i] = zero ? 0.0f : fy;
    redo |= in ? hard : !zero;
  }
  if (redo) {
#pragma unroll
    for (int i = 0; i < N; ++i) y[i] = exp2_cr_t(x[i], g_exp2_frac64);
  }
}

__device__ __forceinline__ float exp2_cr_fast(float x) { return exp2_cr_fast_t(x, g_exp2_t256); }

__device__ __forceinline__ float exp2_cr(float x) { return exp2_cr_t(x, g_exp2_frac64); }

// exp as amulx(log2e) + aexp2 (ref_qwen3.py:27-29)
__device__ __forceinline__ float exp_ref(float x) {
  return exp2_cr(__fmul_rn(x, __uint_as_float(kLog2eBits)));
}
__device__ __forceinline__ float exp_ref_fast(float x) {
  return exp2_cr_fast(__fmul_rn(x, __uint_as_float(kLog2eBits)));
}
__device__ __forceinline__ float exp_ref_fast_t(float x, const unsigned long long *tab) {
  return exp2_cr_fast_t(__fmul_rn(x, __uint_as_float(kLog2eBits)), tab);
}
// exp(v[i]) in place for N values (exp_ref_fast_t value by value); NONPOS as
// for exp2_cr_fast_n (log2(e) v keeps the sign of v)
template <int N, bool NONPOS = false>
__device__ __forceinline__ void exp_ref_fast_n(float (&v)[N], const unsigned long long *tab) {
  float x[N];
#pragma unroll
  for (int i = 0; i < N; ++i) x[i] = __fmul_rn(v[i], __uint_as_float(kLog2eBits));
  exp2_cr_fast_n<N, NONPOS>(x, v, tab);
}

// rne(x / scale) saturated to +-127, NaN -> 0 (ref_qwen3.py:69-76).  The
// quotient is clamped to [-127, 127] in float and rounded to an integer by the
// 1.5 * 2^23 shifter: ties to even, as rint, and clamping to integer bounds
// before the rounding gives what clamping after it does.  No float -> int
// conversion runs (those issue on a narrow pipe).
__device__ __forceinline__ int quant1_from_quotient(float q) {
  const float c = fminf(fmaxf(q, -127.0f), 127.0f);
  const int v = __float_as_int(__fadd_rn(c, 12582912.0f)) - 0x4B400000;
  return q != q ? 0 : v;                 // (selects, no branch)
}
__device__ __forceinline__ int quant1(float x, float scale) {
  return quant1_from_quotient(__fdiv_rn(x, scale));
}

// quant1 of a value x under the scale s = RN(amax * RN(1/127)) of an absolute
// maximum amax >= |x| (every requantisation of the path has this form), from
// a correctly rounded reciprocal r = 1/s shared by the values of the scale and
// Markstein's correction: with r within half an ulp of 1/s and q0 = x r within
// one ulp of x/s, the residual e = x - q0 s is exact and fma(e, r, q0) is the
// correctly rounded x/s (P. Markstein, IBM J. Res. Dev. 34(1), 1990).  The
// caller keeps s within [2^-100, 2^100] (quant_rcp_ok: s is normal, so its two
// roundings are relative errors below 2^-24 each, and e does not underflow).
// Then |x/s| <= 127 / (1 - 2^-24)^2 < 127.5, so the rounded quotient needs no
// clamp to +-127 and cannot overflow; it is rounded to an integer by the
// 1.5 * 2^23 shifter (ties to even, as rint).  NaN x gives 0.  Equal to
// quant1(x, s) for every such x (q3_quant_selfcheck).
__device__ __forceinline__ int quant1_rcp_absmax(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q0, s, x);
  const float q = __fmaf_rn(e, r, q0);
  const int v = __float_as_int(__fadd_rn(q, 12582912.0f)) - 0x4B400000;
  return x != x ? 0 : v;
}
__host__ __device__ __forceinline__ bool quant_rcp_ok(float s) {
  return s >= 7.888609052210118e-31f && s <= 1.2676506002282294e30f;   // 2^-100 .. 2^100
}
// quant1 of N values under the scale of their absolute maximum (s =
// RN(amax * kInv127), amax = max |x[i]| over these values and any others of
// the scale; a warp-uniform choice): from one reciprocal where quant_rcp_ok
// allows it, else from the quotients.
template <int N>
__device__ __forceinline__ void quant_n_absmax(const float (&x)[N], float s, int (&q)[N]) {
  if (quant_rcp_ok(s)) {
    const float r = __frcp_rn(s);
#pragma unroll
    for (int i = 0; i < N; ++i) q[i] = quant1_rcp_absmax(x[i], s, r);
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) q[i] = quant1(x[i], s);
  }
}

// The codes of quant_n_absmax for N values (N a multiple of 4) packed four to a
// word, code i in byte i % 4 of word i / 4.  The float bits of q + 1.5 * 2^23
// carry the code in their low byte (0x4B400000 has a zero low byte), so byte
// permutes gather them without the subtraction; a NaN among the values (one
// check of their sum: NaN propagates, and a false alarm only costs time) sends
// this thread through the per-value selects that give NaN the code 0.
template <int N>
__device__ __forceinline__ void quant_pack_absmax(const float (&x)[N], float s, uint32_t (&w)[N / 4]) {
  uint32_t b[N];
  if (quant_rcp_ok(s)) {
    const float r = __frcp_rn(s);
    float chk = 0.0f;
#pragma unroll
    for (int i = 0; i < N; ++i) {
      const float q0 = __fmul_rn(x[i], r);
      const float e = __fmaf_rn(-q0, s, x[i]);
      b[i] = __float_as_uint(__fadd_rn(__fmaf_rn(e, r, q0), 12582912.0f));
      chk = __fadd_rn(chk, x[i]);
    }
    if (chk != chk) {
#pragma unroll
      for (int i = 0; i < N; ++i) b[i] = x[i] != x[i] ? 0u : b[i];
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) b[i] = static_cast<uint32_t>(quant1(x[i], s));
  }
#pragma unroll
  for (int c = 0; c < N / 4; ++c)
    w[c] = __byte_perm(__byte_perm(b[4 * c], b[4 * c + 1], 0x0040),
                       __byte_perm(b[4 * c + 2], b[4 * c + 3], 0x0040), 0x5410);
}

// 1/sqrt with two roundings (ref_qwen3.py:37-38)
__device__ __forceinline__ float rsqrt_ref(float x) {
  return __frcp_rn(__fsqrt_rn(x));
}

// max as np.where(b > a, b, a) (ref_qwen3.py:57-58)
__device__ __forceinline__ float max_ref(float a, float b) { return b > a ? b : a; }

// Warp adjacent-pair reduction tree (ref_qwen3.py:41-63): a butterfly over
// lanes 1,2,4,8,16 pairs exactly the reference's tree when absent lanes hold
// the identity (0); every lane gets the result.
__device__ __forceinline__ float warp_tree_sum(float v) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// Maximum over the warp (every lane gets it) in one redux.sync (the sm_100a
// float form).  A maximum does not depend on the order of comparisons: callers
// take maxima of magnitudes, or of scores whose maximum only enters as
// exp(s - m) and m == m' tests, where the sign of a zero maximum cannot show.
// NaN inputs are passed over, as by fmaxf.
__device__ __forceinline__ float warp_tree_max(float v) {
  float r;
  asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(r) : "f"(v));
  return r;
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

// Streaming multiprocessors of the current device (cached per device).
inline int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

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
enum TimerFamily { TIMER_NONE = 0, TIMER_ATTENTION = 1, TIMER_GEMM = 2, TIMER_EXCHANGE = 3 };
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
