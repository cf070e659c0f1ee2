// Row-wise operators of the Qwen3 w8a8 path: RMSNorm, per-group int8
// quantisation, embedding + RMSNorm, paged KV scatter, logits argmax.
// All are HBM-bound; one warp owns one row (or one row-group), which makes
// the reference's 32-column block trees map onto warp butterflies.
#include <stdio.h>

#include "q3_common.cuh"

namespace q3 {

// ---------------------------------------------------------------------------
// kernels/rmsnorm.h:34-81 ; tools/ref_qwen3.py:161-177
// ss = sum over 32-column blocks, in order, of tree(x^2); r = 1/sqrt(ss*inv+eps);
// out = (x * r) * w.  out may alias x.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float row_sumsq_blocks(const float *x, int cols, int lane) {
  float ss = 0.0f;
  for (int c0 = 0; c0 < cols; c0 += 32) {
    const int c = c0 + lane;
    const float v = c < cols ? x[c] : 0.0f;
    ss = __fadd_rn(ss, warp_tree_sum(__fmul_rn(v, v)));
  }
  return ss;
}

__global__ void k_rmsnorm_rows(const char *__restrict__ x, long x_rb,
                               const char *__restrict__ w, long w_es,
                               char *out, long out_rb, int rows, int cols, float inv) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const float *xr = reinterpret_cast<const float *>(x + warp * x_rb);
  float *orow = reinterpret_cast<float *>(out + warp * out_rb);
  float ss = row_sumsq_blocks(xr, cols, lane);
  ss = __fmul_rn(ss, inv);
  ss = __fadd_rn(ss, kEps);
  const float r = rsqrt_ref(ss);
  for (int c = lane; c < cols; c += 32) {
    const float wv = *reinterpret_cast<const float *>(w + c * w_es);
    orow[c] = __fmul_rn(__fmul_rn(xr[c], r), wv);
  }
}

// ---------------------------------------------------------------------------
// kernels/quant.h:89-138 ; tools/ref_qwen3.py:86-97
// one warp per (row, group): scale = absmax * (1/127); q = sat(rne(x/scale))
// ---------------------------------------------------------------------------
__global__ void k_quant_rows_heads(const char *__restrict__ x, long x_rb, char *q, long q_rb,
                                   char *s, long s_rb, int rows, int cols, int group) {
  const int groups = (cols + group - 1) / group;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows * groups) return;
  const int r = warp / groups, g = warp % groups;
  const int c0 = g * group;
  const int gc = min(group, cols - c0);
  const float *xr = reinterpret_cast<const float *>(x + r * x_rb) + c0;
  float m = 0.0f;
  for (int c = lane; c < gc; c += 32) m = fmaxf(m, fabsf(xr[c]));
  m = warp_tree_max(m);
  const float scale = __fmul_rn(m, kInv127);
  int8_t *qr = reinterpret_cast<int8_t *>(q + r * q_rb) + c0;
  for (int c = lane; c < gc; c += 32) qr[c] = static_cast<int8_t>(quant1(xr[c], scale));
  if (lane == 0) reinterpret_cast<float *>(s + r * s_rb)[g] = scale;
}

// ---------------------------------------------------------------------------
// kernels/embedding.h:99-168 ; tools/ref_qwen3.py:292-296
// x = f32(table[id]) * scale[id] (written to tmp), then the RMSNorm of x.
// ---------------------------------------------------------------------------
__global__ void k_embedding_rmsnorm(const int8_t *__restrict__ table, long t_rb,
                                    const char *__restrict__ tscale, long ts_es,
                                    const char *__restrict__ ids, long ids_es,
                                    char *tmp, long tmp_rb, const char *__restrict__ w,
                                    long w_es, char *out, long out_rb, int rows, int cols,
                                    float inv) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int id = *reinterpret_cast<const int *>(ids + warp * ids_es);
  const float es = *reinterpret_cast<const float *>(tscale + static_cast<long>(id) * ts_es);
  const int8_t *er = table + static_cast<long>(id) * t_rb;
  float *xr = reinterpret_cast<float *>(tmp + warp * tmp_rb);
  float ss = 0.0f;
  for (int c0 = 0; c0 < cols; c0 += 32) {
    const int c = c0 + lane;
    float v = 0.0f;
    if (c < cols) {
      v = __fmul_rn(static_cast<float>(er[c]), es);
      xr[c] = v;
    }
    ss = __fadd_rn(ss, warp_tree_sum(__fmul_rn(v, v)));
  }
  ss = __fmul_rn(ss, inv);
  ss = __fadd_rn(ss, kEps);
  const float r = rsqrt_ref(ss);
  float *orow = reinterpret_cast<float *>(out + warp * out_rb);
  for (int c = lane; c < cols; c += 32) {
    const float wv = *reinterpret_cast<const float *>(w + c * w_es);
    orow[c] = __fmul_rn(__fmul_rn(xr[c], r), wv);
  }
}

// ---------------------------------------------------------------------------
// kernels/kv_pages.h:63-131 — copy K/V rows (+ per-head scales) into pages.
// ---------------------------------------------------------------------------
struct ScatterRow {
  const uint16_t *table;
  uint32_t token;
};
struct ScatterArgs {
  const char *k, *v, *ks, *vs;
  long k_rb, v_rb, ks_rb, vs_rb;
  char *pk, *pv, *pks, *pvs;
  uint32_t page_tokens, page_bytes, row_bytes, scale_page_bytes, scale_row_bytes;
  int rows, kv_dim, kv_heads;
};

__global__ void k_paged_kv_scatter(ScatterArgs a, const uint16_t *table, uint32_t start) {
  const int r = blockIdx.x;
  const uint32_t tok = start + r;
  const uint32_t page = table[tok / a.page_tokens], slot = tok % a.page_tokens;
  char *dk = a.pk + static_cast<size_t>(page) * a.page_bytes + slot * a.row_bytes;
  char *dv = a.pv + static_cast<size_t>(page) * a.page_bytes + slot * a.row_bytes;
  for (int c = threadIdx.x; c < a.kv_dim; c += blockDim.x) {
    dk[c] = a.k[r * a.k_rb + c];
    dv[c] = a.v[r * a.v_rb + c];
  }
  char *dks = a.pks + static_cast<size_t>(page) * a.scale_page_bytes + slot * a.scale_row_bytes;
  char *dvs = a.pvs + static_cast<size_t>(page) * a.scale_page_bytes + slot * a.scale_row_bytes;
  for (int h = threadIdx.x; h < a.kv_heads; h += blockDim.x) {
    reinterpret_cast<float *>(dks)[h] = reinterpret_cast<const float *>(a.ks + r * a.ks_rb)[h];
    reinterpret_cast<float *>(dvs)[h] = reinterpret_cast<const float *>(a.vs + r * a.vs_rb)[h];
  }
}

struct BatchTables {
  ScatterRow row[128];
};

__global__ void k_paged_kv_scatter_batch(ScatterArgs a, BatchTables t) {
  const int r = blockIdx.x;
  const uint32_t tok = t.row[r].token;
  const uint32_t page = t.row[r].table[tok / a.page_tokens], slot = tok % a.page_tokens;
  char *dk = a.pk + static_cast<size_t>(page) * a.page_bytes + slot * a.row_bytes;
  char *dv = a.pv + static_cast<size_t>(page) * a.page_bytes + slot * a.row_bytes;
  for (int c = threadIdx.x; c < a.kv_dim; c += blockDim.x) {
    dk[c] = a.k[r * a.k_rb + c];
    dv[c] = a.v[r * a.v_rb + c];
  }
  char *dks = a.pks + static_cast<size_t>(page) * a.scale_page_bytes + slot * a.scale_row_bytes;
  char *dvs = a.pvs + static_cast<size_t>(page) * a.scale_page_bytes + slot * a.scale_row_bytes;
  for (int h = threadIdx.x; h < a.kv_heads; h += blockDim.x) {
    reinterpret_cast<float *>(dks)[h] = reinterpret_cast<const float *>(a.ks + r * a.ks_rb)[h];
    reinterpret_cast<float *>(dvs)[h] = reinterpret_cast<const float *>(a.vs + r * a.vs_rb)[h];
  }
}

// ---------------------------------------------------------------------------
// src/main_big.cpp:300-322 ; tools/ref_qwen3.py:447-464
// per 32-column block: first index of the block maximum; across blocks the
// first block with the largest monotone key wins.  One CTA.
// ---------------------------------------------------------------------------
__device__ __forceinline__ unsigned mono_key(float v) {
  const unsigned b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void k_argmax_logits(const float *__restrict__ row, int n, int32_t *out_id) {
  __shared__ unsigned long long red[32];
  const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
  unsigned long long best = 0ull;
  for (int b0 = wid * 32; b0 < n; b0 += nw * 32) {
    const int c = b0 + lane;
    float v = c < n ? row[c] : kNegInf;
    int idx = c < n ? lane : 32;
    // first index of the maximum inside the block (np.argmax semantics)
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
    }
    const unsigned long long key =
        (static_cast<unsigned long long>(mono_key(v)) << 32) | (0xffffffffu - static_cast<unsigned>(b0 + idx));
    best = key > best ? key : best;
  }
  if (lane == 0) red[wid] = best;
  __syncthreads();
  if (wid == 0) {
    unsigned long long k = lane < nw ? red[lane] : 0ull;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
      k = ok > k ? ok : k;
    }
    if (lane == 0) *out_id = static_cast<int32_t>(0xffffffffu - static_cast<unsigned>(k & 0xffffffffu));
  }
}

// element-wise exp / exp2 over a 2-D f32 view (value ops)
__global__ void k_exp_rows(const char *__restrict__ x, long x_rb, char *out, long o_rb, int rows,
                           int cols, int base2) {
  const long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<long>(rows) * cols) return;
  const int r = static_cast<int>(i / cols), c = static_cast<int>(i % cols);
  const float v = reinterpret_cast<const float *>(x + r * x_rb)[c];
  reinterpret_cast<float *>(out + r * o_rb)[c] = base2 ? exp2_cr(v) : exp_ref(v);
}

}  // namespace q3

// ===========================================================================
// C ABI
// ===========================================================================
using namespace q3;
using namespace q3h;

namespace q3h {
static thread_local char g_err[256] = "";
const char *set_cuda_error(cudaError_t e) {
  snprintf(g_err, sizeof g_err, "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return g_err;
}
void set_error_message(const char *msg) { snprintf(g_err, sizeof g_err, "%s", msg); }
}  // namespace q3h

static inline long vec_stride(const q3_view *v) {
  // a [n][1] column (row_bytes = elem) or a [1][n] row (col_bytes = elem)
  return v->rows > 1 ? v->row_bytes : v->col_bytes;
}

extern "C" const char *q3_last_cuda_error(void) { return q3h::g_err; }

extern "C" int q3_device_check(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return Q3_ERR_CUDA;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, dev) != cudaSuccess) return Q3_ERR_CUDA;
  return (p.major == 10 && p.minor == 0) ? Q3_OK : Q3_ERR_ARCH;
}

extern "C" int q3_rmsnorm_rows(const q3_view *x, const q3_view *w, const q3_view *out,
                               float inv, void *stream) {
  Q3_TRY(check_view(x, Q3_DT_F32));
  Q3_TRY(check_view(out, Q3_DT_F32));
  if (!w || !w->data) return Q3_ERR_NULL;
  if (w->dtype != Q3_DT_F32) return Q3_ERR_DTYPE;
  if (out->rows < x->rows || out->cols < x->cols || w->rows * w->cols < x->cols)
    return Q3_ERR_SHAPE;
  if (x->rows == 0) return Q3_OK;
  const int threads = 256, wpb = threads / 32;
  k_rmsnorm_rows<<<(x->rows + wpb - 1) / wpb, threads, 0, (cudaStream_t)stream>>>(
      (const char *)x->data, x->row_bytes, (const char *)w->data, vec_stride(w),
      (char *)out->data, out->row_bytes, x->rows, x->cols, inv);
  return launch_status();
}

extern "C" int q3_quant_rows_heads(const q3_view *x, const q3_view *qi8, const q3_view *scale,
                                   uint32_t group_cols, void *stream) {
  Q3_TRY(check_view(x, Q3_DT_F32));
  Q3_TRY(check_view(qi8, Q3_DT_I8, 1));
  Q3_TRY(check_view(scale, Q3_DT_F32));
  if (group_cols == 0) return Q3_ERR_SHAPE;
  const uint32_t groups = (x->cols + group_cols - 1) / group_cols;
  if (qi8->rows < x->rows || qi8->cols < x->cols || scale->cols < groups ||
      (x->rows > 1 && scale->rows < x->rows))
    return Q3_ERR_SHAPE;
  if (x->rows == 0) return Q3_OK;
  const long warps = static_cast<long>(x->rows) * groups;
  const int threads = 256, wpb = threads / 32;
  k_quant_rows_heads<<<(warps + wpb - 1) / wpb, threads, 0, (cudaStream_t)stream>>>(
      (const char *)x->data, x->row_bytes, (char *)qi8->data, qi8->row_bytes,
      (char *)scale->data, scale->row_bytes, x->rows, x->cols, group_cols);
  return launch_status();
}

extern "C" int q3_embedding_rmsnorm_rows(const q3_view *table, const q3_view *scale,
                                         const q3_view *ids, const q3_view *tmp,
                                         const q3_view *w, const q3_view *out, float inv,
                                         void *stream) {
  Q3_TRY(check_view(table, Q3_DT_I8, 1));
  Q3_TRY(check_view(tmp, Q3_DT_F32));
  Q3_TRY(check_view(out, Q3_DT_F32));
  if (!scale || !scale->data || !ids || !ids->data || !w || !w->data) return Q3_ERR_NULL;
  if (scale->dtype != Q3_DT_F32 || w->dtype != Q3_DT_F32) return Q3_ERR_DTYPE;
  if (ids->dtype != Q3_DT_I32 && ids->dtype != Q3_DT_U32) return Q3_ERR_DTYPE;
  const uint32_t rows = ids->rows * ids->cols;
  if (tmp->rows < rows || out->rows < rows || tmp->cols < table->cols || out->cols < table->cols)
    return Q3_ERR_SHAPE;
  if (rows == 0) return Q3_OK;
  const int threads = 256, wpb = threads / 32;
  k_embedding_rmsnorm<<<(rows + wpb - 1) / wpb, threads, 0, (cudaStream_t)stream>>>(
      (const int8_t *)table->data, table->row_bytes, (const char *)scale->data,
      vec_stride(scale), (const char *)ids->data, vec_stride(ids), (char *)tmp->data,
      tmp->row_bytes, (const char *)w->data, vec_stride(w), (char *)out->data, out->row_bytes,
      rows, table->cols, inv);
  return launch_status();
}

static int scatter_args(ScatterArgs &a, const q3_view *k, const q3_view *v, const q3_view *ks,
                        const q3_view *vs, const q3_paged_kv *kv, uint32_t rows,
                        uint32_t kv_dim, uint32_t kv_heads) {
  Q3_TRY(check_view(k, Q3_DT_I8, 1));
  Q3_TRY(check_view(v, Q3_DT_I8, 1));
  Q3_TRY(check_view(ks, Q3_DT_F32));
  Q3_TRY(check_view(vs, Q3_DT_F32));
  if (!kv || !kv->k || !kv->v || !kv->ks || !kv->vs) return Q3_ERR_NULL;
  if (kv->page_tokens == 0 || kv_dim > kv->row_bytes || kv_heads * 4 > kv->scale_row_bytes)
    return Q3_ERR_SHAPE;
  if (k->rows < rows || v->rows < rows || ks->rows < rows || vs->rows < rows) return Q3_ERR_SHAPE;
  a = ScatterArgs{(const char *)k->data, (const char *)v->data, (const char *)ks->data,
                  (const char *)vs->data, k->row_bytes, v->row_bytes, ks->row_bytes,
                  vs->row_bytes, (char *)kv->k, (char *)kv->v, (char *)kv->ks, (char *)kv->vs,
                  kv->page_tokens, kv->page_bytes, kv->row_bytes, kv->scale_page_bytes,
                  kv->scale_row_bytes, (int)rows, (int)kv_dim, (int)kv_heads};
  return Q3_OK;
}

extern "C" int q3_paged_kv_scatter(const q3_view *k, const q3_view *v, const q3_view *ks,
                                   const q3_view *vs, const q3_paged_kv *kv,
                                   uint32_t start_token, uint32_t rows, uint32_t kv_dim,
                                   uint32_t kv_heads, void *stream) {
  ScatterArgs a;
  Q3_TRY(scatter_args(a, k, v, ks, vs, kv, rows, kv_dim, kv_heads));
  if (!kv->table) return Q3_ERR_NULL;
  if (rows == 0) return Q3_OK;
  k_paged_kv_scatter<<<rows, 128, 0, (cudaStream_t)stream>>>(a, kv->table, start_token);
  return launch_status();
}

extern "C" int q3_paged_kv_scatter_batch(const q3_view *k, const q3_view *v, const q3_view *ks,
                                         const q3_view *vs, const q3_paged_kv *tables,
                                         const uint32_t *tokens, uint32_t rows,
                                         uint32_t kv_dim, uint32_t kv_heads, void *stream) {
  if (!tables || !tokens) return Q3_ERR_NULL;
  if (rows > 128) return Q3_ERR_SHAPE;
  ScatterArgs a;
  Q3_TRY(scatter_args(a, k, v, ks, vs, &tables[0], rows, kv_dim, kv_heads));
  BatchTables t;
  for (uint32_t r = 0; r < rows; ++r) {
    // every row must live in the same page pool (same bases and strides)
    const q3_paged_kv &p = tables[r];
    if (p.k != tables[0].k || p.v != tables[0].v || p.ks != tables[0].ks ||
        p.vs != tables[0].vs || p.page_bytes != tables[0].page_bytes ||
        p.row_bytes != tables[0].row_bytes || p.page_tokens != tables[0].page_tokens ||
        p.scale_page_bytes != tables[0].scale_page_bytes ||
        p.scale_row_bytes != tables[0].scale_row_bytes)
      return Q3_ERR_SHAPE;
    if (!p.table) return Q3_ERR_NULL;
    t.row[r] = ScatterRow{p.table, tokens[r]};
  }
  if (rows == 0) return Q3_OK;
  k_paged_kv_scatter_batch<<<rows, 128, 0, (cudaStream_t)stream>>>(a, t);
  return launch_status();
}

static int exp_common(const q3_view *x, const q3_view *out, int base2, void *stream) {
  Q3_TRY(check_view(x, Q3_DT_F32));
  Q3_TRY(check_view(out, Q3_DT_F32));
  if (out->rows < x->rows || out->cols < x->cols) return Q3_ERR_SHAPE;
  const long n = static_cast<long>(x->rows) * x->cols;
  if (n == 0) return Q3_OK;
  k_exp_rows<<<(n + 255) / 256, 256, 0, (cudaStream_t)stream>>>(
      (const char *)x->data, x->row_bytes, (char *)out->data, out->row_bytes, x->rows, x->cols,
      base2);
  return launch_status();
}

extern "C" int q3_exp_rows(const q3_view *x, const q3_view *out, void *stream) {
  return exp_common(x, out, 0, stream);
}

extern "C" int q3_exp2_rows(const q3_view *x, const q3_view *out, void *stream) {
  return exp_common(x, out, 1, stream);
}

// every float32 bit pattern b in [lo, hi): exp2_cr_fast(b), exp2_cr_fast_n and (for
// b <= 0, -inf and the negative NaNs) its NONPOS form against exp2_cr_t(b)
__global__ void k_exp2_selfcheck(uint32_t lo, uint32_t hi, unsigned long long *count,
                                 uint32_t *first_bad) {
  const uint64_t n = static_cast<uint64_t>(hi) - lo;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t b = lo + static_cast<uint32_t>(i);
    const float x = __uint_as_float(b);
    const float f = exp2_cr_fast(x);
    const float d = exp2_cr_t(x, g_exp2_frac64);
    // the batched form too: x as element 0 of 8 neighbouring bit patterns
    float xs[8], ys[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) xs[j] = __uint_as_float(b ^ static_cast<uint32_t>(j));
    exp2_cr_fast_n(xs, ys, g_exp2_t256);
    bool bad = __float_as_uint(f) != __float_as_uint(d) || __float_as_uint(ys[0]) != __float_as_uint(d);
    if ((b >> 31) || b == 0u) {   // and the form for inputs <= 0, -inf or NaN
      exp2_cr_fast_n<8, true>(xs, ys, g_exp2_t256);
      bad |= __float_as_uint(ys[0]) != __float_as_uint(d);
    }
    if (bad) {
      atomicAdd(count, 1ull);
      atomicMin(first_bad, b);
    }
  }
}

// The int8 code as the reference forms it: the IEEE quotient, rounded to
// nearest even by the float -> int conversion, then saturated; NaN -> 0.
__device__ int quant1_conv(float x, float s) {
  const float q = __fdiv_rn(x, s);
  int v = __float2int_rn(q);
  v = v > 127 ? 127 : v;
  v = v < -127 ? -127 : v;
  return q != q ? 0 : v;
}

// For every float32 x in [lo, hi) and the scale s = RN(amax * kInv127), as the
// kernels form it: quant1 against quant1_conv, and, for |x| <= amax and NaN x,
// the form of quant_n_absmax (from the reciprocal when quant_rcp_ok(s), else
// quant1) against quant1_conv.
__global__ void k_quant_selfcheck(uint32_t lo, uint32_t hi, float amax, unsigned long long *count,
                                  uint32_t *first_bad) {
  const float s = __fmul_rn(amax, kInv127);
  const bool rcp = quant_rcp_ok(s);
  const float r = rcp ? __frcp_rn(s) : 0.0f;
  const uint64_t n = static_cast<uint64_t>(hi) - lo;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint32_t b = lo + static_cast<uint32_t>(i);
    const float x = __uint_as_float(b);
    const int want = quant1_conv(x, s);
    bool bad = quant1(x, s) != want;
    if (!(fabsf(x) > amax)) bad |= (rcp ? quant1_rcp_absmax(x, s, r) : quant1(x, s)) != want;
    if (bad) {
      atomicAdd(count, 1ull);
      atomicMin(first_bad, b);
    }
  }
}

extern "C" int q3_quant_selfcheck(uint32_t lo_bits, uint32_t hi_bits, float amax,
                                  unsigned long long *count, uint32_t *first_bad, void *stream) {
  if (!count || !first_bad) return Q3_ERR_NULL;
  if (hi_bits < lo_bits || !(amax >= 0.0f && amax < INFINITY)) return Q3_ERR_SHAPE;
  if (hi_bits == lo_bits) return Q3_OK;
  k_quant_selfcheck<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(lo_bits, hi_bits, amax, count,
                                                                first_bad);
  return launch_status();
}

extern "C" int q3_exp2_selfcheck(uint32_t lo_bits, uint32_t hi_bits, unsigned long long *count,
                                 uint32_t *first_bad, void *stream) {
  if (!count || !first_bad) return Q3_ERR_NULL;
  if (hi_bits < lo_bits) return Q3_ERR_SHAPE;
  if (hi_bits == lo_bits) return Q3_OK;
  k_exp2_selfcheck<<<148 * 8, 256, 0, (cudaStream_t)stream>>>(lo_bits, hi_bits, count, first_bad);
  return launch_status();
}

extern "C" int q3_argmax_logits(const q3_view *logits, int32_t *out_id, void *stream) {
  Q3_TRY(check_view(logits, Q3_DT_F32));
  if (!out_id) return Q3_ERR_NULL;
  if (logits->cols == 0) return Q3_ERR_SHAPE;
  k_argmax_logits<<<1, 1024, 0, (cudaStream_t)stream>>>((const float *)logits->data,
                                                        logits->cols, out_id);
  return launch_status();
}

namespace q3h {
// used by the model runner: same kernels, raw pointers
int launch_argmax_row(const float *row, int n, int32_t *out_id, cudaStream_t s) {
  k_argmax_logits<<<1, 1024, 0, s>>>(row, n, out_id);
  return launch_status();
}
}  // namespace q3h
