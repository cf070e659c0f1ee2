// C-ABI entry points of the GEMM family: argument checks and dispatch.
#include "q3_common.cuh"
#include "q3_gemm.h"

using namespace q3;
using namespace q3h;

namespace q3 {
int gemm_dispatch(const GemmArgs &p, cudaStream_t s);
}

static int contiguous_f32(const q3_view *v, uint32_t n) {
  if (!v || !v->data) return Q3_ERR_NULL;
  if (v->dtype != Q3_DT_F32) return Q3_ERR_DTYPE;
  const bool col = (v->rows >= n && (v->row_bytes == 4 || v->rows == 1) && v->cols >= 1);
  const bool row = (v->cols >= n && v->col_bytes == 4);
  if (!col && !row) return Q3_ERR_SHAPE;
  if (reinterpret_cast<uintptr_t>(v->data) % 4) return Q3_ERR_ALIGN;
  return Q3_OK;
}

static int base_args(GemmArgs &p, const q3_view *a, const q3_view *a_scale, const q3_view *b,
                     const q3_view *b_scale, uint32_t group_k, uint32_t N) {
  Q3_TRY(check_view(a, Q3_DT_I8, 16));
  Q3_TRY(check_view(b, Q3_DT_I8, 16));
  Q3_TRY(check_view(a_scale, Q3_DT_F32));
  const uint32_t K = a->cols;
  if (group_k == 0 || group_k % 64 || K % group_k || K == 0) return Q3_ERR_SHAPE;
  if (b->cols < K || b->rows < N) return Q3_ERR_SHAPE;
  if (a_scale->cols < K / group_k || (a->rows > 1 && a_scale->rows < a->rows)) return Q3_ERR_SHAPE;
  Q3_TRY(contiguous_f32(b_scale, N));
  p = GemmArgs{};
  p.M = a->rows;
  p.N = N;
  p.K = K;
  p.group = group_k;
  p.a = (const int8_t *)a->data;
  p.a_rb = a->row_bytes;
  p.a_scale = (const char *)a_scale->data;
  p.as_rb = a_scale->row_bytes;
  p.b = (const int8_t *)b->data;
  p.b_rb = b->row_bytes;
  p.b_scale = (const float *)b_scale->data;
  return Q3_OK;
}

extern "C" int q3_gemm_nt_group_store(const q3_view *a, const q3_view *a_scale,
                                      const q3_view *b, const q3_view *b_scale,
                                      const q3_view *out, uint32_t group_k, const q3_view *add,
                                      const q3_view *q8, const q3_view *qs, const q3_view *nw,
                                      const q3_view *cos, const q3_view *sin, float inv_hd,
                                      void *stream) {
  if (!b) return Q3_ERR_NULL;
  const uint32_t N = b->rows;
  if (N % 128) return Q3_ERR_SHAPE;
  GemmArgs p;
  Q3_TRY(base_args(p, a, a_scale, b, b_scale, group_k, N));
  const uint32_t M = p.M;
  if (nw && nw->data) {
    Q3_TRY(check_view(q8, Q3_DT_I8, 1));
    Q3_TRY(check_view(qs, Q3_DT_F32));
    Q3_TRY(check_view(cos, Q3_DT_F32));
    Q3_TRY(check_view(sin, Q3_DT_F32));
    Q3_TRY(contiguous_f32(nw, 128));
    if (q8->cols < N || q8->rows < M || qs->cols < N / 128 || cos->cols < 64 ||
        sin->cols < 64 || (M > 1 && (qs->rows < M || cos->rows < M || sin->rows < M)))
      return Q3_ERR_SHAPE;
    p.mode = EPI_NORMROPE;
    p.q8 = (char *)q8->data;
    p.q8_rb = q8->row_bytes;
    p.qs = (char *)qs->data;
    p.qs_rb = qs->row_bytes;
    p.nw = (const float *)nw->data;
    p.cos = (const char *)cos->data;
    p.cos_rb = cos->row_bytes;
    p.sin = (const char *)sin->data;
    p.sin_rb = sin->row_bytes;
    p.inv_hd = inv_hd;
  } else if (q8 && q8->data) {
    Q3_TRY(check_view(q8, Q3_DT_I8, 1));
    Q3_TRY(check_view(qs, Q3_DT_F32));
    if (q8->cols < N || q8->rows < M || qs->cols < N / 128 || (M > 1 && qs->rows < M))
      return Q3_ERR_SHAPE;
    p.mode = EPI_QUANT;
    p.q8 = (char *)q8->data;
    p.q8_rb = q8->row_bytes;
    p.qs = (char *)qs->data;
    p.qs_rb = qs->row_bytes;
  } else if (add && add->data) {
    Q3_TRY(check_view(add, Q3_DT_F32));
    if (add->cols < N || add->rows < M) return Q3_ERR_SHAPE;
    p.mode = EPI_ADD;
    p.out = (char *)add->data;
    p.out_rb = add->row_bytes;
  } else {
    Q3_TRY(check_view(out, Q3_DT_F32));
    if (out->cols < N || out->rows < M) return Q3_ERR_SHAPE;
    p.mode = EPI_STORE;
    p.out = (char *)out->data;
    p.out_rb = out->row_bytes;
  }
  if (M == 0) return Q3_OK;
  return gemm_dispatch(p, (cudaStream_t)stream);
}

extern "C" int q3_gemm_gate_up_swiglu_quant(const q3_view *a, const q3_view *a_scale,
                                            const q3_view *wg, const q3_view *wgs,
                                            const q3_view *wu, const q3_view *wus,
                                            const q3_view *s8, const q3_view *ss,
                                            uint32_t group_k, void *stream) {
  Q3_TRY(check_view(s8, Q3_DT_I8, 1));
  Q3_TRY(check_view(ss, Q3_DT_F32));
  const uint32_t N = s8->cols;
  if (N % 256) return Q3_ERR_SHAPE;
  GemmArgs p;
  Q3_TRY(base_args(p, a, a_scale, wg, wgs, group_k, N));
  Q3_TRY(check_view(wu, Q3_DT_I8, 16));
  Q3_TRY(contiguous_f32(wus, N));
  if (wu->rows < N || wu->cols < p.K || wu->row_bytes != wg->row_bytes) return Q3_ERR_SHAPE;
  if (s8->rows < (uint32_t)p.M || ss->cols < N / 256 || (p.M > 1 && ss->rows < (uint32_t)p.M))
    return Q3_ERR_SHAPE;
  p.mode = EPI_SWIGLU;
  p.b2 = (const int8_t *)wu->data;
  p.b2_scale = (const float *)wus->data;
  p.q8 = (char *)s8->data;
  p.q8_rb = s8->row_bytes;
  p.qs = (char *)ss->data;
  p.qs_rb = ss->row_bytes;
  if (p.M == 0) return Q3_OK;
  return gemm_dispatch(p, (cudaStream_t)stream);
}

extern "C" size_t q3_gemm_nt_group_argmax_workspace_bytes(uint32_t rows) {
  return static_cast<size_t>(rows) * sizeof(unsigned long long);
}

extern "C" int q3_gemm_nt_group_argmax(const q3_view *a, const q3_view *a_scale,
                                       const q3_view *b, const q3_view *b_scale, float *best,
                                       int32_t *bidx, uint32_t group_k, void *workspace,
                                       size_t workspace_bytes, void *stream) {
  if (!b || !best || !bidx) return Q3_ERR_NULL;
  const uint32_t N = b->rows;
  if (N % 128) return Q3_ERR_SHAPE;
  GemmArgs p;
  Q3_TRY(base_args(p, a, a_scale, b, b_scale, group_k, N));
  if (!workspace) return Q3_ERR_NULL;
  if (reinterpret_cast<uintptr_t>(workspace) % 8) return Q3_ERR_ALIGN;
  if (workspace_bytes < q3_gemm_nt_group_argmax_workspace_bytes(p.M)) return Q3_ERR_CAPACITY;
  p.mode = EPI_ARGMAX;
  p.arg_keys = (unsigned long long *)workspace;
  p.best = best;
  p.bidx = bidx;
  if (p.M == 0) return Q3_OK;
  return gemm_dispatch(p, (cudaStream_t)stream);
}

namespace q3 {
// tensor cores where the shape allows, the CUDA-core kernel otherwise (same bits)
int gemm_dispatch(const GemmArgs &p, cudaStream_t s) {
  if (p.mode == EPI_ARGMAX) Q3_TRY(argmax_begin(p, s));
  const int st = gemm_tc_eligible(p) ? gemm_tc(p, s) : gemm_simt(p, s);
  if (st != Q3_OK) return st;
  if (p.mode == EPI_ARGMAX) return argmax_end(p, s);
  return Q3_OK;
}
}  // namespace q3
