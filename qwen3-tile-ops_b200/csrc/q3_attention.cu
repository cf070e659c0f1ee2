// GQA hd128 attention over a paged int8 KV cache with the reference's
// online softmax (kernels/attention_gqa.h:404-572 ; tools/ref_qwen3.py:210-289):
// per 32-key block j, in key order, for each query row
//   s    = ((f32(q8.k8) * ks) * qs) * qk_scale, causal mask -> -inf
//   nmm  = max(tree_max(s), m);  corr = exp(m - nmm);  den *= corr; res *= corr
//   p    = exp(s - nmm);  den += tree_sum(p);  m = nmm
//   p   *= vs;  pmax = tree_max(|p|)/127;  pq = quant(p, pmax)
//   res += f32(int32(pq . v8)) * pmax
// then res * (1/den), quantised per head into o8/os.
//
// Rows are independent, and a block that lies wholly beyond a row's causal
// horizon is an exact no-op for it (corr = 1, p = 0), so every row can skip
// such blocks regardless of how rows are grouped.
//
// Mapping: one CTA per (sequence, kv head, tile of query rows); one warp per
// (query row, q head of the GQA group); lane c of a warp owns key j+c while
// scoring and output columns 4c..4c+3 while accumulating P.V.
#include "q3_attention.h"
#include "q3_common.cuh"

namespace q3 {

constexpr int HD = 128;
constexpr int KROW = HD + 4;  // padded K row in shared memory (bank-conflict free)

__global__ void __launch_bounds__(512) k_attention_paged(AttnArgs p) {
  __shared__ __align__(16) int8_t sK[32][KROW];
  __shared__ __align__(16) int8_t sV[32][HD];
  __shared__ float sKs[32], sVs[32];

  const int seq = blockIdx.z;
  const int kvh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int grp = p.heads / p.kv_heads;
  const int rows_per_cta = nwarps / grp;
  const int lr = blockIdx.x * rows_per_cta + warp / grp;   // row within the sequence
  const int h = kvh * grp + warp % grp;                    // q head
  const int kv_len = p.kv_len_dev ? p.kv_len_dev[seq] : p.kv_len;
  const int q_rows = p.item_rows ? p.item_rows[seq] : p.q_rows;
  if (static_cast<int>(blockIdx.x) * rows_per_cta >= q_rows) return;   // (uniform) no rows here
  const bool active = lr < q_rows;
  const int qpos = p.causal ? (kv_len - q_rows + lr) : (kv_len - 1);
  const long qrow = (p.item_row0 ? static_cast<long>(p.item_row0[seq]) : static_cast<long>(seq) * q_rows) + lr;
  const uint16_t *table = p.table + static_cast<long>(seq) * p.table_stride;

  // this CTA's last visible key (blocks beyond it are skipped by every row)
  const int last_row = min(q_rows, (int)(blockIdx.x + 1) * rows_per_cta) - 1;
  const int kv_end = p.causal ? min(kv_len, kv_len - q_rows + last_row + 1) : kv_len;

  int qw[32];
  float qsc = 0.0f;
  if (active) {
    const int *qr = reinterpret_cast<const int *>(p.q8 + qrow * p.q_rb + h * HD);
#pragma unroll
    for (int w = 0; w < 32; ++w) qw[w] = qr[w];
    qsc = *reinterpret_cast<const float *>(p.qs + qrow * p.qs_rb + h * 4);
  }
  float m = kNegFltMax, den = 0.0f;
  float res[4] = {0.0f, 0.0f, 0.0f, 0.0f};

  for (int j = 0; j < kv_end; j += 32) {
    // ---- stage the K/V block of this kv head (page-table lookup per key)
    for (int i = threadIdx.x; i < 32 * 8; i += blockDim.x) {
      const int c = i >> 3, v = i & 7;
      const int t = j + c;
      int4 kk = make_int4(0, 0, 0, 0), vv = make_int4(0, 0, 0, 0);
      if (t < kv_len) {
        const uint32_t page = table[t / p.page_tokens], slot = t % p.page_tokens;
        const size_t off = static_cast<size_t>(page) * p.page_bytes + static_cast<size_t>(slot) * p.row_bytes +
                           kvh * HD + v * 16;
        kk = *reinterpret_cast<const int4 *>(p.k + off);
        vv = *reinterpret_cast<const int4 *>(p.v + off);
      }
      int *dk = reinterpret_cast<int *>(&sK[c][v * 16]);
      dk[0] = kk.x; dk[1] = kk.y; dk[2] = kk.z; dk[3] = kk.w;
      *reinterpret_cast<int4 *>(&sV[c][v * 16]) = vv;
    }
    if (threadIdx.x < 32) {
      const int t = j + threadIdx.x;
      float ks = 0.0f, vs = 0.0f;
      if (t < kv_len) {
        const uint32_t page = table[t / p.page_tokens], slot = t % p.page_tokens;
        const size_t off = static_cast<size_t>(page) * p.scale_page_bytes +
                           static_cast<size_t>(slot) * p.scale_row_bytes + kvh * 4;
        ks = *reinterpret_cast<const float *>(p.ks + off);
        vs = *reinterpret_cast<const float *>(p.vs + off);
      }
      sKs[threadIdx.x] = ks;
      sVs[threadIdx.x] = vs;
    }
    __syncthreads();

    if (active && j <= qpos) {
      // ---- scores for key j+lane
      const int *kr = reinterpret_cast<const int *>(&sK[lane][0]);
      int acc = 0;
#pragma unroll
      for (int w = 0; w < 32; ++w) acc = __dp4a(qw[w], kr[w], acc);
      float s = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(acc), sKs[lane]), qsc), p.qk_scale);
      const int t = j + lane;
      if (t > qpos || t >= kv_len) s = kNegInf;
      // ---- online softmax update
      const float nmm = fmaxf(warp_tree_max(s), m);
      const float corr = exp_ref(__fsub_rn(m, nmm));
      den = __fmul_rn(den, corr);
#pragma unroll
      for (int i = 0; i < 4; ++i) res[i] = __fmul_rn(res[i], corr);
      float pr = exp_ref(__fsub_rn(s, nmm));
      den = __fadd_rn(den, warp_tree_sum(pr));
      m = nmm;
      // ---- fold the V scale, requantise P per row
      pr = __fmul_rn(pr, sVs[lane]);
      const float pmax = __fmul_rn(warp_tree_max(fabsf(pr)), kInv127);
      const int pq = quant1(pr, pmax);
      // ---- P.V for output columns 4*lane .. 4*lane+3
      int part[4] = {0, 0, 0, 0};
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int pc = __shfl_sync(0xffffffffu, pq, c);
        const int vw = *reinterpret_cast<const int *>(&sV[c][lane * 4]);
        part[0] += pc * ((vw << 24) >> 24);
        part[1] += pc * ((vw << 16) >> 24);
        part[2] += pc * ((vw << 8) >> 24);
        part[3] += pc * (vw >> 24);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) res[i] = __fadd_rn(res[i], __fmul_rn(i2f_small(part[i]), pmax));
    }
    __syncthreads();
  }

  if (!active) return;
  // ---- 1/den, per-head output quantisation (attention_gqa.h:522-546)
  const float rden = __frcp_rn(den);
  float o[4];
  float mx = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    o[i] = __fmul_rn(res[i], rden);
    mx = fmaxf(mx, fabsf(o[i]));
  }
  mx = warp_tree_max(mx);
  const float scale = __fmul_rn(mx, kInv127);
  char4 q;
  q.x = static_cast<char>(quant1(o[0], scale));
  q.y = static_cast<char>(quant1(o[1], scale));
  q.z = static_cast<char>(quant1(o[2], scale));
  q.w = static_cast<char>(quant1(o[3], scale));
  *reinterpret_cast<char4 *>(p.o8 + qrow * p.o_rb + h * HD + lane * 4) = q;
  if (lane == 0) *reinterpret_cast<float *>(p.os + qrow * p.os_rb + h * 4) = scale;
}

int attention_launch(const AttnArgs &p, int n_seqs, cudaStream_t s) {
  const int grp = p.heads / p.kv_heads;
  int rows_per_cta = 16 / grp;
  if (rows_per_cta < 1) rows_per_cta = 1;
  if (rows_per_cta > p.q_rows) rows_per_cta = p.q_rows;
  const int threads = 32 * grp * rows_per_cta;
  dim3 grid((p.q_rows + rows_per_cta - 1) / rows_per_cta, p.kv_heads, n_seqs);
  q3h::timer_begin(q3h::TIMER_ATTENTION, s);
  k_attention_paged<<<grid, threads, 0, s>>>(p);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_ATTENTION, s);
  return st;
}

}  // namespace q3

using namespace q3;
using namespace q3h;

extern "C" int q3_attention_heads_gqa_tokscale_paged(const q3_view *q8, const q3_view *q_scale,
                                                     const q3_paged_kv *kv, uint32_t kv_len,
                                                     const q3_view *o8, const q3_view *os,
                                                     int heads, int kv_heads, int head_dim,
                                                     int causal, float qk_scale, void *stream) {
  Q3_TRY(check_view(q8, Q3_DT_I8, 4));
  Q3_TRY(check_view(q_scale, Q3_DT_F32));
  Q3_TRY(check_view(o8, Q3_DT_I8, 4));
  Q3_TRY(check_view(os, Q3_DT_F32));
  if (!kv || !kv->k || !kv->v || !kv->ks || !kv->vs || !kv->table) return Q3_ERR_NULL;
  if (head_dim != 128 || heads <= 0 || kv_heads <= 0 || heads % kv_heads ||
      heads / kv_heads > 16)
    return Q3_ERR_SHAPE;
  const uint32_t rows = q8->rows;
  if (q8->cols < (uint32_t)(heads * 128) || o8->cols < (uint32_t)(heads * 128) ||
      o8->rows < rows || q_scale->cols < (uint32_t)heads || os->cols < (uint32_t)heads ||
      (rows > 1 && (q_scale->rows < rows || os->rows < rows)))
    return Q3_ERR_SHAPE;
  if (kv->page_tokens == 0 || kv->row_bytes < (uint32_t)(kv_heads * 128) ||
      kv->scale_row_bytes < (uint32_t)(kv_heads * 4))
    return Q3_ERR_SHAPE;
  if (kv->page_bytes % 16 || kv->row_bytes % 16 || reinterpret_cast<uintptr_t>(kv->k) % 16 ||
      reinterpret_cast<uintptr_t>(kv->v) % 16 || kv->scale_page_bytes % 4 ||
      kv->scale_row_bytes % 4)
    return Q3_ERR_ALIGN;
  if (causal && kv_len < rows) return Q3_ERR_SHAPE;
  if (rows == 0 || kv_len == 0) return Q3_OK;
  AttnArgs p{};
  p.q8 = (const char *)q8->data;
  p.q_rb = q8->row_bytes;
  p.qs = (const char *)q_scale->data;
  p.qs_rb = q_scale->row_bytes;
  p.o8 = (char *)o8->data;
  p.o_rb = o8->row_bytes;
  p.os = (char *)os->data;
  p.os_rb = os->row_bytes;
  p.k = (const char *)kv->k;
  p.v = (const char *)kv->v;
  p.ks = (const char *)kv->ks;
  p.vs = (const char *)kv->vs;
  p.table = kv->table;
  p.table_stride = 0;
  p.page_tokens = kv->page_tokens;
  p.page_bytes = kv->page_bytes;
  p.row_bytes = kv->row_bytes;
  p.scale_page_bytes = kv->scale_page_bytes;
  p.scale_row_bytes = kv->scale_row_bytes;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.q_rows = rows;
  p.kv_len = kv_len;
  p.kv_len_dev = nullptr;
  p.causal = causal ? 1 : 0;
  p.qk_scale = qk_scale;
  return attention_launch(p, 1, (cudaStream_t)stream);
}

extern "C" int q3_attention_decode_batch(const q3_view *q8, const q3_view *q_scale,
                                         const q3_paged_kv *kv, uint32_t num_pages,
                                         const uint16_t *tables, uint32_t max_pages,
                                         const int32_t *kv_len, uint32_t n_seqs,
                                         const q3_view *o8, const q3_view *os, int heads,
                                         int kv_heads, float qk_scale, void *stream) {
  Q3_TRY(check_view(q8, Q3_DT_I8, 4));
  Q3_TRY(check_view(q_scale, Q3_DT_F32));
  Q3_TRY(check_view(o8, Q3_DT_I8, 4));
  Q3_TRY(check_view(os, Q3_DT_F32));
  if (!kv || !kv->k || !kv->v || !kv->ks || !kv->vs || !tables || !kv_len) return Q3_ERR_NULL;
  if (heads <= 0 || kv_heads <= 0 || heads % kv_heads || heads / kv_heads > 16 || max_pages == 0)
    return Q3_ERR_SHAPE;
  if (q8->rows < n_seqs || o8->rows < n_seqs || q8->cols < (uint32_t)(heads * 128) ||
      o8->cols < (uint32_t)(heads * 128) || q_scale->cols < (uint32_t)heads ||
      os->cols < (uint32_t)heads ||
      (n_seqs > 1 && (q_scale->rows < n_seqs || os->rows < n_seqs)))
    return Q3_ERR_SHAPE;
  if (kv->page_tokens == 0 || kv->row_bytes < (uint32_t)(kv_heads * 128) ||
      kv->scale_row_bytes < (uint32_t)(kv_heads * 4))
    return Q3_ERR_SHAPE;
  if (kv->page_bytes % 16 || kv->row_bytes % 16 || reinterpret_cast<uintptr_t>(kv->k) % 16 ||
      reinterpret_cast<uintptr_t>(kv->v) % 16 || kv->scale_page_bytes % 4 ||
      kv->scale_row_bytes % 4)
    return Q3_ERR_ALIGN;
  if (n_seqs == 0) return Q3_OK;
  cudaStream_t s = (cudaStream_t)stream;
  if (heads == 2 * kv_heads && kv->page_tokens == 32 && num_pages > 0) {
    DecodeAttnArgs d{};
    d.q8 = (const char *)q8->data;
    d.q_rb = q8->row_bytes;
    d.qs = (const char *)q_scale->data;
    d.qs_rb = q_scale->row_bytes;
    d.o8 = (char *)o8->data;
    d.o_rb = o8->row_bytes;
    d.os = (char *)os->data;
    d.os_rb = os->row_bytes;
    d.ks = (const char *)kv->ks;
    d.vs = (const char *)kv->vs;
    d.table = tables;
    d.table_stride = max_pages;
    d.page_bytes = kv->page_bytes;
    d.row_bytes = kv->row_bytes;
    d.scale_page_bytes = kv->scale_page_bytes;
    d.scale_row_bytes = kv->scale_row_bytes;
    d.kv_len = kv_len;
    d.qk_scale = qk_scale;
    return attention_decode_launch(d, kv->k, kv->v, num_pages, kv_heads, n_seqs, s);
  }
  AttnArgs p{};
  p.q8 = (const char *)q8->data;
  p.q_rb = q8->row_bytes;
  p.qs = (const char *)q_scale->data;
  p.qs_rb = q_scale->row_bytes;
  p.o8 = (char *)o8->data;
  p.o_rb = o8->row_bytes;
  p.os = (char *)os->data;
  p.os_rb = os->row_bytes;
  p.k = (const char *)kv->k;
  p.v = (const char *)kv->v;
  p.ks = (const char *)kv->ks;
  p.vs = (const char *)kv->vs;
  p.table = tables;
  p.table_stride = max_pages;
  p.page_tokens = kv->page_tokens;
  p.page_bytes = kv->page_bytes;
  p.row_bytes = kv->row_bytes;
  p.scale_page_bytes = kv->scale_page_bytes;
  p.scale_row_bytes = kv->scale_row_bytes;
  p.heads = heads;
  p.kv_heads = kv_heads;
  p.q_rows = 1;
  p.kv_len = 0;
  p.kv_len_dev = kv_len;
  p.causal = 1;
  p.qk_scale = qk_scale;
  return attention_launch(p, n_seqs, s);
}
