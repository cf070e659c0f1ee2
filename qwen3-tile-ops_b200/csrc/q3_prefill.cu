// Batched prompt prefill: n_seqs independent sequences, each with a T-token
// prompt at positions 0..T-1, written into a shared KV page pool under
// per-sequence page tables (kernels/kv_pages.h:98-131 semantics), and the
// greedy next token of every sequence.
//
// Per row the arithmetic is forward_chunk's (src/main_big.cpp:145-296): rows
// never interact except through attention, and a prompt processed as one
// chunk of T rows gives the same bits as the reference's 32-row chunks — every
// row's K/V is written before attention, which masks each row to the keys at
// or before its position (tools/ref_qwen3.py:269-289).  The GEMMs run with all
// n_seqs * T rows stacked (M = n_seqs * T); attention is the causal batched
// paged kernel over the pool; only each sequence's last row goes through the
// final norm and the lm_head argmax.
#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_gemm.h"
#include "q3_tp.h"

namespace {

constexpr uint32_t kPT = 32;   // page tokens
constexpr float kInvSqrt128 = 0.08838834764831845f;

struct PrefillWs {
  float *x, *h;          // [M][H]
  int8_t *h8;            // [M][H]
  float *hs;             // [M][H/256]
  int8_t *q8, *o8;       // [M][QW]
  float *qs, *os;        // [M][heads]
  int8_t *k8, *v8;       // [M][KW] staging of the new K/V rows
  float *ks, *vs;        // [M][kv_heads]
  int8_t *s8;            // [M][I]
  float *ss;             // [M][I/256]
  float *cos, *sin;      // [M][64] rows at each row's position
  float *xl, *hl;        // [B][H] last rows
  int8_t *h8l;           // [B][H]
  float *hsl;            // [B][H/256]
  float *best;           // [B]
  unsigned long long *keys;  // [B]
  size_t total;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

PrefillWs carve(const q3_layout &L, size_t M, uint32_t B, char *base) {
  const size_t H = L.hidden, QW = L.heads * L.head_dim, KW = L.kv_heads * L.head_dim, I = L.inter;
  PrefillWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
  w.x = (float *)take(4 * M * H);
  w.h = (float *)take(4 * M * H);
  w.h8 = (int8_t *)take(M * H);
  w.hs = (float *)take(4 * M * (H / 256));
  w.q8 = (int8_t *)take(M * QW);
  w.o8 = (int8_t *)take(M * QW);
  w.qs = (float *)take(4 * M * L.heads);
  w.os = (float *)take(4 * M * L.heads);
  w.k8 = (int8_t *)take(M * KW);
  w.v8 = (int8_t *)take(M * KW);
  w.ks = (float *)take(4 * M * L.kv_heads);
  w.vs = (float *)take(4 * M * L.kv_heads);
  w.s8 = (int8_t *)take(M * I);
  w.ss = (float *)take(4 * M * (I / 256));
  w.cos = (float *)take(4 * M * (L.head_dim / 2));
  w.sin = (float *)take(4 * M * (L.head_dim / 2));
  w.xl = (float *)take(4 * B * H);
  w.hl = (float *)take(4 * B * H);
  w.h8l = (int8_t *)take(B * H);
  w.hsl = (float *)take(4 * B * (H / 256));
  w.best = (float *)take(4 * B);
  w.keys = (unsigned long long *)take(8 * B);
  w.total = off;
  return w;
}

q3_view v2(void *p, uint32_t rows, uint32_t cols, uint8_t dt) {
  const int es = (dt == Q3_DT_I8 || dt == Q3_DT_U8) ? 1 : 4;
  return q3_view{p, static_cast<int32_t>(cols * es), es, rows, cols, dt};
}

// rope rows of row m (position m % T)
__global__ void k_prefill_rope_rows(const float *cos_t, const float *sin_t, int half, int T,
                                    float *cos, float *sin) {
  const int m = blockIdx.x, t = m % T;
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    cos[(size_t)m * half + j] = cos_t[(size_t)t * half + j];
    sin[(size_t)m * half + j] = sin_t[(size_t)t * half + j];
  }
}

// K/V row m = s*T + t -> page tables[s][t/32], slot t%32
__global__ void k_prefill_scatter(const int8_t *k8, const int8_t *v8, const float *ks,
                                  const float *vs, const uint16_t *tables, uint32_t max_pages,
                                  int T, char *pk, char *pv, char *pks, char *pvs, int kw,
                                  int kvh) {
  const int m = blockIdx.x, s = m / T, t = m % T;
  const uint32_t page = tables[static_cast<size_t>(s) * max_pages + t / kPT], slot = t % kPT;
  const size_t row = static_cast<size_t>(page) * kPT + slot;
  for (int i = threadIdx.x; i < kw / 16; i += blockDim.x) {
    reinterpret_cast<int4 *>(pk + row * kw)[i] = reinterpret_cast<const int4 *>(k8 + (size_t)m * kw)[i];
    reinterpret_cast<int4 *>(pv + row * kw)[i] = reinterpret_cast<const int4 *>(v8 + (size_t)m * kw)[i];
  }
  for (int h = threadIdx.x; h < kvh; h += blockDim.x) {
    reinterpret_cast<float *>(pks + row * kvh * 4)[h] = ks[(size_t)m * kvh + h];
    reinterpret_cast<float *>(pvs + row * kvh * 4)[h] = vs[(size_t)m * kvh + h];
  }
}

// x row s*T + T-1 -> xl[s]; best[s] = -3e38, next_ids[s] = 0 (argmax state)
using q3::kEps;
using q3::kInv127;
using q3::quant1;
using q3::quant_pack_absmax;
using q3::rsqrt_ref;
using q3::warp_tree_max;

// RMSNorm (kernels/rmsnorm.h:34-81) and the per-256-column int8 quantisation
// (kernels/quant.h:89-138) of 1024-column rows in one pass, without the f32
// rows in between: one warp per row, lane l holding columns 4l .. 4l+3 of
// each 128-column chunk (float4 loads, packed int8 stores).  A 32-column
// block's tree of squares is the in-lane (v0+v1)+(v2+v3) followed by the
// butterfly over its 8 lanes (offsets 1, 2, 4): the reference's adjacent-pair
// tree; the 32 block sums are added in column order.  Bit-identical to
// q3_rmsnorm_rows followed by q3_quant_rows_heads with group 256.
__global__ void k_norm_quant_1024(const float *__restrict__ x, const float *__restrict__ w,
                                  float inv, int rows, int8_t *h8, float *hs) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(row) * 1024);
  float4 v[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) v[k] = xr[32 * k + lane];
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    float t = __fadd_rn(__fadd_rn(__fmul_rn(v[k].x, v[k].x), __fmul_rn(v[k].y, v[k].y)),
                        __fadd_rn(__fmul_rn(v[k].z, v[k].z), __fmul_rn(v[k].w, v[k].w)));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) t = __fadd_rn(t, __shfl_xor_sync(0xffffffffu, t, o));
#pragma unroll
    for (int q = 0; q < 4; ++q) ss = __fadd_rn(ss, __shfl_sync(0xffffffffu, t, 8 * q));
  }
  ss = __fadd_rn(__fmul_rn(ss, inv), kEps);
  const float r = rsqrt_ref(ss);
  const float4 *wr = reinterpret_cast<const float4 *>(w);
  int8_t *qrow = h8 + static_cast<size_t>(row) * 1024;
#pragma unroll
  for (int g = 0; g < 4; ++g) {                    // 256-column groups = chunk pairs
    float hv[8];
    float am = 0.0f;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int k = 2 * g + c;
      const float4 wv = wr[32 * k + lane];
      hv[4 * c + 0] = __fmul_rn(__fmul_rn(v[k].x, r), wv.x);
      hv[4 * c + 1] = __fmul_rn(__fmul_rn(v[k].y, r), wv.y);
      hv[4 * c + 2] = __fmul_rn(__fmul_rn(v[k].z, r), wv.z);
      hv[4 * c + 3] = __fmul_rn(__fmul_rn(v[k].w, r), wv.w);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) am = fmaxf(am, fabsf(hv[i]));
    const float scale = __fmul_rn(warp_tree_max(am), kInv127);
    uint32_t w[2];
    quant_pack_absmax(hv, scale, w);
#pragma unroll
    for (int c = 0; c < 2; ++c) reinterpret_cast<uint32_t *>(qrow + 128 * (2 * g + c))[lane] = w[c];
    if (lane == 0) hs[static_cast<size_t>(row) * 4 + g] = scale;
  }
}

__global__ void k_prefill_last_rows(const float *x, int T, int H, float *xl, float *best,
                                    int32_t *next_ids) {
  const int s = blockIdx.x;
  const float *src = x + (static_cast<size_t>(s) * T + T - 1) * H;
  for (int j = threadIdx.x; j < H; j += blockDim.x) xl[(size_t)s * H + j] = src[j];
  if (threadIdx.x == 0) {
    best[s] = -3.0e38f;
    next_ids[s] = 0;
  }
}

}  // namespace

extern "C" size_t q3_prefill_workspace_bytes(const q3_layout *L, uint32_t n_seqs, uint32_t T) {
  if (!L) return 0;
  return carve(*L, static_cast<size_t>(n_seqs) * T, n_seqs, nullptr).total;
}

extern "C" int q3_prefill_batch(void *blob, const q3_layout *layout, const q3_kv_pool *pool,
                                const uint16_t *tables, uint32_t max_pages, const int32_t *ids,
                                uint32_t n_seqs, uint32_t T, int32_t *next_ids, void *workspace,
                                size_t workspace_bytes, void *stream) {
  if (!blob || !layout || !pool || !tables || !ids || !next_ids || !workspace) return Q3_ERR_NULL;
  const q3_layout &L = *layout;
  if (L.head_dim != 128 || L.hidden % 256 || L.inter % 256 || L.max_seq % kPT) return Q3_ERR_SHAPE;
  if (n_seqs == 0 || T == 0) return Q3_OK;
  if (T > L.max_seq || (size_t)(T + kPT - 1) / kPT > max_pages) return Q3_ERR_CAPACITY;
  if ((size_t)n_seqs * T > 0x7fffffffu / L.inter) return Q3_ERR_CAPACITY;
  if (workspace_bytes < q3_prefill_workspace_bytes(layout, n_seqs, T)) return Q3_ERR_CAPACITY;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return Q3_ERR_ALIGN;
  if (!pool->k || !pool->v || !pool->ks || !pool->vs) return Q3_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *s = st;
  const int64_t *o = L.off;
  const uint32_t B = n_seqs, H = L.hidden, HD = L.head_dim, QW = L.heads * HD,
                 KW = L.kv_heads * HD, I = L.inter, V = L.vocab, HALF = HD / 2;
  const uint32_t M = B * T;
  char *bl = static_cast<char *>(blob);
  PrefillWs w = carve(L, M, B, static_cast<char *>(workspace));

  k_prefill_rope_rows<<<M, 64, 0, st>>>(reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]),
                                        reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]), HALF,
                                        T, w.cos, w.sin);
  Q3_TRY(q3h::launch_status());

  const q3_view x = v2(w.x, M, H, Q3_DT_F32), h = v2(w.h, M, H, Q3_DT_F32);
  const q3_view h8 = v2(w.h8, M, H, Q3_DT_I8), hs = v2(w.hs, M, H / 256, Q3_DT_F32);
  const q3_view q8 = v2(w.q8, M, QW, Q3_DT_I8), qs = v2(w.qs, M, L.heads, Q3_DT_F32);
  const q3_view o8 = v2(w.o8, M, QW, Q3_DT_I8), os = v2(w.os, M, L.heads, Q3_DT_F32);
  const q3_view k8 = v2(w.k8, M, KW, Q3_DT_I8), ks = v2(w.ks, M, L.kv_heads, Q3_DT_F32);
  const q3_view v8 = v2(w.v8, M, KW, Q3_DT_I8), vs = v2(w.vs, M, L.kv_heads, Q3_DT_F32);
  const q3_view s8 = v2(w.s8, M, I, Q3_DT_I8), ss = v2(w.ss, M, I / 256, Q3_DT_F32);
  const q3_view cosv = v2(w.cos, M, HALF, Q3_DT_F32), sinv = v2(w.sin, M, HALF, Q3_DT_F32);
  const q3_view idv = v2(const_cast<int32_t *>(ids), M, 1, Q3_DT_I32);
  const q3_view emb = v2(bl + o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = v2(bl + o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view lm = v2(bl + o[Q3_OFF_LM], V, H, Q3_DT_I8);
  const q3_view lm_s = v2(bl + o[Q3_OFF_LM] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view nf = v2(bl + o[Q3_OFF_NF], H, 1, Q3_DT_F32);
  const float inv_h = 1.0f / static_cast<float>(H), inv_hd = 1.0f / static_cast<float>(HD);

  {
    const q3_view n1_0 = v2(bl + o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &idv, &x, &n1_0, &h, inv_h, s));
  }
  // RMSNorm + quant of x into h8/hs: one pass for 1024-column rows, else the
  // two row operators through h
  auto norm_quant = [&](const float *nw, const q3_view &xv, const q3_view &nv) -> int {
    if (H == 1024) {
      k_norm_quant_1024<<<(M + 7) / 8, 256, 0, st>>>(w.x, nw, inv_h, (int)M, w.h8, w.hs);
      return q3h::launch_status();
    }
    Q3_TRY(q3_rmsnorm_rows(&xv, &nv, &h, inv_h, s));
    return q3_quant_rows_heads(&h, &h8, &hs, 256, s);
  };
  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    char *lw = bl + o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    char *ln = bl + o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    auto W = [&](int key, uint32_t r, uint32_t c) { return v2(lw + (o[key] - o[Q3_OFF_LQ]), r, c, Q3_DT_I8); };
    auto S = [&](int key, uint32_t r) { return v2(lw + (o[key] - o[Q3_OFF_LQ]), r, 1, Q3_DT_F32); };
    const q3_view wq = W(Q3_OFF_LQ, QW, H), wk = W(Q3_OFF_LK, KW, H), wv = W(Q3_OFF_LV, KW, H);
    const q3_view wo = W(Q3_OFF_LO, H, QW), wg = W(Q3_OFF_LG, I, H), wu = W(Q3_OFF_LU, I, H);
    const q3_view wd = W(Q3_OFF_LD, H, I);
    const q3_view wqs = S(Q3_OFF_LQ_SCALE, QW), wks = S(Q3_OFF_LK_SCALE, KW);
    const q3_view wvs = S(Q3_OFF_LV_SCALE, KW), wos = S(Q3_OFF_LO_SCALE, H);
    const q3_view wgs = S(Q3_OFF_LG_SCALE, I), wus = S(Q3_OFF_LU_SCALE, I);
    const q3_view wds = S(Q3_OFF_LD_SCALE, H);
    const q3_view n1 = v2(ln, H, 1, Q3_DT_F32);
    const q3_view nq = v2(ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view nk = v2(ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view n2 = v2(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]), H, 1, Q3_DT_F32);
    char *pk = static_cast<char *>(pool->k) + Li * pool->layer_stride;
    char *pv = static_cast<char *>(pool->v) + Li * pool->layer_stride;
    char *pks = static_cast<char *>(pool->ks) + Li * pool->scale_layer_stride;
    char *pvs = static_cast<char *>(pool->vs) + Li * pool->scale_layer_stride;

    if (Li != 0) Q3_TRY(norm_quant(reinterpret_cast<const float *>(ln), x, n1));
    else Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wv, &wvs, nullptr, 256, nullptr, &v8, &vs, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wk, &wks, nullptr, 256, nullptr, &k8, &ks, &nk,
                                  &cosv, &sinv, inv_hd, s));
    k_prefill_scatter<<<M, 64, 0, st>>>(w.k8, w.v8, w.ks, w.vs, tables, max_pages, (int)T, pk, pv,
                                        pks, pvs, KW, L.kv_heads);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wq, &wqs, nullptr, 256, nullptr, &q8, &qs, &nq, &cosv,
                                  &sinv, inv_hd, s));
    if (pool->num_pages > 0 && L.heads % L.kv_heads == 0 && (T + kPT - 1) / kPT <= max_pages) {
      q3::PrefillAttnArgs a{};
      a.qs = reinterpret_cast<const char *>(w.qs);
      a.qs_rb = 4 * L.heads;
      a.o8 = reinterpret_cast<char *>(w.o8);
      a.o_rb = QW;
      a.os = reinterpret_cast<char *>(w.os);
      a.os_rb = 4 * L.heads;
      a.ks = pks;
      a.vs = pvs;
      a.table = tables;
      a.table_stride = max_pages;
      a.scale_page_bytes = kPT * 4 * L.kv_heads;
      a.scale_row_bytes = 4 * L.kv_heads;
      a.num_pages = pool->num_pages;
      a.heads = L.heads;
      a.kv_heads = L.kv_heads;
      a.T = (int)T;
      a.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_prefill_launch(a, w.q8, QW, (int)M, pk, pv, kPT * KW, KW, (int)B, st));
    } else {
      q3::AttnArgs a{};
      a.q8 = reinterpret_cast<const char *>(w.q8);
      a.q_rb = QW;
      a.qs = reinterpret_cast<const char *>(w.qs);
      a.qs_rb = 4 * L.heads;
      a.o8 = reinterpret_cast<char *>(w.o8);
      a.o_rb = QW;
      a.os = reinterpret_cast<char *>(w.os);
      a.os_rb = 4 * L.heads;
      a.k = pk;
      a.v = pv;
      a.ks = pks;
      a.vs = pvs;
      a.table = tables;
      a.table_stride = max_pages;
      a.page_tokens = kPT;
      a.page_bytes = kPT * KW;
      a.row_bytes = KW;
      a.scale_page_bytes = kPT * 4 * L.kv_heads;
      a.scale_row_bytes = 4 * L.kv_heads;
      a.heads = L.heads;
      a.kv_heads = L.kv_heads;
      a.q_rows = (int)T;
      a.kv_len = (int)T;
      a.kv_len_dev = nullptr;
      a.causal = 1;
      a.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_launch(a, (int)B, st));
    }
    Q3_TRY(q3_gemm_nt_group_store(&o8, &os, &wo, &wos, nullptr, 128, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(norm_quant(reinterpret_cast<const float *>(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1])), x, n2));
    Q3_TRY(q3_gemm_gate_up_swiglu_quant(&h8, &hs, &wg, &wgs, &wu, &wus, &s8, &ss, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&s8, &ss, &wd, &wds, nullptr, 256, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
  }
  // last row of every sequence: final norm + quant, lm_head fused with argmax
  k_prefill_last_rows<<<B, 256, 0, st>>>(w.x, (int)T, (int)H, w.xl, w.best, next_ids);
  Q3_TRY(q3h::launch_status());
  const q3_view xl = v2(w.xl, B, H, Q3_DT_F32), hl = v2(w.hl, B, H, Q3_DT_F32);
  const q3_view h8l = v2(w.h8l, B, H, Q3_DT_I8), hsl = v2(w.hsl, B, H / 256, Q3_DT_F32);
  Q3_TRY(q3_rmsnorm_rows(&xl, &nf, &hl, inv_h, s));
  Q3_TRY(q3_quant_rows_heads(&hl, &h8l, &hsl, 256, s));
  return q3_gemm_nt_group_argmax(&h8l, &hsl, &lm, &lm_s, w.best, next_ids, 256, w.keys, 8 * B, s);
}

// ---------------------------------------------------------------------------
// Tensor-parallel prefill: the same batched prefill with the layer split over
// the ranks of a q3::PfComm, bit-identical to q3_prefill_batch on one GPU.
// Rank r owns the KV heads and q heads of its shard (q3_tp_shard_of), the
// MLP groups of its shard, a slice of H / world residual columns and its
// vocabulary rows.  Per layer, every rank:
//   RMSNorm + quant of the full residual x (replicated, same bits everywhere);
//   V, K (head norm/rope/quant) and Q GEMMs for its heads only, its K/V into
//   its own page pool, causal attention over its heads -> its o8/os columns;
//   all-gather of o8/os;
//   O for its residual columns, every K group summed in the reference's
//   order by the one GEMM (ref_qwen3.py:152-157) -> its x columns; all-gather;
//   RMSNorm + quant (replicated); gate/up SwiGLU for its MLP groups -> its
//   s8/ss columns; all-gather; down for its x columns; all-gather.
// Every output element is computed by exactly one rank with the single-GPU
// arithmetic, so no sum changes order.  The exchanges copy each rank's
// columns into every other rank's region over NVLink (CUDA IPC) and signal
// with system-scope counters (q3_tp.cu); the last rows' lm_head runs over
// the rank's vocabulary rows and the (max, first index) keys are exchanged.
// ---------------------------------------------------------------------------
namespace {

using q3::kEps;
using q3::kInv127;
using q3::quant1;
using q3::rsqrt_ref;
using q3::warp_tree_max;
using q3::warp_tree_sum;

// RMSNorm + per-256 quant (rmsnorm.h:34-81, quant.h:89-138) of a residual
// stream whose columns [c0, c0 + nc) are this rank's, in three steps with an
// all-gather after each (the reference's arithmetic, split at its exchange
// points):
//   1. the tree sum of x^2 of each of this rank's 32-column blocks;
//   2. with every block sum: ss summed over the blocks in order, r, h = (x r) w
//      for this rank's columns, and the maximum of |h| per 128 columns;
//   3. with every maximum: the scale of each 256-column group (every rank
//      computes all of them) and the int8 codes of this rank's columns.
// One warp per (row, 32-column block) in step 1, per (row, 128-column chunk)
// in steps 2 and 3.
__global__ void k_pf_block_sums(const float *x, int M, int H, int c0, int nc, float *bsum) {
  const int nbl = nc / 32;
  const long wi = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= static_cast<long>(M) * nbl) return;
  const int m = static_cast<int>(wi / nbl), b = c0 / 32 + static_cast<int>(wi % nbl);
  const float v = x[static_cast<size_t>(m) * H + 32 * b + lane];
  const float t = warp_tree_sum(__fmul_rn(v, v));
  if (lane == 0) bsum[static_cast<size_t>(m) * (H / 32) + b] = t;
}

__global__ void k_pf_norm_amax(const float *x, const float *bsum, const float *w, float inv, int M,
                               int H, int c0, int nc, float *hc, float *amax) {
  const int nch = nc / 128;
  const long wi = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= static_cast<long>(M) * nch) return;
  const int m = static_cast<int>(wi / nch), ch = static_cast<int>(wi % nch);
  const float *bs = bsum + static_cast<size_t>(m) * (H / 32);
  float ss = 0.0f;
  if (H == 1024) {                                   // 32 block sums loaded at once
    float4 b4[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) b4[i] = reinterpret_cast<const float4 *>(bs)[i];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ss = __fadd_rn(ss, b4[i].x);
      ss = __fadd_rn(ss, b4[i].y);
      ss = __fadd_rn(ss, b4[i].z);
      ss = __fadd_rn(ss, b4[i].w);
    }
  } else {
    for (int b = 0; b < H / 32; ++b) ss = __fadd_rn(ss, bs[b]);  // blocks in order
  }
  ss = __fmul_rn(ss, inv);
  ss = __fadd_rn(ss, kEps);
  const float r = rsqrt_ref(ss);
  float mx = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int col = c0 + 128 * ch + 32 * k + lane;
    const float h = __fmul_rn(__fmul_rn(x[static_cast<size_t>(m) * H + col], r), w[col]);
    hc[static_cast<size_t>(m) * nc + (col - c0)] = h;
    mx = fmaxf(mx, fabsf(h));
  }
  mx = warp_tree_max(mx);
  if (lane == 0) amax[static_cast<size_t>(m) * (H / 128) + (c0 / 128 + ch)] = mx;
}

__global__ void k_pf_quant_cols(const float *hc, const float *amax, int M, int H, int c0, int nc,
                                int8_t *h8, float *hs) {
  const int nch = nc / 128;
  const long wi = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (wi >= static_cast<long>(M) * nch) return;
  const int m = static_cast<int>(wi / nch), ch = static_cast<int>(wi % nch);
  const float *am = amax + static_cast<size_t>(m) * (H / 128);
  const int gc = (c0 / 128 + ch) / 2;                                 // this chunk's 256-group
  const float scale = __fmul_rn(fmaxf(am[2 * gc], am[2 * gc + 1]), kInv127);
  if (ch == 0 && lane < H / 256)                                     // every group's scale
    hs[static_cast<size_t>(m) * (H / 256) + lane] =
        __fmul_rn(fmaxf(am[2 * lane], am[2 * lane + 1]), kInv127);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int col = c0 + 128 * ch + 32 * k + lane;
    h8[static_cast<size_t>(m) * H + col] =
        static_cast<int8_t>(quant1(hc[static_cast<size_t>(m) * nc + (col - c0)], scale));
  }
}

inline unsigned warps_grid(long warps) { return static_cast<unsigned>((warps * 32 + 255) / 256); }

}  // namespace

extern "C" int q3_tp_prefill_batch(void *comm, void *blob, const q3_layout *layout,
                                   const q3_kv_pool *pool, const uint16_t *tables,
                                   uint32_t max_pages, const int32_t *ids, uint32_t n_seqs,
                                   uint32_t T, int32_t *next_ids, void *workspace,
                                   size_t workspace_bytes, void *stream) {
  if (!comm || !blob || !layout || !pool || !tables || !ids || !next_ids || !workspace)
    return Q3_ERR_NULL;
  q3::PfComm &c = *static_cast<q3::PfComm *>(comm);
  const q3_layout &L = *layout;
  if (L.head_dim != 128 || L.hidden % 256 || L.inter % 256 || L.max_seq % kPT ||
      L.hidden != c.hidden || L.heads != c.heads || L.inter != c.inter)
    return Q3_ERR_SHAPE;
  if (n_seqs == 0 || T == 0) return Q3_OK;
  for (int q = 0; q < c.world; ++q)
    if (!c.peer[q]) return Q3_ERR_NULL;   // not connected
  if (T > L.max_seq || (size_t)(T + kPT - 1) / kPT > max_pages) return Q3_ERR_CAPACITY;
  if ((size_t)n_seqs * T > c.max_rows || n_seqs > c.max_seqs) return Q3_ERR_CAPACITY;
  if ((size_t)n_seqs * T > 0x7fffffffu / L.inter) return Q3_ERR_CAPACITY;
  if (workspace_bytes < q3_prefill_workspace_bytes(layout, n_seqs, T)) return Q3_ERR_CAPACITY;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return Q3_ERR_ALIGN;
  if (!pool->k || !pool->v || !pool->ks || !pool->vs || pool->num_pages == 0) return Q3_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *s = st;
  const int64_t *o = L.off;
  const q3_tp_shard &sh = c.shard[c.rank];
  const uint32_t B = n_seqs, H = L.hidden, HD = L.head_dim, QW = L.heads * HD, I = L.inter,
                 V = L.vocab, HALF = HD / 2, HEADS = L.heads, G = I / 256;
  const uint32_t QH = sh.q_heads, KVH = sh.kv_heads, QWl = QH * HD, KWl = KVH * HD;
  const uint32_t c0 = c.col0[c.rank], NC = c.cols[c.rank];
  const uint32_t g0 = sh.mlp_group0, NG = sh.mlp_groups;
  const uint32_t M = B * T;
  char *bl = static_cast<char *>(blob);
  PrefillWs w = carve(L, M, B, static_cast<char *>(workspace));
  char *R = c.local;
  int8_t *o8f = reinterpret_cast<int8_t *>(R + c.off_o8);
  float *osf = reinterpret_cast<float *>(R + c.off_os);
  float *xf = reinterpret_cast<float *>(R + c.off_x);
  int8_t *s8f = reinterpret_cast<int8_t *>(R + c.off_s8);
  float *ssf = reinterpret_cast<float *>(R + c.off_ss);
  int8_t *h8f = reinterpret_cast<int8_t *>(R + c.off_h8);
  float *bsumf = reinterpret_cast<float *>(R + c.off_bsum);
  float *amaxf = reinterpret_cast<float *>(R + c.off_amax);

  k_prefill_rope_rows<<<M, 64, 0, st>>>(reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]),
                                        reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]), HALF,
                                        T, w.cos, w.sin);
  Q3_TRY(q3h::launch_status());

  const q3_view x = v2(xf, M, H, Q3_DT_F32), h = v2(w.h, M, H, Q3_DT_F32);
  const q3_view h8 = v2(h8f, M, H, Q3_DT_I8), hs = v2(w.hs, M, H / 256, Q3_DT_F32);
  const q3_view q8 = v2(w.q8, M, QWl, Q3_DT_I8), qs = v2(w.qs, M, QH, Q3_DT_F32);
  const q3_view k8 = v2(w.k8, M, KWl, Q3_DT_I8), ks = v2(w.ks, M, KVH, Q3_DT_F32);
  const q3_view v8 = v2(w.v8, M, KWl, Q3_DT_I8), vs = v2(w.vs, M, KVH, Q3_DT_F32);
  const q3_view o8 = v2(o8f, M, QW, Q3_DT_I8), os = v2(osf, M, HEADS, Q3_DT_F32);
  const q3_view s8 = v2(s8f, M, I, Q3_DT_I8), ss = v2(ssf, M, G, Q3_DT_F32);
  // this rank's columns of the exchanged buffers
  q3_view xc = v2(xf + c0, M, NC, Q3_DT_F32);
  xc.row_bytes = static_cast<int32_t>(4 * H);
  q3_view s8c = v2(s8f + g0 * 256, M, NG * 256, Q3_DT_I8);
  s8c.row_bytes = static_cast<int32_t>(I);
  q3_view ssc = v2(ssf + g0, M, NG, Q3_DT_F32);
  ssc.row_bytes = static_cast<int32_t>(4 * G);
  const q3_view cosv = v2(w.cos, M, HALF, Q3_DT_F32), sinv = v2(w.sin, M, HALF, Q3_DT_F32);
  const q3_view idv = v2(const_cast<int32_t *>(ids), M, 1, Q3_DT_I32);
  const q3_view emb = v2(bl + o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = v2(bl + o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view lm = v2(bl + o[Q3_OFF_LM] + (int64_t)sh.vocab0 * H, sh.vocab_rows, H, Q3_DT_I8);
  const q3_view lm_s = v2(bl + o[Q3_OFF_LM] + (int64_t)V * H + (int64_t)sh.vocab0 * 4,
                          sh.vocab_rows, 1, Q3_DT_F32);
  const q3_view nf = v2(bl + o[Q3_OFF_NF], H, 1, Q3_DT_F32);
  const float inv_h = 1.0f / static_cast<float>(H), inv_hd = 1.0f / static_cast<float>(HD);
  const q3::PfSeg seg_o8{c.off_o8, sh.q_head0 * HD, QWl, QW};
  const q3::PfSeg seg_os{c.off_os, sh.q_head0 * 4, QH * 4, HEADS * 4};
  const q3::PfSeg seg_s8{c.off_s8, g0 * 256, NG * 256, I};
  const q3::PfSeg seg_bsum{c.off_bsum, c0 / 32 * 4, NC / 32 * 4, H / 32 * 4};
  const q3::PfSeg seg_amax{c.off_amax, c0 / 128 * 4, NC / 128 * 4, H / 128 * 4};
  const q3::PfSeg seg_h8{c.off_h8, c0, NC, H};
  // RMSNorm(nw) + quant of the column-sharded residual into h8 (all columns) / hs
  auto sharded_norm = [&](const float *nw) -> int {
    k_pf_block_sums<<<warps_grid((long)M * (NC / 32)), 256, 0, st>>>(xf, (int)M, (int)H, (int)c0,
                                                                     (int)NC, bsumf);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3::pf_push(c, q3::PF_NB, &seg_bsum, 1, M, st));
    Q3_TRY(q3::pf_wait(c, q3::PF_NB, st));
    k_pf_norm_amax<<<warps_grid((long)M * (NC / 128)), 256, 0, st>>>(
        xf, bsumf, nw, 1.0f / static_cast<float>(H), (int)M, (int)H, (int)c0, (int)NC, w.h, amaxf);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3::pf_push(c, q3::PF_NA, &seg_amax, 1, M, st));
    Q3_TRY(q3::pf_wait(c, q3::PF_NA, st));
    k_pf_quant_cols<<<warps_grid((long)M * (NC / 128)), 256, 0, st>>>(w.h, amaxf, (int)M, (int)H,
                                                                      (int)c0, (int)NC, h8f, w.hs);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3::pf_push(c, q3::PF_NH, &seg_h8, 1, M, st));
    return q3::pf_wait(c, q3::PF_NH, st);
  };
  const q3::PfSeg seg_ss{c.off_ss, g0 * 4, NG * 4, G * 4};

  {
    const q3_view n1_0 = v2(bl + o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &idv, &x, &n1_0, &h, inv_h, s));
  }
  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    char *lw = bl + o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    char *ln = bl + o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    // rows [r0, r0 + r) of a weight matrix (K = c columns) and of its scales
    auto W = [&](int key, uint32_t r0, uint32_t r, uint32_t cc) {
      return v2(lw + (o[key] - o[Q3_OFF_LQ]) + static_cast<int64_t>(r0) * cc, r, cc, Q3_DT_I8);
    };
    auto S = [&](int key, uint32_t r0, uint32_t r) {
      return v2(lw + (o[key] - o[Q3_OFF_LQ]) + static_cast<int64_t>(r0) * 4, r, 1, Q3_DT_F32);
    };
    const q3_view wq = W(Q3_OFF_LQ, sh.q_head0 * HD, QWl, H), wqs = S(Q3_OFF_LQ_SCALE, sh.q_head0 * HD, QWl);
    const q3_view wk = W(Q3_OFF_LK, sh.kv_head0 * HD, KWl, H), wks = S(Q3_OFF_LK_SCALE, sh.kv_head0 * HD, KWl);
    const q3_view wv = W(Q3_OFF_LV, sh.kv_head0 * HD, KWl, H), wvs = S(Q3_OFF_LV_SCALE, sh.kv_head0 * HD, KWl);
    const q3_view wo = W(Q3_OFF_LO, c0, NC, QW), wos = S(Q3_OFF_LO_SCALE, c0, NC);
    const q3_view wg = W(Q3_OFF_LG, g0 * 256, NG * 256, H), wgs = S(Q3_OFF_LG_SCALE, g0 * 256, NG * 256);
    const q3_view wu = W(Q3_OFF_LU, g0 * 256, NG * 256, H), wus = S(Q3_OFF_LU_SCALE, g0 * 256, NG * 256);
    const q3_view wd = W(Q3_OFF_LD, c0, NC, I), wds = S(Q3_OFF_LD_SCALE, c0, NC);
    const q3_view n1 = v2(ln, H, 1, Q3_DT_F32);
    const q3_view nq = v2(ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view nk = v2(ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view n2 = v2(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]), H, 1, Q3_DT_F32);
    char *pk = static_cast<char *>(pool->k) + Li * pool->layer_stride;
    char *pv = static_cast<char *>(pool->v) + Li * pool->layer_stride;
    char *pks = static_cast<char *>(pool->ks) + Li * pool->scale_layer_stride;
    char *pvs = static_cast<char *>(pool->vs) + Li * pool->scale_layer_stride;

    // layer 0: x is the embedding, whole on every rank (h from the embedding
    // step); later layers: the column-sharded residual
    if (Li == 0) Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    else Q3_TRY(sharded_norm(reinterpret_cast<const float *>(ln)));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wv, &wvs, nullptr, 256, nullptr, &v8, &vs, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wk, &wks, nullptr, 256, nullptr, &k8, &ks, &nk,
                                  &cosv, &sinv, inv_hd, s));
    k_prefill_scatter<<<M, 64, 0, st>>>(w.k8, w.v8, w.ks, w.vs, tables, max_pages, (int)T, pk, pv,
                                        pks, pvs, KWl, KVH);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wq, &wqs, nullptr, 256, nullptr, &q8, &qs, &nq, &cosv,
                                  &sinv, inv_hd, s));
    {
      q3::PrefillAttnArgs a{};
      a.qs = reinterpret_cast<const char *>(w.qs);
      a.qs_rb = 4 * QH;
      a.o8 = reinterpret_cast<char *>(o8f + sh.q_head0 * HD);
      a.o_rb = QW;
      a.os = reinterpret_cast<char *>(osf + sh.q_head0);
      a.os_rb = 4 * HEADS;
      a.ks = pks;
      a.vs = pvs;
      a.table = tables;
      a.table_stride = max_pages;
      a.scale_page_bytes = kPT * 4 * KVH;
      a.scale_row_bytes = 4 * KVH;
      a.num_pages = pool->num_pages;
      a.heads = (int)QH;
      a.kv_heads = (int)KVH;
      a.T = (int)T;
      a.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_prefill_launch(a, w.q8, QWl, (int)M, pk, pv, kPT * KWl, KWl, (int)B, st));
    }
    {
      const q3::PfSeg sg[2] = {seg_o8, seg_os};
      Q3_TRY(q3::pf_push(c, q3::PF_O, sg, 2, M, st));
      Q3_TRY(q3::pf_wait(c, q3::PF_O, st));
    }
    Q3_TRY(q3_gemm_nt_group_store(&o8, &os, &wo, &wos, nullptr, 128, &xc, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(sharded_norm(reinterpret_cast<const float *>(n2.data)));
    Q3_TRY(q3_gemm_gate_up_swiglu_quant(&h8, &hs, &wg, &wgs, &wu, &wus, &s8c, &ssc, 256, s));
    {
      const q3::PfSeg sg[2] = {seg_s8, seg_ss};
      Q3_TRY(q3::pf_push(c, q3::PF_S, sg, 2, M, st));
      Q3_TRY(q3::pf_wait(c, q3::PF_S, st));
    }
    Q3_TRY(q3_gemm_nt_group_store(&s8, &ss, &wd, &wds, nullptr, 256, &xc, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
  }
  // last row of every sequence: its residual columns gathered, final norm +
  // quant (replicated), lm_head over this rank's vocabulary rows, key exchange
  {
    const q3::PfSeg seg_xl{c.off_x + static_cast<size_t>(T - 1) * H * 4, c0 * 4, NC * 4, T * H * 4};
    Q3_TRY(q3::pf_push(c, q3::PF_XL, &seg_xl, 1, B, st));
    Q3_TRY(q3::pf_wait(c, q3::PF_XL, st));
  }
  k_prefill_last_rows<<<B, 256, 0, st>>>(xf, (int)T, (int)H, w.xl, w.best, next_ids);
  Q3_TRY(q3h::launch_status());
  const q3_view xl = v2(w.xl, B, H, Q3_DT_F32), hl = v2(w.hl, B, H, Q3_DT_F32);
  const q3_view h8l = v2(w.h8l, B, H, Q3_DT_I8), hsl = v2(w.hsl, B, H / 256, Q3_DT_F32);
  Q3_TRY(q3_rmsnorm_rows(&xl, &nf, &hl, inv_h, s));
  Q3_TRY(q3_quant_rows_heads(&hl, &h8l, &hsl, 256, s));
  Q3_TRY(q3_gemm_nt_group_argmax(&h8l, &hsl, &lm, &lm_s, w.best, next_ids, 256, w.keys, 8 * B, s));
  return q3::pf_argmax_exchange(c, w.best, next_ids, sh.vocab0, (int)B, st);
}
