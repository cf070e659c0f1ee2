// Batched paged decode: one new token for each of n_seqs independent
// sequences, every sequence with its own page table into a shared KV page
// pool (kernels/kv_pages.h:98-131 semantics, tools/engine.py's PagePool
// layout).  Per row the arithmetic is exactly forward_chunk's for rows = 1
// (src/main_big.cpp:145-296): rows never interact, so batching them through
// one GEMM is bit-identical to running the sequences one by one.
#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_decode_gemm.h"
#include "q3_gemm.h"
#include "q3_tp.h"

namespace q3 {
struct NormQuantArgs {
  const float *x;
  const float *bsum;
  const float *w;
  float inv;
  int B, H;
  int8_t *h8;
  float *hs;
};
int norm_quant(const NormQuantArgs &a, cudaStream_t s);
}  // namespace q3

namespace {

constexpr uint32_t kPT = 32;   // page tokens
constexpr float kInvSqrt128 = 0.08838834764831845f;

struct DecodeWs {
  float *x, *h;          // [B][H]
  int8_t *h8;            // [B][H]
  float *hs;             // [B][H/256]
  int8_t *q8, *o8;       // [B][QW]
  float *qs, *os;        // [B][heads]
  int8_t *k8, *v8;       // [B][KW] staging of the new K/V rows
  float *ks, *vs;        // [B][kv_heads]
  int8_t *s8;            // [B][I]
  float *ss;             // [B][I/256]
  float *cos, *sin;      // [B][64] rows at each sequence's position
  int *kv_len;           // [B]
  float *best;           // [B]
  unsigned long long *keys;  // [B]
  float *bsum;           // [B][H/32] tree sums of x^2 per 32-column block
  int32_t *lidx;         // [B] argmax index within this rank's vocabulary slice
  size_t total;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

DecodeWs carve(const q3_layout &L, uint32_t B, char *base) {
  const size_t H = L.hidden, QW = L.heads * L.head_dim, KW = L.kv_heads * L.head_dim, I = L.inter;
  DecodeWs w{};
  size_t off = 0;
  auto take = [&](size_t bytes) { char *p = base ? base + off : nullptr; off += align256(bytes); return p; };
  w.x = (float *)take(4 * B * H);
  w.h = (float *)take(4 * B * H);
  w.h8 = (int8_t *)take(B * H);
  w.hs = (float *)take(4 * B * (H / 256));
  w.q8 = (int8_t *)take(B * QW);
  w.o8 = (int8_t *)take(B * QW);
  w.qs = (float *)take(4 * B * L.heads);
  w.os = (float *)take(4 * B * L.heads);
  w.k8 = (int8_t *)take(B * KW);
  w.v8 = (int8_t *)take(B * KW);
  w.ks = (float *)take(4 * B * L.kv_heads);
  w.vs = (float *)take(4 * B * L.kv_heads);
  w.s8 = (int8_t *)take(B * I);
  w.ss = (float *)take(4 * B * (I / 256));
  w.cos = (float *)take(4 * B * (L.head_dim / 2));
  w.sin = (float *)take(4 * B * (L.head_dim / 2));
  w.kv_len = (int *)take(4 * B);
  w.best = (float *)take(4 * B);
  w.keys = (unsigned long long *)take(8 * B);
  w.bsum = (float *)take(4 * B * (H / 32));
  w.lidx = (int32_t *)take(4 * B);
  w.total = off;
  return w;
}

q3_view v2(void *p, uint32_t rows, uint32_t cols, uint8_t dt) {
  const int es = (dt == Q3_DT_I8 || dt == Q3_DT_U8) ? 1 : 4;
  return q3_view{p, static_cast<int32_t>(cols * es), es, rows, cols, dt};
}

// rope rows at each sequence's position; kv_len = pos + 1; best = -3e38
__global__ void k_decode_prep(const int32_t *pos, const float *cos_t, const float *sin_t, int half,
                              float *cos, float *sin, int *kv_len, float *best,
                              int32_t *next_ids, int B) {
  const int s = blockIdx.x;
  const int p = pos[s];
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    cos[s * half + j] = cos_t[p * half + j];
    sin[s * half + j] = sin_t[p * half + j];
  }
  if (threadIdx.x == 0) {
    kv_len[s] = p + 1;
    best[s] = -3.0e38f;
    next_ids[s] = 0;
  }
}

// new K/V row of sequence s -> its page (tables[s][pos/32], slot pos%32)
__global__ void k_decode_scatter(const int8_t *k8, const int8_t *v8, const float *ks,
                                 const float *vs, const int32_t *pos, const uint16_t *tables,
                                 uint32_t max_pages, char *pk, char *pv, char *pks, char *pvs,
                                 int kw, int kvh) {
  const int s = blockIdx.x;
  const int p = pos[s];
  const uint32_t page = tables[static_cast<size_t>(s) * max_pages + p / kPT], slot = p % kPT;
  const size_t row = static_cast<size_t>(page) * kPT + slot;
  for (int i = threadIdx.x; i < kw / 16; i += blockDim.x) {
    reinterpret_cast<int4 *>(pk + row * kw)[i] = reinterpret_cast<const int4 *>(k8 + (size_t)s * kw)[i];
    reinterpret_cast<int4 *>(pv + row * kw)[i] = reinterpret_cast<const int4 *>(v8 + (size_t)s * kw)[i];
  }
  for (int h = threadIdx.x; h < kvh; h += blockDim.x) {
    reinterpret_cast<float *>(pks + row * kvh * 4)[h] = ks[s * kvh + h];
    reinterpret_cast<float *>(pvs + row * kvh * 4)[h] = vs[s * kvh + h];
  }
}

__global__ void k_keys_to_ids(const unsigned long long *keys, int32_t *next_ids, int B) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s < B) next_ids[s] = static_cast<int32_t>(0xffffffffu - static_cast<unsigned>(keys[s] & 0xffffffffu));
}

// The batched step: per layer RMSNorm+quant, QKV (head norm/rope/quant into the
// KV pages), attention, O (+ residual), RMSNorm+quant, gate/up (SwiGLU+quant),
// down (+ residual) -- 7 launches, each a programmatic dependent of the one
// before.  Same arithmetic as the operator-by-operator path.
int decode_fused(char *bl, const q3_layout &L, const q3_kv_pool *pool, const uint16_t *tables,
                 uint32_t max_pages, const int32_t *ids, const int32_t *pos, uint32_t B,
                 int32_t *next_ids, const DecodeWs &w, cudaStream_t st) {
  void *s = st;
  const int64_t *o = L.off;
  const uint32_t H = L.hidden, HD = L.head_dim, QW = L.heads * HD, KW = L.kv_heads * HD,
                 I = L.inter, V = L.vocab;
  const float inv_h = 1.0f / static_cast<float>(H), inv_hd = 1.0f / static_cast<float>(HD);
  const q3_view x = v2(w.x, B, H, Q3_DT_F32), h = v2(w.h, B, H, Q3_DT_F32);
  const q3_view h8 = v2(w.h8, B, H, Q3_DT_I8), hs = v2(w.hs, B, H / 256, Q3_DT_F32);
  const q3_view q8 = v2(w.q8, B, QW, Q3_DT_I8), qs = v2(w.qs, B, L.heads, Q3_DT_F32);
  const q3_view idv = v2(const_cast<int32_t *>(ids), B, 1, Q3_DT_I32);
  const q3_view emb = v2(bl + o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = v2(bl + o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view lm = v2(bl + o[Q3_OFF_LM], V, H, Q3_DT_I8);
  const q3_view lm_s = v2(bl + o[Q3_OFF_LM] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const float *cos_t = reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]);
  const float *sin_t = reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]);
  {
    const q3_view n1_0 = v2(bl + o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &idv, &x, &n1_0, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
  }
  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    char *lw = bl + o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    char *ln = bl + o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    auto Wp = [&](int key) { return reinterpret_cast<const int8_t *>(lw + (o[key] - o[Q3_OFF_LQ])); };
    auto Sp = [&](int key) { return reinterpret_cast<const float *>(lw + (o[key] - o[Q3_OFF_LQ])); };
    const float *nq = reinterpret_cast<const float *>(ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]));
    const float *nk = reinterpret_cast<const float *>(ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]));
    const float *n2 = reinterpret_cast<const float *>(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]));
    char *pk = static_cast<char *>(pool->k) + Li * pool->layer_stride;
    char *pv = static_cast<char *>(pool->v) + Li * pool->layer_stride;
    char *pks = static_cast<char *>(pool->ks) + Li * pool->scale_layer_stride;
    char *pvs = static_cast<char *>(pool->vs) + Li * pool->scale_layer_stride;

    // RMSNorm(n1) + quant of x -> h8/hs (layer 0: the embedding step did it)
    if (Li > 0) {
      q3::NormQuantArgs a{w.x, w.bsum, reinterpret_cast<const float *>(ln), inv_h, (int)B, (int)H,
                          w.h8, w.hs};
      Q3_TRY(q3::norm_quant(a, st));
    }
    // Q | K | V, head norm/rope/quant into q8 and the KV pages
    {
      const int8_t *wts[3] = {Wp(Q3_OFF_LQ), Wp(Q3_OFF_LK), Wp(Q3_OFF_LV)};
      const int rows[3] = {(int)QW, (int)KW, (int)KW};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.hs);
      a.as_rb = 4 * (H / 256);
      a.ws[0] = Sp(Q3_OFF_LQ_SCALE);
      a.ws[1] = Sp(Q3_OFF_LK_SCALE);
      a.ws[2] = Sp(Q3_OFF_LV_SCALE);
      a.heads = (int)L.heads;
      a.kv_heads = (int)L.kv_heads;
      a.nq = nq;
      a.nk = nk;
      a.cos_t = cos_t;
      a.sin_t = sin_t;
      a.pos = pos;
      a.inv_hd = inv_hd;
      a.q8 = w.q8;
      a.qs = w.qs;
      a.pk = pk;
      a.pv = pv;
      a.pks = pks;
      a.pvs = pvs;
      a.tables = tables;
      a.max_pages = max_pages;
      Q3_TRY(q3::dgemm_launch(q3::DG_QKV, 3, wts, rows, w.h8, H, (int)H, 256, a, st));
    }
    // attention
    {
      q3::DecodeAttnArgs d{};
      d.q8 = reinterpret_cast<const char *>(w.q8);
      d.q_rb = QW;
      d.qs = reinterpret_cast<const char *>(w.qs);
      d.qs_rb = 4 * L.heads;
      d.o8 = reinterpret_cast<char *>(w.o8);
      d.o_rb = QW;
      d.os = reinterpret_cast<char *>(w.os);
      d.os_rb = 4 * L.heads;
      d.ks = pks;
      d.vs = pvs;
      d.table = tables;
      d.table_stride = max_pages;
      d.page_bytes = kPT * KW;
      d.row_bytes = KW;
      d.scale_page_bytes = kPT * 4 * L.kv_heads;
      d.scale_row_bytes = 4 * L.kv_heads;
      d.kv_len = w.kv_len;
      d.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_decode_launch(d, pk, pv, pool->num_pages, L.kv_heads, B, st, true));
    }
    // O + residual -> x (and its block sums)
    {
      const int8_t *wts[1] = {Wp(Q3_OFF_LO)};
      const int rows[1] = {(int)H};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.os);
      a.as_rb = 4 * L.heads;
      a.ws[0] = Sp(Q3_OFF_LO_SCALE);
      a.x = w.x;
      a.bsum = w.bsum;
      a.H = (int)H;
      Q3_TRY(q3::dgemm_launch(q3::DG_RESID, 1, wts, rows, w.o8, QW, (int)QW, 128, a, st));
    }
    // RMSNorm(n2) + quant -> h8/hs
    {
      q3::NormQuantArgs a{w.x, w.bsum, n2, inv_h, (int)B, (int)H, w.h8, w.hs};
      Q3_TRY(q3::norm_quant(a, st));
    }
    // gate/up -> SwiGLU + quant -> s8/ss
    {
      const int8_t *wts[2] = {Wp(Q3_OFF_LG), Wp(Q3_OFF_LU)};
      const int rows[2] = {(int)I, (int)I};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.hs);
      a.as_rb = 4 * (H / 256);
      a.ws[0] = Sp(Q3_OFF_LG_SCALE);
      a.ws[1] = Sp(Q3_OFF_LU_SCALE);
      a.s8 = w.s8;
      a.ss = w.ss;
      a.I = (int)I;
      Q3_TRY(q3::dgemm_launch(q3::DG_SWIGLU, 2, wts, rows, w.h8, H, (int)H, 256, a, st));
    }
    // down + residual -> x (and its block sums)
    {
      const int8_t *wts[1] = {Wp(Q3_OFF_LD)};
      const int rows[1] = {(int)H};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.ss);
      a.as_rb = 4 * (I / 256);
      a.ws[0] = Sp(Q3_OFF_LD_SCALE);
      a.x = w.x;
      a.bsum = w.bsum;
      a.H = (int)H;
      Q3_TRY(q3::dgemm_launch(q3::DG_RESID, 1, wts, rows, w.s8, I, (int)I, 256, a, st));
    }
  }
  // final RMSNorm + quant, then lm_head fused with argmax
  {
    q3::NormQuantArgs a{w.x, w.bsum, reinterpret_cast<const float *>(bl + o[Q3_OFF_NF]), inv_h,
                        (int)B, (int)H, w.h8, w.hs};
    Q3_TRY(q3::norm_quant(a, st));
  }
  Q3_TRY(q3_gemm_nt_group_argmax(&h8, &hs, &lm, &lm_s, w.best, next_ids, 256, w.keys, 8 * B, s));
  return Q3_OK;
}

// One rank's share of the batched step under tensor parallelism (the shard of
// q3_tp_shard_of): Q/K/V, the head epilogues and attention for its heads only,
// O and down as per-group partials stored to every rank (PART GEMM mode) and
// summed in group order by the reduce kernel, which also adds the residual and
// runs the next RMSNorm + quant; gate/up for its 256-wide groups; lm_head for
// its vocabulary rows, then the exchange of the (max, index) keys.
int tp_decode(const q3::TpComm &c, char *bl, const q3_layout &L, const q3_kv_pool *pool,
              const uint16_t *tables, uint32_t max_pages, const int32_t *ids, const int32_t *pos,
              uint32_t B, int32_t *next_ids, const DecodeWs &w, cudaStream_t st) {
  void *s = st;
  const int64_t *o = L.off;
  const q3_tp_shard &sh = c.shard[c.rank];
  const uint32_t H = L.hidden, HD = L.head_dim, QW = L.heads * HD, I = L.inter, V = L.vocab;
  const uint32_t QH = sh.q_heads, KVH = sh.kv_heads, QWl = QH * HD, KWl = KVH * HD;
  const uint32_t Gl = sh.mlp_groups, Il = Gl * 256;
  const float inv_h = 1.0f / static_cast<float>(H), inv_hd = 1.0f / static_cast<float>(HD);
  const q3_view x = v2(w.x, B, H, Q3_DT_F32), h = v2(w.h, B, H, Q3_DT_F32);
  const q3_view h8 = v2(w.h8, B, H, Q3_DT_I8), hs = v2(w.hs, B, H / 256, Q3_DT_F32);
  const q3_view idv = v2(const_cast<int32_t *>(ids), B, 1, Q3_DT_I32);
  const q3_view emb = v2(bl + o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = v2(bl + o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const float *cos_t = reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]);
  const float *sin_t = reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]);
  {
    const q3_view n1_0 = v2(bl + o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &idv, &x, &n1_0, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
  }
  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    char *lw = bl + o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    char *ln = bl + o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    auto Wp = [&](int key) { return reinterpret_cast<const int8_t *>(lw + (o[key] - o[Q3_OFF_LQ])); };
    auto Sp = [&](int key) { return reinterpret_cast<const float *>(lw + (o[key] - o[Q3_OFF_LQ])); };
    const float *nq = reinterpret_cast<const float *>(ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]));
    const float *nk = reinterpret_cast<const float *>(ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]));
    const float *n2 = reinterpret_cast<const float *>(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]));
    const float *n_next = Li + 1 < L.layers
                              ? reinterpret_cast<const float *>(ln + o[Q3_OFF_LAYERN_STRIDE])
                              : reinterpret_cast<const float *>(bl + o[Q3_OFF_NF]);
    char *pk = static_cast<char *>(pool->k) + Li * pool->layer_stride;
    char *pv = static_cast<char *>(pool->v) + Li * pool->layer_stride;
    char *pks = static_cast<char *>(pool->ks) + Li * pool->scale_layer_stride;
    char *pvs = static_cast<char *>(pool->vs) + Li * pool->scale_layer_stride;

    // this rank's Q | K | V heads, head norm/rope/quant into q8 and its KV pages
    {
      const int8_t *wts[3] = {Wp(Q3_OFF_LQ) + (size_t)sh.q_head0 * HD * H,
                              Wp(Q3_OFF_LK) + (size_t)sh.kv_head0 * HD * H,
                              Wp(Q3_OFF_LV) + (size_t)sh.kv_head0 * HD * H};
      const int rows[3] = {(int)QWl, (int)KWl, (int)KWl};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.hs);
      a.as_rb = 4 * (H / 256);
      a.ws[0] = Sp(Q3_OFF_LQ_SCALE) + sh.q_head0 * HD;
      a.ws[1] = Sp(Q3_OFF_LK_SCALE) + sh.kv_head0 * HD;
      a.ws[2] = Sp(Q3_OFF_LV_SCALE) + sh.kv_head0 * HD;
      a.heads = (int)QH;
      a.kv_heads = (int)KVH;
      a.nq = nq;
      a.nk = nk;
      a.cos_t = cos_t;
      a.sin_t = sin_t;
      a.pos = pos;
      a.inv_hd = inv_hd;
      a.q8 = w.q8;
      a.qs = w.qs;
      a.pk = pk;
      a.pv = pv;
      a.pks = pks;
      a.pvs = pvs;
      a.tables = tables;
      a.max_pages = max_pages;
      Q3_TRY(q3::dgemm_launch(q3::DG_QKV, 3, wts, rows, w.h8, H, (int)H, 256, a, st));
    }
    {
      q3::DecodeAttnArgs d{};
      d.q8 = reinterpret_cast<const char *>(w.q8);
      d.q_rb = QWl;
      d.qs = reinterpret_cast<const char *>(w.qs);
      d.qs_rb = 4 * QH;
      d.o8 = reinterpret_cast<char *>(w.o8);
      d.o_rb = QWl;
      d.os = reinterpret_cast<char *>(w.os);
      d.os_rb = 4 * QH;
      d.ks = pks;
      d.vs = pvs;
      d.table = tables;
      d.table_stride = max_pages;
      d.page_bytes = kPT * KWl;
      d.row_bytes = KWl;
      d.scale_page_bytes = kPT * 4 * KVH;
      d.scale_row_bytes = 4 * KVH;
      d.kv_len = w.kv_len;
      d.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_decode_launch(d, pk, pv, pool->num_pages, KVH, B, st, true));
    }
    auto part_args = [&](int buf, const float *a_scale, long as_rb, const float *wscale,
                         int slot0) {
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(a_scale);
      a.as_rb = as_rb;
      a.ws[0] = wscale;
      a.H = (int)H;
      a.expect = q3::tp_expect(c, buf);
      if (c.reduce_nccl) {
        // comparison variant: this rank's group partials stay local (slots
        // 0..), counted on the producer-0 counter, summed and all-reduced below
        a.ndst = 1;
        a.slot0 = 0;
        a.dst[0] = reinterpret_cast<float *>(c.local + (buf == q3::TP_O ? c.off_orecv : c.off_drecv));
        a.sig[0] = q3::tp_sig(c, c.rank, buf, 0);
        a.inc[0] = q3::dgemm_part_ctas((int)H, (int)(buf == q3::TP_O ? sh.q_heads : sh.mlp_groups));
        return a;
      }
      a.ndst = c.world;
      a.slot0 = slot0;
      for (int q = 0; q < c.world; ++q) {
        a.dst[q] = reinterpret_cast<float *>(c.peer[q] + (buf == q3::TP_O ? c.off_orecv : c.off_drecv));
        a.sig[q] = q3::tp_sig(c, q, buf, c.rank);
        a.inc[q] = q3::dgemm_part_ctas((int)H, (int)(buf == q3::TP_O ? c.shard[q].q_heads
                                                                      : c.shard[q].mlp_groups));
      }
      return a;
    };
    auto reduce = [&](int buf, int slots, const float *nw) {
      q3::TpReduceArgs r{};
      r.recv = reinterpret_cast<const float *>(c.local + (buf == q3::TP_O ? c.off_orecv : c.off_drecv));
      r.slots = slots;
      r.sig = q3::tp_sig(c, c.rank, buf, 0);
      r.expect = q3::tp_expect(c, buf);
      r.world = c.world;
      if (c.reduce_nccl) {
        const int own = (int)(buf == q3::TP_O ? sh.q_heads : sh.mlp_groups);
        float *red = reinterpret_cast<float *>(c.local + c.off_nccl);
        Q3_TRY(q3::tp_nccl_reduce(c, r.recv, own, (int)B, (int)H, red, st));
        r.recv = red;
        r.slots = 1;
        r.world = 0;                   // complete already: nothing to wait for
      }
      r.x = w.x;
      r.w = nw;
      r.inv = inv_h;
      r.B = (int)B;
      r.H = (int)H;
      r.h8 = w.h8;
      r.hs = w.hs;
      r.wait_ns = c.wait_ns;
      return q3::tp_reduce_norm(r, st);
    };
    // O: partials of this rank's heads (one 128-wide K group each) -> every rank
    {
      const int8_t *wts[1] = {Wp(Q3_OFF_LO) + sh.q_head0 * HD};
      const int rows[1] = {(int)H};
      const q3::DgemmArgs a = part_args(q3::TP_O, w.os, 4 * QH, Sp(Q3_OFF_LO_SCALE), (int)sh.q_head0);
      Q3_TRY(q3::dgemm_launch(q3::DG_PART, 1, wts, rows, w.o8, QWl, (int)QWl, 128, a, st, QW));
    }
    Q3_TRY(reduce(q3::TP_O, (int)L.heads, n2));
    // gate/up for this rank's 256-wide groups -> SwiGLU + quant
    {
      const int8_t *wts[2] = {Wp(Q3_OFF_LG) + (size_t)sh.mlp_group0 * 256 * H,
                              Wp(Q3_OFF_LU) + (size_t)sh.mlp_group0 * 256 * H};
      const int rows[2] = {(int)Il, (int)Il};
      q3::DgemmArgs a{};
      a.M = (int)B;
      a.a_scale = reinterpret_cast<const char *>(w.hs);
      a.as_rb = 4 * (H / 256);
      a.ws[0] = Sp(Q3_OFF_LG_SCALE) + sh.mlp_group0 * 256;
      a.ws[1] = Sp(Q3_OFF_LU_SCALE) + sh.mlp_group0 * 256;
      a.s8 = w.s8;
      a.ss = w.ss;
      a.I = (int)Il;
      Q3_TRY(q3::dgemm_launch(q3::DG_SWIGLU, 2, wts, rows, w.h8, H, (int)H, 256, a, st));
    }
    // down: partials of this rank's groups -> every rank
    {
      const int8_t *wts[1] = {Wp(Q3_OFF_LD) + sh.mlp_group0 * 256};
      const int rows[1] = {(int)H};
      const q3::DgemmArgs a =
          part_args(q3::TP_DOWN, w.ss, 4 * Gl, Sp(Q3_OFF_LD_SCALE), (int)sh.mlp_group0);
      Q3_TRY(q3::dgemm_launch(q3::DG_PART, 1, wts, rows, w.s8, Il, (int)Il, 256, a, st, I));
    }
    Q3_TRY(reduce(q3::TP_DOWN, (int)(I / 256), n_next));
  }
  // lm_head over this rank's vocabulary rows, then the key exchange
  {
    const q3_view lm = v2(bl + o[Q3_OFF_LM] + (int64_t)sh.vocab0 * H, sh.vocab_rows, H, Q3_DT_I8);
    const q3_view lm_s = v2(bl + o[Q3_OFF_LM] + (int64_t)V * H + (int64_t)sh.vocab0 * 4,
                            sh.vocab_rows, 1, Q3_DT_F32);
    Q3_TRY(q3_gemm_nt_group_argmax(&h8, &hs, &lm, &lm_s, w.best, w.lidx, 256, w.keys, 8 * B, s));
  }
  return q3::tp_argmax_exchange(c, w.best, w.lidx, sh.vocab0, (int)B, next_ids, st);
}

}  // namespace

extern "C" int q3_tp_decode_step_batch(void *comm, void *blob, const q3_layout *layout,
                                       const q3_kv_pool *pool, const uint16_t *tables,
                                       uint32_t max_pages, const int32_t *ids, const int32_t *pos,
                                       uint32_t n_seqs, int32_t *next_ids, void *workspace,
                                       size_t workspace_bytes, void *stream) {
  if (!comm || !blob || !layout || !pool || !tables || !ids || !pos || !next_ids || !workspace)
    return Q3_ERR_NULL;
  const q3::TpComm &c = *static_cast<const q3::TpComm *>(comm);
  const q3_layout &L = *layout;
  if (L.head_dim != 128 || L.hidden != 1024 || L.inter % 256 || L.max_seq % kPT ||
      L.heads != c.heads || L.inter / 256 != c.mlp_groups || L.hidden != c.hidden)
    return Q3_ERR_SHAPE;
  if (n_seqs == 0) return Q3_OK;
  if (n_seqs > c.max_seqs || n_seqs > 64) return Q3_ERR_CAPACITY;
  if (workspace_bytes < q3_decode_workspace_bytes(layout, n_seqs)) return Q3_ERR_CAPACITY;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return Q3_ERR_ALIGN;
  if (!pool->k || !pool->v || !pool->ks || !pool->vs || pool->num_pages == 0) return Q3_ERR_NULL;
  for (int q = 0; q < c.world; ++q)
    if (!c.peer[q]) return Q3_ERR_NULL;   // not connected
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  char *bl = static_cast<char *>(blob);
  DecodeWs w = carve(L, n_seqs, static_cast<char *>(workspace));
  k_decode_prep<<<n_seqs, 64, 0, st>>>(pos, reinterpret_cast<const float *>(bl + L.off[Q3_OFF_COS]),
                                       reinterpret_cast<const float *>(bl + L.off[Q3_OFF_SIN]),
                                       L.head_dim / 2, w.cos, w.sin, w.kv_len, w.best, next_ids,
                                       n_seqs);
  Q3_TRY(q3h::launch_status());
  return tp_decode(c, bl, L, pool, tables, max_pages, ids, pos, n_seqs, next_ids, w, st);
}

namespace {
// sequence 0's stage rows of the last decode step -> the blob's stage buffers
__global__ void k_decode_stages_to_blob(const float *x, const int8_t *s8, const float *ss,
                                        const int8_t *o8, const float *os, const float *best,
                                        const int32_t *id, int H, int I, int QW, int heads,
                                        float *bx, int8_t *bs8, float *bss, int8_t *bo8,
                                        float *bos, float *argf, int32_t *argi) {
  for (int i = threadIdx.x; i < H; i += blockDim.x) bx[i] = x[i];
  for (int i = threadIdx.x; i < I; i += blockDim.x) bs8[i] = s8[i];
  for (int i = threadIdx.x; i < QW; i += blockDim.x) bo8[i] = o8[i];
  for (int i = threadIdx.x; i < I / 256; i += blockDim.x) bss[i] = ss[i];
  for (int i = threadIdx.x; i < heads; i += blockDim.x) bos[i] = os[i];
  if (threadIdx.x == 0) {
    *argf = best[0];
    *argi = *id;
  }
}
}  // namespace

namespace q3 {
// After a one-sequence q3_decode_step_batch with this workspace: copy the rows
// the reference's greedy loop leaves in its blob (x, s8/ss, o8/os of the last
// layer, the argmax value and index) into the blob's stage buffers.
int decode_stages_to_blob(const q3_layout &L, void *workspace, void *blob, const int32_t *id,
                          cudaStream_t st) {
  const DecodeWs w = carve(L, 1, static_cast<char *>(workspace));
  char *bl = static_cast<char *>(blob);
  const int64_t *o = L.off;
  k_decode_stages_to_blob<<<1, 256, 0, st>>>(
      w.x, w.s8, w.ss, w.o8, w.os, w.best, id, (int)L.hidden, (int)L.inter,
      (int)(L.heads * L.head_dim), (int)L.heads, reinterpret_cast<float *>(bl + o[Q3_OFF_X]),
      reinterpret_cast<int8_t *>(bl + o[Q3_OFF_S8]), reinterpret_cast<float *>(bl + o[Q3_OFF_SS]),
      reinterpret_cast<int8_t *>(bl + o[Q3_OFF_O8]), reinterpret_cast<float *>(bl + o[Q3_OFF_OS]),
      reinterpret_cast<float *>(bl + o[Q3_OFF_ARGF]), reinterpret_cast<int32_t *>(bl + o[Q3_OFF_ARGI]));
  return q3h::launch_status();
}
}  // namespace q3

extern "C" size_t q3_decode_workspace_bytes(const q3_layout *L, uint32_t n_seqs) {
  if (!L) return 0;
  return carve(*L, n_seqs, nullptr).total;
}

extern "C" int q3_decode_step_batch(void *blob, const q3_layout *layout, const q3_kv_pool *pool,
                                    const uint16_t *tables, uint32_t max_pages,
                                    const int32_t *ids, const int32_t *pos, uint32_t n_seqs,
                                    int32_t *next_ids, void *workspace, size_t workspace_bytes,
                                    void *stream) {
  if (!blob || !layout || !pool || !tables || !ids || !pos || !next_ids || !workspace)
    return Q3_ERR_NULL;
  const q3_layout &L = *layout;
  // max_seq % 32 keeps every pqwf blob offset 16-byte aligned (the GEMMs load
  // 16-byte vectors); head_dim 128 and 256-column groups are the path's shapes
  if (L.head_dim != 128 || L.hidden % 256 || L.inter % 256 || L.max_seq % kPT) return Q3_ERR_SHAPE;
  if (n_seqs == 0) return Q3_OK;
  if (workspace_bytes < q3_decode_workspace_bytes(layout, n_seqs)) return Q3_ERR_CAPACITY;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return Q3_ERR_ALIGN;
  if (!pool->k || !pool->v || !pool->ks || !pool->vs) return Q3_ERR_NULL;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void *s = st;
  const int64_t *o = L.off;
  const uint32_t B = n_seqs, H = L.hidden, HD = L.head_dim, QW = L.heads * HD,
                 KW = L.kv_heads * HD, I = L.inter, V = L.vocab, HALF = HD / 2;
  char *bl = static_cast<char *>(blob);
  DecodeWs w = carve(L, B, static_cast<char *>(workspace));

  k_decode_prep<<<B, 64, 0, st>>>(pos, reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]),
                                  reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]), HALF, w.cos,
                                  w.sin, w.kv_len, w.best, next_ids, B);
  Q3_TRY(q3h::launch_status());
  // fast path: the Qwen3-0.6B shapes with tensor-core split-K GEMMs
  if (B <= 64 && H == 1024 && HD == 128 && L.heads == 2 * L.kv_heads && I % 256 == 0 &&
      QW % 128 == 0 && QW / 128 <= 16 && I / 256 <= 16 && pool->num_pages > 0)
    return decode_fused(bl, L, pool, tables, max_pages, ids, pos, B, next_ids, w, st);

  const q3_view x = v2(w.x, B, H, Q3_DT_F32), h = v2(w.h, B, H, Q3_DT_F32);
  const q3_view h8 = v2(w.h8, B, H, Q3_DT_I8), hs = v2(w.hs, B, H / 256, Q3_DT_F32);
  const q3_view q8 = v2(w.q8, B, QW, Q3_DT_I8), qs = v2(w.qs, B, L.heads, Q3_DT_F32);
  const q3_view o8 = v2(w.o8, B, QW, Q3_DT_I8), os = v2(w.os, B, L.heads, Q3_DT_F32);
  const q3_view k8 = v2(w.k8, B, KW, Q3_DT_I8), ks = v2(w.ks, B, L.kv_heads, Q3_DT_F32);
  const q3_view v8 = v2(w.v8, B, KW, Q3_DT_I8), vs = v2(w.vs, B, L.kv_heads, Q3_DT_F32);
  const q3_view s8 = v2(w.s8, B, I, Q3_DT_I8), ss = v2(w.ss, B, I / 256, Q3_DT_F32);
  const q3_view cosv = v2(w.cos, B, HALF, Q3_DT_F32), sinv = v2(w.sin, B, HALF, Q3_DT_F32);
  const q3_view idv = v2(const_cast<int32_t *>(ids), B, 1, Q3_DT_I32);
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

    if (Li != 0) Q3_TRY(q3_rmsnorm_rows(&x, &n1, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wv, &wvs, nullptr, 256, nullptr, &v8, &vs, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wk, &wks, nullptr, 256, nullptr, &k8, &ks, &nk,
                                  &cosv, &sinv, inv_hd, s));
    k_decode_scatter<<<B, 64, 0, st>>>(w.k8, w.v8, w.ks, w.vs, pos, tables, max_pages, pk, pv, pks,
                                       pvs, KW, L.kv_heads);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wq, &wqs, nullptr, 256, nullptr, &q8, &qs, &nq, &cosv,
                                  &sinv, inv_hd, s));
    if (L.heads == 2 * L.kv_heads && pool->num_pages > 0) {
      q3::DecodeAttnArgs d{};
      d.q8 = reinterpret_cast<const char *>(w.q8);
      d.q_rb = QW;
      d.qs = reinterpret_cast<const char *>(w.qs);
      d.qs_rb = 4 * L.heads;
      d.o8 = reinterpret_cast<char *>(w.o8);
      d.o_rb = QW;
      d.os = reinterpret_cast<char *>(w.os);
      d.os_rb = 4 * L.heads;
      d.ks = pks;
      d.vs = pvs;
      d.table = tables;
      d.table_stride = max_pages;
      d.page_bytes = kPT * KW;
      d.row_bytes = KW;
      d.scale_page_bytes = kPT * 4 * L.kv_heads;
      d.scale_row_bytes = 4 * L.kv_heads;
      d.kv_len = w.kv_len;
      d.qk_scale = kInvSqrt128;
      Q3_TRY(q3::attention_decode_launch(d, pk, pv, pool->num_pages, L.kv_heads, B, st));
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
    a.q_rows = 1;
    a.kv_len = 0;
    a.kv_len_dev = w.kv_len;
    a.causal = 1;
    a.qk_scale = kInvSqrt128;
    Q3_TRY(q3::attention_launch(a, B, st));
    }
    Q3_TRY(q3_gemm_nt_group_store(&o8, &os, &wo, &wos, nullptr, 128, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_rmsnorm_rows(&x, &n2, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    Q3_TRY(q3_gemm_gate_up_swiglu_quant(&h8, &hs, &wg, &wgs, &wu, &wus, &s8, &ss, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&s8, &ss, &wd, &wds, nullptr, 256, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
  }
  Q3_TRY(q3_rmsnorm_rows(&x, &nf, &h, inv_h, s));
  Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
  Q3_TRY(q3_gemm_nt_group_argmax(&h8, &hs, &lm, &lm_s, w.best, next_ids, 256, w.keys, 8 * B, s));
  return Q3_OK;
}
