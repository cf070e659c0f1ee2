// Model-level entry points: the pqwf blob layout (tools/pqwf.py:95-218), the
// per-chunk forward (src/main_big.cpp:145-296) and the greedy loop
// (src/main_big.cpp:332-369), all enqueued on one stream through the operator
// C ABI.  The host only reads CTRL once per generate call; everything else
// (ids, page table, argmax hand-off) stays on the device.
#include <string.h>

#include "q3_common.cuh"

namespace q3 {
int decode_stages_to_blob(const q3_layout &L, void *workspace, void *blob, const int32_t *id,
                          cudaStream_t st);
}

namespace {

constexpr uint32_t kPageTokens = 32;
constexpr float kInvSqrt128 = 0.08838834764831845f;   // kernels/config.h:82

q3_view view(void *base, int64_t off, uint32_t rows, uint32_t cols, uint8_t dt) {
  const int es = (dt == Q3_DT_I8 || dt == Q3_DT_U8) ? 1 : 4;
  return q3_view{static_cast<char *>(base) + off, static_cast<int32_t>(cols * es), es, rows, cols, dt};
}
q3_view rows_of(const q3_view &v, uint32_t r0, uint32_t n) {
  q3_view s = v;
  s.data = static_cast<char *>(v.data) + static_cast<int64_t>(r0) * v.row_bytes;
  s.rows = n;
  return s;
}
q3_view sub_cols(const q3_view &v, uint32_t n) {
  q3_view s = v;
  s.cols = n;
  return s;
}

__global__ void k_fill_ptab(uint16_t *t, int pages) {
  const int p = blockIdx.x * blockDim.x + threadIdx.x;
  if (p < pages) t[p] = static_cast<uint16_t>(pages - 1 - p);   // main_big.cpp:168-171
}

__global__ void k_init_best(float *best, int32_t *bidx) {
  *best = -3.0e38f;   // main_big.cpp:281-290
  *bidx = 0;
}

__global__ void k_copy_id(const int32_t *src, int32_t *dst) { *dst = *src; }

// graph-replayed greedy decode: the step reads its id and position from
// fixed words (cur_id, cur_pos) and leaves the picked id in next_id; this
// kernel then stores it at ids[pos + 1] and moves the words on by one token
__global__ void k_gen_advance(const int32_t *next_id, int32_t *cur_id, int32_t *cur_pos,
                              int32_t *ids) {
  const int32_t pos = *cur_pos, id = *next_id;
  ids[pos + 1] = id;
  *cur_id = id;
  *cur_pos = pos + 1;
}
__global__ void k_gen_start(const int32_t *id, int32_t pos, int32_t *cur_id, int32_t *cur_pos) {
  *cur_id = *id;
  *cur_pos = pos;
}

__global__ void k_iota(int32_t *v, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) v[i] = i;
}

// ptab | argmax keys | positions 0..max_seq-1 | last id | one-sequence decode workspace
struct Ws {
  uint16_t *ptab;
  void *argmax_ws;
  size_t argmax_bytes;
  int32_t *positions;
  int32_t *last_id;
  void *dec_ws;
  size_t dec_bytes;
};

size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

size_t ws_bytes(const q3_layout *L) {
  const size_t pages = L->max_seq / kPageTokens;
  return a256(pages * 2) + 256 + a256(4 * static_cast<size_t>(L->max_seq)) + 256 +
         a256(q3_decode_workspace_bytes(L, 1));
}

int carve(const q3_layout *L, void *ws, size_t bytes, Ws &w) {
  if (!ws) return Q3_ERR_NULL;
  if (bytes < ws_bytes(L)) return Q3_ERR_CAPACITY;
  if (reinterpret_cast<uintptr_t>(ws) % 256) return Q3_ERR_ALIGN;
  const size_t pages = L->max_seq / kPageTokens;
  char *b = static_cast<char *>(ws);
  w.ptab = reinterpret_cast<uint16_t *>(b);
  b += a256(pages * 2);
  w.argmax_ws = b;
  w.argmax_bytes = 256;
  b += 256;
  w.positions = reinterpret_cast<int32_t *>(b);
  b += a256(4 * static_cast<size_t>(L->max_seq));
  w.last_id = reinterpret_cast<int32_t *>(b);
  b += 256;
  w.dec_ws = b;
  w.dec_bytes = a256(q3_decode_workspace_bytes(L, 1));
  return Q3_OK;
}

}  // namespace

extern "C" int q3_layout_compute(q3_layout *L) {
  if (!L) return Q3_ERR_NULL;
  if (!L->hidden || !L->layers || !L->heads || !L->kv_heads || !L->head_dim || !L->inter ||
      !L->vocab || !L->seq || !L->max_seq)
    return Q3_ERR_SHAPE;
  const int64_t H = L->hidden, HD = L->head_dim, QW = L->heads * HD, KW = L->kv_heads * HD;
  const int64_t I = L->inter, V = L->vocab, N = L->seq, MS = L->max_seq, HALF = HD / 2;
  int64_t *o = L->off;
  int64_t off = 0;
  auto place = [&](int idx, int64_t size) { o[idx] = off; off += size; };
  place(Q3_OFF_IDS, 4 * MS);
  place(Q3_OFF_CTRL, 16);
  place(Q3_OFF_X, 4 * N * H);
  place(Q3_OFF_EMB, V * H + 4 * V);
  place(Q3_OFF_LM, V * H + 4 * V);
  place(Q3_OFF_NF, 4 * H);
  place(Q3_OFF_COS, 4 * MS * HALF);
  place(Q3_OFF_SIN, 4 * MS * HALF);
  o[Q3_OFF_LAYERW_BASE] = off;
  const int64_t layer_start = off;
  place(Q3_OFF_LQ, QW * H);
  place(Q3_OFF_LQ_SCALE, 4 * QW);
  place(Q3_OFF_LK, KW * H);
  place(Q3_OFF_LK_SCALE, 4 * KW);
  place(Q3_OFF_LV, KW * H);
  place(Q3_OFF_LV_SCALE, 4 * KW);
  place(Q3_OFF_LO, H * QW);
  place(Q3_OFF_LO_SCALE, 4 * H);
  place(Q3_OFF_LG, I * H);
  place(Q3_OFF_LG_SCALE, 4 * I);
  place(Q3_OFF_LU, I * H);
  place(Q3_OFF_LU_SCALE, 4 * I);
  place(Q3_OFF_LD, H * I);
  place(Q3_OFF_LD_SCALE, 4 * H);
  o[Q3_OFF_LAYERW_STRIDE] = off - layer_start;
  off = layer_start + static_cast<int64_t>(L->layers) * o[Q3_OFF_LAYERW_STRIDE];
  const int64_t norm_stride = 4 * (H + HD + HD + H);
  o[Q3_OFF_LAYERN_BASE] = off;
  o[Q3_OFF_LAYERN_STRIDE] = norm_stride;
  off += static_cast<int64_t>(L->layers) * norm_stride;
  o[Q3_OFF_N1] = o[Q3_OFF_LAYERN_BASE];
  o[Q3_OFF_NQ] = o[Q3_OFF_N1] + 4 * H;
  o[Q3_OFF_NK] = o[Q3_OFF_NQ] + 4 * HD;
  o[Q3_OFF_N2] = o[Q3_OFF_NK] + 4 * HD;
  place(Q3_OFF_LOGITS, 4 * N * V);
  o[Q3_OFF_BLOCK_END] = off;
  off = (off + 0xFFFF) & ~static_cast<int64_t>(0xFFFF);
  place(Q3_OFF_H, 4 * N * H);
  place(Q3_OFF_H8, N * H);
  place(Q3_OFF_HS, 4 * N * (H / 256));
  place(Q3_OFF_Q, 4 * N * QW);
  place(Q3_OFF_K, 4 * N * KW);
  place(Q3_OFF_V, 4 * N * KW);
  place(Q3_OFF_Q8, N * QW);
  place(Q3_OFF_K8, N * KW);
  place(Q3_OFF_V8, N * KW);
  place(Q3_OFF_QS, 4 * N * L->heads);
  place(Q3_OFF_KS, 4 * N * L->kv_heads);
  place(Q3_OFF_VS, 4 * N * L->kv_heads);
  place(Q3_OFF_ATTN, 4 * N * QW);
  place(Q3_OFF_O, 4 * N * H);
  place(Q3_OFF_O8, N * QW);
  place(Q3_OFF_OS, 4 * N * L->heads);
  place(Q3_OFF_G, 4 * N * I);
  place(Q3_OFF_U, 4 * N * I);
  place(Q3_OFF_SW, 4 * N * I);
  place(Q3_OFF_S8, N * I);
  place(Q3_OFF_SS, 4 * N * (I / 256));
  place(Q3_OFF_ARGF, 256);
  place(Q3_OFF_ARGI, 256);
  const int64_t kv_scale_off = MS * KW, kv_scale_bytes = 4 * MS * L->kv_heads;
  o[Q3_OFF_KV_BASE] = off;
  o[Q3_OFF_KV_SOFF] = kv_scale_off;
  o[Q3_OFF_KV_VOFF] = kv_scale_off + kv_scale_bytes;
  o[Q3_OFF_KV_STRIDE] = 2 * (kv_scale_off + kv_scale_bytes);
  off += static_cast<int64_t>(L->layers) * o[Q3_OFF_KV_STRIDE];
  o[Q3_OFF_SCRATCH_END] = off;
  return Q3_OK;
}

extern "C" size_t q3_forward_workspace_bytes(const q3_layout *L) { return L ? ws_bytes(L) : 0; }

namespace {

int forward_chunk_impl(void *blob, const q3_layout *Lp, const Ws &ws, uint32_t pos, uint32_t rows,
                       int lm_out, int optimize_tail, cudaStream_t st) {
  const q3_layout &L = *Lp;
  const int64_t *o = L.off;
  const uint32_t H = L.hidden, HD = L.head_dim, QW = L.heads * HD, KW = L.kv_heads * HD;
  const uint32_t N = L.seq, V = L.vocab, I = L.inter, MS = L.max_seq, HALF = HD / 2;
  void *s = st;

  const q3_view x_all = view(blob, o[Q3_OFF_X], N, H, Q3_DT_F32);
  const q3_view h_all = view(blob, o[Q3_OFF_H], N, H, Q3_DT_F32);
  const q3_view h8_all = view(blob, o[Q3_OFF_H8], N, H, Q3_DT_I8);
  const q3_view hs_all = view(blob, o[Q3_OFF_HS], N, H / 256, Q3_DT_F32);
  const q3_view q_all = view(blob, o[Q3_OFF_Q], N, QW, Q3_DT_F32);
  const q3_view k_all = view(blob, o[Q3_OFF_K], N, KW, Q3_DT_F32);
  const q3_view v_all = view(blob, o[Q3_OFF_V], N, KW, Q3_DT_F32);
  const q3_view q8_all = view(blob, o[Q3_OFF_Q8], N, QW, Q3_DT_I8);
  const q3_view qs_all = view(blob, o[Q3_OFF_QS], N, L.heads, Q3_DT_F32);
  const q3_view o_all = view(blob, o[Q3_OFF_O], N, H, Q3_DT_F32);
  const q3_view o8_all = view(blob, o[Q3_OFF_O8], N, QW, Q3_DT_I8);
  const q3_view os_all = view(blob, o[Q3_OFF_OS], N, L.heads, Q3_DT_F32);
  const q3_view s8_all = view(blob, o[Q3_OFF_S8], N, I, Q3_DT_I8);
  const q3_view ss_all = view(blob, o[Q3_OFF_SS], N, I / 256, Q3_DT_F32);
  const q3_view logits = view(blob, o[Q3_OFF_LOGITS], N, V, Q3_DT_F32);
  const q3_view ids = view(blob, o[Q3_OFF_IDS], MS, 1, Q3_DT_I32);
  const q3_view cos_t = view(blob, o[Q3_OFF_COS], MS, HALF, Q3_DT_F32);
  const q3_view sin_t = view(blob, o[Q3_OFF_SIN], MS, HALF, Q3_DT_F32);
  const q3_view emb = view(blob, o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = view(blob, o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view lm = view(blob, o[Q3_OFF_LM], V, H, Q3_DT_I8);
  const q3_view lm_s = view(blob, o[Q3_OFF_LM] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view nf = view(blob, o[Q3_OFF_NF], H, 1, Q3_DT_F32);

  const q3_view x = rows_of(x_all, 0, rows), h = rows_of(h_all, 0, rows);
  const q3_view h8 = rows_of(h8_all, 0, rows), hs = rows_of(hs_all, 0, rows);
  const q3_view cos_p = rows_of(cos_t, pos, rows), sin_p = rows_of(sin_t, pos, rows);
  const q3_view ids_p = rows_of(ids, pos, rows);
  const float inv_h = 1.0f / static_cast<float>(H);
  const float inv_hd = 1.0f / static_cast<float>(HD);

  {
    const q3_view n1_0 = view(blob, o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &ids_p, &x, &n1_0, &h, inv_h, s));
  }

  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    const int64_t lw = o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    const int64_t ln = o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    const int64_t kv = o[Q3_OFF_KV_BASE] + static_cast<int64_t>(Li) * o[Q3_OFF_KV_STRIDE];
    auto W = [&](int key, uint32_t r, uint32_t c) {
      return view(blob, lw + (o[key] - o[Q3_OFF_LQ]), r, c, Q3_DT_I8);
    };
    auto S = [&](int key, uint32_t r) {
      return view(blob, lw + (o[key] - o[Q3_OFF_LQ]), r, 1, Q3_DT_F32);
    };
    const q3_view wq = W(Q3_OFF_LQ, QW, H), wk = W(Q3_OFF_LK, KW, H), wv = W(Q3_OFF_LV, KW, H);
    const q3_view wo = W(Q3_OFF_LO, H, QW), wg = W(Q3_OFF_LG, I, H), wu = W(Q3_OFF_LU, I, H);
    const q3_view wd = W(Q3_OFF_LD, H, I);
    const q3_view wqs = S(Q3_OFF_LQ_SCALE, QW), wks = S(Q3_OFF_LK_SCALE, KW);
    const q3_view wvs = S(Q3_OFF_LV_SCALE, KW), wos = S(Q3_OFF_LO_SCALE, H);
    const q3_view wgs = S(Q3_OFF_LG_SCALE, I), wus = S(Q3_OFF_LU_SCALE, I);
    const q3_view wds = S(Q3_OFF_LD_SCALE, H);
    const q3_view n1 = view(blob, ln, H, 1, Q3_DT_F32);
    const q3_view nq = view(blob, ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view nk = view(blob, ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view n2 = view(blob, ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]), H, 1, Q3_DT_F32);
    char *kc_base = static_cast<char *>(blob) + kv;
    char *kcs_base = kc_base + o[Q3_OFF_KV_SOFF];
    char *vc_base = kc_base + o[Q3_OFF_KV_VOFF];
    char *vcs_base = vc_base + o[Q3_OFF_KV_SOFF];

    if (Li != 0) Q3_TRY(q3_rmsnorm_rows(&x, &n1, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));

    // K/V straight into the physical page (main_big.cpp:183-209)
    const uint32_t kv_row = KW, ks_row = 4 * L.kv_heads;
    const uint32_t page = (MS / kPageTokens) - 1 - pos / kPageTokens;   // ptab[pos/32]
    const uint32_t slot = pos % kPageTokens;
    const int64_t koff = static_cast<int64_t>(page) * kPageTokens * kv_row + slot * kv_row;
    const int64_t soff = static_cast<int64_t>(page) * kPageTokens * ks_row + slot * ks_row;
    const q3_view kk = rows_of(k_all, 0, rows), vv = rows_of(v_all, 0, rows);
    q3_view vc8{vc_base + koff, (int32_t)kv_row, 1, rows, KW, Q3_DT_I8};
    q3_view vcs{vcs_base + soff, (int32_t)ks_row, 4, rows, L.kv_heads, Q3_DT_F32};
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wv, &wvs, &vv, 256, nullptr, &vc8, &vcs, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    q3_view kc{kc_base + koff, (int32_t)kv_row, 1, rows, KW, Q3_DT_I8};
    q3_view kcs{kcs_base + soff, (int32_t)ks_row, 4, rows, L.kv_heads, Q3_DT_F32};
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wk, &wks, &kk, 256, nullptr, &kc, &kcs, &nk, &cos_p,
                                  &sin_p, inv_hd, s));

    const bool is_last = (Li == L.layers - 1);
    if (is_last && lm_out == Q3_LM_NONE) continue;
    const bool tail_last_row = optimize_tail && is_last;
    const uint32_t tr0 = tail_last_row ? rows - 1 : 0, tr = tail_last_row ? 1 : rows;
    const q3_view h8t = rows_of(h8_all, tr0, tr), hst = rows_of(hs_all, tr0, tr);
    const q3_view xt = rows_of(x_all, tr0, tr), ht = rows_of(h_all, tr0, tr);
    const q3_view qt = rows_of(q_all, tr0, tr), q8t = rows_of(q8_all, tr0, tr);
    const q3_view qst = rows_of(qs_all, tr0, tr), o8t = rows_of(o8_all, tr0, tr);
    const q3_view ost = rows_of(os_all, tr0, tr), ot = rows_of(o_all, tr0, tr);
    const q3_view s8t = rows_of(s8_all, tr0, tr), sst = rows_of(ss_all, tr0, tr);
    const q3_view cos_r = rows_of(cos_t, pos + tr0, tr), sin_r = rows_of(sin_t, pos + tr0, tr);

    Q3_TRY(q3_gemm_nt_group_store(&h8t, &hst, &wq, &wqs, &qt, 256, nullptr, &q8t, &qst, &nq,
                                  &cos_r, &sin_r, inv_hd, s));
    const uint32_t kv_len = pos + rows;
    q3_paged_kv paged{kc_base, vc_base, kcs_base, vcs_base, ws.ptab, kPageTokens,
                      kPageTokens * kv_row, kv_row, kPageTokens * ks_row, ks_row};
    Q3_TRY(q3_attention_heads_gqa_tokscale_paged(&q8t, &qst, &paged, kv_len, &o8t, &ost, L.heads,
                                                 L.kv_heads, HD, 1, kInvSqrt128, s));
    Q3_TRY(q3_gemm_nt_group_store(&o8t, &ost, &wo, &wos, &ot, 128, &xt, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_rmsnorm_rows(&xt, &n2, &ht, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&ht, &h8t, &hst, 256, s));
    Q3_TRY(q3_gemm_gate_up_swiglu_quant(&h8t, &hst, &wg, &wgs, &wu, &wus, &s8t, &sst, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&s8t, &sst, &wd, &wds, &ot, 256, &xt, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
  }

  if (lm_out != Q3_LM_NONE) {
    const q3_view xl = rows_of(x_all, rows - 1, 1);
    const q3_view hl = rows_of(o_all, 0, 1);                  // o borrowed for h
    const q3_view h8l = sub_cols(rows_of(q8_all, 0, 1), H);   // q8 row 0, first H columns
    q3_view hsl{qs_all.data, qs_all.row_bytes, 4, 1, H / 256, Q3_DT_F32};
    Q3_TRY(q3_rmsnorm_rows(&xl, &nf, &hl, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&hl, &h8l, &hsl, 256, s));
    if (lm_out == Q3_LM_LOGITS) {
      const q3_view lg = rows_of(logits, 0, 1);
      Q3_TRY(q3_gemm_nt_group_store(&h8l, &hsl, &lm, &lm_s, &lg, 256, nullptr, nullptr, nullptr,
                                    nullptr, nullptr, nullptr, 0.0f, s));
    } else {
      float *argf = reinterpret_cast<float *>(static_cast<char *>(blob) + o[Q3_OFF_ARGF]);
      int32_t *argi = reinterpret_cast<int32_t *>(static_cast<char *>(blob) + o[Q3_OFF_ARGI]);
      k_init_best<<<1, 1, 0, st>>>(argf, argi);
      Q3_TRY(q3h::launch_status());
      Q3_TRY(q3_gemm_nt_group_argmax(&h8l, &hsl, &lm, &lm_s, argf, argi, 256, ws.argmax_ws,
                                     ws.argmax_bytes, s));
    }
  }
  return Q3_OK;
}

int check_layout(const q3_layout *L) {
  if (!L) return Q3_ERR_NULL;
  if (L->head_dim != 128 || L->hidden % 256 || L->inter % 256 || L->max_seq % kPageTokens ||
      L->seq > kPageTokens || L->max_seq / kPageTokens > 65535)
    return Q3_ERR_SHAPE;
  return Q3_OK;
}

}  // namespace

extern "C" int q3_forward_chunk(void *blob, const q3_layout *layout, uint32_t pos, uint32_t rows,
                                int lm_out, int optimize_tail, void *workspace,
                                size_t workspace_bytes, void *stream) {
  if (!blob) return Q3_ERR_NULL;
  Q3_TRY(check_layout(layout));
  if (rows == 0 || rows > layout->seq) return Q3_ERR_SHAPE;
  if (pos + rows > layout->max_seq) return Q3_ERR_CAPACITY;
  if ((pos % kPageTokens) + rows > kPageTokens) return Q3_ERR_SHAPE;   // one page per chunk
  if (lm_out < Q3_LM_NONE || lm_out > Q3_LM_ARGMAX) return Q3_ERR_MODE;
  Ws ws;
  Q3_TRY(carve(layout, workspace, workspace_bytes, ws));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int pages = layout->max_seq / kPageTokens;
  k_fill_ptab<<<(pages + 127) / 128, 128, 0, st>>>(ws.ptab, pages);
  Q3_TRY(q3h::launch_status());
  return forward_chunk_impl(blob, layout, ws, pos, rows, lm_out, optimize_tail, st);
}

namespace {
constexpr int kGraphUnavailable = -1000;   // capture not possible: run the steps eagerly

// A private capture stream per thread and device (the caller's stream may be
// the legacy default stream, which cannot be captured).
cudaStream_t capture_stream() {
  thread_local cudaStream_t per_dev[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!per_dev[dev] && cudaStreamCreateWithFlags(&per_dev[dev], cudaStreamNonBlocking) != cudaSuccess)
    per_dev[dev] = nullptr;
  return per_dev[dev];
}

// The n_gen decode steps of q3_generate (positions n_prompt .. n_prompt + n_gen - 1,
// ids[n_prompt] already picked): step 0 eagerly, steps 1 .. n_gen - 2 as replays of
// one captured step, the last step eagerly into last_id + the stage rows.
int generate_by_graph(void *blob, const q3_layout *layout, const q3_kv_pool &cache, const Ws &ws,
                      int32_t *ids, uint32_t n_prompt, uint32_t n_gen, cudaStream_t st) {
  cudaStreamCaptureStatus cs_st = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs_st) != cudaSuccess || cs_st != cudaStreamCaptureStatusNone)
    return kGraphUnavailable;      // the caller is capturing: no nested capture
  cudaStream_t cs = capture_stream();
  if (!cs) return kGraphUnavailable;
  const uint32_t max_pages = layout->max_seq / kPageTokens;
  int32_t *cur_id = ws.last_id + 1, *cur_pos = ws.last_id + 2, *next_id = ws.last_id + 3;
  auto step = [&](int32_t *nxt, cudaStream_t s) {
    return q3_decode_step_batch(blob, layout, &cache, ws.ptab, max_pages, cur_id, cur_pos, 1, nxt,
                                ws.dec_ws, ws.dec_bytes, s);
  };
  k_gen_start<<<1, 1, 0, st>>>(ids + n_prompt, static_cast<int32_t>(n_prompt), cur_id, cur_pos);
  Q3_TRY(q3h::launch_status());
  Q3_TRY(step(next_id, st));                                   // step 0
  k_gen_advance<<<1, 1, 0, st>>>(next_id, cur_id, cur_pos, ids);
  Q3_TRY(q3h::launch_status());
  // steps 1 .. n_gen - 2: replays of one captured step (eagerly if capture fails)
  cudaGraphExec_t ge = nullptr;
  if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) == cudaSuccess) {
    int rc = step(next_id, cs);
    if (rc == Q3_OK) {
      k_gen_advance<<<1, 1, 0, cs>>>(next_id, cur_id, cur_pos, ids);
      rc = q3h::launch_status();
    }
    cudaGraph_t g = nullptr;
    const cudaError_t ec = cudaStreamEndCapture(cs, &g);
    if (rc != Q3_OK) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (ec == cudaSuccess && g && cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) ge = nullptr;
    if (g) cudaGraphDestroy(g);
  }
  cudaGetLastError();             // a failed capture leaves nothing behind
  if (ge) {
    cudaError_t e = cudaSuccess;
    for (uint32_t i = 1; i + 1 < n_gen && e == cudaSuccess; ++i) e = cudaGraphLaunch(ge, st);
    cudaGraphExecDestroy(ge);     // freed once the launches above complete
    if (e != cudaSuccess) {
      q3h::set_cuda_error(e);
      return Q3_ERR_CUDA;
    }
  } else {
    for (uint32_t i = 1; i + 1 < n_gen; ++i) {
      Q3_TRY(step(next_id, st));
      k_gen_advance<<<1, 1, 0, st>>>(next_id, cur_id, cur_pos, ids);
      Q3_TRY(q3h::launch_status());
    }
  }
  Q3_TRY(step(ws.last_id, st));                                // the last step
  return q3::decode_stages_to_blob(*layout, ws.dec_ws, blob, ws.last_id, st);
}
}  // namespace

extern "C" int q3_generate(void *blob, const q3_layout *layout, void *workspace,
                           size_t workspace_bytes, void *stream) {
  if (!blob) return Q3_ERR_NULL;
  Q3_TRY(check_layout(layout));
  Ws ws;
  Q3_TRY(carve(layout, workspace, workspace_bytes, ws));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t ctrl[4];
  if (cudaMemcpyAsync(ctrl, static_cast<char *>(blob) + layout->off[Q3_OFF_CTRL], sizeof ctrl,
                      cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess) {
    q3h::set_cuda_error(cudaGetLastError());
    return Q3_ERR_CUDA;
  }
  const uint32_t n_prompt = static_cast<uint32_t>(ctrl[0]), n_gen = static_cast<uint32_t>(ctrl[1]);
  const uint32_t mode = static_cast<uint32_t>(ctrl[3]);
  if (mode > 1) return Q3_ERR_MODE;
  const bool fused = (mode == 0);
  const uint32_t total = n_prompt + n_gen;
  if (total > layout->max_seq) return Q3_ERR_CAPACITY;
  const int pages = layout->max_seq / kPageTokens;
  k_fill_ptab<<<(pages + 127) / 128, 128, 0, st>>>(ws.ptab, pages);
  Q3_TRY(q3h::launch_status());
  k_iota<<<(layout->max_seq + 255) / 256, 256, 0, st>>>(ws.positions, (int)layout->max_seq);
  Q3_TRY(q3h::launch_status());
  int32_t *ids = reinterpret_cast<int32_t *>(static_cast<char *>(blob) + layout->off[Q3_OFF_IDS]);
  // decode steps (one row after the prompt) of the fused mode run the batched
  // decode kernels with one sequence over the blob's own cache: the cache is a
  // page pool in the reference's layout and ptab its page table
  char *kvb = static_cast<char *>(blob) + layout->off[Q3_OFF_KV_BASE];
  const q3_kv_pool cache{kvb, kvb + layout->off[Q3_OFF_KV_VOFF], kvb + layout->off[Q3_OFF_KV_SOFF],
                         kvb + layout->off[Q3_OFF_KV_VOFF] + layout->off[Q3_OFF_KV_SOFF],
                         static_cast<uint64_t>(layout->off[Q3_OFF_KV_STRIDE]),
                         static_cast<uint64_t>(layout->off[Q3_OFF_KV_STRIDE]),
                         layout->max_seq / kPageTokens};
  const bool batched_decode = fused && reinterpret_cast<uintptr_t>(kvb) % 16 == 0 &&
                              layout->off[Q3_OFF_KV_VOFF] % 16 == 0 &&
                              layout->off[Q3_OFF_KV_STRIDE] % 16 == 0;
  const int32_t *argi =
      reinterpret_cast<const int32_t *>(static_cast<char *>(blob) + layout->off[Q3_OFF_ARGI]);
  const float *logits0 =
      reinterpret_cast<const float *>(static_cast<char *>(blob) + layout->off[Q3_OFF_LOGITS]);
  const uint32_t N = layout->seq;
  uint32_t pos = 0;
  while (pos < total) {
    // four or more decode steps: the first runs eagerly (it also sets up the
    // kernels' attributes), the middle ones replay one captured step, the last
    // runs eagerly and copies the stage rows back to the blob
    if (batched_decode && pos == n_prompt && n_gen >= 4) {
      const int st_rc = generate_by_graph(blob, layout, cache, ws, ids, n_prompt, n_gen, st);
      if (st_rc == Q3_OK) break;
      if (st_rc != kGraphUnavailable) return st_rc;
    }
    if (batched_decode && pos >= n_prompt) {
      // the id picked for the next position goes straight into ids[pos + 1]
      const bool last = (pos + 1 == total);
      int32_t *nxt = last ? ws.last_id : ids + pos + 1;
      Q3_TRY(q3_decode_step_batch(blob, layout, &cache, ws.ptab, layout->max_seq / kPageTokens,
                                  ids + pos, ws.positions + pos, 1, nxt, ws.dec_ws, ws.dec_bytes,
                                  st));
      pos += 1;
      if (last) Q3_TRY(q3::decode_stages_to_blob(*layout, ws.dec_ws, blob, nxt, st));
      continue;
    }
    const uint32_t rows = (pos < n_prompt) ? ((n_prompt - pos < N) ? (n_prompt - pos) : N) : 1;
    const bool need_out = (pos + rows >= n_prompt);
    const int lm_out = need_out ? (fused ? Q3_LM_ARGMAX : Q3_LM_LOGITS) : Q3_LM_NONE;
    Q3_TRY(forward_chunk_impl(blob, layout, ws, pos, rows, lm_out, fused ? 1 : 0, st));
    pos += rows;
    if (pos >= n_prompt && pos < total) {
      if (fused) {
        k_copy_id<<<1, 1, 0, st>>>(argi, ids + pos);
        Q3_TRY(q3h::launch_status());
      } else {
        Q3_TRY(q3h::launch_argmax_row(logits0, layout->vocab, ids + pos, st));
      }
    }
  }
  return Q3_OK;
}
