/*
 * q3_ops.h — C ABI of the B200-native Qwen3 w8a8 forward path.
 *
 * One entry point per operator of the reference's operator API (kernels/*.h
 * of mland2333/qwen3-tile-ops), plus its forward_chunk()/greedy-generate entry
 * points (src/main_big.cpp) and a batched paged-decode extension.  Every
 * function is `extern "C"`, takes plain pointers and sizes, enqueues work on the
 * given CUDA stream (`cudaStream_t` passed as `void *`, NULL = legacy default
 * stream) and returns a status code.  All data pointers inside views are
 * DEVICE pointers.  Operators allocate nothing: where an operator needs scratch
 * memory the caller passes a workspace whose size the matching *_workspace_bytes()
 * query returns.
 *
 * Numerics follow the reference bit for bit (tools/ref_qwen3.py): int32 group
 * partials, float32 steps rounded one at a time in the reference's order, and
 * exp(x) = exp2(f32(x*log2e)) with a correctly rounded float32 exp2.
 *
 * Errors: the reference's operators return silently on unsupported shapes
 * (group_gemm.h:47-49, lm_argmax.h:82); these return a non-zero status instead
 * and enqueue nothing.
 */
#ifndef Q3_OPS_H
#define Q3_OPS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* MatrixView dtype codes (kernels/config.h:86-90; tools/pqwf.py:28-33). */
enum { Q3_DT_I8 = 0, Q3_DT_U8 = 1, Q3_DT_I32 = 2, Q3_DT_U32 = 3, Q3_DT_F32 = 4 };

/* Status codes. */
enum {
  Q3_OK = 0,
  Q3_ERR_NULL = 1,     /* a required view/pointer is null                     */
  Q3_ERR_MODE = 2,     /* CTRL mode > 1 (main_big.cpp:346-348 returns 2), or an unknown flag */
  Q3_ERR_SHAPE = 3,    /* sizes do not fit the operator                       */
  Q3_ERR_DTYPE = 4,    /* view dtype code does not match the operand          */
  Q3_ERR_ALIGN = 5,    /* pointer/stride alignment the kernels need is missing */
  Q3_ERR_CUDA = 6,     /* a CUDA launch or call failed (q3_last_cuda_error)   */
  Q3_ERR_CAPACITY = 7, /* workspace too small, or position beyond max_seq     */
  Q3_ERR_ARCH = 8      /* device is not sm_100                                */
};

/* kernels/matrix.h:27-34 — a strided 2-D view; strides in BYTES. */
typedef struct q3_view {
  void *data;
  int32_t row_bytes;
  int32_t col_bytes;
  uint32_t rows;
  uint32_t cols;
  uint8_t dtype;
} q3_view;

/* kernels/kv_pages.h:13-24 — paged KV cache: 32-token pages, logical->physical
 * page table (device memory). */
typedef struct q3_paged_kv {
  void *k;                    /* [page][page_tokens][row_bytes] i8            */
  void *v;
  void *ks;                   /* [page][page_tokens][kv_heads] f32            */
  void *vs;
  const uint16_t *table;      /* logical page -> physical page (device)      */
  uint32_t page_tokens;       /* 32                                          */
  uint32_t page_bytes;        /* page_tokens * row_bytes                     */
  uint32_t row_bytes;         /* kv_heads * head_dim                         */
  uint32_t scale_page_bytes;  /* page_tokens * scale_row_bytes               */
  uint32_t scale_row_bytes;   /* kv_heads * 4                                */
} q3_paged_kv;

/* ---- operators (kernels/*.h) -------------------------------------------- */

/* kernels/rmsnorm.h:34-81 — out = x * rsqrt(mean(x^2)+eps) * w, row-wise. */
int q3_rmsnorm_rows(const q3_view *x, const q3_view *w, const q3_view *out,
                    float inv, void *stream);

/* kernels/quant.h:89-138 — per-row, per-group_cols int8 quantisation:
 * scale = absmax * (1/127), q = sat127(rne(x / scale)). */
int q3_quant_rows_heads(const q3_view *x, const q3_view *qi8,
                        const q3_view *scale, uint32_t group_cols, void *stream);

/* kernels/embedding.h:99-168 — gather int8 rows by id, dequantise into tmp
 * (the residual stream x), fused RMSNorm with w into out. */
int q3_embedding_rmsnorm_rows(const q3_view *table, const q3_view *scale,
                              const q3_view *ids, const q3_view *tmp,
                              const q3_view *w, const q3_view *out, float inv,
                              void *stream);

/* kernels/group_gemm.h:27-222 — per-K-group w8a8 GEMM
 *   out[m][n] = sum_g ((f32(A_g . B_g) * b_scale[n]) * a_scale[m][g])
 * Epilogue by which optional views are non-null (same precedence as the
 * reference): nw -> per-head RMSNorm(inv_hd)*nw + RoPE(cos, sin) + per-head
 * int8 quant into q8/qs; else q8 -> per-head int8 quant into q8/qs; else
 * add -> add += result (residual); else store into out.  The reference's
 * NPU-register outputs (Acc* ao0..ao3) have no counterpart. */
int q3_gemm_nt_group_store(const q3_view *a, const q3_view *a_scale,
                           const q3_view *b, const q3_view *b_scale,
                           const q3_view *out, uint32_t group_k,
                           const q3_view *add, const q3_view *q8,
                           const q3_view *qs, const q3_view *nw,
                           const q3_view *cos, const q3_view *sin, float inv_hd,
                           void *stream);

/* kernels/swiglu_quant.h:164-255 — gate and up GEMMs (per group), SwiGLU,
 * per-256-column int8 quant into s8/ss. */
int q3_gemm_gate_up_swiglu_quant(const q3_view *a, const q3_view *a_scale,
                                 const q3_view *wg, const q3_view *wgs,
                                 const q3_view *wu, const q3_view *wus,
                                 const q3_view *s8, const q3_view *ss,
                                 uint32_t group_k, void *stream);

/* kernels/attention_gqa.h:549-572 (+404-547) — GQA hd128 attention over a
 * paged int8 KV cache, online softmax over 32-key blocks with P requantised
 * per block; output quantised per head into o8/os. */
int q3_attention_heads_gqa_tokscale_paged(const q3_view *q8,
                                          const q3_view *q_scale,
                                          const q3_paged_kv *kv,
                                          uint32_t kv_len, const q3_view *o8,
                                          const q3_view *os, int heads,
                                          int kv_heads, int head_dim,
                                          int causal, float qk_scale,
                                          void *stream);

/* Batch of decode rows (extension of the operator above with the per-request
 * page tables of kernels/kv_pages.h:98-131): row s of q8/q_scale is the one new
 * query row of sequence s, which sees keys 0..kv_len[s]-1 of its own table
 * tables[s*max_pages ...] (device uint16) in the shared pool `kv` (kv->table is
 * ignored; pages 0..num_pages-1).  kv_len is a device int32 array.  Output per
 * head into o8/os exactly as the operator above computes it for that row. */
int q3_attention_decode_batch(const q3_view *q8, const q3_view *q_scale,
                              const q3_paged_kv *kv, uint32_t num_pages,
                              const uint16_t *tables, uint32_t max_pages,
                              const int32_t *kv_len, uint32_t n_seqs,
                              const q3_view *o8, const q3_view *os, int heads,
                              int kv_heads, float qk_scale, void *stream);

/* kernels/kv_pages.h:63-93 — scatter contiguous K/V rows (+scales) into pages. */
int q3_paged_kv_scatter(const q3_view *k, const q3_view *v, const q3_view *ks,
                        const q3_view *vs, const q3_paged_kv *kv,
                        uint32_t start_token, uint32_t rows, uint32_t kv_dim,
                        uint32_t kv_heads, void *stream);

/* kernels/kv_pages.h:98-131 — batch scatter: row r goes to tables[r] at
 * tokens[r].  `tables` and `tokens` are HOST arrays of `rows` entries
 * (rows <= 128); the page tables they point to are device memory. */
int q3_paged_kv_scatter_batch(const q3_view *k, const q3_view *v,
                              const q3_view *ks, const q3_view *vs,
                              const q3_paged_kv *tables, const uint32_t *tokens,
                              uint32_t rows, uint32_t kv_dim, uint32_t kv_heads,
                              void *stream);

/* kernels/lm_argmax.h:72-182 — lm_head per-group GEMM fused with a running
 * (best, bidx) per row: in/out device arrays of a->rows entries, updated like
 * the reference's `best < tmax` per-32-column-block rule (net effect: the
 * first index of the row maximum replaces (best, bidx) when it exceeds best).
 * Needs q3_gemm_nt_group_argmax_workspace_bytes(a->rows) bytes of workspace. */
size_t q3_gemm_nt_group_argmax_workspace_bytes(uint32_t rows);
int q3_gemm_nt_group_argmax(const q3_view *a, const q3_view *a_scale,
                            const q3_view *b, const q3_view *b_scale,
                            float *best, int32_t *bidx, uint32_t group_k,
                            void *workspace, size_t workspace_bytes,
                            void *stream);

/* No counterpart in the reference: the same lm_head + argmax as
 * q3_gemm_nt_group_argmax, for callers that cannot call cudaMalloc (a host
 * that only owns one fixed, pre-planned device buffer, or a serving loop that
 * must keep allocation calls, which can synchronize the device, off its hot
 * path).  It allocates nothing: its scratch is a built-in device array of
 * Q3_NOALLOC_ARGMAX_MAX_ROWS keys (8 bytes each), one per device, shared by
 * every call.  More rows -> Q3_ERR_CAPACITY.  Each call clears the keys it
 * uses; calls that overlap on the GPU race on the array.  The first call on a
 * device looks the array's address up (cudaGetSymbolAddress) with that device
 * current, and so does the first call after the device's context changed (a
 * device reset): make such a call before any stream capture. */
#define Q3_NOALLOC_ARGMAX_MAX_ROWS 4096
int q3_gemm_nt_group_argmax_noalloc(const q3_view *a, const q3_view *a_scale,
                                    const q3_view *b, const q3_view *b_scale,
                                    float *best, int32_t *bidx, uint32_t group_k,
                                    void *stream);

/* src/main_big.cpp:300-322 — greedy pick over a logits row by 32-column blocks
 * (monotone float key); writes the id to *out_id (device). */
int q3_argmax_logits(const q3_view *logits, int32_t *out_id, void *stream);

/* ---- model level (src/main_big.cpp, tools/pqwf.py) ---------------------- */

/* tools/pqwf.py:95-218 — model dimensions; q3_layout_compute fills `off` with
 * the blob offsets of config/model_big.h (indices Q3_OFF_*). */
enum {
  Q3_OFF_IDS, Q3_OFF_CTRL, Q3_OFF_X, Q3_OFF_EMB, Q3_OFF_LM, Q3_OFF_NF,
  Q3_OFF_COS, Q3_OFF_SIN, Q3_OFF_LAYERW_BASE, Q3_OFF_LAYERW_STRIDE,
  Q3_OFF_LQ, Q3_OFF_LQ_SCALE, Q3_OFF_LK, Q3_OFF_LK_SCALE, Q3_OFF_LV,
  Q3_OFF_LV_SCALE, Q3_OFF_LO, Q3_OFF_LO_SCALE, Q3_OFF_LG, Q3_OFF_LG_SCALE,
  Q3_OFF_LU, Q3_OFF_LU_SCALE, Q3_OFF_LD, Q3_OFF_LD_SCALE,
  Q3_OFF_LAYERN_BASE, Q3_OFF_LAYERN_STRIDE, Q3_OFF_N1, Q3_OFF_NQ, Q3_OFF_NK,
  Q3_OFF_N2, Q3_OFF_LOGITS, Q3_OFF_BLOCK_END,
  Q3_OFF_H, Q3_OFF_H8, Q3_OFF_HS, Q3_OFF_Q, Q3_OFF_K, Q3_OFF_V, Q3_OFF_Q8,
  Q3_OFF_K8, Q3_OFF_V8, Q3_OFF_QS, Q3_OFF_KS, Q3_OFF_VS, Q3_OFF_ATTN,
  Q3_OFF_O, Q3_OFF_O8, Q3_OFF_OS, Q3_OFF_G, Q3_OFF_U, Q3_OFF_SW, Q3_OFF_S8,
  Q3_OFF_SS, Q3_OFF_ARGF, Q3_OFF_ARGI, Q3_OFF_KV_BASE, Q3_OFF_KV_STRIDE,
  Q3_OFF_KV_VOFF, Q3_OFF_KV_SOFF, Q3_OFF_SCRATCH_END, Q3_OFF_COUNT
};

typedef struct q3_layout {
  uint32_t hidden, layers, heads, kv_heads, head_dim, inter, vocab, seq, max_seq;
  int64_t off[Q3_OFF_COUNT];
} q3_layout;

int q3_layout_compute(q3_layout *layout);

/* ---- blob producer (tools/convert_pqwf.py:125-219, tools/pqwf.py:279-360) --
 * q3_blob_from_safetensors writes the weight regions of a device blob laid
 * out by `layout` from an HF Qwen3 `model.safetensors`: per-row int8 codes and
 * scales of the embedding, lm_head (embed_tokens when the file has no
 * lm_head.weight) and the seven projections of layers [0, layout->layers),
 * vocab rows [0, layout->vocab); the five norm vectors as float32; RoPE cos/sin
 * tables for rope_theta (config.json "rope_theta", 1e6 by default).  BF16, F16
 * and F32 tensors are read; F16 is decoded as IEEE half unless `flags` holds
 * Q3_CONVERT_F16_AS_UINT16, which widens the 16-bit patterns as unsigned
 * integers the way pqwf.SafeTensors.block_f32 / vector_f32 do (pqwf.py:302,
 * 313, 320).  IDS / CTRL / scratch are left to the caller.
 * Synchronous on `stream`; Q3_ERR_SHAPE when a tensor is missing or its shape
 * or file range does not fit.
 * q3_safetensors_tensor (host only) reports one tensor of the file's header:
 * dtype 0 F32, 1 BF16, 2 F16, -1 other; up to 4 dims of shape. */
enum { Q3_CONVERT_F16_AS_UINT16 = 1 };
int q3_blob_from_safetensors(const char *path, const q3_layout *layout, double rope_theta,
                             uint32_t flags, void *blob, void *stream);
int q3_safetensors_tensor(const char *path, const char *name, int32_t *dtype, uint64_t *shape,
                          int32_t *ndim);

/* LmHeadOut of main_big.cpp:142. */
enum { Q3_LM_NONE = 0, Q3_LM_LOGITS = 1, Q3_LM_ARGMAX = 2 };

/* Workspace (device) needed by q3_forward_chunk / q3_generate. */
size_t q3_forward_workspace_bytes(const q3_layout *layout);

/* src/main_big.cpp:145-296 — one prefill chunk or decode step over the blob
 * (device copy of the pqwf blob).  pos = absolute position of the first row,
 * rows <= layout->seq.  KV goes into the blob's per-layer cache through the
 * reference's reversed page table (main_big.cpp:168-171). */
int q3_forward_chunk(void *blob, const q3_layout *layout, uint32_t pos,
                     uint32_t rows, int lm_out, int optimize_tail,
                     void *workspace, size_t workspace_bytes, void *stream);

/* src/main_big.cpp:332-369 — the greedy loop: reads CTRL [n_prompt, n_gen,
 * max_seq, mode] from the blob (one 16-byte device->host read), then runs
 * every chunk asynchronously, writing each picked id into ids[pos].
 * In mode 0 (fused lm_head + argmax) the one-row decode steps after the
 * prompt run the batched decode kernels with one sequence over the blob's
 * own cache (same bits as q3_forward_chunk); of the blob's stage buffers the
 * call then leaves x, s8/ss, o8/os (last layer, last step) and argf/argi, as
 * the reference's loop does.  Returns Q3_ERR_MODE for mode > 1. */
int q3_generate(void *blob, const q3_layout *layout, void *workspace,
                size_t workspace_bytes, void *stream);

/* ---- batched paged decode (extension; kernels/kv_pages.h:98-131) --------- */

/* A pool of 32-token KV pages for every layer, shared by many sequences.
 * Page p of layer L: K at k + L*layer_stride + p*32*kv_width, its scales at
 * ks + L*scale_layer_stride + p*32*kv_heads*4; V likewise. */
typedef struct q3_kv_pool {
  void *k, *v, *ks, *vs;
  uint64_t layer_stride;        /* bytes between layers in k / v             */
  uint64_t scale_layer_stride;  /* bytes between layers in ks / vs           */
  uint32_t num_pages;
} q3_kv_pool;

/* One decode step for n_seqs independent sequences (one new token each):
 * ids[s] at position pos[s] of sequence s, whose page table is
 * tables[s*max_pages ...] (device).  Writes the greedy next id of every
 * sequence to next_ids[s] (device).  Weights come from the blob. */
size_t q3_decode_workspace_bytes(const q3_layout *layout, uint32_t n_seqs);
int q3_decode_step_batch(void *blob, const q3_layout *layout,
                         const q3_kv_pool *pool, const uint16_t *tables,
                         uint32_t max_pages, const int32_t *ids,
                         const int32_t *pos, uint32_t n_seqs, int32_t *next_ids,
                         void *workspace, size_t workspace_bytes, void *stream);

/* Prompt prefill for n_seqs independent sequences (extension; the batched form
 * of src/main_big.cpp:332-348's prompt chunks): ids[s*T + t] is token t of
 * sequence s, at position t.  Writes every layer's K/V rows 0..T-1 into the
 * pages tables[s*max_pages ...] (device) of the pool and the greedy next id of
 * every sequence to next_ids[s] (device).  Same bits as prefilling each
 * sequence alone in 32-row chunks.  Needs T <= max_seq, ceil(T/32) <= max_pages
 * and q3_prefill_workspace_bytes(layout, n_seqs, T) bytes of workspace. */
size_t q3_prefill_workspace_bytes(const q3_layout *layout, uint32_t n_seqs, uint32_t T);
int q3_prefill_batch(void *blob, const q3_layout *layout, const q3_kv_pool *pool,
                     const uint16_t *tables, uint32_t max_pages, const int32_t *ids,
                     uint32_t n_seqs, uint32_t T, int32_t *next_ids, void *workspace,
                     size_t workspace_bytes, void *stream);

/* ---- host batching engine (extension; tools/engine.py:81-243) -------------
 * The reference's PagePool / Scheduler / Sampler / Engine.step in native code:
 * requests in admission order, prompts fed in chunks of up to 32 rows, one
 * decode row per generating request, at most max_rows rows per step, 32-token
 * pages taken from the end of the free list and returned when a request
 * finishes (the reference's policy exactly; a request that cannot get its
 * pages waits).  Each step runs the batch's rows through the model on the GPU
 * (blob non-null: the engine owns a page pool of num_pages pages for every
 * layer, q3_engine_device_bytes() of device memory, allocated at create) or
 * through a guest callback that fills the logits of the rows that need them
 * (the reference's guest_step; blob may be null).  Greedy picks
 * (temperature <= 0) are the first maximum, as np.argmax; sampling applies
 * temperature, repetition penalty, top-k and top-p as tools/engine.py:118-149
 * does, in float64, and draws one uniform per sample from the request's
 * np.random.default_rng(seed) stream (the same stream as the reference's
 * Request.rng), so a request's sampled ids follow the reference's for the same
 * logits.  On the GPU step the sampler runs on the device after the lm_head
 * (q3_sample_logits); with a guest it runs on the host.  Greedy ids per
 * request are bit-identical to running the request alone through
 * forward_chunk. */
typedef struct q3_sampling_params {
  uint32_t max_new;
  double temperature;
  uint32_t top_k;
  double top_p;
  double repetition_penalty;
  uint64_t seed;
  const int32_t *stop_tokens;   /* copied at add_request */
  uint32_t n_stop;
} q3_sampling_params;

typedef struct q3_engine_item {  /* one request's rows in a step (BatchItem) */
  int32_t rid;
  uint32_t row_start, rows, pos;
  int32_t prefill, needs_logits;
  const int32_t *tokens;         /* rows ids, valid until the next step       */
} q3_engine_item;

/* logits: one row of layout->vocab floats for each item with needs_logits, in
 * item order; return 0 (non-zero aborts the step with that status) */
typedef int (*q3_engine_guest_fn)(void *user, const q3_engine_item *items, uint32_t n_items,
                                  float *logits);

size_t q3_engine_device_bytes(const q3_layout *layout, uint32_t num_pages, uint32_t max_rows);
int q3_engine_create(void *blob, const q3_layout *layout, uint32_t num_pages, uint32_t max_rows,
                     void **engine);
int q3_engine_set_guest(void *engine, q3_engine_guest_fn fn, void *user);
/* Q3_ERR_CAPACITY when n_prompt + max_new exceeds layout->max_seq */
int q3_engine_add_request(void *engine, const int32_t *prompt, uint32_t n_prompt,
                          const q3_sampling_params *params, int32_t *rid);
/* one Engine.step; *did_work = 0 when no request could run (the step then
 * finishes requests that reached max_new, as the reference does) */
int q3_engine_step(void *engine, int32_t *did_work, void *stream);
int q3_engine_run(void *engine, uint32_t max_steps, void *stream);
int q3_engine_last_batch(const void *engine, q3_engine_item *items, uint32_t cap,
                         uint32_t *n_items);
int q3_engine_result(const void *engine, int32_t rid, int32_t *ids, uint32_t cap,
                     uint32_t *n_generated, int32_t *finished);
uint32_t q3_engine_free_pages(const void *engine);
uint64_t q3_engine_steps(const void *engine);
int q3_engine_destroy(void *engine);

/* ---- sampling after the lm_head (tools/engine.py:118-149) -----------------
 * q3_sample_logits picks one id per row of `logits` (rows x vocab f32) on the
 * device, with the Sampler's steps in float64: temperature <= 0 -> the first
 * maximum; else x = logits / temperature, the repetition penalty on the row's
 * generated ids (x / rp where x > 0, else x * rp), top-k (every x below the
 * k-th largest dropped), top-p (in descending order, every element whose
 * cumulative normalised probability exceeds top_p dropped, the first always
 * kept; equal values are ordered by index), then the first index whose
 * cumulative probability (index order) exceeds u, as Generator.choice(V, p)
 * does with its uniform u.  `params` and `generated` are DEVICE arrays; row r's
 * generated ids are generated[gen_offset .. gen_offset + gen_count).  Results
 * agree with the reference's float64 numpy arithmetic except where u or top_p
 * falls within a few float64 ulps of a cumulative sum (summation order). */
typedef struct q3_sample_row {
  double temperature, top_p, repetition_penalty;
  double u;                 /* the draw: Generator.random() of the request   */
  int32_t top_k;
  uint32_t gen_offset, gen_count, pad;
} q3_sample_row;

size_t q3_sample_workspace_bytes(uint32_t rows, uint32_t vocab);
int q3_sample_logits(const q3_view *logits, const q3_sample_row *params, const int32_t *generated,
                     int32_t *out_ids, void *workspace, size_t workspace_bytes, void *stream);

/* The first n draws of np.random.default_rng(seed).random() (host). */
int q3_rng_uniforms(uint64_t seed, uint32_t n, double *out);

/* ---- tokenizer (tools/tokenizer.py:39-192), host only ---------------------
 * The byte-level BPE of an HF tokenizer.json: added tokens matched literally
 * (leftmost-longest), the GPT-2 style pretokenizer split, byte symbols merged
 * by rank.  Text is UTF-8.  encode/decode report the needed size in *n_ids /
 * *n_bytes and return Q3_ERR_CAPACITY when `cap` is smaller; an id or symbol
 * outside the vocabulary, or malformed input, gives Q3_ERR_SHAPE.  Decoding
 * replaces invalid UTF-8 as Python's errors="replace" does.  eos_id is the id
 * of <|im_end|> (151645 when the file has none). */
int q3_tokenizer_load(const char *tokenizer_json, void **tokenizer);
int q3_tokenizer_encode(const void *tokenizer, const char *text, size_t text_bytes, int32_t *ids,
                        uint32_t cap, uint32_t *n_ids);
int q3_tokenizer_decode(const void *tokenizer, const int32_t *ids, uint32_t n, char *text,
                        size_t cap, size_t *n_bytes);
int32_t q3_tokenizer_eos_id(const void *tokenizer);
int q3_tokenizer_destroy(void *tokenizer);

/* ---- tensor-parallel batched decode (extension) ---------------------------
 * The batched decode step split over `world` GPUs of one node, one process per
 * GPU.  The reference runs one hart and has no such split; this follows its
 * arithmetic exactly (src/main_big.cpp:173-262 per layer):
 *   - Q/K/V, head norm/rope/quant, the KV pages and attention: by KV head (a
 *     rank owns kv_heads/world KV heads and their 2 Q heads each);
 *   - gate/up + SwiGLU + quant: by 256-wide quant group;
 *   - O and down: every rank computes the dequantised partials of its own K
 *     groups and stores them into every rank's receive buffer over NVLink;
 *     each rank then adds all groups in group order (group_gemm.h:194-214 /
 *     ref_qwen3.py:151-157 order), so x stays bit-identical on every rank;
 *   - lm_head: by vocabulary rows; the (max, first index) pairs of the ranks
 *     are exchanged and the largest value, then the smallest index, wins.
 * The rank's pool holds only its own KV heads: row width kv_heads*128 of the
 * shard.  next_ids comes out identical on every rank and identical to
 * q3_decode_step_batch on one GPU. */
typedef struct q3_tp_shard {
  int32_t rank, world;
  uint32_t q_head0, q_heads;        /* Q heads [q_head0, q_head0 + q_heads)        */
  uint32_t kv_head0, kv_heads;      /* KV heads                                    */
  uint32_t mlp_group0, mlp_groups;  /* 256-wide intermediate groups                */
  uint32_t vocab0, vocab_rows;      /* lm_head rows, whole 128-row tiles           */
} q3_tp_shard;

/* Host only.  Q3_ERR_SHAPE unless world divides kv_heads, heads = 2*kv_heads,
 * and every rank gets at least one MLP group and one 128-row vocabulary tile. */
int q3_tp_shard_of(const q3_layout *layout, int32_t rank, int32_t world, q3_tp_shard *out);

/* Bytes of the opaque handle q3_tp_comm_create writes (a CUDA IPC handle). */
size_t q3_tp_handle_bytes(void);

/* Communicator of one rank on the current device: allocates the rank's
 * exchange region (receive buffers for up to max_seqs <= 64 sequences and the
 * signal counters) and writes its handle.  The caller gathers every rank's
 * handle (rank order) by any means and passes them to q3_tp_comm_connect,
 * which maps the peers' regions.  reset zeroes this rank's counters (all ranks
 * reset between the same two host barriers, with no step in flight); after a
 * timed-out wait (device status bit 20) the counters disagree until reset. */
int q3_tp_comm_create(const q3_layout *layout, int32_t rank, int32_t world,
                      uint32_t max_seqs, void **comm, void *handle);
int q3_tp_comm_connect(void *comm, const void *handles);
int q3_tp_comm_reset(void *comm, void *stream);
int q3_tp_comm_destroy(void *comm);

/* No counterpart in the reference (it runs on one NPU): failure detection of
 * the exchange.  set_wait_ns sets how long this rank's kernels wait for a
 * peer's signal before they give up, set device status bit 20 and return
 * (default 2 s; 1 ms .. 60 s, else Q3_ERR_SHAPE).  inject_missing_signals
 * raises this rank's expected signal count of one exchange buffer (0 = O
 * partials, 1 = down partials, 2 = argmax keys) from `producer` by `count`,
 * stream-ordered, exactly as if that producer had fallen behind: the next
 * consumer of the buffer times out.  It exists to test the recovery path
 * (timeout -> status bit 20 -> q3_tp_comm_reset -> clean step) without a
 * peer process or a GPU fault. */
int q3_tp_comm_set_wait_ns(void *comm, uint64_t ns);

/* Comparison variant of the decode step's O / down reductions
 * (src/main_big.cpp:255,261 reduction points): mode 1 sums each rank's own
 * group partials in order, then sums the ranks' results with ncclAllReduce
 * (NCCL's ring/tree order, so the residual stream matches the exact path only
 * within float32 rounding, and greedy ids can differ where two logits tie
 * within it); mode 0 (default) is the exact ordered exchange.  The first
 * switch to mode 1 is collective: every rank passes the same 128-byte NCCL
 * unique id, made on one rank by q3_tp_nccl_unique_id and sent to the others
 * by the host.  NCCL is loaded from the process (libnccl.so.2) at that point;
 * nothing else in the library uses it. */
int q3_tp_nccl_unique_id(void *out128);
int q3_tp_comm_set_reduction(void *comm, int32_t mode, const void *nccl_unique_id);
int q3_tp_comm_inject_missing_signals(void *comm, int32_t buf, int32_t producer,
                                      uint32_t count, void *stream);

/* One decode step of this rank (same arguments as q3_decode_step_batch; the
 * workspace size is q3_decode_workspace_bytes).  Every rank calls it with the
 * same ids, pos and tables; the kernels wait for the peers' partials on the
 * device (bounded, about two seconds). */
int q3_tp_decode_step_batch(void *comm, void *blob, const q3_layout *layout,
                            const q3_kv_pool *pool, const uint16_t *tables,
                            uint32_t max_pages, const int32_t *ids, const int32_t *pos,
                            uint32_t n_seqs, int32_t *next_ids, void *workspace,
                            size_t workspace_bytes, void *stream);

/* Tensor-parallel batched prefill (config 5 at 2/4/8 GPUs): the layer chain
 * of q3_prefill_batch split over the ranks, bit-identical to it.  Rank r owns
 * the q/KV heads and MLP groups of its shard (q3_tp_shard_of), the residual
 * columns [r*H/world, (r+1)*H/world) and its vocabulary rows.  Per layer:
 * RMSNorm + quant of the full residual on every rank; V, K and Q GEMMs and
 * causal attention for the rank's heads (its pool holds only its KV heads);
 * all-gather of the attention output o8/os; the O GEMM for the rank's residual
 * columns (every K group summed in the reference's order, group_gemm.h:194-214);
 * all-gather of x; RMSNorm + quant; gate/up SwiGLU for the rank's groups;
 * all-gather of s8/ss; down for the rank's columns; all-gather of x.  The last
 * rows' lm_head runs over the rank's vocabulary rows and the (max, first
 * index) keys are exchanged, as in the decode step.  Every element is computed
 * by one rank with the single-GPU arithmetic, so no sum changes order.
 *
 * The communicator holds the exchanged buffers of up to max_rows = n_seqs*T
 * rows and max_seqs sequences (about max_rows * 7.2 KB at the Qwen3-0.6B
 * shape) in a region every rank maps (CUDA IPC); create / connect / reset /
 * destroy work like the decode communicator's.  Exchanges are copies into the
 * other ranks' regions over NVLink, ordered by system-scope counters; a wait
 * gives up after wait_ns (2 s by default), sets device status bit 20 and
 * returns.  The workspace is q3_prefill_workspace_bytes(layout, n_seqs, T). */
int q3_tp_prefill_comm_create(const q3_layout *layout, int32_t rank, int32_t world,
                              uint32_t max_rows, uint32_t max_seqs, void **comm, void *handle);
int q3_tp_prefill_comm_connect(void *comm, const void *handles);
int q3_tp_prefill_comm_reset(void *comm, void *stream);
int q3_tp_prefill_comm_set_wait_ns(void *comm, uint64_t ns);
int q3_tp_prefill_comm_destroy(void *comm);
int q3_tp_prefill_batch(void *comm, void *blob, const q3_layout *layout,
                        const q3_kv_pool *pool, const uint16_t *tables, uint32_t max_pages,
                        const int32_t *ids, uint32_t n_seqs, uint32_t T, int32_t *next_ids,
                        void *workspace, size_t workspace_bytes, void *stream);

/* ---- value ops (include/tile.h exp_/exp2 semantics; tests/guest/value_ops.cpp)
 * out[i] = exp(x[i]) as the path computes it: exp2(f32(x * log2e))
 * (tools/ref_qwen3.py:27-29), or out[i] = exp2(x[i]); both correctly rounded
 * float32.  Element-wise over every element of a view (f32). */
int q3_exp_rows(const q3_view *x, const q3_view *out, void *stream);
int q3_exp2_rows(const q3_view *x, const q3_view *out, void *stream);

/* No counterpart in the reference: self-check of the device evaluations of
 * the correctly rounded exp2 (the short one, also in its batched branch-free
 * form and, for inputs <= 0, -inf and NaN, in the batched form for such
 * inputs, against the longer double-precision one it falls back to near
 * rounding midpoints).  Every float32 bit pattern in [lo_bits, hi_bits) is evaluated
 * each way; *count (device, caller-zeroed)
 * gains the number of results that differ and *first_bad (device, caller-set
 * to 0xffffffff) the smallest differing bit pattern. */
int q3_exp2_selfcheck(uint32_t lo_bits, uint32_t hi_bits, unsigned long long *count,
                      uint32_t *first_bad, void *stream);

/* No counterpart in the reference: self-check of the library's int8
 * requantisation against the IEEE quotient rounded by the float -> int
 * conversion and saturated.  With the scale s = amax * (1/127) formed as the
 * kernels form it: the code from the quotient rounded in float, for every
 * float32 bit pattern x in [lo_bits, hi_bits); and the code from a shared
 * reciprocal of s (Markstein's correction, no clamp), used where s is the scale
 * of the values' own absolute maximum, for those x with |x| <= amax and NaN.
 * amax finite and >= 0; *count (device, caller-zeroed) gains the codes that
 * differ and *first_bad (device, caller-set to 0xffffffff) the smallest
 * differing x. */
int q3_quant_selfcheck(uint32_t lo_bits, uint32_t hi_bits, float amax, unsigned long long *count,
                       uint32_t *first_bad, void *stream);

/* ---- misc ---------------------------------------------------------------- */
const char *q3_last_cuda_error(void);
int q3_device_check(void); /* Q3_OK on an sm_100 device, else Q3_ERR_ARCH */

/* Device-side error word of the library's kernels (0 = none; bit 1: a page
 * index beyond the pool was skipped; bit 2: a sequence needs more pages than
 * its table holds; bit 3 and bits 16-19: a bounded wait in a tensor-core GEMM or
 * attention pipeline timed out and the kernel gave up; bit 20: a
 * tensor-parallel exchange wait for another rank timed out).  Reading
 * synchronises with the device and clears
 * the word; -1 if it cannot be read. */
int q3_device_status(void);

/* Number of kernels this library has launched in this process (all threads). */
uint64_t q3_launch_count(void);

/* Kernel timing hook for benchmarks: while attached, the i-th launch of the
 * named kernel family ("attention", "gemm", "exchange": the tensor-parallel
 * reduce and key-exchange kernels) records cudaEvent_t start[i]
 * before it and stop[i] after it on its own stream, for i < capacity.
 * q3_timer_detach() returns how many launches were recorded. */
int q3_timer_attach(const char *family, void *const *start_events,
                    void *const *stop_events, int capacity);
int q3_timer_detach(void);

#ifdef __cplusplus
}
#endif

#endif /* Q3_OPS_H */
