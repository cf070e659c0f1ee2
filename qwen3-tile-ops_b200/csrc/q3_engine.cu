// Host batching engine: a page pool, the continuous-batching scheduler and the
// sampler of tools/engine.py:81-243, in C++, with the model step on the GPU.
//
// Scheduling is the reference's policy step for step (Scheduler.build_batch,
// Engine.step, PagePool): requests in admission order; a request still in its
// prompt gets a chunk of min(32, rest of the prompt, rows left) rows, a request
// in decode one row (its last generated id); pages are taken from the end of
// the free list as a request grows and returned when it finishes; a request
// that cannot get its pages waits.  One batch mixes prompt chunks and decode
// rows of many requests (kernels/kv_pages.h:98-131 semantics).
//
// The step runs every row of the batch through the layers with the operator
// entry points (the same arithmetic as forward_chunk for each row): embedding,
// RMSNorm/quant, Q/K/V with head norm/rope/quant, the new K/V rows scattered
// into each request's pages, one paged attention launch over all requests
// (each row sees its own request's keys up to its position), O + residual, the
// MLP, and for the requests that need logits the final norm and the lm_head:
// the fused argmax when every pick is greedy, else the logits and the device
// sampler (q3_sample_logits), so only the picked ids come back.
//
// Instead of the GPU step, a guest callback may produce the logits (the
// reference's guest_step), which runs the scheduler and sampler on the host.
// Either way a sampled pick draws its uniform from the request's
// np.random.default_rng(seed) stream (q3_rng.h), as the reference's
// Request.rng does.
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <new>
#include <vector>

#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_rng.h"

namespace {

constexpr uint32_t kPT = 32;
constexpr float kInvSqrt128 = 0.08838834764831845f;

enum ReqState { S_WAITING = 0, S_PREFILL = 1, S_DECODE = 2, S_FINISHED = 3 };

struct Req {
  int32_t rid = 0;
  std::vector<int32_t> prompt, generated, stop;
  q3_sampling_params sp{};
  uint32_t n_fed = 0;
  std::vector<uint32_t> pages;
  ReqState state = S_WAITING;
  q3rng::Pcg64 rng;
};

struct Item {
  Req *req;
  uint32_t row_start, rows, pos;
  std::vector<int32_t> tokens;
  bool prefill, needs_logits;
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// device buffers of one engine (offsets into one allocation)
struct Dev {
  // rows of a batch
  size_t x, h, h8, hs, q8, qs, k8, ks, v8, vs, o8, os, s8, ss, cosr, sinr;
  // step inputs, copied in one piece
  size_t in, ids, pos, row_item, item_rows, item_row0, item_kvlen, logit_rows, tables, sparams,
      in_bytes;
  // generated ids of the sampled rows (repetition penalty), copied after `in`
  size_t gen, gen_bytes;
  // lm_head rows, sampler
  size_t lx, lh, lh8, lhs, best, bidx, keys, logits, sout, sws;
  // page pool
  size_t pk, pv, pks, pvs;
  size_t total;
};

}  // namespace

struct q3_engine {
  char *blob = nullptr;
  q3_layout L{};
  uint32_t num_pages = 0, max_rows = 0, max_pages = 0;
  std::vector<uint32_t> free_list;
  std::vector<char> used;
  std::vector<Req *> reqs;
  std::vector<Item> last;
  std::vector<q3_engine_item> last_c;
  int32_t next_rid = 0;
  uint64_t steps = 0;
  q3_engine_guest_fn guest = nullptr;
  void *guest_user = nullptr;
  char *dev = nullptr;
  Dev d{};
  char *host_in = nullptr;        // pinned staging of the step inputs
  cudaEvent_t in_copied = nullptr;  // the last copy out of host_in has completed
  char *host_out = nullptr;       // pinned ids + logits
  size_t host_out_bytes = 0;
  std::vector<float> host_logits; // guest mode
};

namespace {

// ------------------------------------------------------------------ kernels
__global__ void k_eng_rope(const int32_t *pos, const float *cos_t, const float *sin_t, float *cosr,
                           float *sinr, int half) {
  const int r = blockIdx.x, p = pos[r];
  for (int j = threadIdx.x; j < half; j += blockDim.x) {
    cosr[r * half + j] = cos_t[static_cast<size_t>(p) * half + j];
    sinr[r * half + j] = sin_t[static_cast<size_t>(p) * half + j];
  }
}

// row r's new K/V -> page tables[item(r)][pos/32], slot pos%32
__global__ void k_eng_scatter(const int8_t *k8, const int8_t *v8, const float *ks, const float *vs,
                              const int32_t *pos, const int32_t *row_item, const uint16_t *tables,
                              uint32_t max_pages, char *pk, char *pv, char *pks, char *pvs, int kw,
                              int kvh) {
  const int r = blockIdx.x, p = pos[r];
  const uint32_t page = tables[static_cast<size_t>(row_item[r]) * max_pages + p / kPT];
  const size_t row = static_cast<size_t>(page) * kPT + (p % kPT);
  for (int i = threadIdx.x; i < kw / 16; i += blockDim.x) {
    reinterpret_cast<int4 *>(pk + row * kw)[i] = reinterpret_cast<const int4 *>(k8 + (size_t)r * kw)[i];
    reinterpret_cast<int4 *>(pv + row * kw)[i] = reinterpret_cast<const int4 *>(v8 + (size_t)r * kw)[i];
  }
  for (int h = threadIdx.x; h < kvh; h += blockDim.x) {
    reinterpret_cast<float *>(pks + row * kvh * 4)[h] = ks[r * kvh + h];
    reinterpret_cast<float *>(pvs + row * kvh * 4)[h] = vs[r * kvh + h];
  }
}

__global__ void k_eng_gather(const float *x, const int32_t *rows, float *out, int H, float *best) {
  const int i = blockIdx.x;
  const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<size_t>(rows[i]) * H);
  float4 *dst = reinterpret_cast<float4 *>(out + static_cast<size_t>(i) * H);
  for (int c = threadIdx.x; c < H / 4; c += blockDim.x) dst[c] = src[c];
  if (threadIdx.x == 0) best[i] = -3.0e38f;
}

q3_view vw(char *p, uint32_t rows, uint32_t cols, uint8_t dt) {
  const int es = (dt == Q3_DT_I8 || dt == Q3_DT_U8) ? 1 : 4;
  return q3_view{p, static_cast<int32_t>(cols * es), es, rows, cols, dt};
}

Dev carve(const q3_layout &L, uint32_t R, uint32_t num_pages) {
  const size_t H = L.hidden, QW = L.heads * L.head_dim, KW = L.kv_heads * L.head_dim, I = L.inter;
  const size_t HALF = L.head_dim / 2, MP = L.max_seq / kPT, V = L.vocab;
  Dev d{};
  size_t off = 0;
  auto take = [&](size_t bytes) { const size_t o = off; off += align256(bytes); return o; };
  d.x = take(4 * R * H);
  d.h = take(4 * R * H);
  d.h8 = take(R * H);
  d.hs = take(4 * R * (H / 256));
  d.q8 = take(R * QW);
  d.qs = take(4 * R * L.heads);
  d.k8 = take(R * KW);
  d.ks = take(4 * R * L.kv_heads);
  d.v8 = take(R * KW);
  d.vs = take(4 * R * L.kv_heads);
  d.o8 = take(R * QW);
  d.os = take(4 * R * L.heads);
  d.s8 = take(R * I);
  d.ss = take(4 * R * (I / 256));
  d.cosr = take(4 * R * HALF);
  d.sinr = take(4 * R * HALF);
  // step inputs: one contiguous block (offsets relative to d.in)
  d.in = off;
  size_t io = 0;
  auto itake = [&](size_t bytes) { const size_t o = io; io += align256(bytes); return o; };
  d.ids = itake(4 * R);
  d.pos = itake(4 * R);
  d.row_item = itake(4 * R);
  d.item_rows = itake(4 * R);
  d.item_row0 = itake(4 * R);
  d.item_kvlen = itake(4 * R);
  d.logit_rows = itake(4 * R);
  d.tables = itake(2 * R * MP);
  d.sparams = itake(sizeof(q3_sample_row) * R);
  d.in_bytes = io;
  off += align256(io);
  d.gen_bytes = 4 * R * static_cast<size_t>(L.max_seq);
  d.gen = take(d.gen_bytes);
  d.lx = take(4 * R * H);
  d.lh = take(4 * R * H);
  d.lh8 = take(R * H);
  d.lhs = take(4 * R * (H / 256));
  d.best = take(4 * R);
  d.bidx = take(4 * R);
  d.keys = take(8 * R);
  d.logits = take(4 * R * V);
  d.sout = take(4 * R);
  d.sws = take(q3_sample_workspace_bytes(R, static_cast<uint32_t>(V)));
  const size_t pool_rows = static_cast<size_t>(L.layers) * num_pages * kPT;
  d.pk = take(pool_rows * KW);
  d.pv = take(pool_rows * KW);
  d.pks = take(pool_rows * 4 * L.kv_heads);
  d.pvs = take(pool_rows * 4 * L.kv_heads);
  d.total = off;
  return d;
}

// ------------------------------------------------------------ page pool
uint32_t alloc_page(q3_engine &e, bool &ok) {
  if (e.free_list.empty()) {
    ok = false;
    return 0;
  }
  const uint32_t p = e.free_list.back();   // list.pop()
  e.free_list.pop_back();
  e.used[p] = 1;
  ok = true;
  return p;
}
bool ensure(q3_engine &e, Req &r, uint32_t n_tokens) {
  const uint32_t need = (n_tokens + kPT - 1) / kPT;
  while (r.pages.size() < need) {
    bool ok;
    const uint32_t p = alloc_page(e, ok);
    if (!ok) return false;
    r.pages.push_back(p);
  }
  return true;
}
void release(q3_engine &e, Req &r) {
  for (uint32_t p : r.pages)
    if (e.used[p]) {
      e.used[p] = 0;
      e.free_list.push_back(p);
    }
  r.pages.clear();
}
void finish(q3_engine &e, Req &r) {
  if (r.state != S_FINISHED) {
    r.state = S_FINISHED;
    release(e, r);
  }
}

// ------------------------------------------------------------ scheduler
std::vector<Item> build_batch(q3_engine &e) {
  std::vector<Item> items;
  uint32_t rows = 0;
  for (Req *rp : e.reqs) {
    Req &r = *rp;
    if (r.state == S_FINISHED) continue;
    const uint32_t n_prompt = static_cast<uint32_t>(r.prompt.size());
    if (r.n_fed < n_prompt) {                      // prompt chunk
      if (rows >= e.max_rows) continue;
      const uint32_t chunk = std::min(std::min(32u, n_prompt - r.n_fed), e.max_rows - rows);
      if (chunk == 0) continue;
      if (!ensure(e, r, r.n_fed + chunk)) continue;
      const bool last = r.n_fed + chunk == n_prompt;
      items.push_back(Item{&r, rows, chunk, r.n_fed,
                           std::vector<int32_t>(r.prompt.begin() + r.n_fed,
                                                r.prompt.begin() + r.n_fed + chunk),
                           true, last});
      rows += chunk;
      continue;
    }
    if (r.generated.size() >= r.sp.max_new) {      // decode: feed the last id
      finish(e, r);
      continue;
    }
    if (rows >= e.max_rows) continue;
    if (r.generated.empty()) continue;
    if (!ensure(e, r, r.n_fed + 1)) continue;
    items.push_back(Item{&r, rows, 1, r.n_fed, {r.generated.back()}, false, true});
    rows += 1;
  }
  return items;
}

// ------------------------------------------------------------ sampler
// numpy's pairwise summation of a float64 array (the loop np.sum runs)
double pairwise_sum(const double *a, size_t n) {
  if (n < 8) {
    double s = 0.0;
    for (size_t i = 0; i < n; ++i) s += a[i];
    return s;
  }
  if (n <= 128) {
    double r[8];
    for (int j = 0; j < 8; ++j) r[j] = a[j];
    size_t i = 8;
    for (; i < n - n % 8; i += 8)
      for (int j = 0; j < 8; ++j) r[j] += a[i + j];
    double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += a[i];
    return res;
  }
  size_t n2 = n / 2;
  n2 -= n2 % 8;
  return pairwise_sum(a, n2) + pairwise_sum(a + n2, n - n2);
}

// tools/engine.py:118-149 in float64 with numpy's operation order: greedy =
// np.argmax; x / T; penalty over set(generated); top-k threshold at
// np.partition's k-th largest; top-p over the descending order (equal values
// by index; numpy's default argsort leaves them to its introsort); then
// Generator.choice(V, p): cdf = cumsum(p) / cdf[-1], the first index whose
// cdf exceeds u.  u is the request's next default_rng(seed).random().
int32_t sample(const float *logits, uint32_t V, Req &r) {
  const q3_sampling_params &p = r.sp;
  if (!(p.temperature > 0.0)) {
    uint32_t best = 0;
    for (uint32_t i = 1; i < V; ++i)
      if (static_cast<double>(logits[i]) > static_cast<double>(logits[best])) best = i;
    return static_cast<int32_t>(best);
  }
  std::vector<double> x(logits, logits + V);
  for (double &v : x) v /= p.temperature;
  if (p.repetition_penalty != 1.0) {
    std::vector<int32_t> seen(r.generated);
    std::sort(seen.begin(), seen.end());
    seen.erase(std::unique(seen.begin(), seen.end()), seen.end());
    for (int32_t t : seen) {
      if (t < 0 || static_cast<uint32_t>(t) >= V) continue;
      if (x[t] > 0) x[t] /= p.repetition_penalty;
      else x[t] *= p.repetition_penalty;
    }
  }
  if (p.top_k > 0 && p.top_k < V) {
    std::vector<double> s(x);
    std::nth_element(s.begin(), s.end() - p.top_k, s.end());
    const double kth = *(s.end() - p.top_k);
    for (double &v : x)
      if (v < kth) v = -INFINITY;
  }
  std::vector<double> probs(V);
  if (p.top_p < 1.0) {
    std::vector<uint32_t> order(V);
    for (uint32_t i = 0; i < V; ++i) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](uint32_t a, uint32_t b) { return x[a] > x[b]; });
    const double top = x[order[0]];
    for (uint32_t i = 0; i < V; ++i) probs[i] = std::exp(x[order[i]] - top);
    const double sum = pairwise_sum(probs.data(), V);
    double cum = 0.0;
    for (uint32_t i = 0; i < V; ++i) {
      cum += probs[i] / sum;
      if (i > 0 && !(cum <= p.top_p)) x[order[i]] = -INFINITY;
    }
  }
  const double m = *std::max_element(x.begin(), x.end());
  for (uint32_t i = 0; i < V; ++i) probs[i] = std::exp(x[i] - m);
  const double sum = pairwise_sum(probs.data(), V);
  double cum = 0.0;
  for (double &v : probs) v = cum += v / sum;
  const double last = probs[V - 1];
  const double u = r.rng.random();
  for (uint32_t i = 0; i < V; ++i)
    if (probs[i] / last > u) return static_cast<int32_t>(i);
  return static_cast<int32_t>(V - 1);
}

// ------------------------------------------------------------ GPU step
int gpu_step(q3_engine &e, const std::vector<Item> &items, std::vector<int32_t> &ids_out,
             const float *&logits_out, cudaStream_t st) {
  const q3_layout &L = e.L;
  const int64_t *o = L.off;
  const Dev &d = e.d;
  char *D = e.dev;
  void *s = st;
  const uint32_t H = L.hidden, HD = L.head_dim, QW = L.heads * HD, KW = L.kv_heads * HD,
                 I = L.inter, V = L.vocab, MP = e.max_pages, HALF = HD / 2;
  const float inv_h = 1.0f / static_cast<float>(H), inv_hd = 1.0f / static_cast<float>(HD);

  // ---- step inputs
  uint32_t R = 0, maxr = 0, n_logit = 0;
  bool any_sampled = false;
  char *in = e.host_in;
  // the previous step's copy of the staging buffer must have left it
  cudaError_t ce = cudaEventSynchronize(e.in_copied);
  if (ce != cudaSuccess) {
    q3h::set_cuda_error(ce);
    return Q3_ERR_CUDA;
  }
  memset(in, 0, d.in_bytes);
  int32_t *ids = reinterpret_cast<int32_t *>(in + d.ids), *pos = reinterpret_cast<int32_t *>(in + d.pos);
  int32_t *row_item = reinterpret_cast<int32_t *>(in + d.row_item);
  int32_t *item_rows = reinterpret_cast<int32_t *>(in + d.item_rows);
  int32_t *item_row0 = reinterpret_cast<int32_t *>(in + d.item_row0);
  int32_t *item_kvlen = reinterpret_cast<int32_t *>(in + d.item_kvlen);
  int32_t *logit_rows = reinterpret_cast<int32_t *>(in + d.logit_rows);
  uint16_t *tables = reinterpret_cast<uint16_t *>(in + d.tables);
  q3_sample_row *sp = reinterpret_cast<q3_sample_row *>(in + d.sparams);
  int32_t *gen = reinterpret_cast<int32_t *>(in + d.in_bytes);
  uint32_t n_gen = 0;
  for (size_t i = 0; i < items.size(); ++i) {
    const Item &it = items[i];
    for (uint32_t t = 0; t < it.rows; ++t) {
      ids[it.row_start + t] = it.tokens[t];
      pos[it.row_start + t] = static_cast<int32_t>(it.pos + t);
      row_item[it.row_start + t] = static_cast<int32_t>(i);
    }
    item_rows[i] = static_cast<int32_t>(it.rows);
    item_row0[i] = static_cast<int32_t>(it.row_start);
    item_kvlen[i] = static_cast<int32_t>(it.pos + it.rows);
    for (size_t pg = 0; pg < it.req->pages.size(); ++pg)
      tables[i * MP + pg] = static_cast<uint16_t>(it.req->pages[pg]);
    if (it.needs_logits) {
      // the sampler's inputs; u is drawn only for a sampled pick, as the
      // reference's rng.choice is only reached then
      Req &rq = *it.req;
      q3_sample_row &row = sp[n_logit];
      row.temperature = rq.sp.temperature;
      row.top_p = rq.sp.top_p;
      row.repetition_penalty = rq.sp.repetition_penalty;
      row.top_k = static_cast<int32_t>(std::min<uint32_t>(rq.sp.top_k, 0x7FFFFFFF));
      row.gen_offset = n_gen;
      row.gen_count = 0;
      if (rq.sp.temperature > 0.0) {
        any_sampled = true;
        row.u = rq.rng.random();
        if (rq.sp.repetition_penalty != 1.0) {
          memcpy(gen + n_gen, rq.generated.data(), 4 * rq.generated.size());
          row.gen_count = static_cast<uint32_t>(rq.generated.size());
          n_gen += row.gen_count;
        }
      }
      logit_rows[n_logit++] = static_cast<int32_t>(it.row_start + it.rows - 1);
    }
    R = std::max(R, it.row_start + it.rows);
    maxr = std::max(maxr, it.rows);
  }
  ce = cudaMemcpyAsync(D + d.in, in, d.in_bytes, cudaMemcpyHostToDevice, st);
  if (ce == cudaSuccess && n_gen)
    ce = cudaMemcpyAsync(D + d.gen, gen, 4 * static_cast<size_t>(n_gen), cudaMemcpyHostToDevice, st);
  if (ce == cudaSuccess) ce = cudaEventRecord(e.in_copied, st);
  if (ce != cudaSuccess) {
    q3h::set_cuda_error(ce);
    return Q3_ERR_CUDA;
  }
  const int32_t *dpos = reinterpret_cast<const int32_t *>(D + d.in + d.pos);

  const q3_view x = vw(D + d.x, R, H, Q3_DT_F32), h = vw(D + d.h, R, H, Q3_DT_F32);
  const q3_view h8 = vw(D + d.h8, R, H, Q3_DT_I8), hs = vw(D + d.hs, R, H / 256, Q3_DT_F32);
  const q3_view q8 = vw(D + d.q8, R, QW, Q3_DT_I8), qs = vw(D + d.qs, R, L.heads, Q3_DT_F32);
  const q3_view k8 = vw(D + d.k8, R, KW, Q3_DT_I8), ks = vw(D + d.ks, R, L.kv_heads, Q3_DT_F32);
  const q3_view v8 = vw(D + d.v8, R, KW, Q3_DT_I8), vs = vw(D + d.vs, R, L.kv_heads, Q3_DT_F32);
  const q3_view o8 = vw(D + d.o8, R, QW, Q3_DT_I8), os = vw(D + d.os, R, L.heads, Q3_DT_F32);
  const q3_view s8 = vw(D + d.s8, R, I, Q3_DT_I8), ss = vw(D + d.ss, R, I / 256, Q3_DT_F32);
  const q3_view cosr = vw(D + d.cosr, R, HALF, Q3_DT_F32), sinr = vw(D + d.sinr, R, HALF, Q3_DT_F32);
  const q3_view idv = vw(D + d.in + d.ids, R, 1, Q3_DT_I32);
  char *bl = e.blob;
  const q3_view emb = vw(bl + o[Q3_OFF_EMB], V, H, Q3_DT_I8);
  const q3_view emb_s = vw(bl + o[Q3_OFF_EMB] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view lm = vw(bl + o[Q3_OFF_LM], V, H, Q3_DT_I8);
  const q3_view lm_s = vw(bl + o[Q3_OFF_LM] + (int64_t)V * H, V, 1, Q3_DT_F32);
  const q3_view nf = vw(bl + o[Q3_OFF_NF], H, 1, Q3_DT_F32);

  k_eng_rope<<<R, 64, 0, st>>>(dpos, reinterpret_cast<const float *>(bl + o[Q3_OFF_COS]),
                               reinterpret_cast<const float *>(bl + o[Q3_OFF_SIN]),
                               reinterpret_cast<float *>(D + d.cosr), reinterpret_cast<float *>(D + d.sinr),
                               HALF);
  Q3_TRY(q3h::launch_status());
  {
    const q3_view n1_0 = vw(bl + o[Q3_OFF_N1], H, 1, Q3_DT_F32);
    Q3_TRY(q3_embedding_rmsnorm_rows(&emb, &emb_s, &idv, &x, &n1_0, &h, inv_h, s));
  }
  const size_t layer_rows = static_cast<size_t>(e.num_pages) * kPT;
  for (uint32_t Li = 0; Li < L.layers; ++Li) {
    char *lw = bl + o[Q3_OFF_LQ] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERW_STRIDE];
    char *ln = bl + o[Q3_OFF_N1] + static_cast<int64_t>(Li) * o[Q3_OFF_LAYERN_STRIDE];
    auto W = [&](int key, uint32_t r, uint32_t c) { return vw(lw + (o[key] - o[Q3_OFF_LQ]), r, c, Q3_DT_I8); };
    auto S = [&](int key, uint32_t r) { return vw(lw + (o[key] - o[Q3_OFF_LQ]), r, 1, Q3_DT_F32); };
    const q3_view wq = W(Q3_OFF_LQ, QW, H), wk = W(Q3_OFF_LK, KW, H), wv = W(Q3_OFF_LV, KW, H);
    const q3_view wo = W(Q3_OFF_LO, H, QW), wg = W(Q3_OFF_LG, I, H), wu = W(Q3_OFF_LU, I, H);
    const q3_view wd = W(Q3_OFF_LD, H, I);
    const q3_view wqs = S(Q3_OFF_LQ_SCALE, QW), wks = S(Q3_OFF_LK_SCALE, KW);
    const q3_view wvs = S(Q3_OFF_LV_SCALE, KW), wos = S(Q3_OFF_LO_SCALE, H);
    const q3_view wgs = S(Q3_OFF_LG_SCALE, I), wus = S(Q3_OFF_LU_SCALE, I);
    const q3_view wds = S(Q3_OFF_LD_SCALE, H);
    const q3_view n1 = vw(ln, H, 1, Q3_DT_F32);
    const q3_view nq = vw(ln + (o[Q3_OFF_NQ] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view nk = vw(ln + (o[Q3_OFF_NK] - o[Q3_OFF_N1]), HD, 1, Q3_DT_F32);
    const q3_view n2 = vw(ln + (o[Q3_OFF_N2] - o[Q3_OFF_N1]), H, 1, Q3_DT_F32);
    char *pk = D + d.pk + Li * layer_rows * KW, *pv = D + d.pv + Li * layer_rows * KW;
    char *pks = D + d.pks + Li * layer_rows * 4 * L.kv_heads;
    char *pvs = D + d.pvs + Li * layer_rows * 4 * L.kv_heads;

    if (Li != 0) Q3_TRY(q3_rmsnorm_rows(&x, &n1, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wv, &wvs, nullptr, 256, nullptr, &v8, &vs, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wk, &wks, nullptr, 256, nullptr, &k8, &ks, &nk, &cosr,
                                  &sinr, inv_hd, s));
    k_eng_scatter<<<R, 64, 0, st>>>(reinterpret_cast<const int8_t *>(k8.data),
                                    reinterpret_cast<const int8_t *>(v8.data),
                                    reinterpret_cast<const float *>(ks.data),
                                    reinterpret_cast<const float *>(vs.data), dpos,
                                    reinterpret_cast<const int32_t *>(D + d.in + d.row_item),
                                    reinterpret_cast<const uint16_t *>(D + d.in + d.tables), MP, pk,
                                    pv, pks, pvs, KW, L.kv_heads);
    Q3_TRY(q3h::launch_status());
    Q3_TRY(q3_gemm_nt_group_store(&h8, &hs, &wq, &wqs, nullptr, 256, nullptr, &q8, &qs, &nq, &cosr,
                                  &sinr, inv_hd, s));
    {
      q3::AttnArgs a{};
      a.q8 = static_cast<const char *>(q8.data);
      a.q_rb = QW;
      a.qs = static_cast<const char *>(qs.data);
      a.qs_rb = 4 * L.heads;
      a.o8 = static_cast<char *>(o8.data);
      a.o_rb = QW;
      a.os = static_cast<char *>(os.data);
      a.os_rb = 4 * L.heads;
      a.k = pk;
      a.v = pv;
      a.ks = pks;
      a.vs = pvs;
      a.table = reinterpret_cast<const uint16_t *>(D + d.in + d.tables);
      a.table_stride = MP;
      a.page_tokens = kPT;
      a.page_bytes = kPT * KW;
      a.row_bytes = KW;
      a.scale_page_bytes = kPT * 4 * L.kv_heads;
      a.scale_row_bytes = 4 * L.kv_heads;
      a.heads = L.heads;
      a.kv_heads = L.kv_heads;
      a.q_rows = maxr;
      a.kv_len_dev = reinterpret_cast<const int *>(D + d.in + d.item_kvlen);
      a.causal = 1;
      a.qk_scale = kInvSqrt128;
      a.item_rows = reinterpret_cast<const int *>(D + d.in + d.item_rows);
      a.item_row0 = reinterpret_cast<const int *>(D + d.in + d.item_row0);
      Q3_TRY(q3::attention_launch(a, static_cast<int>(items.size()), st));
    }
    Q3_TRY(q3_gemm_nt_group_store(&o8, &os, &wo, &wos, nullptr, 128, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_rmsnorm_rows(&x, &n2, &h, inv_h, s));
    Q3_TRY(q3_quant_rows_heads(&h, &h8, &hs, 256, s));
    Q3_TRY(q3_gemm_gate_up_swiglu_quant(&h8, &hs, &wg, &wgs, &wu, &wus, &s8, &ss, 256, s));
    Q3_TRY(q3_gemm_nt_group_store(&s8, &ss, &wd, &wds, nullptr, 256, &x, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, 0.0f, s));
  }
  // ---- lm_head for the last row of every request that needs logits
  ids_out.assign(n_logit, 0);
  logits_out = nullptr;
  if (n_logit == 0) return Q3_OK;
  k_eng_gather<<<n_logit, 256, 0, st>>>(reinterpret_cast<const float *>(D + d.x),
                                        reinterpret_cast<const int32_t *>(D + d.in + d.logit_rows),
                                        reinterpret_cast<float *>(D + d.lx), H,
                                        reinterpret_cast<float *>(D + d.best));
  Q3_TRY(q3h::launch_status());
  const q3_view lx = vw(D + d.lx, n_logit, H, Q3_DT_F32), lh = vw(D + d.lh, n_logit, H, Q3_DT_F32);
  const q3_view lh8 = vw(D + d.lh8, n_logit, H, Q3_DT_I8);
  const q3_view lhs = vw(D + d.lhs, n_logit, H / 256, Q3_DT_F32);
  Q3_TRY(q3_rmsnorm_rows(&lx, &nf, &lh, inv_h, s));
  Q3_TRY(q3_quant_rows_heads(&lh, &lh8, &lhs, 256, s));
  Q3_TRY(q3_gemm_nt_group_argmax(&lh8, &lhs, &lm, &lm_s, reinterpret_cast<float *>(D + d.best),
                                 reinterpret_cast<int32_t *>(D + d.bidx), 256, D + d.keys,
                                 8 * static_cast<size_t>(e.max_rows), s));
  const char *picked = D + d.bidx;
  if (any_sampled) {
    // full logits of the rows, then the sampler on the device: only the
    // picked ids come back
    const q3_view lg = vw(D + d.logits, n_logit, V, Q3_DT_F32);
    Q3_TRY(q3_gemm_nt_group_store(&lh8, &lhs, &lm, &lm_s, &lg, 256, nullptr, nullptr, nullptr,
                                  nullptr, nullptr, nullptr, 0.0f, s));
    Q3_TRY(q3_sample_logits(&lg, reinterpret_cast<const q3_sample_row *>(D + d.in + d.sparams),
                            reinterpret_cast<const int32_t *>(D + d.gen),
                            reinterpret_cast<int32_t *>(D + d.sout), D + d.sws,
                            q3_sample_workspace_bytes(e.max_rows, V), s));
    picked = D + d.sout;
  }
  ce = cudaMemcpyAsync(e.host_out, picked, 4 * n_logit, cudaMemcpyDeviceToHost, st);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(st);
  if (ce != cudaSuccess) {
    q3h::set_cuda_error(ce);
    return Q3_ERR_CUDA;
  }
  memcpy(ids_out.data(), e.host_out, 4 * n_logit);
  return Q3_OK;
}

}  // namespace

// ======================================================================= C ABI
extern "C" size_t q3_engine_device_bytes(const q3_layout *layout, uint32_t num_pages,
                                         uint32_t max_rows) {
  if (!layout || max_rows == 0) return 0;
  return carve(*layout, max_rows, num_pages).total;
}

extern "C" int q3_engine_create(void *blob, const q3_layout *layout, uint32_t num_pages,
                                uint32_t max_rows, void **engine) {
  if (!layout || !engine) return Q3_ERR_NULL;
  *engine = nullptr;
  const q3_layout &L = *layout;
  if (num_pages == 0 || num_pages > 65536 || max_rows == 0 || max_rows > 1024 ||
      L.max_seq % kPT || L.max_seq / kPT == 0)
    return Q3_ERR_SHAPE;
  if (blob && (L.head_dim != 128 || L.hidden % 256 || L.inter % 256 || L.heads % L.kv_heads ||
               L.vocab % 128))
    return Q3_ERR_SHAPE;
  q3_engine *e = new (std::nothrow) q3_engine;
  if (!e) return Q3_ERR_CAPACITY;
  e->blob = static_cast<char *>(blob);
  e->L = L;
  e->num_pages = num_pages;
  e->max_rows = max_rows;
  e->max_pages = L.max_seq / kPT;
  e->free_list.resize(num_pages);
  for (uint32_t i = 0; i < num_pages; ++i) e->free_list[i] = i;
  e->used.assign(num_pages, 0);
  if (blob) {   // device step: pool, row buffers and pinned staging
    e->d = carve(L, max_rows, num_pages);
    e->host_out_bytes = align256(4 * max_rows);
    cudaError_t ce = cudaMalloc(&e->dev, e->d.total);
    if (ce == cudaSuccess) ce = cudaMemset(e->dev, 0, e->d.total);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->host_in, e->d.in_bytes + e->d.gen_bytes);
    if (ce == cudaSuccess) ce = cudaMallocHost(&e->host_out, e->host_out_bytes);
    if (ce == cudaSuccess) ce = cudaEventCreateWithFlags(&e->in_copied, cudaEventDisableTiming);
    if (ce == cudaSuccess) ce = cudaEventRecord(e->in_copied, 0);
    if (ce == cudaSuccess) ce = cudaDeviceSynchronize();
    if (ce != cudaSuccess) {
      q3h::set_cuda_error(ce);
      if (e->dev) cudaFree(e->dev);
      if (e->host_in) cudaFreeHost(e->host_in);
      if (e->host_out) cudaFreeHost(e->host_out);
      if (e->in_copied) cudaEventDestroy(e->in_copied);
      delete e;
      return Q3_ERR_CUDA;
    }
  }
  *engine = e;
  return Q3_OK;
}

extern "C" int q3_engine_set_guest(void *engine, q3_engine_guest_fn fn, void *user) {
  if (!engine) return Q3_ERR_NULL;
  q3_engine *e = static_cast<q3_engine *>(engine);
  e->guest = fn;
  e->guest_user = user;
  return Q3_OK;
}

extern "C" int q3_engine_add_request(void *engine, const int32_t *prompt, uint32_t n_prompt,
                                     const q3_sampling_params *params, int32_t *rid) {
  if (!engine || !prompt || !params || !rid) return Q3_ERR_NULL;
  q3_engine *e = static_cast<q3_engine *>(engine);
  if (n_prompt == 0) return Q3_ERR_SHAPE;
  if (static_cast<uint64_t>(n_prompt) + params->max_new > e->L.max_seq) return Q3_ERR_CAPACITY;
  if (e->blob)   // ids index the embedding table
    for (uint32_t i = 0; i < n_prompt; ++i)
      if (prompt[i] < 0 || static_cast<uint32_t>(prompt[i]) >= e->L.vocab) return Q3_ERR_SHAPE;
  if (params->n_stop && !params->stop_tokens) return Q3_ERR_NULL;
  Req *r = new (std::nothrow) Req;
  if (!r) return Q3_ERR_CAPACITY;
  r->rid = e->next_rid++;
  r->prompt.assign(prompt, prompt + n_prompt);
  r->sp = *params;
  r->stop.assign(params->stop_tokens, params->stop_tokens + params->n_stop);
  r->sp.stop_tokens = nullptr;
  r->rng = q3rng::Pcg64(params->seed);
  e->reqs.push_back(r);
  *rid = r->rid;
  return Q3_OK;
}

extern "C" int q3_engine_step(void *engine, int32_t *did_work, void *stream) {
  if (!engine || !did_work) return Q3_ERR_NULL;
  q3_engine *e = static_cast<q3_engine *>(engine);
  *did_work = 0;
  if (!e->guest && !e->dev) return Q3_ERR_NULL;         // neither a model nor a guest
  std::vector<Item> items = build_batch(*e);
  e->last = items;
  if (items.empty()) {
    for (Req *r : e->reqs)
      if (r->state != S_FINISHED && r->n_fed >= r->prompt.size() &&
          r->generated.size() >= r->sp.max_new)
        finish(*e, *r);
    return Q3_OK;
  }
  const uint32_t V = e->L.vocab;
  std::vector<int32_t> greedy;
  const float *logits = nullptr;
  if (e->guest) {
    std::vector<q3_engine_item> ci(items.size());
    uint32_t n_logit = 0;
    for (size_t i = 0; i < items.size(); ++i) {
      const Item &it = items[i];
      ci[i] = q3_engine_item{it.req->rid, it.row_start, it.rows, it.pos, it.prefill ? 1 : 0,
                             it.needs_logits ? 1 : 0, it.tokens.data()};
      n_logit += it.needs_logits ? 1u : 0u;
    }
    e->host_logits.assign(static_cast<size_t>(n_logit) * V, 0.0f);
    const int rc = e->guest(e->guest_user, ci.data(), static_cast<uint32_t>(ci.size()),
                            e->host_logits.data());
    if (rc != 0) return rc;
    logits = e->host_logits.data();
  } else {
    Q3_TRY(gpu_step(*e, items, greedy, logits, static_cast<cudaStream_t>(stream)));
  }
  uint32_t li = 0;
  for (Item &it : items) {
    Req &r = *it.req;
    r.n_fed += it.rows;
    if (it.needs_logits) {
      int32_t tok;
      if (!e->guest) tok = greedy[li];   // picked on the device
      else tok = sample(logits + static_cast<size_t>(li) * V, V, r);
      ++li;
      r.generated.push_back(tok);
      if (std::find(r.stop.begin(), r.stop.end(), tok) != r.stop.end() ||
          r.generated.size() >= r.sp.max_new)
        finish(*e, r);
      else
        r.state = S_DECODE;
    } else if (r.n_fed < r.prompt.size()) {
      r.state = S_PREFILL;
    }
  }
  ++e->steps;
  *did_work = 1;
  return Q3_OK;
}

extern "C" int q3_engine_run(void *engine, uint32_t max_steps, void *stream) {
  if (!engine) return Q3_ERR_NULL;
  q3_engine *e = static_cast<q3_engine *>(engine);
  int32_t work = 1;
  while (e->steps < max_steps && work) Q3_TRY(q3_engine_step(engine, &work, stream));
  return Q3_OK;
}

extern "C" int q3_engine_last_batch(const void *engine, q3_engine_item *items, uint32_t cap,
                                    uint32_t *n_items) {
  if (!engine || !n_items) return Q3_ERR_NULL;
  const q3_engine *e = static_cast<const q3_engine *>(engine);
  *n_items = static_cast<uint32_t>(e->last.size());
  if (cap < e->last.size()) return e->last.empty() ? Q3_OK : Q3_ERR_CAPACITY;
  if (!items && !e->last.empty()) return Q3_ERR_NULL;
  for (size_t i = 0; i < e->last.size(); ++i) {
    const Item &it = e->last[i];
    items[i] = q3_engine_item{it.req->rid, it.row_start, it.rows, it.pos, it.prefill ? 1 : 0,
                              it.needs_logits ? 1 : 0, it.tokens.data()};
  }
  return Q3_OK;
}

extern "C" int q3_engine_result(const void *engine, int32_t rid, int32_t *ids, uint32_t cap,
                                uint32_t *n_generated, int32_t *finished) {
  if (!engine || !n_generated || !finished) return Q3_ERR_NULL;
  const q3_engine *e = static_cast<const q3_engine *>(engine);
  for (const Req *r : e->reqs) {
    if (r->rid != rid) continue;
    *n_generated = static_cast<uint32_t>(r->generated.size());
    *finished = r->state == S_FINISHED ? 1 : 0;
    if (ids) std::copy_n(r->generated.begin(), std::min<size_t>(cap, r->generated.size()), ids);
    return Q3_OK;
  }
  return Q3_ERR_SHAPE;
}

extern "C" uint32_t q3_engine_free_pages(const void *engine) {
  return engine ? static_cast<uint32_t>(static_cast<const q3_engine *>(engine)->free_list.size()) : 0;
}

extern "C" uint64_t q3_engine_steps(const void *engine) {
  return engine ? static_cast<const q3_engine *>(engine)->steps : 0;
}

extern "C" int q3_engine_destroy(void *engine) {
  if (!engine) return Q3_OK;
  q3_engine *e = static_cast<q3_engine *>(engine);
  for (Req *r : e->reqs) delete r;
  if (e->in_copied) {
    cudaEventSynchronize(e->in_copied);
    cudaEventDestroy(e->in_copied);
  }
  if (e->dev) {
    cudaDeviceSynchronize();   // no step of this engine may still use its memory
    cudaFree(e->dev);
  }
  if (e->host_in) cudaFreeHost(e->host_in);
  if (e->host_out) cudaFreeHost(e->host_out);
  delete e;
  return Q3_OK;
}
