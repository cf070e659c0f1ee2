// Tensor-parallel decode: shard plan, communicator (exchange regions mapped
// between the ranks' processes with CUDA IPC) and the kernels that consume the
// exchanged data.  The producers are the PART mode of the decode GEMM
// (q3_decode_gemm.cu), which stores each rank's dequantised K-group partials
// straight into every rank's receive buffer, and the argmax exchange below.
//
// Ordering protocol (no host collective on the data path).  Region of every
// rank: sig[buf][producer] counters, expect[buf][producer] (local only), the
// receive buffers.  A producer CTA stores its data to every rank, passes a
// CTA barrier, and one thread adds 1 (release, system scope: cumulative over
// the stores the barrier ordered before it) to sig[buf][me] at every rank.  The consumer of `buf` on a rank waits until sig[buf][q] has reached
// expect[buf][q] for every q (acquire, system scope; bounded at ~2 s), the
// expected count having been advanced by this rank's own producer kernel of the
// buffer, which runs just before the consumer in stream order.  A rank can
// reuse a buffer only after every rank has consumed its previous contents:
// the next write into `buf` comes after the writer waited for data that each
// reader produces only after its own consumer of `buf` finished (stream order).
#include <dlfcn.h>
#include <string.h>

#include <new>

#include "q3_common.cuh"
#include "q3_tc.cuh"
#include "q3_tp.h"

namespace q3 {

static __device__ unsigned int g_tp_error = 0;
constexpr unsigned kErrTpWait = 1u << 20;

int tp_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_tp_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_tp_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace {

// wait (bounded by limit_ns, 2 s by default) until the counter has reached
// `target` (wrap-safe)
__device__ bool wait_count(const unsigned *ctr, unsigned target, unsigned long long limit_ns) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (static_cast<int>(v - target) >= 0) return true;
    if ((it & 63) == 0) {
      const uint64_t t = tcx::gtime();
      if (t0 == 0) t0 = t;
      else if (t - t0 > limit_ns) return false;
    }
  }
}

__device__ __forceinline__ void sys_signal(unsigned *ctr) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

// CTA per row, 1024 threads, H == 1024: thread t owns feature t, so warp w is
// the 32-column block w (lane = column in the block) and warps 8g..8g+7 the
// quant group g; all the partials of a thread are loaded before the first add
__global__ void __launch_bounds__(1024) k_tp_reduce_norm(TpReduceArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ __align__(16) float bsum[32];
  __shared__ float gmax[32];
  const int m = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  if (t < a.world && !wait_count(a.sig + t, a.expect[t], a.wait_ns))
    atomicOr(&g_tp_error, kErrTpWait);
  __syncthreads();
  // group-ordered sum of the partials (ref_qwen3.py:151-157)
  const float *base = a.recv + static_cast<size_t>(m) * a.H + t;
  const size_t sstride = static_cast<size_t>(a.B) * a.H;
  float v[kTpMaxSlots];
#pragma unroll
  for (int s = 0; s < kTpMaxSlots; ++s) v[s] = s < a.slots ? __ldcg(base + s * sstride) : 0.0f;
  float acc = 0.0f;
#pragma unroll
  for (int s = 0; s < kTpMaxSlots; ++s)
    if (s < a.slots) acc = __fadd_rn(acc, v[s]);
  // x += sum; tree sum of x^2 over this warp's 32-column block (rmsnorm.h:34-81)
  float *xr = a.x + static_cast<size_t>(m) * a.H;
  const float xv = __fadd_rn(xr[t], acc);
  xr[t] = xv;
  const float b = warp_tree_sum(__fmul_rn(xv, xv));
  if (lane == 0) bsum[warp] = b;
  __syncthreads();
  float4 b4[8];                           // the 32 block sums at once, then in block order
#pragma unroll
  for (int i = 0; i < 8; ++i) b4[i] = reinterpret_cast<const float4 *>(bsum)[i];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ss = __fadd_rn(ss, b4[i].x);
    ss = __fadd_rn(ss, b4[i].y);
    ss = __fadd_rn(ss, b4[i].z);
    ss = __fadd_rn(ss, b4[i].w);
  }
  ss = __fadd_rn(__fmul_rn(ss, a.inv), kEps);
  const float r = rsqrt_ref(ss);
  const float hv = __fmul_rn(__fmul_rn(xv, r), a.w[t]);
  const float mx = warp_tree_max(fabsf(hv));
  if (lane == 0) gmax[warp] = mx;
  __syncthreads();
  const int g = warp >> 3;                // quant group = features [256g, 256g + 256)
  float gm = 0.0f;
#pragma unroll
  for (int w = 0; w < 8; ++w) gm = fmaxf(gm, gmax[8 * g + w]);
  const float scale = __fmul_rn(gm, kInv127);
  a.h8[static_cast<size_t>(m) * a.H + t] = static_cast<int8_t>(quant1(hv, scale));
  if ((t & 255) == 0) a.hs[static_cast<size_t>(m) * (a.H / 256) + g] = scale;
}

struct TpArgmaxArgs {
  const float *best;
  const int32_t *bidx;
  uint32_t v0;
  int B, world, me, max_seqs;
  unsigned long long *keys_dst[kTpMaxRanks];   // rank q's key buffer [ranks][max_seqs]
  unsigned *sig_dst[kTpMaxRanks];              // rank q's sig[TP_KEYS][me]
  const unsigned long long *keys;              // this rank's key buffer
  const unsigned *sig;                         // this rank's sig[TP_KEYS][.]
  unsigned *expect;                            // this rank's expect[TP_KEYS][.]
  int32_t *next_ids;
  unsigned long long wait_ns;
};

// (max, first index) of every rank's slice as one key (monotone value << 32 |
// ~global index): the largest key is the largest value, then the smallest
// index -- the first maximum of the whole row, as np.argmax picks it
// (ref_qwen3.py:447-464).  One CTA, thread i = sequence i.
__global__ void __launch_bounds__(64) k_tp_argmax_exchange(TpArgmaxArgs a) {
  const int i = threadIdx.x;
  if (i < a.B) {
    const float v = __fadd_rn(a.best[i], 0.0f);
    const unsigned b = __float_as_uint(v);
    const unsigned key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    const unsigned long long k = (static_cast<unsigned long long>(key) << 32) |
                                 (0xffffffffu - (static_cast<unsigned>(a.bidx[i]) + a.v0));
    for (int q = 0; q < a.world; ++q) a.keys_dst[q][a.me * a.max_seqs + i] = k;
  }
  __syncthreads();   // every store before thread 0's system-scope release
  if (i == 0)
    for (int q = 0; q < a.world; ++q) sys_signal(a.sig_dst[q]);
  if (i < a.world) {
    const unsigned target = a.expect[i] + 1u;
    if (!wait_count(a.sig + i, target, a.wait_ns)) atomicOr(&g_tp_error, kErrTpWait);
    a.expect[i] = target;
  }
  __syncthreads();
  if (i < a.B) {
    unsigned long long best = 0ull;
    for (int q = 0; q < a.world; ++q) {
      const unsigned long long k = __ldcg(a.keys + q * a.max_seqs + i);
      best = k > best ? k : best;
    }
    a.next_ids[i] = static_cast<int32_t>(0xffffffffu - static_cast<unsigned>(best & 0xffffffffu));
  }
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

__global__ void k_tp_expect_add(unsigned *expect, unsigned count) { *expect += count; }

// out[m][t] = ((0 + recv[0][m][t]) + recv[1][m][t]) + ... (slot order)
__global__ void k_tp_sum_slots(const float *recv, int slots, int B, int H, float *out) {
  const size_t n = static_cast<size_t>(B) * H;
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    float acc = 0.0f;
    for (int sl = 0; sl < slots; ++sl) acc = __fadd_rn(acc, __ldcg(recv + sl * n + i));
    out[i] = acc;
  }
}

// ---- NCCL, loaded at run time from the process (the copy torch loaded), so
// the library itself does not depend on it.  Only the comparison variant uses it.
struct NcclUid { char internal[128]; };
using NcclGetUid = int (*)(NcclUid *);
using NcclInit = int (*)(void **, int, NcclUid, int);
using NcclAllReduce = int (*)(const void *, void *, size_t, int, int, void *, cudaStream_t);
using NcclDestroy = int (*)(void *);
constexpr int kNcclFloat32 = 7, kNcclSum = 0;
struct NcclApi {
  NcclGetUid get_uid = nullptr;
  NcclInit init = nullptr;
  NcclAllReduce all_reduce = nullptr;
  NcclDestroy destroy = nullptr;
};
const NcclApi *nccl_api() {
  static NcclApi api;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW);
    if (h) {
      api.get_uid = reinterpret_cast<NcclGetUid>(dlsym(h, "ncclGetUniqueId"));
      api.init = reinterpret_cast<NcclInit>(dlsym(h, "ncclCommInitRank"));
      api.all_reduce = reinterpret_cast<NcclAllReduce>(dlsym(h, "ncclAllReduce"));
      api.destroy = reinterpret_cast<NcclDestroy>(dlsym(h, "ncclCommDestroy"));
    }
  }
  return (api.get_uid && api.init && api.all_reduce && api.destroy) ? &api : nullptr;
}

// ---- prefill exchanges
struct PfPushArgs {
  const char *src;                  // this rank's region
  char *dst[kTpMaxRanks];           // every rank's region as mapped here
  unsigned *sig[kTpMaxRanks];       // rank q's counter of (exchange, this rank)
  PfSeg seg[2];
  int nseg, world, me;
  uint32_t rows;
};

// rows are spread over the CTAs; a row's segment goes to every other rank in
// 16-byte words when the segment allows it, else in 4-byte words.  Each CTA
// then fences its stores at system scope, passes a barrier, and one thread
// adds 1 (release, system scope) to this rank's counter at every rank.
__global__ void __launch_bounds__(256) k_pf_push(PfPushArgs a) {
  for (int si = 0; si < a.nseg; ++si) {
    const PfSeg sg = a.seg[si];
    const bool v16 = (sg.offset % 16 == 0) && (sg.width % 16 == 0) && (sg.row_bytes % 16 == 0) &&
                     (sg.base % 16 == 0);
    const uint32_t words = v16 ? sg.width / 16 : sg.width / 4;
    const size_t total = static_cast<size_t>(a.rows) * words;
    for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<size_t>(gridDim.x) * blockDim.x) {
      const size_t r = i / words, w = i % words;
      const size_t off = sg.base + r * sg.row_bytes + sg.offset + w * (v16 ? 16 : 4);
      if (v16) {
        const int4 v = __ldcg(reinterpret_cast<const int4 *>(a.src + off));
        for (int q = 0; q < a.world; ++q)
          if (q != a.me) *reinterpret_cast<int4 *>(a.dst[q] + off) = v;
      } else {
        const int v = __ldcg(reinterpret_cast<const int *>(a.src + off));
        for (int q = 0; q < a.world; ++q)
          if (q != a.me) *reinterpret_cast<int *>(a.dst[q] + off) = v;
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int q = 0; q < a.world; ++q) sys_signal(a.sig[q]);
}

__global__ void k_pf_wait(const unsigned *sig, int world, unsigned target, unsigned long long wait_ns) {
  const int q = threadIdx.x;
  if (q < world && !wait_count(sig + q, target, wait_ns)) atomicOr(&g_tp_error, kErrTpWait);
}

struct PfKeyArgs {
  const float *best;
  int32_t *idx;                                // in: local index; out: the greedy id
  uint32_t v0;
  int B, world, me, max_seqs;
  unsigned long long *keys_dst[kTpMaxRanks];   // rank q's key buffer [ranks][max_seqs]
  unsigned *sig_dst[kTpMaxRanks];              // rank q's counter of (PF_KEYS, me)
  const unsigned long long *keys;              // this rank's key buffer
  const unsigned *sig;                         // this rank's counters of PF_KEYS
  unsigned target;
  unsigned long long wait_ns;
};

// (max, first index) of every rank's vocabulary slice as one key (monotone
// value << 32 | ~global index): the largest key is the first maximum of the
// whole row, as np.argmax picks it (ref_qwen3.py:447-464).  One CTA, thread i =
// sequence i.
__global__ void __launch_bounds__(256) k_pf_argmax_exchange(PfKeyArgs a) {
  const int i = threadIdx.x;
  if (i < a.B) {
    const float v = __fadd_rn(a.best[i], 0.0f);
    const unsigned b = __float_as_uint(v);
    const unsigned key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    const unsigned long long k = (static_cast<unsigned long long>(key) << 32) |
                                 (0xffffffffu - (static_cast<unsigned>(a.idx[i]) + a.v0));
    for (int q = 0; q < a.world; ++q) a.keys_dst[q][a.me * a.max_seqs + i] = k;
  }
  __threadfence_system();
  __syncthreads();
  if (i == 0)
    for (int q = 0; q < a.world; ++q) sys_signal(a.sig_dst[q]);
  if (i < a.world && !wait_count(a.sig + i, a.target, a.wait_ns)) atomicOr(&g_tp_error, kErrTpWait);
  __syncthreads();
  if (i < a.B) {
    unsigned long long best = 0ull;
    for (int q = 0; q < a.world; ++q) {
      const unsigned long long k = __ldcg(a.keys + q * a.max_seqs + i);
      best = k > best ? k : best;
    }
    a.idx[i] = static_cast<int32_t>(0xffffffffu - static_cast<unsigned>(best & 0xffffffffu));
  }
}

}  // namespace

unsigned *pf_sig(const PfComm &c, int q, int ex, int producer) {
  return reinterpret_cast<unsigned *>(c.peer[q] + c.off_sig) + ex * kTpMaxRanks + producer;
}

int pf_push(PfComm &c, int ex, const PfSeg *segs, int nseg, uint32_t rows, cudaStream_t s) {
  if (nseg < 1 || nseg > 2) return Q3_ERR_SHAPE;
  PfPushArgs a{};
  a.src = c.local;
  for (int q = 0; q < c.world; ++q) {
    a.dst[q] = c.peer[q];
    a.sig[q] = pf_sig(c, q, ex, c.rank);
  }
  for (int i = 0; i < nseg; ++i) {
    if (segs[i].width % 4 || segs[i].offset % 4 || segs[i].row_bytes % 4 || segs[i].base % 4)
      return Q3_ERR_ALIGN;
    a.seg[i] = segs[i];
  }
  a.nseg = nseg;
  a.world = c.world;
  a.me = c.rank;
  a.rows = rows;
  c.gen[ex] += 1;
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  k_pf_push<<<kPfPushCtas, 256, 0, s>>>(a);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

int pf_wait(const PfComm &c, int ex, cudaStream_t s) {
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  k_pf_wait<<<1, 32, 0, s>>>(pf_sig(c, c.rank, ex, 0), c.world, c.gen[ex] * kPfPushCtas, c.wait_ns);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

int pf_argmax_exchange(PfComm &c, const float *best, int32_t *idx, uint32_t v0, int B, cudaStream_t s) {
  if (B < 1 || B > 256 || static_cast<uint32_t>(B) > c.max_seqs) return Q3_ERR_SHAPE;
  PfKeyArgs a{};
  a.best = best;
  a.idx = idx;
  a.v0 = v0;
  a.B = B;
  a.world = c.world;
  a.me = c.rank;
  a.max_seqs = static_cast<int>(c.max_seqs);
  for (int q = 0; q < c.world; ++q) {
    a.keys_dst[q] = reinterpret_cast<unsigned long long *>(c.peer[q] + c.off_keys);
    a.sig_dst[q] = pf_sig(c, q, PF_KEYS, c.rank);
  }
  a.keys = reinterpret_cast<const unsigned long long *>(c.local + c.off_keys);
  a.sig = pf_sig(c, c.rank, PF_KEYS, 0);
  c.gen[PF_KEYS] += 1;
  a.target = c.gen[PF_KEYS];
  a.wait_ns = c.wait_ns;
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  k_pf_argmax_exchange<<<1, 256, 0, s>>>(a);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

int tp_nccl_reduce(const TpComm &c, const float *recv, int slots, int B, int H, float *out,
                   cudaStream_t s) {
  const NcclApi *api = nccl_api();
  if (!api || !c.nccl) return Q3_ERR_NULL;
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  k_tp_sum_slots<<<64, 256, 0, s>>>(recv, slots, B, H, out);
  int st = q3h::launch_status();
  if (st == Q3_OK && api->all_reduce(out, out, static_cast<size_t>(B) * H, kNcclFloat32, kNcclSum,
                                     c.nccl, s) != 0) {
    q3h::set_error_message("ncclAllReduce failed");
    st = Q3_ERR_CUDA;
  }
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

int tp_reduce_norm(const TpReduceArgs &a, cudaStream_t s) {
  // world 0: the partials are already complete (no counters to wait for)
  if (a.H != 1024 || a.B < 1 || a.slots < 1 || a.slots > kTpMaxSlots || a.world < 0 ||
      a.world > kTpMaxRanks)
    return Q3_ERR_SHAPE;
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  const int st = q3h::launch_ex(true, k_tp_reduce_norm, dim3(a.B), dim3(1024), 0, s, a);
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

int tp_argmax_exchange(const TpComm &c, const float *best, const int32_t *bidx, uint32_t v0,
                       int B, int32_t *next_ids, cudaStream_t s) {
  if (B < 1 || B > 64 || static_cast<uint32_t>(B) > c.max_seqs) return Q3_ERR_SHAPE;
  TpArgmaxArgs a{};
  a.best = best;
  a.bidx = bidx;
  a.v0 = v0;
  a.B = B;
  a.world = c.world;
  a.me = c.rank;
  a.max_seqs = static_cast<int>(c.max_seqs);
  for (int q = 0; q < c.world; ++q) {
    a.keys_dst[q] = reinterpret_cast<unsigned long long *>(c.peer[q] + c.off_keys);
    a.sig_dst[q] = tp_sig(c, q, TP_KEYS, c.rank);
  }
  a.keys = reinterpret_cast<const unsigned long long *>(c.local + c.off_keys);
  a.sig = tp_sig(c, c.rank, TP_KEYS, 0);
  a.expect = tp_expect(c, TP_KEYS);
  a.next_ids = next_ids;
  a.wait_ns = c.wait_ns;
  q3h::timer_begin(q3h::TIMER_EXCHANGE, s);
  k_tp_argmax_exchange<<<1, 64, 0, s>>>(a);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_EXCHANGE, s);
  return st;
}

}  // namespace q3

using q3::TpComm;

extern "C" int q3_tp_shard_of(const q3_layout *L, int32_t rank, int32_t world, q3_tp_shard *out) {
  if (!L || !out) return Q3_ERR_NULL;
  if (world < 1 || world > q3::kTpMaxRanks || rank < 0 || rank >= world) return Q3_ERR_SHAPE;
  if (L->kv_heads == 0 || L->kv_heads % world || L->heads != 2 * L->kv_heads || L->inter % 256 ||
      L->vocab % 128)
    return Q3_ERR_SHAPE;
  const uint32_t G = L->inter / 256, T = L->vocab / 128, w = static_cast<uint32_t>(world),
                 r = static_cast<uint32_t>(rank);
  if (G < w || T < w) return Q3_ERR_SHAPE;
  q3_tp_shard s{};
  s.rank = rank;
  s.world = world;
  s.kv_heads = L->kv_heads / w;
  s.kv_head0 = r * s.kv_heads;
  s.q_heads = 2 * s.kv_heads;
  s.q_head0 = 2 * s.kv_head0;
  s.mlp_group0 = r * G / w;
  s.mlp_groups = (r + 1) * G / w - s.mlp_group0;
  const uint32_t t0 = r * T / w, t1 = (r + 1) * T / w;
  s.vocab0 = t0 * 128;
  s.vocab_rows = (t1 - t0) * 128;
  *out = s;
  return Q3_OK;
}

extern "C" size_t q3_tp_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" int q3_tp_comm_create(const q3_layout *L, int32_t rank, int32_t world,
                                 uint32_t max_seqs, void **comm, void *handle) {
  if (!L || !comm || !handle) return Q3_ERR_NULL;
  *comm = nullptr;
  if (max_seqs < 1 || max_seqs > 64 || L->hidden != 1024 || L->head_dim != 128 ||
      L->heads > static_cast<uint32_t>(q3::kTpMaxSlots) ||
      L->inter / 256 > static_cast<uint32_t>(q3::kTpMaxSlots))
    return Q3_ERR_SHAPE;
  TpComm *c = new (std::nothrow) TpComm{};
  if (!c) return Q3_ERR_CAPACITY;
  for (int q = 0; q < world && q < q3::kTpMaxRanks; ++q) {
    const int st = q3_tp_shard_of(L, q, world, &c->shard[q]);
    if (st != Q3_OK) {
      delete c;
      return st;
    }
  }
  if (world < 1 || world > q3::kTpMaxRanks || rank < 0 || rank >= world) {
    delete c;
    return Q3_ERR_SHAPE;
  }
  c->rank = rank;
  c->world = world;
  c->wait_ns = q3::kTpDefaultWaitNs;
  c->max_seqs = max_seqs;
  c->hidden = L->hidden;
  c->heads = L->heads;
  c->mlp_groups = L->inter / 256;
  const size_t slot = static_cast<size_t>(max_seqs) * L->hidden * 4;
  c->off_sig = 0;
  c->off_expect = 256;
  c->off_orecv = 512;
  c->off_drecv = q3::align256(c->off_orecv + c->heads * slot);
  c->off_keys = q3::align256(c->off_drecv + c->mlp_groups * slot);
  c->off_nccl = q3::align256(c->off_keys + static_cast<size_t>(q3::kTpMaxRanks) * max_seqs * 8);
  c->bytes = q3::align256(c->off_nccl + slot);
  cudaError_t e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  c->peer[rank] = c->local;
  *comm = c;
  return Q3_OK;
}

extern "C" int q3_tp_comm_connect(void *comm, const void *handles) {
  if (!comm || !handles) return Q3_ERR_NULL;
  TpComm *c = static_cast<TpComm *>(comm);
  const cudaIpcMemHandle_t *h = static_cast<const cudaIpcMemHandle_t *>(handles);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank || c->opened[q]) continue;
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      q3h::set_cuda_error(e);
      return Q3_ERR_CUDA;
    }
    c->peer[q] = static_cast<char *>(p);
    c->opened[q] = true;
  }
  return Q3_OK;
}

extern "C" int q3_tp_comm_reset(void *comm, void *stream) {
  if (!comm) return Q3_ERR_NULL;
  TpComm *c = static_cast<TpComm *>(comm);
  const cudaError_t e = cudaMemsetAsync(c->local, 0, c->off_orecv, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  return Q3_OK;
}

extern "C" int q3_tp_comm_set_wait_ns(void *comm, uint64_t ns) {
  if (!comm) return Q3_ERR_NULL;
  if (ns < 1000000ull || ns > 60000000000ull) return Q3_ERR_SHAPE;
  static_cast<TpComm *>(comm)->wait_ns = ns;
  return Q3_OK;
}

extern "C" int q3_tp_comm_inject_missing_signals(void *comm, int32_t buf, int32_t producer,
                                                 uint32_t count, void *stream) {
  if (!comm) return Q3_ERR_NULL;
  TpComm *c = static_cast<TpComm *>(comm);
  if (buf < 0 || buf >= q3::TP_NBUF || producer < 0 || producer >= c->world || count == 0)
    return Q3_ERR_SHAPE;
  q3::k_tp_expect_add<<<1, 1, 0, static_cast<cudaStream_t>(stream)>>>(
      q3::tp_expect(*c, buf) + producer, count);
  return q3h::launch_status();
}

// ---- tensor-parallel prefill communicator
extern "C" int q3_tp_prefill_comm_create(const q3_layout *L, int32_t rank, int32_t world,
                                         uint32_t max_rows, uint32_t max_seqs, void **comm,
                                         void *handle) {
  if (!L || !comm || !handle) return Q3_ERR_NULL;
  *comm = nullptr;
  if (world < 1 || world > q3::kTpMaxRanks || rank < 0 || rank >= world) return Q3_ERR_SHAPE;
  if (max_rows < 1 || max_seqs < 1 || max_seqs > 256 || L->head_dim != 128 ||
      L->hidden % (128u * static_cast<uint32_t>(world)) || L->inter % 256)
    return Q3_ERR_SHAPE;
  q3::PfComm *c = new (std::nothrow) q3::PfComm{};
  if (!c) return Q3_ERR_CAPACITY;
  for (int q = 0; q < world; ++q) {
    const int st = q3_tp_shard_of(L, q, world, &c->shard[q]);
    if (st != Q3_OK) {
      delete c;
      return st;
    }
    c->cols[q] = L->hidden / static_cast<uint32_t>(world);
    c->col0[q] = static_cast<uint32_t>(q) * c->cols[q];
  }
  c->rank = rank;
  c->world = world;
  c->max_rows = max_rows;
  c->max_seqs = max_seqs;
  c->hidden = L->hidden;
  c->heads = L->heads;
  c->inter = L->inter;
  c->wait_ns = q3::kTpDefaultWaitNs;
  const size_t M = max_rows, QW = static_cast<size_t>(L->heads) * 128;
  size_t off = 4096;                                   // counters
  c->off_sig = 0;
  c->off_o8 = off;   off = q3::align256(off + M * QW);
  c->off_os = off;   off = q3::align256(off + M * L->heads * 4);
  c->off_x = off;    off = q3::align256(off + M * L->hidden * 4);
  c->off_s8 = off;   off = q3::align256(off + M * L->inter);
  c->off_ss = off;   off = q3::align256(off + M * (L->inter / 256) * 4);
  c->off_keys = off; off = q3::align256(off + static_cast<size_t>(q3::kTpMaxRanks) * max_seqs * 8);
  c->off_h8 = off;   off = q3::align256(off + M * L->hidden);
  c->off_bsum = off; off = q3::align256(off + M * (L->hidden / 32) * 4);
  c->off_amax = off; off = q3::align256(off + M * (L->hidden / 128) * 4);
  c->bytes = off;
  cudaError_t e = cudaMalloc(&c->local, c->bytes);
  if (e == cudaSuccess) e = cudaMemset(c->local, 0, 4096);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t *>(handle), c->local);
  if (e != cudaSuccess) {
    if (c->local) cudaFree(c->local);
    delete c;
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  c->peer[rank] = c->local;
  *comm = c;
  return Q3_OK;
}

extern "C" int q3_tp_prefill_comm_connect(void *comm, const void *handles) {
  if (!comm || !handles) return Q3_ERR_NULL;
  q3::PfComm *c = static_cast<q3::PfComm *>(comm);
  const cudaIpcMemHandle_t *h = static_cast<const cudaIpcMemHandle_t *>(handles);
  for (int q = 0; q < c->world; ++q) {
    if (q == c->rank || c->opened[q]) continue;
    void *p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h[q], cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      q3h::set_cuda_error(e);
      return Q3_ERR_CUDA;
    }
    c->peer[q] = static_cast<char *>(p);
    c->opened[q] = true;
  }
  return Q3_OK;
}

extern "C" int q3_tp_prefill_comm_reset(void *comm, void *stream) {
  if (!comm) return Q3_ERR_NULL;
  q3::PfComm *c = static_cast<q3::PfComm *>(comm);
  const cudaError_t e = cudaMemsetAsync(c->local, 0, 4096, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    q3h::set_cuda_error(e);
    return Q3_ERR_CUDA;
  }
  for (int i = 0; i < q3::PF_NEX; ++i) c->gen[i] = 0;
  return Q3_OK;
}

extern "C" int q3_tp_prefill_comm_set_wait_ns(void *comm, uint64_t ns) {
  if (!comm) return Q3_ERR_NULL;
  if (ns < 1000000ull || ns > 60000000000ull) return Q3_ERR_SHAPE;
  static_cast<q3::PfComm *>(comm)->wait_ns = ns;
  return Q3_OK;
}

extern "C" int q3_tp_prefill_comm_destroy(void *comm) {
  if (!comm) return Q3_OK;
  q3::PfComm *c = static_cast<q3::PfComm *>(comm);
  for (int q = 0; q < c->world; ++q)
    if (c->opened[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->local) cudaFree(c->local);
  delete c;
  return Q3_OK;
}

extern "C" int q3_tp_nccl_unique_id(void *out) {
  if (!out) return Q3_ERR_NULL;
  const q3::NcclApi *api = q3::nccl_api();
  if (!api) {
    q3h::set_error_message("libnccl.so.2 is not loadable in this process");
    return Q3_ERR_CUDA;
  }
  q3::NcclUid uid;
  if (api->get_uid(&uid) != 0) {
    q3h::set_error_message("ncclGetUniqueId failed");
    return Q3_ERR_CUDA;
  }
  memcpy(out, &uid, sizeof uid);
  return Q3_OK;
}

extern "C" int q3_tp_comm_set_reduction(void *comm, int32_t mode, const void *nccl_unique_id) {
  if (!comm) return Q3_ERR_NULL;
  TpComm *c = static_cast<TpComm *>(comm);
  if (mode == 0) {
    c->reduce_nccl = 0;
    return Q3_OK;
  }
  if (mode != 1) return Q3_ERR_MODE;
  if (!c->nccl) {
    if (!nccl_unique_id) return Q3_ERR_NULL;
    const q3::NcclApi *api = q3::nccl_api();
    if (!api) {
      q3h::set_error_message("libnccl.so.2 is not loadable in this process");
      return Q3_ERR_CUDA;
    }
    q3::NcclUid uid;
    memcpy(&uid, nccl_unique_id, sizeof uid);
    void *nc = nullptr;
    if (api->init(&nc, c->world, uid, c->rank) != 0 || !nc) {   // collective over the ranks
      q3h::set_error_message("ncclCommInitRank failed");
      return Q3_ERR_CUDA;
    }
    c->nccl = nc;
  }
  c->reduce_nccl = 1;
  return Q3_OK;
}

extern "C" int q3_tp_comm_destroy(void *comm) {
  if (!comm) return Q3_OK;
  TpComm *c = static_cast<TpComm *>(comm);
  if (c->nccl) {
    const q3::NcclApi *api = q3::nccl_api();
    if (api) api->destroy(c->nccl);
    c->nccl = nullptr;
  }
  for (int q = 0; q < c->world; ++q)
    if (c->opened[q]) cudaIpcCloseMemHandle(c->peer[q]);
  if (c->local) cudaFree(c->local);
  delete c;
  return Q3_OK;
}
