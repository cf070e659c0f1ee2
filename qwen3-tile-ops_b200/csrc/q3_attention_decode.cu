// Decode attention (one query row per sequence) over the paged int8 KV pool.
// Same arithmetic as kernels/attention_gqa.h:404-547 / tools/ref_qwen3.py:210-266,
// reorganised for the tensor cores:
//
// The reference walks 32-key blocks in order; block j uses the running maximum
// m_j = max(m_{j-1}, tree_max(s_j)), a prefix max of the block maxima, so the
// block's
//     corr_j = exp(m_{j-1} - m_j),  p_j = exp(s_j - m_j),  psum_j = tree_sum(p_j),
//     pq_j = quant(p_j * vs, pmax_j),  part_j = f32(int32(pq_j . V_j)) * pmax_j
// are known as soon as the maxima of blocks 0..j are, and only the two cheap
// recurrences
//     den_j = (den_{j-1} * corr_j) + psum_j,  res_j = (res_{j-1} * corr_j) + part_j
// run in block order, with exactly the reference's two roundings each.
//
// CTA = one (sequence, kv head); the two q heads of the GQA group share every
// K/V page.  Blocks go in groups of 4 pages (128 keys).  Warp roles:
//   warp 4    producer: cp.async of the K pages (ring of 2 groups) and the V
//             pages (ring of 1) into shared memory, rows in the tensor cores'
//             128-byte swizzle; completion is tracked by mbarriers
//             (cp.async.mbarrier.arrive), so nothing blocks on a copy group.
//   warp 5    MMA issuer (one lane): QK(g) = K tile (M = 128 keys, K = 128) x
//             the two q rows (N = 16) into one of two TMEM slots; PV(g) = V tile
//             read MN-major (M = 128 value columns, K = 128 keys) x pq, where row
//             2q+h of pq holds block q's requantised probabilities for head h in
//             block q's 32 keys and zeros elsewhere, so column 2q+h of the result
//             is block q's int32 P.V.  QK runs one group ahead of PV.
//   warps 0-3 softmax: warp w takes block w of each group (scale, mask, block
//             max, prefix max, corr, p, psum, pmax, pq); then, with thread
//             d = value column d, the recurrences of the previous group in order.
// All int32 products are exact, so the tensor cores change no bit.  Every
// wait is bounded (about one second); a timeout sets a bit of the device error
// word, the roles stop, copies and MMAs in flight are drained and TMEM freed.
#include <mutex>

#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_tc.cuh"

namespace q3 {

__device__ unsigned int g_device_error = 0;   // read by q3_device_status()

namespace dec {

using namespace tcx;

constexpr int NCW = 4;                  // softmax warps
// With two V slots (at most 3 CTAs per SM) the K and V pages come from two
// producer warps, so a K copy never queues behind a V slot that waits for the
// softmax (256 pairs: 38.9 against 42.1 us); with one V slot (4 CTAs per SM)
// one producer warp interleaves them (the seventh warp cost more than it gave).
template <int VS>
__host__ __device__ constexpr int threads_of() { return (NCW + (VS == 2 ? 3 : 2)) * 32; }
constexpr int PRODUCER = NCW, MMA_WARP = NCW + 1, VPRODUCER = NCW + 2;
constexpr int TAB_CACHE = 512;          // page-table entries kept in shared memory
constexpr int TMEM_COLS = 64;           // QK slots at 0 and 16, PV slots at 32 and 48
constexpr unsigned kErrPage = 2u;       // a page index >= num_pages (copy skipped)
constexpr unsigned kErrTable = 4u;      // kv_len needs more pages than the table holds
constexpr unsigned kErrWait = 8u;       // a pipeline wait timed out
constexpr uint32_t ID_QK = idesc_i8(16);          // A = keys (K-major), B = q rows
constexpr uint32_t ID_PV = idesc_i8(16, true);    // A = V (MN-major), B = pq rows

template <int VS>   // V ring slots: 1, or 2 when fewer CTAs share an SM
struct Smem {
  alignas(1024) int8_t kbuf[2][4][4096];  // K pages of a group, 128-byte swizzled rows
  alignas(1024) int8_t vbuf[VS][4][4096]; // V pages of a group
  // B operands, 8 rows each; rows 8..15 of N = 16 alias rows 0..7 (stride offset 0)
  alignas(1024) int8_t qt[1024];          // 128-byte swizzled: rows 0,1 = q heads
  alignas(1024) int8_t pq[2][1024];       // no swizzle: [16-key chunk][8 rows][16 B]
  uint16_t tab[TAB_CACHE];                // this sequence's page table (first TAB_CACHE entries)
  float bm[2][NCW][2];                    // block maxima
  alignas(16) float corr[2][2][4];        // [slot][head][block]
  alignas(16) float psum[2][2][4];
  alignas(16) float pmax[2][2][4];
  float red[NCW][2];
  unsigned long long kfull[2], kempty[2], vfull[VS], vempty[VS];
  unsigned long long qk_done[2], pv_done[2], pq_ready[2], bm_ready[2], mma_final;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src)
               : "memory");
}
// arrive on `b` once every cp.async this thread issued so far has landed
__device__ __forceinline__ void cp_arrive(unsigned long long *b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void softmax_sync() {   // the 4 softmax warps only
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}
template <class S>
__device__ __forceinline__ bool wait_or_abort(unsigned long long *b, uint32_t par, S &sm) {
  if (mbar_wait(b, par, &sm.abort)) return true;
  if (!*reinterpret_cast<volatile int *>(&sm.abort)) atomicOr(&g_device_error, kErrWait);
  *reinterpret_cast<volatile int *>(&sm.abort) = 1;
  return false;
}

template <class S>
__device__ __forceinline__ uint32_t page_of(const S &sm, const uint16_t *table, int j) {
  return j < TAB_CACHE ? sm.tab[j] : table[j];
}

template <int VS>
__global__ void __launch_bounds__(threads_of<VS>(), VS == 1 ? 4 : 3)
    k_attention_decode(const char *__restrict__ kpool, const char *__restrict__ vpool,
                       DecodeAttnArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem<VS> &sm = *reinterpret_cast<Smem<VS> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int kvh = blockIdx.x, seq = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  pdl_trigger();
  pdl_wait();       // q, the new K/V rows and kv_len come from earlier kernels
  const int kv_len = p.kv_len[seq];
  const int nb = (kv_len + 31) >> 5;
  const uint16_t *table = p.table + static_cast<long>(seq) * p.table_stride;
  if (kv_len <= 0 || nb > p.table_stride) {        // uniform for the whole CTA
    if (tid == 0) atomicOr(&g_device_error, kErrTable);
    return;
  }
  const int G = (nb + 3) >> 2;                     // groups of 4 blocks

  // ---- set-up: B operands (zero except the rows written later), barriers, TMEM
  constexpr int THREADS = threads_of<VS>();
  for (int i = tid * 4; i < 1024; i += THREADS * 4) {
    if (i >= 256) *reinterpret_cast<int *>(sm.qt + i) = 0;
    *reinterpret_cast<int *>(sm.pq[0] + i) = 0;
    *reinterpret_cast<int *>(sm.pq[1] + i) = 0;
  }
  for (int i = tid; i < nb && i < TAB_CACHE; i += THREADS) sm.tab[i] = table[i];
  if (tid < 64) {                                  // q rows of the two heads
    const int hh = tid >> 5, h = kvh * 2 + hh;
    const int v = reinterpret_cast<const int *>(p.q8 + static_cast<long>(seq) * p.q_rb + h * 128)[lane];
    *reinterpret_cast<int *>(sm.qt + hh * 128 + (((lane >> 2) ^ hh) << 4) + (lane & 3) * 4) = v;
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kfull[i], 32);
      mbar_init(&sm.kempty[i], 1);
      mbar_init(&sm.qk_done[i], 1);
      mbar_init(&sm.pv_done[i], 1);
      mbar_init(&sm.pq_ready[i], NCW * 32);
      mbar_init(&sm.bm_ready[i], NCW);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&sm.vfull[i], 32);
      mbar_init(&sm.vempty[i], 1);
    }
    mbar_init(&sm.mma_final, 1);
    sm.abort = 0;
    mbar_init_fence();
  }
  fence_proxy_async();                             // qt / pq stores -> tensor cores
  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  float den[2] = {0.0f, 0.0f}, res[2] = {0.0f, 0.0f};   // softmax threads: value column tid

  if (warp == PRODUCER || (VS == 2 && warp == VPRODUCER)) {
    // ---- producers.  Two V slots: K(0), K(1), ... through the 2-slot K ring
    // (this warp) and V(0), V(1), ... through the V slots (the other producer
    // warp).  One V slot: one warp issues K(0), K(1), V(0), K(2), V(1), ...,
    // K(G-1), V(G-2), V(G-1).
    const int r4 = lane >> 3, c16 = lane & 7;     // lane: 16-byte chunk c16 of rows 4i + r4
    const int n_it = VS == 2 ? G : 2 * G;
    for (int it = 0; it < n_it; ++it) {
      int g, isv;
      if (VS == 2) {
        g = it;
        isv = warp == VPRODUCER;
      } else if (it == 0) {
        g = 0; isv = 0;
      } else if (it == 2 * G - 1) {
        g = G - 1; isv = 1;
      } else {                                    // it odd -> K((it+1)/2), it even -> V(it/2 - 1)
        g = (it + 1) >> 1; isv = !(it & 1); if (isv) g -= 1;
      }
      const char *pool = isv ? vpool : kpool;
      unsigned long long *full;
      int8_t(*dst)[4096];
      if (!isv) {
        const int slot = g & 1;
        if (g >= 2 && !wait_or_abort(&sm.kempty[slot], ((g >> 1) - 1) & 1, sm)) break;
        full = &sm.kfull[slot];
        dst = sm.kbuf[slot];
      } else {
        const int vslot = g % VS;
        if (g >= VS && !wait_or_abort(&sm.vempty[vslot], ((g / VS) - 1) & 1, sm)) break;
        full = &sm.vfull[vslot];
        dst = sm.vbuf[vslot];
      }
      const int first = 4 * g, count = min(4, nb - first);
      for (int q = 0; q < count; ++q) {
        const uint32_t page = page_of(sm, table, first + q);
        if (page >= p.num_pages) {
          if (lane == 0) atomicOr(&g_device_error, kErrPage);
          continue;
        }
        const char *src = pool + static_cast<size_t>(page) * p.page_bytes + kvh * 128 + c16 * 16;
#pragma unroll
        for (int i = 0; i < 8; ++i) {              // 4 whole rows per instruction
          const int row = 4 * i + r4;
          cp_async16(dst[q] + row * 128 + ((c16 ^ (row & 7)) << 4), src + static_cast<size_t>(row) * p.row_bytes);
        }
      }
      cp_arrive(full);
    }
    cp_wait_all();
  } else if (warp == MMA_WARP) {
    // ---- MMA issuer: QK(0), then per g: QK(g+1), PV(g)
    if (lane == 0) {
      const uint32_t bq = su32(sm.qt);
      bool ok = true;
      auto issue_qk = [&](int g) -> bool {
        const int slot = g & 1;
        if (!wait_or_abort(&sm.kfull[slot], (g >> 1) & 1, sm)) return false;
        fence_after();
        const uint32_t a0 = su32(sm.kbuf[slot][0]);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_i8(tmem + 16 * slot, sdesc_sw128(a0 + ks * 32), sdesc_sw128(bq + ks * 32, 0), ID_QK,
                 ks != 0);
        mma_commit(&sm.qk_done[slot]);
        mma_commit(&sm.kempty[slot]);
        return true;
      };
      ok = issue_qk(0);
      for (int g = 0; g < G && ok; ++g) {
        if (g + 1 < G && !(ok = issue_qk(g + 1))) break;
        const int slot = g & 1;
        if (!(ok = wait_or_abort(&sm.vfull[g % VS], (g / VS) & 1, sm))) break;
        if (!(ok = wait_or_abort(&sm.pq_ready[slot], (g >> 1) & 1, sm))) break;
        fence_after();
        const int count = min(4, nb - 4 * g);
        const uint32_t a0 = su32(sm.vbuf[g % VS][0]), b0 = su32(sm.pq[slot]);
        for (int q = 0; q < count; ++q)          // k-step q = block q's 32 keys
          mma_i8(tmem + 32 + 16 * slot, sdesc_sw128(a0 + q * 4096), sdesc_plain(b0 + q * 256, 128, 0),
                 ID_PV, q != 0);
        mma_commit(&sm.pv_done[slot]);
        mma_commit(&sm.vempty[g % VS]);
      }
      mma_commit(&sm.mma_final);                   // every MMA issued above has completed
      mbar_wait(&sm.mma_final, 0, nullptr);        // bounded
    }
    __syncwarp();
  } else {
    // ---- softmax warps
    const float qs0 = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8);
    const float qs1 = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8 + 4);
    const float qk_scale = p.qk_scale;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    float carry0 = kNegFltMax, carry1 = kNegFltMax;
    // scales of block (g, warp), loaded one group ahead
    auto load_scales = [&](int g, float &ks, float &vs) {
      const int j = 4 * g + warp, t = j * 32 + lane;
      ks = vs = 0.0f;
      if (j < nb && t < kv_len) {
        const uint32_t page = page_of(sm, table, j);
        if (page < p.num_pages) {
          const size_t o = static_cast<size_t>(page) * p.scale_page_bytes +
                           static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4;
          ks = *reinterpret_cast<const float *>(p.ks + o);
          vs = *reinterpret_cast<const float *>(p.vs + o);
        }
      }
    };
    auto recur = [&](int g) -> bool {
      const int slot = g & 1, count = min(4, nb - 4 * g);
      if (!wait_or_abort(&sm.pv_done[slot], (g >> 1) & 1, sm)) return false;
      fence_after();
      int v[8];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                     "=r"(v[6]), "=r"(v[7])
                   : "r"(lane_base + 32 + 16 * slot));
      tmem_wait_ld();
      float cv[2][4], sv[2][4], mv[2][4];   // the block terms, one vector load each
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        *reinterpret_cast<float4 *>(cv[h]) = *reinterpret_cast<const float4 *>(sm.corr[slot][h]);
        *reinterpret_cast<float4 *>(sv[h]) = *reinterpret_cast<const float4 *>(sm.psum[slot][h]);
        *reinterpret_cast<float4 *>(mv[h]) = *reinterpret_cast<const float4 *>(sm.pmax[slot][h]);
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < count) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            den[h] = __fadd_rn(__fmul_rn(den[h], cv[h][q]), sv[h][q]);
            res[h] = __fadd_rn(__fmul_rn(res[h], cv[h][q]),
                               __fmul_rn(i2f_small(v[2 * q + h]), mv[h][q]));
          }
        }
      }
      return true;
    };
    float ks_n, vs_n;
    load_scales(0, ks_n, vs_n);
    bool ok = true;
    for (int g = 0; g < G && ok; ++g) {
      const int slot = g & 1, count = min(4, nb - 4 * g);
      const int j = 4 * g + warp, t = j * 32 + lane;
      const float ks = ks_n, vs = vs_n;
      if (g + 1 < G) load_scales(g + 1, ks_n, vs_n);
      if (!(ok = wait_or_abort(&sm.qk_done[slot], (g >> 1) & 1, sm))) break;
      fence_after();
      float s0 = kNegInf, s1 = kNegInf;
      if (warp < count) {
        int a0, a1;
        tmem_ld2(lane_base + 16 * slot, a0, a1);
        tmem_wait_ld();
        if (t < kv_len) {                          // decode: the row sees keys 0..kv_len-1
          s0 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a0), ks), qs0), qk_scale);
          s1 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a1), ks), qs1), qk_scale);
        }
        const float b0 = warp_tree_max(s0), b1 = warp_tree_max(s1);
        if (lane == 0) { sm.bm[slot][warp][0] = b0; sm.bm[slot][warp][1] = b1; }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.bm_ready[slot]);
      if (!(ok = wait_or_abort(&sm.bm_ready[slot], (g >> 1) & 1, sm))) break;
      float mp0 = carry0, mp1 = carry1;            // running max before block j
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        if (w < count) {
          const float c0 = sm.bm[slot][w][0], c1 = sm.bm[slot][w][1];
          if (w < warp) { mp0 = fmaxf(mp0, c0); mp1 = fmaxf(mp1, c1); }
          carry0 = fmaxf(carry0, c0);
          carry1 = fmaxf(carry1, c1);
        }
      }
      if (warp < count) {
        const float mj0 = fmaxf(mp0, sm.bm[slot][warp][0]), mj1 = fmaxf(mp1, sm.bm[slot][warp][1]);
        // lane 0: corr of head 0, lane 1: corr of head 1
        // exp(m_prev - m_new) is exp(0) = 1 exactly when the running maximum of
        // both heads stayed (the common case after the first blocks)
        const float cx = (mp0 == mj0 && mp1 == mj1)
                             ? 1.0f
                             : exp_ref(lane == 1 ? __fsub_rn(mp1, mj1) : __fsub_rn(mp0, mj0));
        float prv[2] = {__fsub_rn(s0, mj0), __fsub_rn(s1, mj1)};   // both heads' p in one batch
        exp_ref_fast_n<2, true>(prv, g_exp2_t256);   // s - m_j <= 0
        const float pr0 = prv[0], pr1 = prv[1];
        const float ps0 = warp_tree_sum(pr0), ps1 = warp_tree_sum(pr1);
        const float pv0 = (t < kv_len) ? __fmul_rn(pr0, vs) : 0.0f;
        const float pv1 = (t < kv_len) ? __fmul_rn(pr1, vs) : 0.0f;
        const float pm0 = __fmul_rn(warp_tree_max(fabsf(pv0)), kInv127);
        const float pm1 = __fmul_rn(warp_tree_max(fabsf(pv1)), kInv127);
        // row 2w+h, keys of block w = 16-key chunks 2w and 2w+1
        int8_t *dst = sm.pq[slot] + (2 * warp + (lane >> 4)) * 128 + 2 * warp * 16 + (lane & 15);
        dst[0] = static_cast<int8_t>(quant1(pv0, pm0));
        dst[16] = static_cast<int8_t>(quant1(pv1, pm1));
        if (lane < 2) sm.corr[slot][lane][warp] = cx;
        if (lane == 0) {
          sm.psum[slot][0][warp] = ps0; sm.psum[slot][1][warp] = ps1;
          sm.pmax[slot][0][warp] = pm0; sm.pmax[slot][1][warp] = pm1;
        }
      }
      fence_proxy_async();                         // pq stores -> tensor cores
      fence_before();                              // QK slot reads done
      mbar_arrive(&sm.pq_ready[slot]);
      if (g >= 1 && !(ok = recur(g - 1))) break;
      fence_before();
    }
    if (ok) ok = recur(G - 1);
    fence_before();
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
  if (*reinterpret_cast<volatile int *>(&sm.abort) || warp >= NCW) return;

  // ---- 1/den, per-head output quantisation (attention_gqa.h:522-546)
  float o[2], mx[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    o[h] = __fmul_rn(res[h], __frcp_rn(den[h]));
    mx[h] = warp_tree_max(fabsf(o[h]));
  }
  if (lane == 0) { sm.red[warp][0] = mx[0]; sm.red[warp][1] = mx[1]; }
  softmax_sync();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float hm = 0.0f;
#pragma unroll
    for (int w = 0; w < NCW; ++w) hm = fmaxf(hm, sm.red[w][h]);
    const float scale = __fmul_rn(hm, kInv127);
    const int hd = kvh * 2 + h;
    p.o8[static_cast<long>(seq) * p.o_rb + hd * 128 + tid] = static_cast<char>(quant1(o[h], scale));
    if (tid == 0) *reinterpret_cast<float *>(p.os + static_cast<long>(seq) * p.os_rb + hd * 4) = scale;
  }
}

}  // namespace dec

// ---------------------------------------------------------------- host side
// The split form's CTAs each stream at most 4 key groups in two phases (K,
// then V) and hand the recurrence state down the cluster; measured on one B200
// at 2112 keys it wins only while the pairs cannot fill the GPU: 64 pairs
// 27.6 us against 36.8 for the single-CTA kernel, 128 pairs 48 against 37.
constexpr long kSplitMaxPairs = 96;

int attention_decode_split_cluster(uint32_t max_pages);
int attention_decode_split_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                                  uint32_t num_pages, int kv_heads, int n_seqs, int cluster,
                                  cudaStream_t s, bool pdl);

template <int VS>
static size_t smem_of() { return sizeof(dec::Smem<VS>) + 1024; }   // + alignment slack
// 4 (one V slot) or 3 (two) CTAs per SM: 228 KB of shared memory, 1 KB of it
// reserved per CTA
static_assert(sizeof(dec::Smem<1>) + 1024 <= 228 * 1024 / 4 - 1024, "4 CTAs per SM");
static_assert(sizeof(dec::Smem<2>) + 1024 <= 228 * 1024 / 3 - 1024, "3 CTAs per SM");

template <int VS>
static int launch_decode(bool pdl, dim3 grid, size_t smem, cudaStream_t s, const void *k_pool,
                         const void *v_pool, const DecodeAttnArgs &a) {
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(dec::k_attention_decode<VS>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr_err != cudaSuccess) {
    q3h::set_cuda_error(attr_err);
    return Q3_ERR_CUDA;
  }
  return q3h::launch_ex(pdl, dec::k_attention_decode<VS>, grid, dim3(dec::threads_of<VS>()), smem, s,
                        static_cast<const char *>(k_pool), static_cast<const char *>(v_pool), a);
}

int attention_decode_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                            uint32_t num_pages, int kv_heads, int n_seqs, cudaStream_t s, bool pdl) {
  // few pairs (tensor parallelism, small batches): split each pair's key range
  // over a cluster (q3_attention_decode_split.cu)
  if (static_cast<long>(n_seqs) * kv_heads <= kSplitMaxPairs) {
    const int cl = attention_decode_split_cluster(static_cast<uint32_t>(p.table_stride));
    if (cl > 1)
      return attention_decode_split_launch(p, k_pool, v_pool, num_pages, kv_heads, n_seqs, cl, s, pdl);
  }
  if (p.row_bytes % 16 || p.page_bytes % 16 || reinterpret_cast<uintptr_t>(k_pool) % 16 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16)
    return Q3_ERR_ALIGN;
  DecodeAttnArgs a = p;
  a.num_pages = num_pages;
  dim3 grid(kv_heads, n_seqs);
  // with at most 3 CTAs per SM (pairs <= 3 x SMs) a CTA has room for a second
  // V slot: the V copy of group g+1 then runs while the P.V of group g waits
  const bool two_v = static_cast<long>(n_seqs) * kv_heads <= 3L * q3h::sm_count();
  q3h::timer_begin(q3h::TIMER_ATTENTION, s);
  const int st = two_v ? launch_decode<2>(pdl, grid, smem_of<2>(), s, k_pool, v_pool, a)
                       : launch_decode<1>(pdl, grid, smem_of<1>(), s, k_pool, v_pool, a);
  q3h::timer_end(q3h::TIMER_ATTENTION, s);
  return st;
}

}  // namespace q3

namespace q3 {
int gemm_device_status_take();
int gemm2_device_status_take();
int dgemm_device_status_take();
int pattn_device_status_take();
int tp_device_status_take();
int dsplit_device_status_take();
}

extern "C" int q3_device_status(void) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q3::g_device_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q3::g_device_error, &zero, sizeof zero);
  const int g = q3::gemm_device_status_take();
  if (g < 0) return -1;
  const int g2 = q3::gemm2_device_status_take();
  if (g2 < 0) return -1;
  v |= static_cast<unsigned int>(g2);
  const int dg = q3::dgemm_device_status_take();
  if (dg < 0) return -1;
  v |= static_cast<unsigned int>(dg);
  const int pa = q3::pattn_device_status_take();
  if (pa < 0) return -1;
  v |= static_cast<unsigned int>(pa);
  const int tp = q3::tp_device_status_take();
  if (tp < 0) return -1;
  v |= static_cast<unsigned int>(tp);
  const int ds = q3::dsplit_device_status_take();
  if (ds < 0) return -1;
  v |= static_cast<unsigned int>(ds);
  return static_cast<int>(v) | g;
}
