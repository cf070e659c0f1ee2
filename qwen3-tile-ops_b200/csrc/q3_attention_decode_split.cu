// Decode attention with the key range of one (sequence, kv head) split over
// the CTAs of a thread-block cluster, bit-identical to k_attention_decode
// (kernels/attention_gqa.h:404-547 / tools/ref_qwen3.py:210-266).
//
// k_attention_decode walks a sequence's ~66 key blocks in one CTA; with few
// (sequence, head) pairs per GPU (tensor parallelism, small batches) that
// serial chain is the floor.  The reference's per-block terms only need the
// running maximum, a prefix max of the block maxima, so the work splits
// exactly into
//   1. every CTA: Q.K of its key groups, block maxima (scores kept in registers);
//   2. cluster barrier; CTA c takes the maximum over the blocks of CTAs < c
//      (distributed shared memory) as its carry-in;
//   3. every CTA: per block corr, p, psum, pmax, pq and P.V on the tensor
//      cores (each group's P.V stays in its own TMEM columns);
//   4. the two recurrences den = den*corr + psum, res = res*corr + part run in
//      block order: CTA c waits for CTA c-1's (den, res), applies its blocks
//      and hands the state to CTA c+1 through its shared memory; the last CTA
//      writes o8/os.
// Per block the arithmetic and its order are the single-CTA kernel's.
//
// CTA c of the cluster takes groups [c*gpc, (c+1)*gpc) of the sequence's
// groups of 4 pages, gpc = ceil(G / cluster size) <= kMaxG.  Warps: 0-3
// softmax (warp w = block w of a group; thread d = value column d in step 4),
// 4 producer (cp.async of the K pages, then the V pages, through one 2-slot
// ring), 5 MMA issuer.  Every wait is bounded (about one second); a timeout
// sets a bit of the device error word and the roles run to the end, so every
// thread reaches both cluster barriers.
#include <mutex>

#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_tc.cuh"

namespace q3 {

// device error word of this file's kernel (q3_device_status ORs it in); same
// bits as k_attention_decode's
static __device__ unsigned int g_dsplit_error = 0;

int dsplit_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_dsplit_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_dsplit_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace dsplit {

using namespace tcx;

constexpr int NCW = 4;                  // softmax warps
constexpr int THREADS = (NCW + 2) * 32;
constexpr int PRODUCER = NCW, MMA_WARP = NCW + 1;
constexpr int kMaxG = 4;                // key groups (of 4 pages) per CTA
constexpr int TAB_CACHE = 512;
constexpr int TMEM_COLS = 128;          // QK slots at 0 and 16, P.V of group g at 32 + 16 g
constexpr unsigned kErrPage = 2u, kErrTable = 4u, kErrWait = 8u;
constexpr uint32_t ID_QK = idesc_i8(16);
constexpr uint32_t ID_PV = idesc_i8(16, true);

struct Smem {
  alignas(1024) int8_t ring[2][4][4096];  // K pages of a group, then V pages (128B swizzle)
  alignas(1024) int8_t qt[1024];
  alignas(1024) int8_t pq[2][1024];
  uint16_t tab[TAB_CACHE];
  float bm[kMaxG][NCW][2];                // block maxima of this CTA
  float cmax[2];                          // this CTA's maximum over its blocks (per head)
  float corr[kMaxG][2][4], psum[kMaxG][2][4], pmax[kMaxG][2][4];
  float st_res[2][128];                   // (den, res) handed in by the previous CTA
  float st_den[2];
  float red[NCW][2];
  unsigned long long full[2], empty[2], qk_done[2], s_read[2], pq_ready[2], pv_done[2];
  unsigned long long pv_all, chain, mma_final;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_arrive(unsigned long long *b) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(b)) : "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void softmax_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NCW * 32) : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_to(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t mbar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(mbar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ bool wait_or_abort(unsigned long long *b, uint32_t par, Smem &sm) {
  if (mbar_wait(b, par, &sm.abort)) return true;
  if (!*reinterpret_cast<volatile int *>(&sm.abort)) atomicOr(&g_dsplit_error, kErrWait);
  *reinterpret_cast<volatile int *>(&sm.abort) = 1;
  return false;
}
// bounded wait for the chain barrier; waits regardless of the abort word (the
// previous CTA always arrives once, also after its own timeout)
__device__ __forceinline__ bool wait_chain(unsigned long long *b) {
  if (mbar_wait(b, 0, nullptr)) return true;
  atomicOr(&g_dsplit_error, kErrWait);
  return false;
}
__device__ __forceinline__ uint32_t page_of(const Smem &sm, const uint16_t *table, int j) {
  return j < TAB_CACHE ? sm.tab[j] : table[j];
}

__global__ void __launch_bounds__(THREADS, 4)
    k_attention_decode_split(const char *__restrict__ kpool, const char *__restrict__ vpool,
                             DecodeAttnArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t C = cluster_size(), c = cluster_rank();
  const int kvh = blockIdx.x / C, seq = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  pdl_trigger();
  pdl_wait();
  const int kv_len = p.kv_len[seq];
  const int nb = (kv_len + 31) >> 5;
  const uint16_t *table = p.table + static_cast<long>(seq) * p.table_stride;
  // no early return: every thread reaches both cluster barriers
  const bool bad = kv_len <= 0 || nb > p.table_stride;
  const int G = bad ? 0 : (nb + 3) >> 2;
  const int gpc = (G + static_cast<int>(C) - 1) / static_cast<int>(C);
  const int g0 = min(G, static_cast<int>(c) * gpc), n = min(G, g0 + gpc) - g0;   // my groups
  if (bad && tid == 0 && c == 0) atomicOr(&g_dsplit_error, kErrTable);
  if (n > kMaxG && tid == 0) atomicOr(&g_dsplit_error, kErrTable);   // host picks C so this cannot happen
  const int ng = n > kMaxG ? 0 : n;

  // ---- set-up
  for (int i = tid * 4; i < 1024; i += THREADS * 4) {
    if (i >= 256) *reinterpret_cast<int *>(sm.qt + i) = 0;
    *reinterpret_cast<int *>(sm.pq[0] + i) = 0;
    *reinterpret_cast<int *>(sm.pq[1] + i) = 0;
  }
  for (int i = 4 * g0 + tid; i < 4 * (g0 + ng) && i < nb && i < TAB_CACHE; i += THREADS)
    sm.tab[i] = table[i];
  if (tid < 64 && ng > 0) {
    const int hh = tid >> 5, h = kvh * 2 + hh;
    const int v = reinterpret_cast<const int *>(p.q8 + static_cast<long>(seq) * p.q_rb + h * 128)[lane];
    *reinterpret_cast<int *>(sm.qt + hh * 128 + (((lane >> 2) ^ hh) << 4) + (lane & 3) * 4) = v;
  }
  if (tid == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.full[i], 32);
      mbar_init(&sm.empty[i], 1);
      mbar_init(&sm.qk_done[i], 1);
      mbar_init(&sm.s_read[i], NCW * 32);
      mbar_init(&sm.pq_ready[i], NCW * 32);
      mbar_init(&sm.pv_done[i], 1);
    }
    mbar_init(&sm.pv_all, 1);
    mbar_init(&sm.chain, 1);
    mbar_init(&sm.mma_final, 1);
    sm.abort = 0;
    sm.cmax[0] = sm.cmax[1] = kNegInf;
    mbar_init_fence();
  }
  fence_proxy_async();
  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == PRODUCER) {
    // cluster barrier 1 (chunk maxima published): nothing to publish, so arrive
    // now and wait only after the copies (the softmax warps need them first)
    cluster_arrive_release();
    // ---- K of groups 0..ng-1, then V of groups 0..ng-1, through the 2-slot ring
    const int r4 = lane >> 3, c16 = lane & 7;
    for (int it = 0; it < 2 * ng; ++it) {
      const bool isv = it >= ng;
      const int g = isv ? it - ng : it, slot = it & 1;
      if (it >= 2 && !wait_or_abort(&sm.empty[slot], ((it >> 1) - 1) & 1, sm)) break;
      const char *pool = isv ? vpool : kpool;
      const int first = 4 * (g0 + g), count = min(4, nb - first);
      for (int q = 0; q < count; ++q) {
        const uint32_t page = page_of(sm, table, first + q);
        if (page >= p.num_pages) {
          if (lane == 0) atomicOr(&g_dsplit_error, kErrPage);
          continue;
        }
        const char *src = pool + static_cast<size_t>(page) * p.page_bytes + kvh * 128 + c16 * 16;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int row = 4 * i + r4;
          cp_async16(sm.ring[slot][q] + row * 128 + ((c16 ^ (row & 7)) << 4),
                     src + static_cast<size_t>(row) * p.row_bytes);
        }
      }
      cp_arrive(&sm.full[slot]);
    }
    cp_wait_all();
    cluster_wait_acquire();
  } else if (warp == MMA_WARP) {
    cluster_arrive_release();                                  // barrier 1, as the producer
    if (lane == 0) {
      const uint32_t bq = su32(sm.qt);
      bool ok = true;
      for (int g = 0; g < ng && ok; ++g) {                     // Q.K of every group
        const int slot = g & 1;
        if (!(ok = wait_or_abort(&sm.full[slot], (g >> 1) & 1, sm))) break;
        if (g >= 2 && !(ok = wait_or_abort(&sm.s_read[slot], ((g >> 1) - 1) & 1, sm))) break;
        fence_after();
        const uint32_t a0 = su32(sm.ring[slot][0]);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_i8(tmem + 16 * slot, sdesc_sw128(a0 + ks * 32), sdesc_sw128(bq + ks * 32, 0), ID_QK,
                 ks != 0);
        mma_commit(&sm.qk_done[slot]);
        mma_commit(&sm.empty[slot]);
      }
      for (int g = 0; g < ng && ok; ++g) {                     // P.V of every group
        const int it = ng + g, slot = it & 1, ps = g & 1;
        if (!(ok = wait_or_abort(&sm.full[slot], (it >> 1) & 1, sm))) break;
        if (!(ok = wait_or_abort(&sm.pq_ready[ps], (g >> 1) & 1, sm))) break;
        fence_after();
        const int count = min(4, nb - 4 * (g0 + g));
        const uint32_t a0 = su32(sm.ring[slot][0]), b0 = su32(sm.pq[ps]);
        for (int q = 0; q < count; ++q)
          mma_i8(tmem + 32 + 16 * g, sdesc_sw128(a0 + q * 4096), sdesc_plain(b0 + q * 256, 128, 0),
                 ID_PV, q != 0);
        mma_commit(&sm.pv_done[ps]);
        mma_commit(&sm.empty[slot]);
      }
      mma_commit(&sm.pv_all);                                  // every P.V above has completed
      mma_commit(&sm.mma_final);
      mbar_wait(&sm.mma_final, 0, nullptr);
    }
    __syncwarp();
    cluster_wait_acquire();
  } else {
    // ---------------------------------------------------------------- softmax warps
    const float qs0 = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8);
    const float qs1 = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8 + 4);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    auto scale_at = [&](const char *base, int g) -> float {
      const int j = 4 * (g0 + g) + warp, t = j * 32 + lane;
      if (j >= nb || t >= kv_len) return 0.0f;
      const uint32_t page = page_of(sm, table, j);
      if (page >= p.num_pages) return 0.0f;
      return *reinterpret_cast<const float *>(base + static_cast<size_t>(page) * p.scale_page_bytes +
                                              static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4);
    };
    bool ok = true;
    // 1. scores and block maxima of my groups (kept in registers)
    float s0r[kMaxG], s1r[kMaxG];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      s0r[g] = s1r[g] = kNegInf;
      if (g < ng && ok) {
        const int slot = g & 1, count = min(4, nb - 4 * (g0 + g));
        const int j = 4 * (g0 + g) + warp, t = j * 32 + lane;
        const float ks = scale_at(p.ks, g);
        ok = wait_or_abort(&sm.qk_done[slot], (g >> 1) & 1, sm);
        fence_after();
        int a0 = 0, a1 = 0;
        tmem_ld2(lane_base + 16 * slot, a0, a1);
        tmem_wait_ld();
        fence_before();
        mbar_arrive(&sm.s_read[slot]);
        if (ok && warp < count && t < kv_len) {
          s0r[g] = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a0), ks), qs0), p.qk_scale);
          s1r[g] = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a1), ks), qs1), p.qk_scale);
        }
        const float b0 = warp_tree_max(s0r[g]), b1 = warp_tree_max(s1r[g]);
        if (lane == 0) { sm.bm[g][warp][0] = b0; sm.bm[g][warp][1] = b1; }
      }
    }
    softmax_sync();
    if (tid == 0) {
      float m0 = kNegInf, m1 = kNegInf;
      for (int g = 0; g < ng; ++g)
        for (int w = 0; w < NCW; ++w) { m0 = fmaxf(m0, sm.bm[g][w][0]); m1 = fmaxf(m1, sm.bm[g][w][1]); }
      sm.cmax[0] = m0;
      sm.cmax[1] = m1;
    }
    softmax_sync();
    // 2. carry-in: the maximum over the blocks of the CTAs before this one
    cluster_arrive_release();
    cluster_wait_acquire();
    float carry0 = kNegFltMax, carry1 = kNegFltMax;             // the reference's initial m
    for (uint32_t q = 0; q < c; ++q) {
      carry0 = fmaxf(carry0, ld_cluster_f32(map_to(su32(&sm.cmax[0]), q)));
      carry1 = fmaxf(carry1, ld_cluster_f32(map_to(su32(&sm.cmax[1]), q)));
    }
    // 3. per block corr, p, psum, pmax, pq; P.V on the tensor cores
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
      if (g < ng && ok) {
        const int ps = g & 1, count = min(4, nb - 4 * (g0 + g));
        const int j = 4 * (g0 + g) + warp, t = j * 32 + lane;
        float mp0 = carry0, mp1 = carry1;                        // running max before block j
        for (int w = 0; w < NCW; ++w) {
          if (w < count) {
            const float c0 = sm.bm[g][w][0], c1 = sm.bm[g][w][1];
            if (w < warp) { mp0 = fmaxf(mp0, c0); mp1 = fmaxf(mp1, c1); }
            carry0 = fmaxf(carry0, c0);
            carry1 = fmaxf(carry1, c1);
          }
        }
        const float vs = scale_at(p.vs, g);
        if (g >= 2) ok = wait_or_abort(&sm.pv_done[ps], ((g >> 1) - 1) & 1, sm);
        if (ok && warp < count) {
          const float mj0 = fmaxf(mp0, sm.bm[g][warp][0]), mj1 = fmaxf(mp1, sm.bm[g][warp][1]);
          const float cx = (mp0 == mj0 && mp1 == mj1)
                               ? 1.0f
                               : exp_ref(lane == 1 ? __fsub_rn(mp1, mj1) : __fsub_rn(mp0, mj0));
          float prv[2] = {__fsub_rn(s0r[g], mj0), __fsub_rn(s1r[g], mj1)};   // one batch
          exp_ref_fast_n<2, true>(prv, g_exp2_t256);   // s - m_j <= 0
          const float pr0 = prv[0], pr1 = prv[1];
          const float psm0 = warp_tree_sum(pr0), psm1 = warp_tree_sum(pr1);
          const float pv0 = (t < kv_len) ? __fmul_rn(pr0, vs) : 0.0f;
          const float pv1 = (t < kv_len) ? __fmul_rn(pr1, vs) : 0.0f;
          const float pm0 = __fmul_rn(warp_tree_max(fabsf(pv0)), kInv127);
          const float pm1 = __fmul_rn(warp_tree_max(fabsf(pv1)), kInv127);
          int8_t *dst = sm.pq[ps] + (2 * warp + (lane >> 4)) * 128 + 2 * warp * 16 + (lane & 15);
          dst[0] = static_cast<int8_t>(quant1(pv0, pm0));
          dst[16] = static_cast<int8_t>(quant1(pv1, pm1));
          if (lane < 2) sm.corr[g][lane][warp] = cx;
          if (lane == 0) {
            sm.psum[g][0][warp] = psm0; sm.psum[g][1][warp] = psm1;
            sm.pmax[g][0][warp] = pm0; sm.pmax[g][1][warp] = pm1;
          }
        }
        fence_proxy_async();
        mbar_arrive(&sm.pq_ready[ps]);
      }
    }
    if (ng > 0 && ok) ok = wait_or_abort(&sm.pv_all, 0, sm);
    fence_after();
    softmax_sync();                                              // corr/psum/pmax of every block
    // 4. the recurrences in block order, state handed down the cluster
    float den[2] = {0.0f, 0.0f}, res[2] = {0.0f, 0.0f};
    if (c > 0) {
      wait_chain(&sm.chain);
      den[0] = sm.st_den[0]; den[1] = sm.st_den[1];
      res[0] = sm.st_res[0][tid]; res[1] = sm.st_res[1][tid];
    }
    for (int g = 0; g < ng; ++g) {
      const int count = min(4, nb - 4 * (g0 + g));
      int v[8];
      asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                   : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                     "=r"(v[6]), "=r"(v[7])
                   : "r"(lane_base + 32 + 16 * g));
      tmem_wait_ld();
      if (!ok) continue;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < count) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float cc = sm.corr[g][h][q];
            den[h] = __fadd_rn(__fmul_rn(den[h], cc), sm.psum[g][h][q]);
            res[h] = __fadd_rn(__fmul_rn(res[h], cc), __fmul_rn(i2f_small(v[2 * q + h]), sm.pmax[g][h][q]));
          }
        }
      }
    }
    if (c + 1 < C) {                                             // hand the state on
      const uint32_t nx = c + 1;
      st_cluster_f32(map_to(su32(&sm.st_res[0][tid]), nx), res[0]);
      st_cluster_f32(map_to(su32(&sm.st_res[1][tid]), nx), res[1]);
      if (tid < 2) st_cluster_f32(map_to(su32(&sm.st_den[tid]), nx), den[tid]);
      softmax_sync();
      if (tid == 0) {
        asm volatile("fence.acq_rel.cluster;" ::: "memory");
        arrive_remote(map_to(su32(&sm.chain), nx));
      }
    } else if (!bad) {
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
  }

  // every CTA of the cluster stays until the others are done with its memory
  fence_before();
  __syncthreads();
  cluster_arrive_release();
  cluster_wait_acquire();
  fence_after();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
}

}  // namespace dsplit

// Clusters per (sequence, kv head) for a page table of max_pages pages, 0 if
// the split form cannot hold it (more than 8 CTAs of kMaxG groups each).
int attention_decode_split_cluster(uint32_t max_pages) {
  const uint32_t G = (max_pages + 3) / 4;
  const uint32_t C = (G + dsplit::kMaxG - 1) / dsplit::kMaxG;
  return C >= 1 && C <= 8 ? static_cast<int>(C) : 0;
}

int attention_decode_split_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                                  uint32_t num_pages, int kv_heads, int n_seqs, int cluster,
                                  cudaStream_t s, bool pdl) {
  if (p.row_bytes % 16 || p.page_bytes % 16 || reinterpret_cast<uintptr_t>(k_pool) % 16 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16 || cluster < 1 || cluster > 8)
    return Q3_ERR_ALIGN;
  const size_t smem = sizeof(dsplit::Smem) + 1024;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(dsplit::k_attention_decode_split,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr_err != cudaSuccess) {
    q3h::set_cuda_error(attr_err);
    return Q3_ERR_CUDA;
  }
  DecodeAttnArgs a = p;
  a.num_pages = num_pages;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(kv_heads * cluster, n_seqs);
  cfg.blockDim = dim3(dsplit::THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  q3h::timer_begin(q3h::TIMER_ATTENTION, s);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, dsplit::k_attention_decode_split,
                                           static_cast<const char *>(k_pool),
                                           static_cast<const char *>(v_pool), a);
  int st;
  if (e != cudaSuccess) {
    q3h::count_launch();
    cudaGetLastError();
    q3h::set_cuda_error(e);
    st = Q3_ERR_CUDA;
  } else {
    st = q3h::launch_status();
  }
  q3h::timer_end(q3h::TIMER_ATTENTION, s);
  return st;
}

}  // namespace q3
