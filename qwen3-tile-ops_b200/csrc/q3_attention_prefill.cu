// Causal prompt attention (prefill) over the paged int8 KV pool, on the tensor
// cores.  Same arithmetic per query row as kernels/attention_gqa.h:404-547 /
// tools/ref_qwen3.py:210-289: per 32-key block j, in key order,
//   s    = ((f32(q8.k8) * ks) * qs) * qk_scale, keys after the row's position -> -inf
//   m'   = max(tree_max(s), m);  corr = exp(m - m');  p = exp(s - m')
//   den  = (den * corr) + tree_sum(p)
//   pv   = p * vs;  pmax = tree_max(|pv|) / 127;  pq = quant(pv, pmax)
//   res  = (res * corr) + f32(int32(pq . v8)) * pmax
// then res * (1/den) and a per-head quant into o8/os.  A block that lies wholly
// after a row's position is an exact no-op for that row (corr = 1, p = 0).
//
// CTA = 128 query rows (positions r0..r0+127) of one q head of one sequence;
// the heaviest row tiles are scheduled first.  Warp roles:
//   warps 0-15 the rows: warp w owns rows 32 (w % 4) + lane (its TMEM lane
//              quadrant) and part pt = w / 4 of every block's 32 keys (8 keys)
//              and of the 128 value columns (32).  The four parts of a row
//              exchange their block max, tree sums and absmax through shared
//              memory (the reference's 32-key trees split exactly at their two
//              top levels: (s0 + s1) + (s2 + s3)), so each part computes corr /
//              pmax itself and runs the res recurrence for its 32 columns in
//              registers.
//   warp 16    tcgen05 issuer: S_j = Q (M = 128 rows, K = 128) x K_j (N = 32
//              keys) into one of two TMEM slots, then P.V of block j-1 =
//              PQ_{j-1} (M = 128, K = 32) x V_{j-1} read MN-major (N = 128).
//   warp 17    producer: Q once, then per block the K and V page tiles by TMA
//              (128-byte swizzle) into a ring of stages, and their scales.
// The rows overlap block j's softmax with block j-1's P.V on the tensor core.
// All int32 products are exact; every wait is bounded (about one second), a
// timeout sets a bit of the device error word and the roles run to the end.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_gemm.h"
#include "q3_tc.cuh"

namespace q3 {

static __device__ unsigned int g_pattn_error = 0;

int pattn_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_pattn_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_pattn_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace pa {

using namespace tcx;

constexpr int ROWS = 128;
constexpr int KP = 4;                      // parts of a block (keys) / of the value columns
constexpr int CW = 4 * KP;                 // row warps
constexpr int KPK = 32 / KP, KPC = 128 / KP;   // keys / value columns per part
constexpr int MMA_WARP = CW, PRODUCER = CW + 1;
constexpr int THREADS = (CW + 2) * 32;
constexpr int NST = 4;                     // K/V stages
constexpr int TMEM_COLS = 256;             // S slots at 0 and 32, P.V at 64..191
constexpr unsigned kErrWait = 1u << 18;
constexpr unsigned kErrPage = 1u << 19;
constexpr uint32_t ID_QK = idesc_i8(32);                   // A = Q rows, B = K rows (K-major)
constexpr uint32_t ID_PV = idesc_i8(128, false, true);     // A = pq (K-major), B = V (MN-major)

struct Smem {
  alignas(1024) int8_t q[ROWS * 128];                // 128-byte swizzled
  alignas(1024) int8_t k[NST][32 * 128];             // page tiles, 128-byte swizzled
  alignas(1024) int8_t v[NST][32 * 128];
  alignas(1024) int8_t pq[2][2 * ROWS * 16];         // [key half][16 row groups][8 rows][16 B]
  alignas(16) float ks[NST][32];
  alignas(16) float vs[NST][32];
  alignas(16) float xmax[2][ROWS][KP];               // [block parity][row][part]
  alignas(16) float xsum[2][ROWS][KP];
  alignas(16) float xam[2][ROWS][KP];
  float xout[KP][ROWS];
  unsigned long long t256[Q3_EXP2_T256_N];           // exp2 table (per-lane indices)
  unsigned long long q_full, kv_full[NST], kv_empty[NST];
  unsigned long long s_full[2], s_free[2], p_full[2], o_full, o_free, final_done;
  uint32_t tmem_base;
  int abort;
};

// the four warps (parts) of one TMEM lane quadrant, which share its 32 rows
__device__ __forceinline__ void rows_sync(int qd) {
  asm volatile("bar.sync %0, %1;" ::"r"(2 + qd), "n"(KP * 32) : "memory");
}
__device__ __forceinline__ bool wait_or_abort(unsigned long long *b, uint32_t par, int *abort) {
  if (mbar_wait(b, par, abort, 1000000u)) return true;   // suspend up to 1 ms per try
  if (!*reinterpret_cast<volatile int *>(abort)) atomicOr(&g_pattn_error, kErrWait);
  *reinterpret_cast<volatile int *>(abort) = 1;
  return false;
}
// adjacent-pair tree over 8 values (the lower levels of the reference's 32-value tree)
__device__ __forceinline__ float tree8_sum(const float (&v)[8]) {
  float t[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) t[i] = __fadd_rn(v[2 * i], v[2 * i + 1]);
#pragma unroll
  for (int i = 0; i < 2; ++i) t[i] = __fadd_rn(t[2 * i], t[2 * i + 1]);
  return __fadd_rn(t[0], t[1]);
}
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, int (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]),
                 "=r"(v[6]), "=r"(v[7])
               : "r"(taddr));
}

__global__ void __launch_bounds__(THREADS, 1)
    k_attention_prefill(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const PrefillAttnArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int tile = gridDim.x - 1 - blockIdx.x;             // heaviest first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (p.heads / p.kv_heads);
  const int r0 = tile * ROWS;
  const int last = min(r0 + ROWS, p.T) - 1;                 // last row position of the tile
  const int J = last / 32 + 1;                              // key blocks 0..J-1
  const uint16_t *table = p.table + static_cast<long>(b) * p.table_stride;

  if (tid == 0) {
    mbar_init(&sm.q_full, 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(&sm.kv_full[i], 1 + 32);
      mbar_init(&sm.kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], CW * 32);
      mbar_init(&sm.p_full[i], CW * 32);
    }
    mbar_init(&sm.o_full, 1);
    mbar_init(&sm.o_free, CW * 32);
    mbar_init(&sm.final_done, 1);
    sm.abort = 0;
    mbar_init_fence();
  }
  for (int i = tid; i < Q3_EXP2_T256_N; i += THREADS) sm.t256[i] = g_exp2_t256[i];
  if (warp == MMA_WARP) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == PRODUCER) {
    // ------------------------------------------------------------------ producer
    if (lane == 0) {
      mbar_expect_tx(&sm.q_full, ROWS * 128);
      tma_2d(sm.q, &qmap, h * 128, b * p.T + r0, &sm.q_full);
    }
    for (int j = 0; j < J; ++j) {
      const int st = j % NST;
      if (j >= NST) wait_or_abort(&sm.kv_empty[st], ((j / NST) - 1) & 1, &sm.abort);
      uint32_t page = table[j];
      if (page >= p.num_pages) {
        if (lane == 0) atomicOr(&g_pattn_error, kErrPage);
        page = 0;
      }
      if (lane == 0) {
        mbar_expect_tx(&sm.kv_full[st], 2 * 32 * 128);
        tma_3d(sm.k[st], &kmap, kvh * 128, 0, static_cast<int>(page), &sm.kv_full[st]);
        tma_3d(sm.v[st], &vmap, kvh * 128, 0, static_cast<int>(page), &sm.kv_full[st]);
      }
      const size_t so = static_cast<size_t>(page) * p.scale_page_bytes +
                        static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4;
      sm.ks[st][lane] = *reinterpret_cast<const float *>(p.ks + so);
      sm.vs[st][lane] = *reinterpret_cast<const float *>(p.vs + so);
      mbar_arrive(&sm.kv_full[st]);
    }
    // every fill has been consumed before the CTA ends (the MMAs wait on them)
  } else if (warp == MMA_WARP) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      wait_or_abort(&sm.q_full, 0, &sm.abort);
      const uint32_t qa = su32(sm.q);
      for (int j = 0; j <= J; ++j) {
        if (j < J) {                                        // S_j = Q . K_j
          const int st = j % NST, slot = j & 1;
          wait_or_abort(&sm.kv_full[st], (j / NST) & 1, &sm.abort);
          if (j >= 2) wait_or_abort(&sm.s_free[slot], ((j >> 1) - 1) & 1, &sm.abort);
          fence_after();
          const uint32_t kb = su32(sm.k[st]);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_i8(tmem + 32 * slot, sdesc_sw128(qa + ks * 32), sdesc_sw128(kb + ks * 32), ID_QK,
                   ks != 0);
          mma_commit(&sm.s_full[slot]);
        }
        if (j >= 1) {                                       // P.V of block j-1
          const int jj = j - 1, st = jj % NST;
          wait_or_abort(&sm.p_full[jj & 1], (jj >> 1) & 1, &sm.abort);
          if (jj >= 1) wait_or_abort(&sm.o_free, (jj - 1) & 1, &sm.abort);
          fence_after();
          mma_i8(tmem + 64, sdesc_plain(su32(sm.pq[jj & 1]), 2 * 8 * ROWS, 128),
                 sdesc_sw128(su32(sm.v[st])), ID_PV, 0);
          mma_commit(&sm.o_full);
          mma_commit(&sm.kv_empty[st]);
        }
      }
      mma_commit(&sm.final_done);                           // every MMA above has completed
      mbar_wait(&sm.final_done, 0, nullptr);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ rows
    const int qd = warp & 3, pt = warp >> 2;
    const int r = qd * 32 + lane, pos = r0 + r;
    const bool active = pos < p.T;
    const long grow = static_cast<long>(b) * p.T + pos;     // row of q8/o8
    const float qsc = active ? *reinterpret_cast<const float *>(p.qs + grow * p.qs_rb + h * 4) : 0.0f;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    float m = kNegFltMax, den = 0.0f;
    float res[KPC];
#pragma unroll
    for (int d = 0; d < KPC; ++d) res[d] = 0.0f;
    float corr_prev = 1.0f, pmax_prev = 0.0f;

    auto pv_update = [&](int jj, float corr, float pm) {   // res recurrence, block jj
      wait_or_abort(&sm.o_full, jj & 1, &sm.abort);
      fence_after();
      int o[KPC];
#pragma unroll
      for (int c = 0; c < KPC / 16; ++c)
        tmem_ld16(lane_base + 64 + KPC * pt + 16 * c, *reinterpret_cast<int(*)[16]>(&o[16 * c]));
      tmem_wait_ld();
      fence_before();
      mbar_arrive(&sm.o_free);
      if (__all_sync(0xffffffffu, corr == 1.0f)) {          // res * 1 = res exactly
#pragma unroll
        for (int d = 0; d < KPC; ++d) res[d] = __fadd_rn(res[d], __fmul_rn(i2f_small(o[d]), pm));
      } else {
#pragma unroll
        for (int d = 0; d < KPC; ++d)
          res[d] = __fadd_rn(__fmul_rn(res[d], corr), __fmul_rn(i2f_small(o[d]), pm));
      }
    };

    for (int j = 0; j < J; ++j) {
      const int st = j % NST, slot = j & 1;
      wait_or_abort(&sm.s_full[slot], (j >> 1) & 1, &sm.abort);
      fence_after();
      int a[KPK];
      tmem_ld8(lane_base + 32 * slot + KPK * pt, a);
      tmem_wait_ld();
      fence_before();
      mbar_arrive(&sm.s_free[slot]);
      wait_or_abort(&sm.kv_full[st], (j / NST) & 1, &sm.abort);   // the block's scales
      float s[KPK], ksv[KPK], vsv[KPK];
      *reinterpret_cast<float4 *>(&ksv[0]) = *reinterpret_cast<const float4 *>(&sm.ks[st][KPK * pt]);
      *reinterpret_cast<float4 *>(&ksv[4]) = *reinterpret_cast<const float4 *>(&sm.ks[st][KPK * pt + 4]);
      // every key of the block at or before every row of this warp: no mask
      const bool open = 32 * j + 31 <= r0 + qd * 32;
      float bm = kNegInf;
      if (open) {
#pragma unroll
        for (int i = 0; i < KPK; ++i) {
          s[i] = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a[i]), ksv[i]), qsc), p.qk_scale);
          bm = fmaxf(bm, s[i]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < KPK; ++i) {
          const int key = 32 * j + KPK * pt + i;
          s[i] = (key <= pos)
                     ? __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a[i]), ksv[i]), qsc), p.qk_scale)
                     : kNegInf;
          bm = fmaxf(bm, s[i]);
        }
      }
      sm.xmax[slot][r][pt] = bm;
      rows_sync(qd);
      const float4 xm = *reinterpret_cast<const float4 *>(sm.xmax[slot][r]);
      const float bmax = fmaxf(fmaxf(xm.x, xm.y), fmaxf(xm.z, xm.w));
      const float mn = fmaxf(m, bmax);
      // exp(m - mn) is exp(0) = 1 exactly when the running maximum did not move
      const float corr = (mn == m) ? 1.0f : exp_ref_fast_t(__fsub_rn(m, mn), sm.t256);
      float pv[KPK];
      float am = 0.0f;
#pragma unroll
      for (int i = 0; i < KPK; ++i) s[i] = __fsub_rn(s[i], mn);
      exp_ref_fast_n<KPK, true>(s, sm.t256);                  // p (s - m' <= 0)
      const float ps = tree8_sum(s);
      *reinterpret_cast<float4 *>(&vsv[0]) = *reinterpret_cast<const float4 *>(&sm.vs[st][KPK * pt]);
      *reinterpret_cast<float4 *>(&vsv[4]) = *reinterpret_cast<const float4 *>(&sm.vs[st][KPK * pt + 4]);
      if (open) {
#pragma unroll
        for (int i = 0; i < KPK; ++i) {
          pv[i] = __fmul_rn(s[i], vsv[i]);
          am = fmaxf(am, fabsf(pv[i]));
        }
      } else {
#pragma unroll
        for (int i = 0; i < KPK; ++i) {
          const int key = 32 * j + KPK * pt + i;
          pv[i] = (key <= pos) ? __fmul_rn(s[i], vsv[i]) : 0.0f;
          am = fmaxf(am, fabsf(pv[i]));
        }
      }
      sm.xsum[slot][r][pt] = ps;
      sm.xam[slot][r][pt] = am;
      rows_sync(qd);
      // the two top levels of the 32-key tree: (s0 + s1) + (s2 + s3)
      const float4 xs = *reinterpret_cast<const float4 *>(sm.xsum[slot][r]);
      const float psum = __fadd_rn(__fadd_rn(xs.x, xs.y), __fadd_rn(xs.z, xs.w));
      const float4 xa = *reinterpret_cast<const float4 *>(sm.xam[slot][r]);
      const float amx = fmaxf(fmaxf(xa.x, xa.y), fmaxf(xa.z, xa.w));
      const float pm = __fmul_rn(amx, kInv127);
      den = __fadd_rn(__fmul_rn(den, corr), psum);
      m = mn;
      uint32_t w2[2];
      quant_pack_absmax(pv, pm, w2);                       // one reciprocal for the 8 codes
      // keys 8 pt .. : 16-key chunk pt / 2, bytes 8 (pt % 2) .. of the row's 16
      *reinterpret_cast<uint2 *>(sm.pq[slot] + (pt >> 1) * (8 * 2 * ROWS) + (r >> 3) * 128 +
                                 (r & 7) * 16 + (pt & 1) * 8) = make_uint2(w2[0], w2[1]);
      fence_proxy_async();
      mbar_arrive(&sm.p_full[slot]);
      if (j >= 1) pv_update(j - 1, corr_prev, pmax_prev);
      corr_prev = corr;
      pmax_prev = pm;
    }
    pv_update(J - 1, corr_prev, pmax_prev);

    // ---- 1/den, per-head output quantisation (attention_gqa.h:522-546)
    const float rden = __frcp_rn(den);
    float mx = 0.0f;
#pragma unroll
    for (int d = 0; d < KPC; ++d) {
      res[d] = __fmul_rn(res[d], rden);
      mx = fmaxf(mx, fabsf(res[d]));
    }
    sm.xout[pt][r] = mx;
    rows_sync(qd);
    float omx = sm.xout[0][r];
#pragma unroll
    for (int q = 1; q < KP; ++q) omx = fmaxf(omx, sm.xout[q][r]);
    const float scale = __fmul_rn(omx, kInv127);
    if (active) {
      uint32_t w4[KPC / 4];
      quant_pack_absmax(res, scale, w4);
      uint4 *dst = reinterpret_cast<uint4 *>(p.o8 + grow * p.o_rb + h * 128 + KPC * pt);
#pragma unroll
      for (int c = 0; c < KPC / 16; ++c) dst[c] = make_uint4(w4[4 * c], w4[4 * c + 1], w4[4 * c + 2], w4[4 * c + 3]);
      if (pt == 0) *reinterpret_cast<float *>(p.os + grow * p.os_rb + h * 4) = scale;
    }
  }

  fence_before();
  __syncthreads();
  fence_after();
  if (warp == MMA_WARP) tmem_dealloc<TMEM_COLS>(tmem);
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// pool [pages][32 rows][row_bytes] int8 (page stride page_bytes); box = 128 bytes x 32 rows
static bool page_map(CUtensorMap *m, const void *base, uint32_t row_bytes, uint32_t page_bytes,
                     uint32_t num_pages) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {row_bytes, 32, num_pages};
  cuuint64_t strides[2] = {row_bytes, page_bytes};
  cuuint32_t box[3] = {128, 32, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace pa

int attention_prefill_launch(const PrefillAttnArgs &p, const void *q8, long q_rb, int M,
                             const void *k_pool, const void *v_pool, uint32_t page_bytes,
                             uint32_t row_bytes, int n_seqs, cudaStream_t s) {
  if (p.heads % p.kv_heads || q_rb % 16 || row_bytes % 16 || page_bytes % 16 ||
      page_bytes < 32 * row_bytes || row_bytes < (uint32_t)p.kv_heads * 128 ||
      reinterpret_cast<uintptr_t>(q8) % 16 || reinterpret_cast<uintptr_t>(k_pool) % 16 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16 || p.T < 1 || (p.T + 31) / 32 > p.table_stride)
    return Q3_ERR_SHAPE;
  CUtensorMap qm, km, vm;
  if (!tc::make_map(&qm, q8, M, p.heads * 128, q_rb, pa::ROWS) ||
      !pa::page_map(&km, k_pool, row_bytes, page_bytes, p.num_pages) ||
      !pa::page_map(&vm, v_pool, row_bytes, page_bytes, p.num_pages))
    return Q3_ERR_CUDA;
  const size_t smem = sizeof(pa::Smem) + 1024;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(pa::k_attention_prefill, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem);
  });
  if (attr != cudaSuccess) {
    q3h::set_cuda_error(attr);
    return Q3_ERR_CUDA;
  }
  dim3 grid((p.T + pa::ROWS - 1) / pa::ROWS, p.heads, n_seqs);
  q3h::timer_begin(q3h::TIMER_ATTENTION, s);
  pa::k_attention_prefill<<<grid, pa::THREADS, smem, s>>>(qm, km, vm, p);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_ATTENTION, s);
  return st;
}

}  // namespace q3
