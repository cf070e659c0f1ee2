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
// CTA = one (sequence, kv head), 4 warps; the two q heads of the GQA group
// share every K/V page.  Pages (32 tokens x 128 bytes of this kv head) stream
// through three buffers of "rounds" of 4 pages with cp.async (16 bytes per
// thread, rows stored in the tensor cores' 128-byte swizzle); rounds alternate
// K and V over the same 4 blocks, two rounds ahead of the one in use.
//   K round  one tcgen05.mma chain (M = 128 keys, N = 16, K = 128) gives q.k of
//            both heads for the 4 pages in TMEM; warp w takes page w: scale,
//            mask, block max, prefix max, then p / psum / pmax / pq and corr.
//   V round  per page one tcgen05.mma with A = V read MN-major (M = 128 value
//            columns, K = 32 keys) and B = the pq rows of both heads, so thread
//            d of the CTA gets the int32 P.V of column d for both heads and runs
//            the recurrences over the round's blocks in order.
// All int32 products are exact, so the tensor cores change no bit.  Thread 0
// waits for each MMA completion with a bound; the outcome reaches the other
// threads through the barrier, and a timeout sets a bit of the device error word.
#include <mutex>

#include "q3_attention.h"
#include "q3_common.cuh"
#include "q3_tc.cuh"

namespace q3 {

__device__ unsigned int g_device_error = 0;   // read by q3_device_status()

namespace dec {

using namespace tcx;

constexpr int NW = 4;               // warps
constexpr int THREADS = NW * 32;
constexpr int NBUF = 3;             // round buffers (two rounds in flight)
constexpr int TMEM_COLS = 64;       // K round: 16 columns; V round: 16 per page
constexpr unsigned kErrPage = 2u;   // a page index >= num_pages (copy skipped)
constexpr unsigned kErrTable = 4u;  // kv_len needs more pages than the table holds
constexpr unsigned kErrMma = 8u;    // a tensor-core completion wait timed out
constexpr uint32_t ID_QK = idesc_i8(16);          // A = keys (K-major), B = q rows
constexpr uint32_t ID_PV = idesc_i8(16, true);    // A = V (MN-major), B = pq rows

struct Smem {
  alignas(1024) int8_t buf[NBUF][4][4096];   // page tiles, 128-byte swizzled rows
  alignas(1024) int8_t qt[2048];             // B of the K round: rows 0,1 = q heads, rest 0
  alignas(1024) int8_t pq[4][512];           // B of the V round per page: [row group][k half][8 rows][16 B]
  float bm[4][2];                            // block maxima of the K round
  float corr[2][4], psum[2][4], pmax[2][4];  // per head, per page of the round
  float red[NW][2];
  unsigned long long mbar;
  uint32_t tmem_base;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_keep2() {
  asm volatile("cp.async.wait_group 2;" ::: "memory");
}
__device__ __forceinline__ void cp_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// byte offset of 16-byte chunk `i` of row `r` in a swizzled 32x128 page tile
__device__ __forceinline__ int swz(int r, int i) { return r * 128 + (((i ^ (r & 7))) << 4); }

// each of the 128 threads copies 2 x 16 bytes of every page of round r
// (rounds: 2g = K pages of blocks 4g..4g+3, 2g+1 = V pages of the same blocks)
__device__ __forceinline__ void issue_round(int r, int nb, int8_t (*dst)[4096],
                                            const DecodeAttnArgs &p, const char *kpool,
                                            const char *vpool, const uint16_t *table, int kvh) {
  const int t = threadIdx.x;
  const int row = t >> 2, c0 = (t & 3) * 2;
  const int first = 4 * (r >> 1), count = min(4, nb - first);
  const char *pool = (r & 1) ? vpool : kpool;
  const size_t off = static_cast<size_t>(row) * p.row_bytes + kvh * 128 + c0 * 16;
  for (int q = 0; q < count; ++q) {
    const uint32_t page = table[first + q];
    if (page >= p.num_pages) {
      if (t == 0) atomicOr(&g_device_error, kErrPage);
      continue;
    }
    const char *src = pool + static_cast<size_t>(page) * p.page_bytes + off;
    cp_async16(dst[q] + swz(row, c0), src);
    cp_async16(dst[q] + swz(row, c0 + 1), src + 16);
  }
}

__global__ void __launch_bounds__(THREADS, 4)
    k_attention_decode(const char *__restrict__ kpool, const char *__restrict__ vpool,
                       DecodeAttnArgs p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int kvh = blockIdx.x, seq = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int kv_len = p.kv_len[seq];
  const int nb = (kv_len + 31) >> 5;
  const uint16_t *table = p.table + static_cast<long>(seq) * p.table_stride;
  const float qk_scale = p.qk_scale;
  if (kv_len <= 0 || nb > p.table_stride) {        // uniform for the whole CTA
    if (tid == 0) atomicOr(&g_device_error, kErrTable);
    return;
  }
  const int R = 2 * ((nb + 3) >> 2);               // K and V rounds
  issue_round(0, nb, sm.buf[0], p, kpool, vpool, table, kvh);
  cp_commit();
  issue_round(1, nb, sm.buf[1], p, kpool, vpool, table, kvh);   // R >= 2 always
  cp_commit();

  // operand B of both products: rows 2..15 stay zero
  for (int i = 256 + tid * 4; i < 2048; i += THREADS * 4) *reinterpret_cast<int *>(sm.qt + i) = 0;
  for (int i = tid * 4; i < 4 * 512; i += THREADS * 4) *reinterpret_cast<int *>(&sm.pq[0][0] + i) = 0;
  float qsc[2];
  {
    const int hh = tid >> 5;                       // threads 0..63: q rows of the two heads
    if (hh < 2) {
      const int h = kvh * 2 + hh;
      const int v = reinterpret_cast<const int *>(p.q8 + static_cast<long>(seq) * p.q_rb + h * 128)[lane];
      *reinterpret_cast<int *>(sm.qt + hh * 128 + (((lane >> 2) ^ hh) << 4) + (lane & 3) * 4) = v;
    }
    qsc[0] = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8);
    qsc[1] = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + kvh * 8 + 4);
  }
  if (tid == 0) {
    mbar_init(&sm.mbar, 1);
    mbar_init_fence();
  }
  if (warp == 0) tmem_alloc<TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);

  float carry[2] = {kNegFltMax, kNegFltMax};
  float den[2] = {0.0f, 0.0f}, res[2] = {0.0f, 0.0f};   // thread = value column tid
  uint32_t phase = 0;
  bool mma_ok = true;       // thread 0's view of the last completion wait
  bool aborted = false;     // uniform

  for (int r = 0; r < R; ++r) {
    if (r + 2 < R) issue_round(r + 2, nb, sm.buf[(r + 2) % NBUF], p, kpool, vpool, table, kvh);
    cp_commit();
    cp_wait_keep2();
    fence_proxy_async();      // this thread's copies and B-operand stores -> tensor cores
    __syncthreads();
    const int first = 4 * (r >> 1), count = min(4, nb - first);
    int8_t(*pages)[4096] = sm.buf[r % NBUF];
    if (tid == 0) {
      fence_after();
      if (!(r & 1)) {
        const uint32_t a0 = su32(pages[0]), b0 = su32(sm.qt);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks)
          mma_i8(tmem, sdesc_sw128(a0 + ks * 32), sdesc_sw128(b0 + ks * 32), ID_QK, ks != 0);
      } else {
        for (int q = 0; q < count; ++q)
          mma_i8(tmem + 16 * q, sdesc_sw128(su32(pages[q])), sdesc_plain(su32(sm.pq[q]), 128, 256),
                 ID_PV, 0);
      }
      mma_commit(&sm.mbar);
      mma_ok = mbar_wait(&sm.mbar, phase, nullptr);
      fence_before();
    }
    if (__syncthreads_or(!mma_ok)) {               // uniform: all threads leave together
      if (tid == 0) atomicOr(&g_device_error, kErrMma);
      aborted = true;
      break;
    }
    phase ^= 1u;
    fence_after();
    if (!(r & 1)) {
      // ---- K round: warp w takes block first + w
      const int j = first + warp;
      const int t = j * 32 + lane;
      float s0 = kNegInf, s1 = kNegInf;
      uint32_t page = 0;
      if (warp < count) {
        int a0, a1;
        tmem_ld2(lane_base, a0, a1);
        tmem_wait_ld();
        page = table[j];
        const float ks = (t < kv_len && page < p.num_pages)
                             ? *reinterpret_cast<const float *>(
                                   p.ks + static_cast<size_t>(page) * p.scale_page_bytes +
                                   static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4)
                             : 0.0f;
        if (t < kv_len) {                          // decode: the row sees keys 0..kv_len-1
          s0 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a0), ks), qsc[0]), qk_scale);
          s1 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(a1), ks), qsc[1]), qk_scale);
        }
        const float b0 = warp_tree_max(s0), b1 = warp_tree_max(s1);
        if (lane == 0) { sm.bm[warp][0] = b0; sm.bm[warp][1] = b1; }
      }
      __syncthreads();
      float mp0 = carry[0], mp1 = carry[1];        // running max before block first + warp
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        if (w < warp && w < count) { mp0 = fmaxf(mp0, sm.bm[w][0]); mp1 = fmaxf(mp1, sm.bm[w][1]); }
      }
      if (warp < count) {
        const float mj0 = fmaxf(mp0, sm.bm[warp][0]), mj1 = fmaxf(mp1, sm.bm[warp][1]);
        // lane 0: corr of head 0, lane 1: corr of head 1
        const float cx = exp_ref(lane == 1 ? __fsub_rn(mp1, mj1) : __fsub_rn(mp0, mj0));
        const float vs = (t < kv_len && page < p.num_pages)
                             ? *reinterpret_cast<const float *>(
                                   p.vs + static_cast<size_t>(page) * p.scale_page_bytes +
                                   static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4)
                             : 0.0f;
        const float pr0 = exp_ref(__fsub_rn(s0, mj0)), pr1 = exp_ref(__fsub_rn(s1, mj1));
        const float ps0 = warp_tree_sum(pr0), ps1 = warp_tree_sum(pr1);
        const float pv0 = (t < kv_len) ? __fmul_rn(pr0, vs) : 0.0f;
        const float pv1 = (t < kv_len) ? __fmul_rn(pr1, vs) : 0.0f;
        const float pm0 = __fmul_rn(warp_tree_max(fabsf(pv0)), kInv127);
        const float pm1 = __fmul_rn(warp_tree_max(fabsf(pv1)), kInv127);
        int8_t *dst = sm.pq[warp] + (lane >> 4) * 128 + (lane & 15);
        dst[0] = static_cast<int8_t>(quant1(pv0, pm0));    // row 0: head 2 kvh
        dst[16] = static_cast<int8_t>(quant1(pv1, pm1));   // row 1: head 2 kvh + 1
        if (lane < 2) sm.corr[lane][warp] = cx;
        if (lane == 0) {
          sm.psum[0][warp] = ps0; sm.psum[1][warp] = ps1;
          sm.pmax[0][warp] = pm0; sm.pmax[1][warp] = pm1;
        }
      }
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        if (w < count) { carry[0] = fmaxf(carry[0], sm.bm[w][0]); carry[1] = fmaxf(carry[1], sm.bm[w][1]); }
      }
    } else {
      // ---- V round: column tid of both heads, blocks in order
      int v[4][2];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (q < count) tmem_ld2(lane_base + 16 * q, v[q][0], v[q][1]);
      tmem_wait_ld();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q < count) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float c = sm.corr[h][q];
            den[h] = __fadd_rn(__fmul_rn(den[h], c), sm.psum[h][q]);
            res[h] = __fadd_rn(__fmul_rn(res[h], c), __fmul_rn(i2f_small(v[q][h]), sm.pmax[h][q]));
          }
        }
      }
    }
    fence_before();   // TMEM reads ordered before the next round's barrier and MMA
  }
  cp_wait_all();
  if (aborted && tid == 0) mbar_wait(&sm.mbar, phase, nullptr);   // drain, bounded
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 0) tmem_dealloc<TMEM_COLS>(tmem);
  if (aborted) return;

  // ---- 1/den, per-head output quantisation (attention_gqa.h:522-546)
  float o[2], mx[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    o[h] = __fmul_rn(res[h], __fdiv_rn(1.0f, den[h]));
    float m = fabsf(o[h]);
#pragma unroll
    for (int k = 1; k < 32; k <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, k));
    mx[h] = m;
  }
  if (lane == 0) { sm.red[warp][0] = mx[0]; sm.red[warp][1] = mx[1]; }
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float hm = 0.0f;
#pragma unroll
    for (int w = 0; w < NW; ++w) hm = fmaxf(hm, sm.red[w][h]);
    const float scale = __fmul_rn(hm, kInv127);
    const int hd = kvh * 2 + h;
    p.o8[static_cast<long>(seq) * p.o_rb + hd * 128 + tid] = static_cast<char>(quant1(o[h], scale));
    if (tid == 0) *reinterpret_cast<float *>(p.os + static_cast<long>(seq) * p.os_rb + hd * 4) = scale;
  }
}

}  // namespace dec

// ---------------------------------------------------------------- host side
int attention_decode_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                            uint32_t num_pages, int kv_heads, int n_seqs, cudaStream_t s) {
  if (p.row_bytes % 16 || p.page_bytes % 16 || reinterpret_cast<uintptr_t>(k_pool) % 16 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16)
    return Q3_ERR_ALIGN;
  const size_t smem = sizeof(dec::Smem) + 1024;   // + alignment slack
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [&] {
    attr_err = cudaFuncSetAttribute(dec::k_attention_decode,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr_err != cudaSuccess) {
    q3h::set_cuda_error(attr_err);
    return Q3_ERR_CUDA;
  }
  DecodeAttnArgs a = p;
  a.num_pages = num_pages;
  dim3 grid(kv_heads, n_seqs);
  q3h::timer_begin(q3h::TIMER_ATTENTION, s);
  dec::k_attention_decode<<<grid, dec::THREADS, smem, s>>>(
      static_cast<const char *>(k_pool), static_cast<const char *>(v_pool), a);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_ATTENTION, s);
  return st;
}

}  // namespace q3

namespace q3 {
int gemm_device_status_take();
}

extern "C" int q3_device_status(void) {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, q3::g_device_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(q3::g_device_error, &zero, sizeof zero);
  const int g = q3::gemm_device_status_take();
  if (g < 0) return -1;
  return static_cast<int>(v) | g;
}
