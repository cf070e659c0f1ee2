// Decode attention (one query row per sequence) over the paged int8 KV pool.
// Same arithmetic as kernels/attention_gqa.h:404-547 / tools/ref_qwen3.py:210-266,
// reorganised:
//
// The reference walks 32-key blocks in order, and every step of block j uses
// the running maximum m_j = max(m_{j-1}, tree_max(s_j)).  m_j depends only on
// block maxima, so it is a prefix max.  Once the m_j are known, each block's
//     corr_j = exp(m_{j-1} - m_j),  p_j = exp(s_j - m_j),  psum_j = tree_sum(p_j),
//     pq_j = quant(p_j * vs, pmax_j),  part_j = f32(int32(pq_j . V_j)) * pmax_j
// can be computed independently, and only the two cheap recurrences
//     den_j = (den_{j-1} * corr_j) + psum_j,  res_j = (res_{j-1} * corr_j) + part_j
// must run in block order — with exactly the reference's two roundings each.
//
// CTA = one (sequence, kv head), 4 warps: the two q heads of the GQA group
// share every K/V page.  Pages (32 tokens x 128 bytes of this kv head) stream
// through a double buffer of "rounds" of 4 pages with cp.async (16 bytes per
// thread, XOR-swizzled rows so that row-wise and column-wise reads are free of
// bank conflicts): the next round is in flight while the current one is used.
// Per chunk of up to CH blocks:
//   pass 1  (K rounds, warp w takes page w)  s = q.k for both heads -> S, block maxima
//   scan    prefix max of the block maxima
//   pass 1b (block-parallel)  corr, p, psum, pq, pmax per block
//   pass 2  (V rounds, column-parallel) each warp owns 32 of the 128 output
//           columns and runs the recurrence over the blocks in order.
#include <mutex>

#include "q3_attention.h"
#include "q3_common.cuh"

namespace q3 {

__device__ unsigned int g_device_error = 0;   // read by q3_device_status()

namespace dec {

constexpr int CH = 48;          // blocks per chunk (1536 keys); a multiple of 4
constexpr int NW = 4;           // warps
constexpr int THREADS = NW * 32;
constexpr int RPC = 2 * (CH / 4);   // rounds of a full chunk (K rounds then V rounds)
constexpr unsigned kErrPage = 2u;   // a page index >= num_pages (copy skipped)
constexpr unsigned kErrTable = 4u;  // kv_len needs more pages than the table holds

struct Smem {
  alignas(128) int8_t buf[2][4][4096];
  float S[2][CH * 32];
  int8_t PQ[2][CH * 32];
  float bmax[2][CH];
  float mrun[2][CH];
  float pmax[2][CH];
  float psum[2][CH];
  float corr[2][CH];
  int8_t q[2][128];
  float qs[2];
  float red[NW][2];
};

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_wait_all_but_newest() {
  asm volatile("cp.async.wait_group 1;" ::: "memory");
}
// byte offset of 16-byte chunk `i` of row `r` in a swizzled 32x128 page tile
__device__ __forceinline__ int swz(int r, int i) { return r * 128 + (((i ^ (r & 7))) << 4); }

__device__ __forceinline__ int sx8(int w, int b) { return (w << (24 - 8 * b)) >> 24; }

struct Round {
  int c0;      // first block of the chunk
  int nbc;     // blocks in the chunk
  int v;       // 0: K round, 1: V round
  int first;   // first block of the round (chunk relative)
  int count;   // pages in the round (1..4)
};

__device__ __forceinline__ Round round_of(int r, int nb) {
  const int nch = (nb + CH - 1) / CH;
  int k = r / RPC;
  if (k > nch - 1) k = nch - 1;
  const int rr = r - k * RPC;
  Round o;
  o.c0 = k * CH;
  o.nbc = min(CH, nb - o.c0);
  const int nrk = (o.nbc + 3) >> 2;
  o.v = rr >= nrk;
  o.first = 4 * (rr - (o.v ? nrk : 0));
  o.count = min(4, o.nbc - o.first);
  return o;
}

__device__ __forceinline__ int rounds_total(int nb) {
  const int nch = (nb + CH - 1) / CH;
  const int last = nb - (nch - 1) * CH;
  return (nch - 1) * RPC + 2 * ((last + 3) >> 2);
}

// each of the 128 threads copies 2 x 16 bytes of every page of the round
__device__ __forceinline__ void issue_round(const Round &rd, int8_t (*dst)[4096],
                                            const DecodeAttnArgs &p, const char *kpool,
                                            const char *vpool, const uint16_t *table, int kvh) {
  const int t = threadIdx.x;
  const int row = t >> 2, c0 = (t & 3) * 2;
  const char *pool = rd.v ? vpool : kpool;
  for (int q = 0; q < rd.count; ++q) {
    const uint32_t page = table[rd.c0 + rd.first + q];
    if (page >= p.num_pages) {
      if (t == 0) atomicOr(&g_device_error, kErrPage);
      continue;
    }
    const char *src = pool + static_cast<size_t>(page) * p.page_bytes +
                      static_cast<size_t>(row) * p.row_bytes + kvh * 128;
    cp_async16(dst[q] + swz(row, c0), src + c0 * 16);
    cp_async16(dst[q] + swz(row, c0 + 1), src + (c0 + 1) * 16);
  }
}

__global__ void __launch_bounds__(THREADS, 4)
    k_attention_decode(const char *__restrict__ kpool, const char *__restrict__ vpool,
                       DecodeAttnArgs p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Smem &sm = *reinterpret_cast<Smem *>(smem_raw);

  const int kvh = blockIdx.x, seq = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kv_len = p.kv_len[seq];
  const int nb = (kv_len + 31) >> 5;
  const uint16_t *table = p.table + static_cast<long>(seq) * p.table_stride;
  const float qk_scale = p.qk_scale;
  if (kv_len <= 0 || nb > p.table_stride) {        // uniform for the whole CTA
    if (threadIdx.x == 0) atomicOr(&g_device_error, kErrTable);
    return;
  }

  if (threadIdx.x < 64) {   // q rows of the two heads (int8) and their scales
    const int hh = threadIdx.x >> 5;
    const int h = kvh * 2 + hh;
    const int *src = reinterpret_cast<const int *>(p.q8 + static_cast<long>(seq) * p.q_rb + h * 128);
    reinterpret_cast<int *>(sm.q[hh])[lane] = src[lane];
    if (lane == 0) sm.qs[hh] = *reinterpret_cast<const float *>(p.qs + static_cast<long>(seq) * p.qs_rb + h * 4);
  }

  float m_carry[2] = {kNegFltMax, kNegFltMax};
  float den_h[2] = {0.0f, 0.0f};     // every lane keeps both heads' denominators
  float res[2] = {0.0f, 0.0f};
  const int dq = lane & 7, kg = lane >> 3;
  const int my_h = kg >> 1;                       // head of the two columns this lane owns
  const int my_d0 = warp * 32 + dq * 4 + (kg & 1) * 2;

  const int R = rounds_total(nb);
  issue_round(round_of(0, nb), sm.buf[0], p, kpool, vpool, table, kvh);
  cp_commit();
  for (int r = 0; r < R; ++r) {
    if (r + 1 < R) issue_round(round_of(r + 1, nb), sm.buf[(r + 1) & 1], p, kpool, vpool, table, kvh);
    cp_commit();
    cp_wait_all_but_newest();
    __syncthreads();
    const Round rd = round_of(r, nb);
    const int c0 = rd.c0, nbc = rd.nbc;
    int8_t(*pages)[4096] = sm.buf[r & 1];
    if (!rd.v) {
      // ---- pass 1: scores (warp w takes page w of the round)
      if (warp < rd.count) {
        const int j = rd.first + warp;
        const int8_t *tile = pages[warp];
        int acc0 = 0, acc1 = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int4 kw = *reinterpret_cast<const int4 *>(tile + swz(lane, i));
          const int4 q0 = *reinterpret_cast<const int4 *>(&sm.q[0][i * 16]);
          const int4 q1 = *reinterpret_cast<const int4 *>(&sm.q[1][i * 16]);
          acc0 = __dp4a(kw.x, q0.x, acc0); acc0 = __dp4a(kw.y, q0.y, acc0);
          acc0 = __dp4a(kw.z, q0.z, acc0); acc0 = __dp4a(kw.w, q0.w, acc0);
          acc1 = __dp4a(kw.x, q1.x, acc1); acc1 = __dp4a(kw.y, q1.y, acc1);
          acc1 = __dp4a(kw.z, q1.z, acc1); acc1 = __dp4a(kw.w, q1.w, acc1);
        }
        const int t = (c0 + j) * 32 + lane;
        const uint32_t page = table[c0 + j];
        const float ks = (t < kv_len && page < p.num_pages)
                             ? *reinterpret_cast<const float *>(
                                   p.ks + static_cast<size_t>(page) * p.scale_page_bytes +
                                   static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4)
                             : 0.0f;
        float s0 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(acc0), ks), sm.qs[0]), qk_scale);
        float s1 = __fmul_rn(__fmul_rn(__fmul_rn(i2f_small(acc1), ks), sm.qs[1]), qk_scale);
        if (t >= kv_len) s0 = s1 = kNegInf;          // decode: the row sees keys 0..kv_len-1
        sm.S[0][j * 32 + lane] = s0;
        sm.S[1][j * 32 + lane] = s1;
        const float b0 = warp_tree_max(s0), b1 = warp_tree_max(s1);
        if (lane == 0) { sm.bmax[0][j] = b0; sm.bmax[1][j] = b1; }
      }
      if (rd.first + rd.count == nbc) {     // last K round of the chunk
        __syncthreads();
        // ---- prefix max of the block maxima (warp h scans head h)
        if (warp < 2) {
          const int h = warp;
          float run = m_carry[h];
          for (int b0 = 0; b0 < nbc; b0 += 32) {
            const int j = b0 + lane;
            float v = j < nbc ? sm.bmax[h][j] : kNegInf;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
              const float u = __shfl_up_sync(0xffffffffu, v, o);
              if (lane >= o) v = fmaxf(v, u);
            }
            v = fmaxf(v, run);
            if (j < nbc) sm.mrun[h][j] = v;
            run = __shfl_sync(0xffffffffu, v, 31);
          }
        }
        __syncthreads();
        // ---- pass 1b: probabilities, requantised P (block-parallel)
        for (int j = warp; j < nbc; j += NW) {
          const int t = (c0 + j) * 32 + lane;
          const uint32_t page = table[c0 + j];
          const float vs = (t < kv_len && page < p.num_pages)
                               ? *reinterpret_cast<const float *>(
                                     p.vs + static_cast<size_t>(page) * p.scale_page_bytes +
                                     static_cast<size_t>(lane) * p.scale_row_bytes + kvh * 4)
                               : 0.0f;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float mj = sm.mrun[h][j];
            const float mp = j ? sm.mrun[h][j - 1] : m_carry[h];
            const float corr = exp_ref(__fsub_rn(mp, mj));
            const float pr = exp_ref(__fsub_rn(sm.S[h][j * 32 + lane], mj));
            const float ps = warp_tree_sum(pr);
            const float pv = (t < kv_len) ? __fmul_rn(pr, vs) : 0.0f;
            const float pm = __fmul_rn(warp_tree_max(fabsf(pv)), kInv127);
            const int q = quant1(pv, pm);
            sm.PQ[h][j * 32 + lane] = static_cast<int8_t>(q);   // 4 keys per word for dp4a
            if (lane == 0) {
              sm.corr[h][j] = corr;
              sm.psum[h][j] = ps;
              sm.pmax[h][j] = pm;
            }
          }
        }
      }
    } else {
      // ---- pass 2: P.V and the in-order recurrences (column-parallel)
      // lane: column quad dq of this warp's 32 columns, key quads kg and kg + 4;
      // 4 key rows x 4 columns are transposed with byte permutes so that one
      // dp4a multiplies 4 keys of one column with their 4 packed P values
      const int chunk = 2 * warp + (dq >> 2), coff = (dq & 3) << 2;
      for (int q = 0; q < rd.count; ++q) {
        const int j = rd.first + q;
        const int8_t *tile = pages[q];
        int a0[4] = {0, 0, 0, 0}, a1[4] = {0, 0, 0, 0};
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int kq = kg + 4 * half;
          int w[4];
#pragma unroll
          for (int r = 0; r < 4; ++r) {
            const int row = 4 * kq + r;
            w[r] = *reinterpret_cast<const int *>(tile + row * 128 + ((chunk ^ (row & 7)) << 4) + coff);
          }
          const int lo01 = __byte_perm(w[0], w[1], 0x5140), hi01 = __byte_perm(w[0], w[1], 0x7362);
          const int lo23 = __byte_perm(w[2], w[3], 0x5140), hi23 = __byte_perm(w[2], w[3], 0x7362);
          const int t[4] = {__byte_perm(lo01, lo23, 0x5410), __byte_perm(lo01, lo23, 0x7632),
                            __byte_perm(hi01, hi23, 0x5410), __byte_perm(hi01, hi23, 0x7632)};
          const int p0 = *reinterpret_cast<const int *>(&sm.PQ[0][j * 32 + 4 * kq]);
          const int p1 = *reinterpret_cast<const int *>(&sm.PQ[1][j * 32 + 4 * kq]);
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            a0[b] = __dp4a(t[b], p0, a0[b]);
            a1[b] = __dp4a(t[b], p1, a1[b]);
          }
        }
#pragma unroll
        for (int b = 0; b < 4; ++b) {
#pragma unroll
          for (int o = 8; o < 32; o <<= 1) {
            a0[b] += __shfl_xor_sync(0xffffffffu, a0[b], o);
            a1[b] += __shfl_xor_sync(0xffffffffu, a1[b], o);
          }
        }
        const int sel = (kg & 1) * 2;
        const int e0 = my_h ? (sel ? a1[2] : a1[0]) : (sel ? a0[2] : a0[0]);
        const int e1 = my_h ? (sel ? a1[3] : a1[1]) : (sel ? a0[3] : a0[1]);
        const float corr = sm.corr[my_h][j], pm = sm.pmax[my_h][j];
        res[0] = __fadd_rn(__fmul_rn(res[0], corr), __fmul_rn(i2f_small(e0), pm));
        res[1] = __fadd_rn(__fmul_rn(res[1], corr), __fmul_rn(i2f_small(e1), pm));
#pragma unroll
        for (int h = 0; h < 2; ++h)
          den_h[h] = __fadd_rn(__fmul_rn(den_h[h], sm.corr[h][j]), sm.psum[h][j]);
      }
      if (rd.first + rd.count == nbc) {      // last V round: carry the running max
        m_carry[0] = sm.mrun[0][nbc - 1];
        m_carry[1] = sm.mrun[1][nbc - 1];
      }
    }
    __syncthreads();   // buffer (r & 1) and the chunk arrays are reused afterwards
  }

  // ---- 1/den, per-head output quantisation (attention_gqa.h:522-546)
  const float rden = __fdiv_rn(1.0f, den_h[my_h]);
  const float o0 = __fmul_rn(res[0], rden), o1 = __fmul_rn(res[1], rden);
  float mx = fmaxf(fabsf(o0), fabsf(o1));
  // lanes of the same head differ in bits 0..3 of the lane id (dq and kg & 1)
#pragma unroll
  for (int o = 1; o < 16; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((lane & 15) == 0) sm.red[warp][lane >> 4] = mx;
  __syncthreads();
  float hm = 0.0f;
#pragma unroll
  for (int w = 0; w < NW; ++w) hm = fmaxf(hm, sm.red[w][my_h]);
  const float scale = __fmul_rn(hm, kInv127);
  const int h = kvh * 2 + my_h;
  char2 qv;
  qv.x = static_cast<char>(quant1(o0, scale));
  qv.y = static_cast<char>(quant1(o1, scale));
  *reinterpret_cast<char2 *>(p.o8 + static_cast<long>(seq) * p.o_rb + h * 128 + my_d0) = qv;
  if (warp == 0 && (lane & 15) == 0)
    *reinterpret_cast<float *>(p.os + static_cast<long>(seq) * p.os_rb + h * 4) = scale;
}

}  // namespace dec

// ---------------------------------------------------------------- host side
int attention_decode_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                            uint32_t num_pages, int kv_heads, int n_seqs, cudaStream_t s) {
  if (p.row_bytes % 16 || p.page_bytes % 16 || reinterpret_cast<uintptr_t>(k_pool) % 16 ||
      reinterpret_cast<uintptr_t>(v_pool) % 16)
    return Q3_ERR_ALIGN;
  const size_t smem = sizeof(dec::Smem);
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
