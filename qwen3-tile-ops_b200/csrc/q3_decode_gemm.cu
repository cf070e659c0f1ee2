// Decode-sized w8a8 GEMMs (one row per sequence, <= 64 rows) with the K-group
// reduction and the path's epilogues inside one kernel.
//
// The GEMM result is the group-ordered sum of per-group dequantised products
//     acc[m][n] = ((0 + pf_0) + pf_1) + ...,  pf_g = (f32(A_g . W_g) * ws[n]) * as[m][g]
// (ref_qwen3.py:151-157).  To stream the weights with many SMs, the K groups of
// one 128-feature output tile are spread over the CTAs of a thread-block cluster:
// each CTA computes the tensor-core products of its groups (tcgen05 kind::i8,
// weights as M = 128, tokens as N = 64), dequantises them into its own shared
// memory, and after a cluster barrier each CTA sums every group in order for a
// slice of the tokens, reading the other CTAs' partials over distributed shared
// memory.  The summing CTA then runs the epilogue for its tokens:
//   QKV     Q heads: head RMSNorm + RoPE + quant -> q8/qs; K heads: the same into
//           the KV page; V heads: quant into the KV page
//           (group_gemm.h:168-193, norm_rope_quant.h:17-86, main_big.cpp:183-209)
//   RESID   x += result (O and down, group_gemm.h:194-214), plus the tree sums of
//           x^2 over each 32-column block for the next RMSNorm (rmsnorm.h:34-81)
//   SWIGLU  silu(gate) * up over the 256 features of a quant group (two 128-
//           feature tiles in one cluster), per-256 quant (swiglu_quant.h:164-255)
// Weights are requested before the kernel waits on the one before it
// (programmatic dependent launch); activations, TMEM and every global write
// after.  Every mbarrier wait is
// bounded; a timeout sets bit 17 of the device error word and the CTA still
// takes part in both cluster barriers, so no peer is left waiting.
#include <cuda.h>

#include <mutex>

#include "q3_common.cuh"
#include "q3_decode_gemm.h"
#include "q3_gemm.h"
#include "q3_tc.cuh"

namespace q3 {

static __device__ unsigned int g_dgemm_error = 0;

int dgemm_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_dgemm_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_dgemm_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace dg {

using namespace tcx;

constexpr int NTOK = 64;
constexpr int EPI_WARPS = 8;                     // two per TMEM lane quadrant
constexpr int THREADS = (EPI_WARPS + 1) * 32;    // warp 8: TMA producer and MMA issuer
constexpr unsigned kErrTimeout = 1u << 17;

template <int NACC, int GPC, int GROUP>
struct Cfg {
  static constexpr int NB = GROUP / 128;                  // 128-byte K boxes per group
  static constexpr int A_BYTES = 128 * GROUP;             // one weight tile, one group
  static constexpr int B_BYTES = NTOK * GROUP;            // the activations of one group
  static constexpr int SLOT = NACC * A_BYTES + B_BYTES;   // operands of one group
  static constexpr int OPER = GPC * SLOT;
  static constexpr int PART = GPC * NACC * NTOK * 128 * 4;
  // each CTA receives, for its slice of the tokens, every group of every tile of
  // the cluster: as many bytes as it sends
  static constexpr int RCV = PART;
  static constexpr int REGION = OPER > PART + RCV ? OPER : PART + RCV;
  static constexpr int TMEM_RAW = GPC * NACC * NTOK;
  static constexpr int TMEM_COLS = TMEM_RAW <= 64 ? 64 : TMEM_RAW <= 128 ? 128 : 256;
};

template <int NACC, int GPC, int GROUP>
struct __align__(1024) Smem {
  // operands while the MMAs run; the dequantised partials [slot][acc][token][128] after
  alignas(1024) unsigned char region[Cfg<NACC, GPC, GROUP>::REGION];
  float as[NTOK][GPC];
  unsigned long long full[GPC], done, rcv_full;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t map_peer(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// bulk copy of `bytes` from this CTA's shared memory to a cluster peer's
// (distributed shared memory, no multicast), completion counted on the peer's
// mbarrier
__device__ __forceinline__ void push_to_peer(uint32_t dst_cluster, uint32_t src_cta, uint32_t bytes,
                                             uint32_t mbar_cluster) {
  asm volatile(
      "cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          dst_cluster),
      "r"(src_cta), "r"(bytes), "r"(mbar_cluster)
      : "memory");
}

// +1 on a counter that another GPU may poll (system scope, release: every write
// this thread made, or saw through a barrier, is visible before the count)
__device__ __forceinline__ void sys_signal(unsigned *ctr) {
  asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

template <int MODE, int NACC, int GPC, int GROUP, int TPCL, int GT>
__global__ void __launch_bounds__(THREADS, 1)
    k_dgemm(const __grid_constant__ CUtensorMap w0, const __grid_constant__ CUtensorMap w1,
            const __grid_constant__ CUtensorMap w2, const __grid_constant__ CUtensorMap act,
            const DgemmArgs p) {
  using C = Cfg<NACC, GPC, GROUP>;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem<NACC, GPC, GROUP> &sm = *reinterpret_cast<Smem<NACC, GPC, GROUP> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int tile = blockIdx.x, gs = blockIdx.y;        // output tile, slice of GPC groups
  constexpr int CL = GT / GPC;                          // group slices (cluster depth)
  constexpr int NC = TPCL * CL;                         // CTAs in the cluster
  const int crx = tile % TPCL;
  const int map = (MODE == DG_SWIGLU) ? 0 : (tile < p.t1 ? 0 : tile < p.t2 ? 1 : 2);
  const int row_in_map = (MODE == DG_SWIGLU)
                             ? tile * 128
                             : (tile - (map == 0 ? 0 : map == 1 ? p.t1 : p.t2)) * 128;

  pdl_trigger();
  if (tid == 0) {
    for (int i = 0; i < GPC; ++i) mbar_init(&sm.full[i], 1);
    mbar_init(&sm.done, 1);
    mbar_init(&sm.rcv_full, 1);
    sm.abort = 0;
    mbar_init_fence();
  }
  __syncthreads();
  // weights first: no earlier kernel writes them
  if (warp == EPI_WARPS && lane == 0) {
    const CUtensorMap *wm = map == 0 ? &w0 : map == 1 ? &w1 : &w2;
    for (int gl = 0; gl < GPC; ++gl) {
      const int g = gs * GPC + gl;
      unsigned char *base = sm.region + gl * C::SLOT;
      mbar_expect_tx(&sm.full[gl], C::SLOT);
      for (int b = 0; b < C::NB; ++b) {
        tma_2d(base + b * 16384, wm, g * GROUP + b * 128, row_in_map, &sm.full[gl]);
        if (NACC == 2)
          tma_2d(base + C::A_BYTES + b * 16384, &w1, g * GROUP + b * 128, row_in_map, &sm.full[gl]);
      }
    }
  }
  // Everything else waits for the kernel before.  TMEM is taken only after the
  // wait: a dependent that held TMEM while waiting could starve a predecessor
  // CTA that still has to allocate.
  pdl_wait();
  if (warp == EPI_WARPS) tmem_alloc<C::TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == EPI_WARPS) {
    // ------------------------------------------------ TMA producer + MMA issuer
    if (lane == 0) {
      for (int gl = 0; gl < GPC; ++gl) {
        const int g = gs * GPC + gl;
        unsigned char *bb = sm.region + gl * C::SLOT + NACC * C::A_BYTES;
        for (int b = 0; b < C::NB; ++b) tma_2d(bb + b * 8192, &act, g * GROUP + b * 128, 0, &sm.full[gl]);
      }
      constexpr uint32_t ID = idesc_i8(NTOK);
      bool ok = true;
      for (int gl = 0; gl < GPC && ok; ++gl) {
        if (!mbar_wait(&sm.full[gl], 0, &sm.abort)) { ok = false; break; }
        fence_after();
        const uint32_t sa = su32(sm.region + gl * C::SLOT), sb = sa + NACC * C::A_BYTES;
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const uint32_t dt = tmem + (gl * NACC + a) * NTOK;
          for (int b = 0; b < C::NB; ++b)
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              mma_i8(dt, sdesc_sw128(sa + a * C::A_BYTES + b * 16384 + ks * 32),
                     sdesc_sw128(sb + b * 8192 + ks * 32), ID, (b | ks) != 0);
        }
      }
      mma_commit(&sm.done);            // arrives once every MMA issued above has completed
      if (!ok) {
        atomicOr(&g_dgemm_error, kErrTimeout);
        sm.abort = 1;
        for (int gl = 0; gl < GPC; ++gl) mbar_wait(&sm.full[gl], 0, nullptr);   // copies landed
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------ dequantised partials -> smem
    // warp w: TMEM lanes 32 (w % 4) .. (feature rows), tokens 32 (w / 4) ..
    const int f = (warp & 3) * 32 + lane, c0 = (warp >> 2) * 32;
    for (int i = tid; i < NTOK * GPC; i += EPI_WARPS * 32) {
      const int m = i / GPC, gl = i % GPC;
      sm.as[m][gl] = m < p.M ? *reinterpret_cast<const float *>(p.a_scale + (long)m * p.as_rb +
                                                                  (gs * GPC + gl) * 4)
                             : 0.0f;
    }
    float wsv[NACC];
#pragma unroll
    for (int a = 0; a < NACC; ++a)
      wsv[a] = (MODE == DG_SWIGLU) ? p.ws[a][row_in_map + f] : p.ws[map][row_in_map + f];
    epi_sync();
    const bool ok = mbar_wait(&sm.done, 0, &sm.abort);
    fence_after();
    fence_proxy_async();               // operands (async proxy) -> partials (generic stores)
    if (ok) {
      if (c0 < p.M) {                  // (token columns of no row: nothing to keep)
      float *part = reinterpret_cast<float *>(sm.region);
      const uint32_t lane_addr = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
#pragma unroll
      for (int gl = 0; gl < GPC; ++gl) {
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          float *dst = part + static_cast<size_t>((gl * NACC + a) * NTOK) * 128 + f;
          int v[32];
          tmem_ld16(lane_addr + (gl * NACC + a) * NTOK + c0, *reinterpret_cast<int(*)[16]>(&v[0]));
          tmem_ld16(lane_addr + (gl * NACC + a) * NTOK + c0 + 16, *reinterpret_cast<int(*)[16]>(&v[16]));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i)
            dst[(c0 + i) * 128] = __fmul_rn(__fmul_rn(i2f_small(v[i]), wsv[a]), sm.as[c0 + i][gl]);
        }
      }
      }
    } else if (lane == 0) {
      atomicOr(&g_dgemm_error, kErrTimeout);
      sm.abort = 1;
    }
    __syncwarp();
  }

  if constexpr (MODE == DG_PART) {
    // ---------------------------------------------- tensor-parallel partials -> every rank
    // Token m of this CTA's partial (512 contiguous bytes of features) goes to
    // row m of slot slot0 + gs of each rank's receive buffer; a CTA whose MMAs
    // timed out still signals (its data is void, the error bit says so), so no
    // rank waits on it for long.
    fence_before();
    __syncthreads();
    fence_after();
    if (warp < EPI_WARPS && !sm.abort) {
      const float *part = reinterpret_cast<const float *>(sm.region);
      for (int m = warp; m < p.M; m += EPI_WARPS) {
        const float4 v = reinterpret_cast<const float4 *>(part + static_cast<size_t>(m) * 128)[lane];
        const size_t off = (static_cast<size_t>(p.slot0 + gs) * p.M + m) * p.H + tile * 128;
        for (int q = 0; q < p.ndst; ++q) reinterpret_cast<float4 *>(p.dst[q] + off)[lane] = v;
      }
    }
    // the barrier orders every thread's stores before thread 0's release at
    // system scope (release is cumulative), which the consumers acquire
    __syncthreads();
    if (tid == 0) {
      for (int q = 0; q < p.ndst; ++q) sys_signal(p.sig[q]);
      if (tile == 0 && gs == 0)
        for (int q = 0; q < p.ndst; ++q) p.expect[q] += static_cast<unsigned>(p.inc[q]);
    }
    if (warp == EPI_WARPS) tmem_dealloc<C::TMEM_COLS>(tmem);
    return;
  }

  // ---------------------------------------------- every partial of the cluster is in smem
  fence_proxy_async();                                  // partial stores -> bulk copies
  constexpr int TPC = NTOK / NC;                        // tokens reduced by each CTA
  const int rank = crx + TPCL * gs;
  // rows of token slice r that exist (a few-row step sends and receives only those)
  auto slice_rows = [&](int r) { return max(0, min(TPC, p.M - r * TPC)); };
  if (tid == 0)                                         // the slices this CTA will receive
    mbar_expect_tx(&sm.rcv_full, static_cast<unsigned>(NC * GPC * NACC * slice_rows(rank) * 128 * 4));
  fence_before();
  cluster_sync();
  fence_after();
  // Push: slice r (tokens r*TPC ..) of each of my partials [gl][a] goes to CTA r,
  // into its receive buffer at [group][acc][my tile][TPC][128].
  if (warp == EPI_WARPS) {
    const uint32_t part0 = su32(sm.region), rcv0 = part0 + C::PART;
    constexpr int NCOPY = GPC * NACC * NC;
    for (int c = lane; c < NCOPY; c += 32) {
      const int r = c % NC, a = (c / NC) % NACC, gl = c / (NC * NACC);
      const int rows = slice_rows(r);
      if (rows == 0) continue;
      const int g = gs * GPC + gl;
      const uint32_t src = part0 + static_cast<uint32_t>((((gl * NACC + a) * NTOK + r * TPC) * 128) * 4);
      const uint32_t dst = rcv0 + static_cast<uint32_t>(((((g * NACC + a) * TPCL + crx) * TPC) * 128) * 4);
      push_to_peer(map_peer(dst, r), src, static_cast<uint32_t>(rows * 128 * 4),
                   map_peer(su32(&sm.rcv_full), r));
    }
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // my sources are read
    __syncwarp();
  }

  if (warp < EPI_WARPS) {
    const bool got = mbar_wait(&sm.rcv_full, 0, nullptr);
    if (!got && tid == 0) atomicOr(&g_dgemm_error, kErrTimeout);
    const float *rcv = reinterpret_cast<const float *>(sm.region + C::PART);
    // group g of cluster tile tt, accumulator a, token mi of my slice; a lane
    // holds features lane + 32k (k < 4); every load is issued before the sums
    auto load_groups = [&](int tt, int a, int mi, float (&v)[GT][4]) {
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        const float *src = rcv + ((((g * NACC + a) * TPCL + tt) * TPC + mi) * 128 + lane);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[g][k] = src[32 * k];
      }
    };
    auto sum_groups = [&](const float (&v)[GT][4], float (&out)[4]) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        out[k] = 0.0f;
#pragma unroll
        for (int g = 0; g < GT; ++g) out[k] = __fadd_rn(out[k], v[g][k]);   // group order
      }
    };
    for (int mi = warp; mi < TPC; mi += EPI_WARPS) {
      const int m = rank * TPC + mi;
      if (m >= p.M) continue;
      if (MODE == DG_QKV) {
        const int h = tile;                              // head: Q heads, then K, then V
        const int pos = p.pos[m];
        const bool is_v = h >= p.heads + p.kv_heads;
        float nwv[4], cs[2], sn[2];
        if (!is_v) {
          const float *nw = h < p.heads ? p.nq : p.nk;
#pragma unroll
          for (int k = 0; k < 4; ++k) nwv[k] = nw[lane + 32 * k];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            cs[k] = p.cos_t[static_cast<size_t>(pos) * 64 + lane + 32 * k];
            sn[k] = p.sin_t[static_cast<size_t>(pos) * 64 + lane + 32 * k];
          }
        }
        float pv[GT][4], v[4];
        load_groups(0, 0, mi, pv);
        sum_groups(pv, v);
        if (!is_v) {
          float ss = 0.0f;
#pragma unroll
          for (int k = 0; k < 4; ++k) ss = __fadd_rn(ss, warp_tree_sum(__fmul_rn(v[k], v[k])));
          ss = __fadd_rn(__fmul_rn(ss, p.inv_hd), kEps);
          const float r = rsqrt_ref(ss);
#pragma unroll
          for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], r), nwv[k]);
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const float l = v[k], rr = v[k + 2];
            v[k] = __fsub_rn(__fmul_rn(l, cs[k]), __fmul_rn(rr, sn[k]));
            v[k + 2] = __fadd_rn(__fmul_rn(l, sn[k]), __fmul_rn(rr, cs[k]));
          }
        }
        float mx = 0.0f;
#pragma unroll
        for (int k = 0; k < 4; ++k) mx = fmaxf(mx, fabsf(v[k]));
        mx = warp_tree_max(mx);
        const float scale = __fmul_rn(mx, kInv127);
        int qv[4];
        quant_n_absmax(v, scale, qv);
        if (h < p.heads) {
          int8_t *dst = p.q8 + static_cast<size_t>(m) * p.heads * 128 + h * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = static_cast<int8_t>(qv[k]);
          if (lane == 0) p.qs[m * p.heads + h] = scale;
        } else {
          const int kvh = is_v ? h - p.heads - p.kv_heads : h - p.heads;
          const uint32_t page = p.tables[static_cast<size_t>(m) * p.max_pages + pos / 32];
          const size_t row = static_cast<size_t>(page) * 32 + (pos % 32);
          const int kw = p.kv_heads * 128;
          int8_t *dst = reinterpret_cast<int8_t *>(is_v ? p.pv : p.pk) + row * kw + kvh * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = static_cast<int8_t>(qv[k]);
          if (lane == 0)
            reinterpret_cast<float *>(is_v ? p.pvs : p.pks)[row * p.kv_heads + kvh] = scale;
        }
      } else if (MODE == DG_RESID) {
        float *xr = p.x + static_cast<size_t>(m) * p.H + tile * 128;
        float xv[4], pv[GT][4], v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) xv[k] = xr[lane + 32 * k];
        load_groups(0, 0, mi, pv);
        sum_groups(pv, v);
        float bs[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          xv[k] = __fadd_rn(xv[k], v[k]);
          bs[k] = warp_tree_sum(__fmul_rn(xv[k], xv[k]));   // block tile*4 + k
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) xr[lane + 32 * k] = xv[k];
        if (lane < 4) {
          const float b = lane == 0 ? bs[0] : lane == 1 ? bs[1] : lane == 2 ? bs[2] : bs[3];
          p.bsum[static_cast<size_t>(m) * (p.H / 32) + tile * 4 + lane] = b;
        }
      } else {
        // SWIGLU: tiles 2j, 2j+1 of the cluster = the 256 features of quant group j
        float gv[2][4], uv[2][4];
        {
          float pg[GT][4], pu[GT][4];
#pragma unroll
          for (int tt = 0; tt < 2; ++tt) {
            load_groups(tt, 0, mi, pg);
            load_groups(tt, 1, mi, pu);
            sum_groups(pg, gv[tt]);
            sum_groups(pu, uv[tt]);
          }
        }
        float sw[8];
        float mx = 0.0f;
        float en[8];                   // exp(-g) of the lane's 8 features in one batch
#pragma unroll
        for (int i = 0; i < 8; ++i) en[i] = __fmul_rn(gv[i / 4][i % 4], -1.0f);
        exp_ref_fast_n(en, g_exp2_t256);
#pragma unroll
        for (int tt = 0; tt < 2; ++tt) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            float e = __fadd_rn(en[tt * 4 + k], 1.0f);
            e = __frcp_rn(e);
            sw[tt * 4 + k] = __fmul_rn(__fmul_rn(gv[tt][k], e), uv[tt][k]);
            mx = fmaxf(mx, fabsf(sw[tt * 4 + k]));
          }
        }
        mx = warp_tree_max(mx);
        const float scale = __fmul_rn(mx, kInv127);
        const int grp = tile / 2;
        int8_t *dst = p.s8 + static_cast<size_t>(m) * p.I + grp * 256;
        int qv[8];
        quant_n_absmax(sw, scale, qv);
#pragma unroll
        for (int k = 0; k < 8; ++k) dst[lane + 32 * k] = static_cast<int8_t>(qv[k]);
        if (lane == 0) p.ss[static_cast<size_t>(m) * (p.I / 256) + grp] = scale;
      }
    }
    __syncwarp();
  }

  // ---------------------------------------------- peers are done reading my partials
  fence_before();
  cluster_sync();
  fence_after();
  if (warp == EPI_WARPS) tmem_dealloc<C::TMEM_COLS>(tmem);
}

// ---------------------------------------------------------------- host side
template <int MODE, int NACC, int GPC, int GROUP, int TPCL, int GT>
static int launch(const CUtensorMap (&wm)[3], const CUtensorMap &am, const DgemmArgs &p, int tiles,
                  cudaStream_t s) {
  using C = Cfg<NACC, GPC, GROUP>;
  auto kern = k_dgemm<MODE, NACC, GPC, GROUP, TPCL, GT>;
  const size_t smem = sizeof(Smem<NACC, GPC, GROUP>) + 1024;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  if (attr != cudaSuccess) {
    q3h::set_cuda_error(attr);
    return Q3_ERR_CUDA;
  }
  static_assert(GT % GPC == 0 && TPCL * (GT / GPC) <= 8 && NTOK % (TPCL * (GT / GPC)) == 0,
                "cluster shape");
  if ((MODE != DG_PART && p.G != GT) || tiles % TPCL) return Q3_ERR_SHAPE;
  static_assert(C::TMEM_RAW <= 256, "TMEM columns");
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(tiles, p.G / GPC);
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = TPCL;
  at[0].val.clusterDim.y = MODE == DG_PART ? 1 : p.G / GPC;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  q3h::timer_begin(q3h::TIMER_GEMM, s);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, wm[0], wm[1], wm[2], am, p);
  int st;
  if (e != cudaSuccess) {
    q3h::count_launch();
    cudaGetLastError();
    q3h::set_cuda_error(e);
    st = Q3_ERR_CUDA;
  } else {
    st = q3h::launch_status();
  }
  q3h::timer_end(q3h::TIMER_GEMM, s);
  return st;
}

}  // namespace dg

int dgemm_launch(int mode, int nmaps, const int8_t *const *w, const int *rows, const int8_t *a,
                 long a_rb, int K, int group, const DgemmArgs &args, cudaStream_t s, long w_rb) {
  DgemmArgs p = args;
  if (w_rb == 0) w_rb = K;
  if (p.M < 1 || p.M > dg::NTOK || K % group || a_rb % 16 || w_rb % 16 || w_rb < K ||
      reinterpret_cast<uintptr_t>(a) % 16)
    return Q3_ERR_SHAPE;
  p.K = K;
  p.G = K / group;
  CUtensorMap wm[3], am;
  int tiles = 0;
  for (int i = 0; i < 3; ++i) {
    const int j = i < nmaps ? i : nmaps - 1;
    if (rows[j] % 128 || reinterpret_cast<uintptr_t>(w[j]) % 16) return Q3_ERR_SHAPE;
    if (!tc::make_map(&wm[i], w[j], rows[j], K, w_rb, 128)) return Q3_ERR_CUDA;
  }
  if (mode == DG_SWIGLU) {
    tiles = rows[0] / 128;
  } else {
    p.t1 = rows[0] / 128;
    p.t2 = p.t1 + (nmaps > 1 ? rows[1] / 128 : 0);
    tiles = p.t2 + (nmaps > 2 ? rows[2] / 128 : 0);
  }
  if (!tc::make_map(&am, a, p.M, K, a_rb, dg::NTOK)) return Q3_ERR_CUDA;
  // the Qwen3-0.6B shapes: QKV K = 1024 (4 groups of 256), O K = 2048 (16 of 128),
  // gate/up K = 1024 (4 of 256), down K = 3072 (12 of 256)
  if (mode == DG_QKV && group == 256 && p.G == 4)
    return dg::launch<DG_QKV, 1, 1, 256, 1, 4>(wm, am, p, tiles, s);
  if (mode == DG_RESID && group == 128 && p.G == 16)
    return dg::launch<DG_RESID, 1, 2, 128, 1, 16>(wm, am, p, tiles, s);
  if (mode == DG_RESID && group == 256 && p.G == 12)
    return dg::launch<DG_RESID, 1, 3, 256, 1, 12>(wm, am, p, tiles, s);
  if (mode == DG_SWIGLU && group == 256 && p.G == 4)
    return dg::launch<DG_SWIGLU, 2, 1, 256, 2, 4>(wm, am, p, tiles, s);
  if (mode == DG_PART) {
    if (p.ndst < 1 || p.ndst > kTpMaxRanks || !p.expect || rows[0] != p.H) return Q3_ERR_SHAPE;
    for (int q = 0; q < p.ndst; ++q) {
      if (!p.dst[q] || !p.sig[q]) return Q3_ERR_NULL;
      if (reinterpret_cast<uintptr_t>(p.dst[q]) % 16) return Q3_ERR_ALIGN;
    }
    if (group == 128) return dg::launch<DG_PART, 1, 1, 128, 1, 1>(wm, am, p, tiles, s);
    if (group == 256) return dg::launch<DG_PART, 1, 1, 256, 1, 1>(wm, am, p, tiles, s);
  }
  return Q3_ERR_SHAPE;
}

}  // namespace q3
