// Per-K-group w8a8 GEMM on a pair of SMs (tcgen05 cta_group::2, kind::i8) for
// the prefill's many-row residual GEMMs (O and down: kernels/group_gemm.h:194-214
// with the bits of q3_gemm_tc.cu and so of the CUDA-core path).
//
// Why a pair.  One CTA's 128-feature x 128-token tile needs 1/64 byte of
// operands per MAC from L2 into shared memory.  A pair computes one MMA of
// M = 256 features x N = NT tokens: each CTA loads its own 128 weight rows and
// its own NT/2 token rows, and the MMA reads the operands of both CTAs, so a
// 256-feature x 192-token tile costs (128 + 96) / (128 x 192) byte per MAC per
// SM, 0.57 of the single CTA's.  Measured on the config-2 shapes at 65536 rows
// it wins for the residual GEMMs, whose many K-groups keep the MMAs ahead of
// the epilogue (O 489 against 573 us, down 477 against 535); the GEMMs with
// four K-groups and a per-token epilogue stay on the single-CTA kernel.
//
// Orientation as in q3_gemm_tc.cu: M = weight rows (output features), N =
// tokens, K = input features.  The accumulator of a K-group lives in both
// CTAs' TMEM (CTA r: features 128 r .. 128 r + 127, all NT tokens), so every
// CTA dequantises its own 128 features for all NT tokens:
//     acc[n][m] = acc[n][m] + (f32(part[n][m]) * b_scale[n]) * a_scale[m][g]
// (ref_qwen3.py:152-157), group after group, while the MMAs of the next groups
// fill the other TMEM buffers.
//
// Roles.  Rank 0 of the pair (the leader) issues every MMA and owns the
// stage-full barriers: both CTAs' TMA copies complete on the leader's barrier
// (the cta_group::2 form of the copy), the leader's producer announces the
// pair's bytes, and each MMA group's completion is committed to the barriers
// of both CTAs.  Both CTAs' epilogue warps release a TMEM buffer on the
// leader's barrier.  Persistent: each pair walks a contiguous run of tiles.
// Every mbarrier wait is bounded (about one second); a timeout sets bit 16 of
// the device error word and tells the peer CTA to stop too.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "q3_common.cuh"
#include "q3_gemm.h"
#include "q3_tc.cuh"

namespace q3 {

static __device__ unsigned int g_gemm2_error = 0;

int gemm2_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm2_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemm2_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace tc2 {

using namespace tcx;

constexpr unsigned kErrPairTimeout = 1u << 16;   // as q3_gemm_tc.cu's timeout
// Epilogue warps (a multiple of 4: one TMEM lane quadrant each, the tokens
// split between the warps of a quadrant).  With the producer and the MMA warp,
// at most ceil(warps / 4) warps share an SM sub-partition's 16K registers,
// which bounds the registers per thread (its running sums stay in registers).
#ifndef Q3_PAIR_EPI_WARPS
#define Q3_PAIR_EPI_WARPS 12
#endif
#ifndef Q3_PAIR_NT
#define Q3_PAIR_NT 192            // tokens of a pair tile (MMA N)
#endif
#ifndef Q3_PAIR_LDW
#define Q3_PAIR_LDW 16            // TMEM columns per load
#endif
constexpr int EPI_WARPS = Q3_PAIR_EPI_WARPS;
constexpr int THREADS = (EPI_WARPS + 2) * 32;
constexpr uint32_t kAccBias = 0x4B400000u;      // accumulators start at 1.5 * 2^23
constexpr float kAccBiasF = 12582912.0f;
constexpr int TMEM_COLS = 512;

template <int MODE>
struct Cfg {
  static constexpr int NACC = 1;
  static constexpr int NT = Q3_PAIR_NT;
  // TMEM accumulator buffers: as many K-groups in flight as TMEM holds (<= 4)
  static constexpr int NBUF = TMEM_COLS / (NACC * NT) >= 4 ? 4 : TMEM_COLS / (NACC * NT);
  static constexpr int HALF = NT / 2;                           // token rows each CTA loads
  static constexpr int A_BYTES = 128 * 128;                     // 128 weight rows x 128 K-bytes
  static constexpr int B_BYTES = HALF * 128;
  static constexpr int STAGE_BYTES = NACC * A_BYTES + B_BYTES;
  static constexpr int HT = NT / (EPI_WARPS / 4);               // tokens per epilogue warp
  static constexpr int LDW = HT % Q3_PAIR_LDW == 0 ? Q3_PAIR_LDW : 16;
  // stage ring: as deep as shared memory allows next to the staging buffers
  static constexpr int OTHER = 16 * NT * 4 + 2048;
  static constexpr int STAGES_FIT = (225 * 1024 - OTHER) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static_assert(HT % LDW == 0 && LDW % 16 == 0, "TMEM load width");
  static_assert(NBUF >= 2 && NBUF * NACC * NT <= TMEM_COLS, "TMEM");
};

template <int MODE>
struct __align__(1024) Smem {
  using C = Cfg<MODE>;
  alignas(1024) int8_t stage[C::STAGES][C::STAGE_BYTES];
  alignas(16) float ascale[16 * C::NT];           // a_scale of the token tile, [group][token]
  unsigned long long full[C::STAGES], empty[C::STAGES], tfull[C::NBUF], tempty[C::NBUF], done;
  uint32_t tmem_base;
  int abort;
};

struct PairArgs {
  GemmArgs g;
  int groups;   // K / group
  int boxes;    // group / 128
};

// ---------------------------------------------------------------- PTX pieces
__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t at_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// arrive on a barrier of another CTA of the cluster (no data handed over with it:
// the TMEM reads it releases are ordered by the tcgen05 fences around it)
__device__ __forceinline__ void arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void st_at_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}
// 2D tile copy into this CTA's shared memory, completing on the barrier at
// `bar` (a cluster address: the leader's stage-full barrier)
__device__ __forceinline__ void tma_2d_to(void *dst, const CUtensorMap *m, int x, int y,
                                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(su32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t dt, uint64_t ad, uint64_t bd, uint32_t id) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, 1, 0;\n"
      " tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(dt),
      "l"(ad), "l"(bd), "r"(id)
      : "memory");
}
// arrive on the barrier at cluster address `bar` once the pair's MMAs so far complete
__device__ __forceinline__ void commit_pair(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem) {   // one warp per CTA
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   su32(dst_smem)),
               "n"(TMEM_COLS)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base) {      // one warp per CTA
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "n"(TMEM_COLS)
               : "memory");
}
// instruction descriptor: s32 accumulate, s8 x s8, K-major A and B, M = 256, N = n
__host__ __device__ constexpr uint32_t idesc_pair(int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         ((256u >> 4) << 24);
}

// LDW consecutive TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, int (&v)[16]) { tmem_ld16(taddr, v); }
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, int (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]),
        "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]),
        "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const PairArgs args) {
  using C = Cfg<MODE>;
  constexpr int STAGES = C::STAGES, NT = C::NT, HT = C::HT, NACC = C::NACC, NBUF = C::NBUF;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem<MODE> &sm = *reinterpret_cast<Smem<MODE> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const GemmArgs &p = args.g;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = args.groups, NB = args.boxes;
  const int tiles_x = p.N / 256;
  const int ntiles = tiles_x * ((p.M + NT - 1) / NT);
  const int tile_it = G * NB;
  // pair p takes a contiguous run of tiles (feature tile fastest), so the token
  // tile and its activation scales change only every tiles_x tiles
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int per_pair = (ntiles + npairs - 1) / npairs;
  const int t_begin = min(ntiles, pair * per_pair), t_end = min(ntiles, t_begin + per_pair);
  auto tile_rows = [&](int tile) { return (tile % tiles_x) * 256; };
  auto tile_m0 = [&](int tile) { return (tile / tiles_x) * NT; };
  const int f = (warp & 3) * 32 + lane, c0 = (warp >> 2) * HT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < NBUF; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], 2 * EPI_WARPS);   // both CTAs' epilogue warps
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == EPI_WARPS + 1) tmem_alloc_pair(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  if (warp < EPI_WARPS) {                        // every accumulator starts at the bias
#pragma unroll
    for (int b = 0; b < NBUF * NACC; ++b)
#pragma unroll
      for (int c = 0; c < HT; c += 16) tmem_st16(lane_addr + b * NT + c0 + c, kAccBias);
    tmem_wait_st();
  }
  fence_before();
  cluster_sync_all();                            // both CTAs: barriers ready, TMEM biased
  fence_after();

  const uint32_t full_l = at_rank(su32(&sm.full[0]), 0);      // leader's barriers
  const uint32_t tempty_l = at_rank(su32(&sm.tempty[0]), 0);
  const uint32_t empty_p = at_rank(su32(&sm.empty[0]), 1);    // rank 1's barriers
  const uint32_t tfull_p = at_rank(su32(&sm.tfull[0]), 1);
  const uint32_t other = rank ^ 1u;
  const uint32_t abort_o = at_rank(su32(&sm.abort), other);
  auto fail = [&]() {
    atomicOr(&g_gemm2_error, kErrPairTimeout);
    sm.abort = 1;
    st_at_u32(abort_o, 1u);
  };

  if (warp == EPI_WARPS) {
    // ------------------------------------------------------------ TMA producer
    int issued = 0;
    bool ok = true;
    int it = 0;
    for (int tile = t_begin; tile < t_end && ok; ++tile) {
      const int row0 = tile_rows(tile) + static_cast<int>(rank) * 128, m0 = tile_m0(tile);
      const int mrow = m0 + static_cast<int>(rank) * C::HALF;
      for (int ti = 0; ti < tile_it && ok; ++ti, ++it) {
        const int st = it % STAGES;
        if (lane == 0) {
          if (!mbar_wait(&sm.empty[st], ((it / STAGES) & 1) ^ 1, &sm.abort)) {
            ok = false;
          } else {
            if (leader) mbar_expect_tx(&sm.full[st], 2 * C::STAGE_BYTES);   // the pair's bytes
            const int k0 = ti * 128;
            const uint32_t fb = full_l + st * 8;
            int8_t *dst = sm.stage[st];
            tma_2d_to(dst, &tmA, k0, row0, fb);
            tma_2d_to(dst + NACC * C::A_BYTES, &tmB, k0, mrow, fb);
            ++issued;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
    }
    if (!ok && lane == 0) {
      fail();
      if (leader) {                              // let the pair's copies land
        for (int i = max(0, issued - STAGES); i < issued; ++i)
          mbar_wait(&sm.full[i % STAGES], (i / STAGES) & 1, nullptr);
      } else {
        const uint64_t t0 = gtime();
        while (gtime() - t0 < 2000000ull) {
        }
      }
    }
  } else if (warp == EPI_WARPS + 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      constexpr uint32_t ID = idesc_pair(NT);
      bool ok = true;
      int it = 0;
      const int my_tiles = t_end - t_begin;
      for (int gi = 0; gi < my_tiles * G && ok; ++gi) {
        const int buf = gi % NBUF;
        if (lane == 0 && !mbar_wait(&sm.tempty[buf], ((gi / NBUF) & 1) ^ 1, &sm.abort)) ok = false;
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        fence_after();
        for (int box = 0; box < NB && ok; ++box, ++it) {
          const int st = it % STAGES;
          if (lane == 0) {
            if (!mbar_wait(&sm.full[st], (it / STAGES) & 1, &sm.abort)) {
              ok = false;
            } else {
              fence_after();
              const uint32_t sa = su32(sm.stage[st]);
              const uint32_t sb = sa + NACC * C::A_BYTES;
#pragma unroll
              for (int a = 0; a < NACC; ++a) {
                const uint32_t dt = tmem + (buf * NACC + a) * NT;
#pragma unroll
                for (int ks = 0; ks < 4; ++ks)
                  mma_pair(dt, sdesc_sw128(sa + a * C::A_BYTES + ks * 32), sdesc_sw128(sb + ks * 32), ID);
              }
              commit_pair(su32(&sm.empty[st]));   // both CTAs may refill the stage
              commit_pair(empty_p + st * 8);
            }
          }
          ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        }
        if (ok && lane == 0) {
          commit_pair(su32(&sm.tfull[buf]));      // the group's sums are in both TMEMs
          commit_pair(tfull_p + buf * 8);
        }
      }
      if (lane == 0) {                           // every MMA issued has completed
        commit_pair(su32(&sm.done));
        mbar_wait(&sm.done, 0, nullptr);
      }
      if (!ok && lane == 0) fail();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    bool ok = true;
    int gi = 0, tcount = 0;
    int scales_m0 = -1;
    for (int tile = t_begin; tile < t_end && ok; ++tile, ++tcount) {
      const int row0 = tile_rows(tile), m0 = tile_m0(tile);
      const int r0 = row0 + static_cast<int>(rank) * 128;   // this CTA's 128 features
      const int mvalid = min(NT, p.M - m0);
      if (m0 != scales_m0) {
        epi_sync();
        for (int i = threadIdx.x; i < NT * G; i += EPI_WARPS * 32) {
          const int g = i / NT, m = i % NT;
          sm.ascale[i] = (m < mvalid)
                             ? *reinterpret_cast<const float *>(p.a_scale + (long)(m0 + m) * p.as_rb + g * 4)
                             : 0.0f;
        }
        epi_sync();
        scales_m0 = m0;
      }
      const int n = r0 + f;
      if (MODE == EPI_ADD) {
        // the residual rows this warp adds to after the groups: into L2 now, so
        // the epilogue's loads do not wait on DRAM (one 128-byte line per row)
        const char *seg = p.out + static_cast<long>(r0 + (warp & 3) * 32) * 4;
#pragma unroll
        for (int i = lane; i < HT; i += 32)
          if (c0 + i < mvalid)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(seg + (long)(m0 + c0 + i) * p.out_rb));
      }
      float bs[NACC];
      bs[0] = p.b_scale[n];
      float accf[NACC][HT];
#pragma unroll
      for (int a = 0; a < NACC; ++a)
#pragma unroll
        for (int i = 0; i < HT; ++i) accf[a][i] = 0.0f;
      for (int g = 0; g < G; ++g, ++gi) {
        const int buf = gi % NBUF;
        if (!mbar_wait(&sm.tfull[buf], (gi / NBUF) & 1, &sm.abort)) {
          ok = false;
          break;
        }
        fence_after();
        const float *asg = sm.ascale + g * NT + c0;
#pragma unroll
        for (int a = 0; a < NACC; ++a) {
          const uint32_t col = lane_addr + (buf * NACC + a) * NT + c0;
#pragma unroll
          for (int c = 0; c < HT; c += C::LDW) {
            int v[C::LDW];
            tmem_ld_cols(col + c, v);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < C::LDW; i += 16) tmem_st16(col + c + i, kAccBias);
#pragma unroll
            for (int i = 0; i < C::LDW; i += 4) {
              const float4 as4 = *reinterpret_cast<const float4 *>(asg + c + i);
              const float asv[4] = {as4.x, as4.y, as4.z, as4.w};
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float x = __fsub_rn(__int_as_float(v[i + j]), kAccBiasF);   // exact
                accf[a][c + i + j] = __fadd_rn(accf[a][c + i + j], __fmul_rn(__fmul_rn(x, bs[a]), asv[j]));
              }
            }
          }
        }
        tmem_wait_st();
        fence_before();
        __syncwarp();
        if (lane == 0) {
          if (leader) mbar_arrive(&sm.tempty[buf]);
          else arrive_remote(tempty_l + buf * 8);
        }
      }
      if (!ok) break;

      {
#pragma unroll
        for (int c = 0; c < HT; c += 16) {     // 16 tokens: every load before its stores
          float xv[16];
          if (MODE == EPI_ADD) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              xv[i] = (c0 + c + i < mvalid)
                          ? reinterpret_cast<const float *>(p.out + (long)(m0 + c0 + c + i) * p.out_rb)[n]
                          : 0.0f;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            if (c0 + c + i < mvalid) {
              float *row = reinterpret_cast<float *>(p.out + (long)(m0 + c0 + c + i) * p.out_rb);
              row[n] = (MODE == EPI_ADD) ? __fadd_rn(xv[i], accf[0][c + i]) : accf[0][c + i];
            }
          }
        }
      }
    }
    if (!ok && lane == 0) fail();
  }

  // ---------------------------------------------------------------- teardown
  fence_before();
  __syncthreads();
  cluster_sync_all();      // the peer is done with this CTA's shared memory and TMEM
  fence_after();
  if (warp == EPI_WARPS + 1) tmem_dealloc_pair(tmem);
}

// ---------------------------------------------------------------- host side
template <int MODE>
static int launch(const GemmArgs &p, cudaStream_t s) {
  using C = Cfg<MODE>;
  CUtensorMap ta, tb;
  const uint64_t K = p.K;
  if (!tc::make_map(&ta, p.b, p.N, K, p.b_rb, 128)) return Q3_ERR_CUDA;
  if (!tc::make_map(&tb, p.a, p.M, K, p.a_rb, C::HALF)) return Q3_ERR_CUDA;
  const size_t smem = sizeof(Smem<MODE>) + 1024;
  cudaLaunchConfig_t cfg{};
  cfg.blockDim = dim3(THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = 2;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  // pairs resident at once (one CTA per SM; an SM without a partner in its
  // cluster group stays idle), found once per mode
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  static int max_pairs = 0;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(k_gemm_pair<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem);
    if (attr != cudaSuccess) return;
    cudaLaunchConfig_t q = cfg;
    q.gridDim = dim3(2);
    int n = 0;
    attr = cudaOccupancyMaxActiveClusters(&n, k_gemm_pair<MODE>, &q);
    max_pairs = n;
  });
  if (attr != cudaSuccess) {
    q3h::set_cuda_error(attr);
    return Q3_ERR_CUDA;
  }
  if (max_pairs < 1) return Q3_ERR_CAPACITY;
  PairArgs a{p, p.K / p.group, p.group / 128};
  const int ntiles = (p.N / 256) * ((p.M + C::NT - 1) / C::NT);
  cfg.gridDim = dim3(2 * (ntiles < max_pairs ? ntiles : max_pairs));
  q3h::timer_begin(q3h::TIMER_GEMM, s);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, k_gemm_pair<MODE>, ta, tb, a);
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

}  // namespace tc2

// Residual GEMMs (O, down) of 1024 rows and more whose features fill 256-row
// pair tiles; q3_gemm_tc.cu's gemm_tc checked the rest.  (A STORE epilogue
// compiles from the same template but measured slower than the single-CTA
// kernel at four K-groups, so it is not dispatched here.)
bool gemm_pair_eligible(const GemmArgs &p) {
  return p.mode == EPI_ADD && p.M >= 1024 && p.N % 256 == 0;
}

int gemm_pair(const GemmArgs &p, cudaStream_t s) {
  if (p.mode == EPI_ADD) return tc2::launch<EPI_ADD>(p, s);
  return Q3_ERR_SHAPE;
}

}  // namespace q3
