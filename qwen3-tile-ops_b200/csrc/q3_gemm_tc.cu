// Per-K-group w8a8 GEMM on the 5th-generation tensor cores (tcgen05, kind::i8),
// with the epilogues of kernels/group_gemm.h:27-222, swiglu_quant.h:105-255 and
// lm_argmax.h:72-182.  Bit-identical to the CUDA-core path (q3_gemm_simt.cu).
//
// Orientation: the MMA's M dimension is 128 WEIGHT rows (output features), its
// N dimension a tile of NTOK tokens (activation rows), K the input features.
// One TMEM accumulator [128 lanes = features][NTOK columns = tokens] int32 per
// K-group; several of them rotate, so the epilogue warps dequantise group g
//     acc[n][m] = acc[n][m] + (f32(part[n][m]) * b_scale[n]) * a_scale[m][g]
// (the reference's order, ref_qwen3.py:152-157) while the MMA warp runs g+1.
// A thread of the epilogue owns one feature row, so every per-feature reduction
// of the reference (head RMSNorm, head/group absmax) is a reduction over lanes.
//
// The dequantisation is the epilogue's inner loop (3 rounded float ops per
// output and group), so it is kept lean: each accumulator starts at the bit
// pattern of 1.5 * 2^23 (written back by the epilogue after it reads a
// buffer), so the int32 group sum converts to float with one exact
// subtraction.  (Packed f32x2 arithmetic is not used: ptxas may contract a
// packed multiply and add into one fused operation, which changes the bits.)
//
// Persistent: one CTA per SM walks the (feature tile, token tile) list; the stage
// ring and the TMEM buffers run on across tiles, so a tile's epilogue overlaps
// the next tile's copies and MMAs.  Warps: 0 .. EPI_WARPS-1 epilogue (EPI_WARPS/4
// per TMEM lane quadrant: warp w reads lanes 32 (w % 4) .. for one slice of the
// tokens), then the TMA producer, then the MMA issuer and TMEM owner.  Operands
// arrive by TMA (no multicast) into 128B-swizzled shared memory, 128 K-bytes
// per stage.  No warp leaves before the others; every
// mbarrier wait is bounded (about one second) and a timeout sets bit 16 of the
// device error word, drains the copies and MMAs in flight and frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "q3_common.cuh"
#include "q3_gemm.h"
#include "q3_tc.cuh"

namespace q3 {

// device error word of this file's kernels (q3_device_status ORs it in)
static __device__ unsigned int g_gemm_error = 0;

int gemm_device_status_take() {
  unsigned int v = 0, zero = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof v) != cudaSuccess) return -1;
  if (v) cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof zero);
  return static_cast<int>(v);
}

namespace tc {

constexpr unsigned kErrGemmTimeout = 1u << 16;
#ifndef Q3_GEMM_EPI_WARPS
#define Q3_GEMM_EPI_WARPS 16
#endif
#ifndef Q3_GEMM_NTOK_BIG
#define Q3_GEMM_NTOK_BIG 128
#endif
#ifndef Q3_GEMM_STAGES_PLAIN
#define Q3_GEMM_STAGES_PLAIN 4
#endif
#ifndef Q3_GEMM_STAGES_64
#define Q3_GEMM_STAGES_64 4
#endif
constexpr int EPI_WARPS = Q3_GEMM_EPI_WARPS;   // a multiple of 4 (TMEM lane quadrants)
constexpr int THREADS = (EPI_WARPS + 2) * 32;
// Accumulators start at the bit pattern of 1.5 * 2^23: the int32 sum of a
// K-group (|sum| <= 256 * 127 * 127 < 2^22) then reads as the float
// 12582912 + sum exactly, so f32(sum) is one exact subtraction.
constexpr uint32_t kAccBias = 0x4B400000u;
constexpr float kAccBiasF = 12582912.0f;

template <int NTOK, int MODE>
struct Cfg {
  static constexpr int NACC = (MODE == EPI_SWIGLU) ? 2 : 1;           // gate + up
  static constexpr int TILES = (MODE == EPI_SWIGLU) ? 2 : 1;          // 128-row tiles per CTA
  static constexpr int A_BYTES = 128 * 128;                           // one weight box
  static constexpr int B_BYTES = NTOK * 128;                          // one activation box
  static constexpr int STAGE_BYTES = NACC * A_BYTES + B_BYTES;
  // accumulator buffers in flight: as many K-groups as TMEM holds (<= 8)
  static constexpr int NBUF = (512 / (NACC * NTOK)) >= 8 ? 8 : (512 / (NACC * NTOK));
  static constexpr int TMEM_COLS_RAW = NBUF * NACC * NTOK;
  static constexpr int TMEM_COLS = TMEM_COLS_RAW <= 32 ? 32 : TMEM_COLS_RAW <= 64 ? 64
                                   : TMEM_COLS_RAW <= 128 ? 128 : TMEM_COLS_RAW <= 256 ? 256 : 512;
  static constexpr int XROWS = (MODE == EPI_SWIGLU) ? 256 : (MODE == EPI_NORMROPE || MODE == EPI_QUANT) ? 128 : 1;
  // stage ring: as deep as shared memory allows next to the staging buffer
  static constexpr int STAGES = (MODE == EPI_SWIGLU) ? 3
                               : XROWS > 1              ? 4
                               : NTOK == 64             ? Q3_GEMM_STAGES_64
                                                        : Q3_GEMM_STAGES_PLAIN;
  static constexpr int HT = NTOK / (EPI_WARPS / 4);                    // tokens per epilogue warp
};

template <int NTOK, int MODE>
struct __align__(1024) Smem {
  alignas(1024) int8_t stage[Cfg<NTOK, MODE>::STAGES][Cfg<NTOK, MODE>::STAGE_BYTES];
  // epilogue staging [feature][token], rows padded by one word (conflict-free)
  float xchg[Cfg<NTOK, MODE>::XROWS][NTOK + 1];
  alignas(16) float ascale[16 * NTOK];     // a_scale of this token tile, [group][token]
  // ARGMAX with one token tile: this CTA's best key per token over all its tiles
  unsigned long long akey[MODE == EPI_ARGMAX ? NTOK : 1];
  unsigned long long full[Cfg<NTOK, MODE>::STAGES], empty[Cfg<NTOK, MODE>::STAGES];
  unsigned long long tfull[Cfg<NTOK, MODE>::NBUF], tempty[Cfg<NTOK, MODE>::NBUF], done;
  uint32_t tmem_base;
  int abort;
};

using namespace tcx;

__device__ __forceinline__ void epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(EPI_WARPS * 32) : "memory");
}

struct TcArgs {
  GemmArgs g;
  int groups;         // K / group
  int boxes;          // group / 128
};

template <int NTOK, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
              const __grid_constant__ CUtensorMap tmB, const TcArgs args) {
  using C = Cfg<NTOK, MODE>;
  constexpr int STAGES = C::STAGES;
  constexpr int HT = C::HT;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Smem<NTOK, MODE> &sm = *reinterpret_cast<Smem<NTOK, MODE> *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const GemmArgs &p = args.g;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = args.groups, NB = args.boxes;
  const int tiles_x = p.N / (128 * C::TILES);     // feature tiles
  const int ntiles = tiles_x * ((p.M + NTOK - 1) / NTOK);
  const int tile_it = C::TILES * G * NB;          // producer / MMA k-iterations per tile
  // persistent: this CTA takes tiles blockIdx.x, blockIdx.x + gridDim.x, ...
  // (feature tile fastest, so the CTAs in flight share weights and activations)
  auto tile_rows = [&](int tile) { return (tile % tiles_x) * 128 * C::TILES; };
  auto tile_m0 = [&](int tile) { return (tile / tiles_x) * NTOK; };
  // epilogue warp w: TMEM lanes (feature rows) 32 (w % 4) .., tokens c0 .. c0 + HT - 1
  const int f = (warp & 3) * 32 + lane, c0 = (warp >> 2) * HT;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], 1);
    }
    for (int i = 0; i < C::NBUF; ++i) {
      mbar_init(&sm.tfull[i], 1);
      mbar_init(&sm.tempty[i], EPI_WARPS);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == EPI_WARPS + 1) tmem_alloc<C::TMEM_COLS>(&sm.tmem_base);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = sm.tmem_base;
  const uint32_t lane_addr = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  if (warp < EPI_WARPS) {                          // every accumulator starts at the bias
#pragma unroll
    for (int b = 0; b < C::NBUF * C::NACC; ++b)
#pragma unroll
      for (int c = 0; c < HT; c += 16) tmem_st16(lane_addr + b * NTOK + c0 + c, kAccBias);
    tmem_wait_st();
  }
  // ARGMAX: with a single token tile the keys are reduced in shared memory over
  // all of this CTA's tiles and written to global memory once (a global atomic
  // per tile and token would serialise ~1200 updates on each token's key)
  const bool cta_keys = MODE == EPI_ARGMAX && p.M <= NTOK;
  if (MODE == EPI_ARGMAX && threadIdx.x < NTOK) sm.akey[threadIdx.x] = 0ull;
  fence_before();
  __syncthreads();
  fence_after();

  if (warp == EPI_WARPS) {
    // ------------------------------------------------------------ TMA producer
    int issued = 0;
    bool ok = true;
    int it = 0;
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
      const int row0 = tile_rows(tile), m0 = tile_m0(tile);
      for (int ti = 0; ti < tile_it && ok; ++ti, ++it) {
        const int st = it % STAGES;
        if (lane == 0) {
          if (!mbar_wait(&sm.empty[st], ((it / STAGES) & 1) ^ 1, &sm.abort)) ok = false;
          else {
            const int t = ti / (G * NB), r = ti % (G * NB);
            const int k0 = r * 128;   // (g * NB + box) * 128
            mbar_expect_tx(&sm.full[st], C::STAGE_BYTES);
            int8_t *dst = sm.stage[st];
            tma_2d(dst, &tmA, k0, row0 + t * 128, &sm.full[st]);
            if (C::NACC == 2) tma_2d(dst + C::A_BYTES, &tmA2, k0, row0 + t * 128, &sm.full[st]);
            tma_2d(dst + C::NACC * C::A_BYTES, &tmB, k0, m0, &sm.full[st]);
            ++issued;
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
    }
    if (!ok && lane == 0) {
      atomicOr(&g_gemm_error, kErrGemmTimeout);
      sm.abort = 1;
      for (int it = max(0, issued - STAGES); it < issued; ++it)   // let issued copies land
        mbar_wait(&sm.full[it % STAGES], (it / STAGES) & 1, nullptr);
    }
  } else if (warp == EPI_WARPS + 1) {
    // ------------------------------------------------------------ MMA issuer
    // every MMA accumulates: the buffers hold the bias, not zero
    constexpr uint32_t ID = idesc_i8(NTOK);
    bool ok = true;
    int it = 0;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    for (int gi = 0; gi < my_tiles * C::TILES * G && ok; ++gi) {
      const int buf = gi % C::NBUF;
      if (lane == 0 && !mbar_wait(&sm.tempty[buf], ((gi / C::NBUF) & 1) ^ 1, &sm.abort)) ok = false;
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      fence_after();
      for (int box = 0; box < NB && ok; ++box, ++it) {
        const int st = it % STAGES;
        if (lane == 0) {
          if (!mbar_wait(&sm.full[st], (it / STAGES) & 1, &sm.abort)) ok = false;
          else {
            fence_after();
            const uint32_t sa = su32(sm.stage[st]);
            const uint32_t sb = sa + C::NACC * C::A_BYTES;
#pragma unroll
            for (int a = 0; a < C::NACC; ++a) {
              const uint32_t dt = tmem + (buf * C::NACC + a) * NTOK;
#pragma unroll
              for (int ks = 0; ks < 4; ++ks)
                mma_i8(dt, sdesc_sw128(sa + a * C::A_BYTES + ks * 32), sdesc_sw128(sb + ks * 32), ID, 1);
            }
            mma_commit(&sm.empty[st]);          // frees the stage when these MMAs finish
          }
        }
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      }
      if (ok && lane == 0) mma_commit(&sm.tfull[buf]);
    }
    if (lane == 0) {                             // every MMA issued has completed
      mma_commit(&sm.done);
      mbar_wait(&sm.done, 0, nullptr);
    }
    if (!ok && lane == 0) {
      atomicOr(&g_gemm_error, kErrGemmTimeout);
      sm.abort = 1;
    }
  } else {
    // ------------------------------------------------------------ epilogue
    constexpr int TPW = NTOK / EPI_WARPS;          // tokens per warp in the per-token passes
    const int etid = threadIdx.x;                  // 0 .. EPI_WARPS*32 - 1
    float nwv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (MODE == EPI_NORMROPE) {
#pragma unroll
      for (int k = 0; k < 4; ++k) nwv[k] = p.nw[lane + 32 * k];
    }
    bool ok = true;
    int gi = 0;
    int scales_m0 = -1;                          // token tile whose scales sm.ascale holds
    for (int tile = blockIdx.x; tile < ntiles && ok; tile += gridDim.x) {
    const int row0 = tile_rows(tile), m0 = tile_m0(tile);
    const int mvalid = min(NTOK, p.M - m0);
    if (m0 != scales_m0) {                       // (uniform: m0 is the CTA's)
      epi_sync();                                // the previous tile's readers are done
      for (int i = etid; i < NTOK * G; i += EPI_WARPS * 32) {   // this tile's activation scales
        const int g = i / NTOK, m = i % NTOK;
        sm.ascale[i] = (m < mvalid)
                           ? *reinterpret_cast<const float *>(p.a_scale + (long)(m0 + m) * p.as_rb + g * 4)
                           : 0.0f;
      }
      epi_sync();
      scales_m0 = m0;
    }
    for (int t = 0; t < C::TILES && ok; ++t) {
      const int n = row0 + t * 128 + f;
      float bs[C::NACC];
      bs[0] = p.b_scale[n];
      if (C::NACC == 2) bs[C::NACC - 1] = p.b2_scale[n];
      float accf[C::NACC][HT];
#pragma unroll
      for (int a = 0; a < C::NACC; ++a)
#pragma unroll
        for (int i = 0; i < HT; ++i) accf[a][i] = 0.0f;
      for (int g = 0; g < G; ++g, ++gi) {
        const int buf = gi % C::NBUF;
        if (!mbar_wait(&sm.tfull[buf], (gi / C::NBUF) & 1, &sm.abort)) { ok = false; break; }
        fence_after();
        const float *asg = sm.ascale + g * NTOK + c0;
#pragma unroll
        for (int a = 0; a < C::NACC; ++a) {
          const uint32_t col = lane_addr + (buf * C::NACC + a) * NTOK + c0;
#pragma unroll
          for (int c = 0; c < HT; c += 16) {       // 16 token columns at a time
            int v[16];
            tmem_ld16(col + c, v);
            tmem_wait_ld();
            tmem_st16(col + c, kAccBias);          // ready for the buffer's next use
            // acc += (f32(part) * b_scale[n]) * a_scale[m][g]   (ref_qwen3.py:152-157)
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
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
        if (lane == 0) mbar_arrive(&sm.tempty[buf]);
      }
      if (!ok) break;

      // -------------------------------------------------------- epilogues
      if (MODE == EPI_STORE || MODE == EPI_ADD) {
        float xv[HT];
        if (MODE == EPI_ADD) {                     // every load before the first store
#pragma unroll
          for (int i = 0; i < HT; ++i)
            xv[i] = (c0 + i < mvalid)
                        ? reinterpret_cast<const float *>(p.out + (long)(m0 + c0 + i) * p.out_rb)[n]
                        : 0.0f;
        }
#pragma unroll
        for (int i = 0; i < HT; ++i) {
          if (c0 + i < mvalid) {
            float *row = reinterpret_cast<float *>(p.out + (long)(m0 + c0 + i) * p.out_rb);
            row[n] = (MODE == EPI_ADD) ? __fadd_rn(xv[i], accf[0][i]) : accf[0][i];
          }
        }
      } else if (MODE == EPI_ARGMAX) {
        // (max, first index) per token over the tile's 128 rows -> atomicMax of a
        // packed key (monotone value << 32 | ~index): largest value, then smallest index
#pragma unroll
        for (int i = 0; i < HT; ++i) {
          const float v = __fadd_rn(accf[0][i], 0.0f);   // -0 -> +0: equal maxima compare equal
          const unsigned b = __float_as_uint(v);
          const unsigned key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
          // the 64-bit maximum over the warp in two 32-bit reductions: the
          // largest value key, then the largest ~index among the lanes holding it
          const unsigned kmax = __reduce_max_sync(0xffffffffu, key);
          const unsigned imax =
              __reduce_max_sync(0xffffffffu, key == kmax ? 0xffffffffu - static_cast<unsigned>(n) : 0u);
          const unsigned long long k = (static_cast<unsigned long long>(kmax) << 32) | imax;
          if (lane == 0 && c0 + i < mvalid) {
            if (cta_keys) atomicMax(&sm.akey[c0 + i], k);
            else atomicMax(p.arg_keys + m0 + c0 + i, k);
          }
        }
      } else {
        // stage this tile's values [feature][token] in shared memory (padded rows)
        // and continue with one warp per token (features l, l+32, l+64, l+96 per lane)
        if (MODE == EPI_SWIGLU) {
          // silu(g)*u (ref_qwen3.py:194-200), element by element, then staged
          // exp(-g) of the thread's HT tokens in one batch (throughput-bound
          // here: one exp per gate output; the short exp2, branch-free)
          float en[HT];
#pragma unroll
          for (int i = 0; i < HT; ++i) en[i] = __fmul_rn(accf[0][i], -1.0f);
          exp_ref_fast_n(en, g_exp2_t256);
#pragma unroll
          for (int i = 0; i < HT; ++i) {
            float sw = 0.0f;
            if (c0 + i < mvalid) {
              const float gt = accf[0][i];
              float e = __fadd_rn(en[i], 1.0f);
              e = __frcp_rn(e);
              sw = __fmul_rn(__fmul_rn(gt, e), accf[C::NACC - 1][i]);
            }
            sm.xchg[t * 128 + f][c0 + i] = sw;
          }
          epi_sync();
          if (t == C::TILES - 1) {
            // per-token absmax over the 256-feature group, quantise both tiles
            for (int m = warp; m < mvalid; m += EPI_WARPS) {
              float v[8];
              float mx = 0.0f;
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                v[k] = sm.xchg[lane + 32 * k][m];
                mx = fmaxf(mx, fabsf(v[k]));
              }
              mx = warp_tree_max(mx);
              const float scale = __fmul_rn(mx, kInv127);
              int8_t *q = reinterpret_cast<int8_t *>(p.q8 + (long)(m0 + m) * p.q8_rb) + row0;
#pragma unroll
              int qv[8];
              quant_n_absmax(v, scale, qv);
#pragma unroll
              for (int k = 0; k < 8; ++k) q[lane + 32 * k] = static_cast<int8_t>(qv[k]);
              if (lane == 0)
                *reinterpret_cast<float *>(p.qs + (long)(m0 + m) * p.qs_rb + (row0 / 256) * 4) = scale;
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < HT; ++i) sm.xchg[f][c0 + i] = accf[0][i];
          // rope rows of this warp's tokens, loaded while the others stage
          float cs[TPW][2], sn[TPW][2];
          if (MODE == EPI_NORMROPE) {
#pragma unroll
            for (int j = 0; j < TPW; ++j) {
              const int m = warp + EPI_WARPS * j;
              const int mm = m < mvalid ? m : 0;
              const float *cr = reinterpret_cast<const float *>(p.cos + (long)(m0 + mm) * p.cos_rb);
              const float *sr = reinterpret_cast<const float *>(p.sin + (long)(m0 + mm) * p.sin_rb);
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                cs[j][k] = cr[lane + 32 * k];
                sn[j][k] = sr[lane + 32 * k];
              }
            }
          }
          epi_sync();
          const int r0 = row0 + t * 128;
#pragma unroll
          for (int j = 0; j < TPW; ++j) {
            const int m = warp + EPI_WARPS * j;
            if (m >= mvalid) break;
            float v[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k] = sm.xchg[lane + 32 * k][m];
            if (MODE == EPI_NORMROPE) {
              // head RMSNorm: tree over each 32-row block (k), blocks summed in order
              float ss = 0.0f;
#pragma unroll
              for (int k = 0; k < 4; ++k) ss = __fadd_rn(ss, warp_tree_sum(__fmul_rn(v[k], v[k])));
              ss = __fadd_rn(__fmul_rn(ss, p.inv_hd), kEps);
              const float r = rsqrt_ref(ss);
#pragma unroll
              for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], r), nwv[k]);
              // rotate-half RoPE: pairs (l, l+64) and (l+32, l+96) live in this lane
#pragma unroll
              for (int k = 0; k < 2; ++k) {
                const float l = v[k], rr = v[k + 2];
                v[k] = __fsub_rn(__fmul_rn(l, cs[j][k]), __fmul_rn(rr, sn[j][k]));
                v[k + 2] = __fadd_rn(__fmul_rn(l, sn[j][k]), __fmul_rn(rr, cs[j][k]));
              }
            }
            float mx = 0.0f;
#pragma unroll
            for (int k = 0; k < 4; ++k) mx = fmaxf(mx, fabsf(v[k]));
            mx = warp_tree_max(mx);
            const float scale = __fmul_rn(mx, kInv127);
            int8_t *q = reinterpret_cast<int8_t *>(p.q8 + (long)(m0 + m) * p.q8_rb) + r0;
#pragma unroll
            int qv[4];
            quant_n_absmax(v, scale, qv);
#pragma unroll
            for (int k = 0; k < 4; ++k) q[lane + 32 * k] = static_cast<int8_t>(qv[k]);
            if (lane == 0)
              *reinterpret_cast<float *>(p.qs + (long)(m0 + m) * p.qs_rb + (r0 / 128) * 4) = scale;
          }
        }
        epi_sync();   // the staging buffer is rewritten by the next tile
      }
    }
    }                                            // tiles
    if (!ok && lane == 0) {
      atomicOr(&g_gemm_error, kErrGemmTimeout);
      sm.abort = 1;
    }
  }

  // ---------------------------------------------------------------- teardown
  fence_before();
  __syncthreads();
  fence_after();
  if (cta_keys && threadIdx.x < p.M && blockIdx.x < ntiles) {
    const unsigned long long k = sm.akey[threadIdx.x];
    if (k) atomicMax(p.arg_keys + threadIdx.x, k);
  }
  if (warp == EPI_WARPS + 1) tmem_dealloc<C::TMEM_COLS>(tmem);
}

// ---------------------------------------------------------------- host side
static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  });
  return fn;
}

// int8 [rows][cols] with row stride `stride` bytes; box = 128 bytes x box_rows
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols,
              uint64_t stride, uint32_t box_rows) {
  auto enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {stride};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NTOK, int MODE>
static int launch(const GemmArgs &p, cudaStream_t s) {
  using C = Cfg<NTOK, MODE>;
  CUtensorMap ta, ta2, tb;
  const uint64_t K = p.K;
  if (!make_map(&ta, p.b, p.N, K, p.b_rb, 128)) return Q3_ERR_CUDA;
  if (!make_map(&ta2, C::NACC == 2 ? p.b2 : p.b, p.N, K, p.b_rb, 128)) return Q3_ERR_CUDA;
  if (!make_map(&tb, p.a, p.M, K, p.a_rb, NTOK)) return Q3_ERR_CUDA;
  const size_t smem = sizeof(Smem<NTOK, MODE>) + 1024;
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [&] {
    attr = cudaFuncSetAttribute(k_gemm_tc<NTOK, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)smem);
  });
  if (attr != cudaSuccess) {
    q3h::set_cuda_error(attr);
    return Q3_ERR_CUDA;
  }
  TcArgs a{p, p.K / p.group, p.group / 128};
  const int ntiles = (p.N / (128 * C::TILES)) * ((p.M + NTOK - 1) / NTOK);
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  dim3 grid(ntiles < sms ? ntiles : sms);       // persistent: one CTA per SM
  q3h::timer_begin(q3h::TIMER_GEMM, s);
  k_gemm_tc<NTOK, MODE><<<grid, THREADS, smem, s>>>(ta, ta2, tb, a);
  const int st = q3h::launch_status();
  q3h::timer_end(q3h::TIMER_GEMM, s);
  return st;
}

}  // namespace tc

// Shapes the tensor-core path takes: 128-byte K boxes within whole groups,
// 16-byte aligned operands, at most 16 groups, whole 128-row (256 for SwiGLU) tiles.
bool gemm_tc_eligible(const GemmArgs &p) {
  if (p.group % 128 || p.K % p.group || p.K / p.group > 16 || p.group > 256) return false;
  if (p.a_rb % 16 || p.b_rb % 16 || reinterpret_cast<uintptr_t>(p.a) % 16 ||
      reinterpret_cast<uintptr_t>(p.b) % 16)
    return false;
  if (p.mode == EPI_SWIGLU) {
    if (p.N % 256 || reinterpret_cast<uintptr_t>(p.b2) % 16) return false;
  } else if (p.N % 128) {
    return false;
  }
  return true;
}

int gemm_tc(const GemmArgs &p, cudaStream_t s) {
  if (gemm_pair_eligible(p)) return gemm_pair(p, s);
  switch (p.mode) {
    // wider token tiles cut the weight traffic per MAC; SwiGLU stages 256
    // features per token and keeps 64, and so do the few-row GEMMs
    case EPI_STORE:
      return p.M > 64 ? tc::launch<Q3_GEMM_NTOK_BIG, EPI_STORE>(p, s) : tc::launch<64, EPI_STORE>(p, s);
    case EPI_ADD:
      return p.M > 64 ? tc::launch<Q3_GEMM_NTOK_BIG, EPI_ADD>(p, s) : tc::launch<64, EPI_ADD>(p, s);
    case EPI_QUANT:
      return p.M > 64 ? tc::launch<Q3_GEMM_NTOK_BIG, EPI_QUANT>(p, s) : tc::launch<64, EPI_QUANT>(p, s);
    case EPI_NORMROPE:
      return p.M > 64 ? tc::launch<Q3_GEMM_NTOK_BIG, EPI_NORMROPE>(p, s)
                      : tc::launch<64, EPI_NORMROPE>(p, s);
    case EPI_SWIGLU: return tc::launch<64, EPI_SWIGLU>(p, s);
    case EPI_ARGMAX: return tc::launch<64, EPI_ARGMAX>(p, s);
  }
  return Q3_ERR_SHAPE;
}

}  // namespace q3
