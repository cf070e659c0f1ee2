// Per-K-group w8a8 GEMM on the CUDA cores (dp4a), with every epilogue of the
// reference's gemm_nt_group_store (kernels/group_gemm.h:27-222), the fused
// gate/up + SwiGLU + quant (kernels/swiglu_quant.h:105-255) and the fused
// lm_head + argmax (kernels/lm_argmax.h:72-182).
//
// This is the general-shape path (any row count, any row strides that keep
// 16-byte alignment).  The tensor-core path (q3_gemm_tc.cu) serves the large
// prefill GEMMs; both produce identical bits.
//
// Tile: NT output columns per CTA (thread t owns column n0 + t), MT rows per
// CTA, K streamed through shared memory 64 bytes at a time.
#include "q3_common.cuh"
#include "q3_gemm.h"

namespace q3 {

constexpr int KC = 64;          // K bytes per shared-memory stage
constexpr int KCW = KC / 4;     // int32 words per stage
constexpr int BPAD = KCW + 1;   // padded row (words) -> conflict-free column reads

template <int NT, int MT, int MODE>
__global__ void __launch_bounds__(NT) k_gemm_group_simt(GemmArgs p) {
  constexpr bool DUAL = (MODE == EPI_SWIGLU);
  __shared__ int sA[MT][KCW];
  __shared__ int sB[DUAL ? 2 : 1][NT][BPAD];
  __shared__ float sRed[MT][NT / 32];
  __shared__ float sY[(MODE == EPI_NORMROPE) ? MT : 1][NT];

  const int t = threadIdx.x;
  const int n0 = blockIdx.x * NT;
  const int m0 = blockIdx.y * MT;
  const int mrows = min(MT, p.M - m0);
  const int lane = t & 31, wid = t >> 5;

  float acc[MT], acc2[DUAL ? MT : 1];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
#pragma unroll
  for (int m = 0; m < (DUAL ? MT : 1); ++m) acc2[m] = 0.0f;

  const int n = n0 + t;
  const float bs = p.b_scale[n];
  const float bs2 = DUAL ? p.b2_scale[n] : 0.0f;
  const int groups = p.K / p.group;

  for (int g = 0; g < groups; ++g) {
    int part[MT], part2[DUAL ? MT : 1];
#pragma unroll
    for (int m = 0; m < MT; ++m) part[m] = 0;
#pragma unroll
    for (int m = 0; m < (DUAL ? MT : 1); ++m) part2[m] = 0;
    for (int kc = 0; kc < p.group; kc += KC) {
      const int k0 = g * p.group + kc;
      // stage A [MT][64 B] and B [NT][64 B] (16-byte vectors)
      for (int i = t; i < MT * 4; i += NT) {
        const int m = i >> 2, v = i & 3;
        int4 val = make_int4(0, 0, 0, 0);
        if (m < mrows) val = *reinterpret_cast<const int4 *>(p.a + (long)(m0 + m) * p.a_rb + k0 + v * 16);
        *reinterpret_cast<int4 *>(&sA[m][v * 4]) = val;
      }
#pragma unroll
      for (int d = 0; d < (DUAL ? 2 : 1); ++d) {
        const int8_t *bb = d ? p.b2 : p.b;
        for (int i = t; i < NT * 4; i += NT) {
          const int r = i >> 2, v = i & 3;
          const int4 val = *reinterpret_cast<const int4 *>(bb + (long)(n0 + r) * p.b_rb + k0 + v * 16);
          sB[d][r][v * 4 + 0] = val.x;
          sB[d][r][v * 4 + 1] = val.y;
          sB[d][r][v * 4 + 2] = val.z;
          sB[d][r][v * 4 + 3] = val.w;
        }
      }
      __syncthreads();
#pragma unroll
      for (int w = 0; w < KCW; ++w) {
        const int bw = sB[0][t][w];
        const int bw2 = DUAL ? sB[DUAL ? 1 : 0][t][w] : 0;
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const int aw = sA[m][w];
          part[m] = __dp4a(aw, bw, part[m]);
          if (DUAL) part2[m] = __dp4a(aw, bw2, part2[m]);
        }
      }
      __syncthreads();
    }
    // dequant: (f32(part) * b_scale[n]) * a_scale[m][g], summed over groups in order
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < mrows) {
        const float as = *reinterpret_cast<const float *>(p.a_scale + (long)(m0 + m) * p.as_rb + g * 4);
        acc[m] = __fadd_rn(acc[m], __fmul_rn(__fmul_rn(__int2float_rn(part[m]), bs), as));
        if (DUAL) acc2[m] = __fadd_rn(acc2[m], __fmul_rn(__fmul_rn(__int2float_rn(part2[m]), bs2), as));
      }
    }
  }

  // ---------------------------------------------------------------- epilogues
  if (MODE == EPI_STORE) {
    for (int m = 0; m < mrows; ++m)
      reinterpret_cast<float *>(p.out + (long)(m0 + m) * p.out_rb)[n] = acc[m];
  } else if (MODE == EPI_ADD) {
    for (int m = 0; m < mrows; ++m) {
      float *xr = reinterpret_cast<float *>(p.out + (long)(m0 + m) * p.out_rb);
      xr[n] = __fadd_rn(xr[n], acc[m]);
    }
  } else if (MODE == EPI_QUANT || MODE == EPI_NORMROPE) {
    // NT == 128 == one head
    if (MODE == EPI_NORMROPE) {
      // per-head RMSNorm: warp w holds the 32-column block w; blocks summed in order
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const float s = warp_tree_sum(__fmul_rn(acc[m], acc[m]));
        if (lane == 0) sRed[m][wid] = s;
      }
      __syncthreads();
      const float wv = p.nw[t];
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float ss = 0.0f;
#pragma unroll
        for (int b = 0; b < NT / 32; ++b) ss = __fadd_rn(ss, sRed[m][b]);
        ss = __fadd_rn(__fmul_rn(ss, p.inv_hd), kEps);
        const float r = rsqrt_ref(ss);
        sY[MODE == EPI_NORMROPE ? m : 0][t] = __fmul_rn(__fmul_rn(acc[m], r), wv);
      }
      __syncthreads();
      // rotate-half RoPE with separately rounded products (ref_qwen3.py:180-191)
      const int j = t & 63;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        if (m < mrows) {
          const float c = reinterpret_cast<const float *>(p.cos + (long)(m0 + m) * p.cos_rb)[j];
          const float s = reinterpret_cast<const float *>(p.sin + (long)(m0 + m) * p.sin_rb)[j];
          const float l = sY[MODE == EPI_NORMROPE ? m : 0][j];
          const float rr = sY[MODE == EPI_NORMROPE ? m : 0][j + 64];
          acc[m] = (t < 64) ? __fsub_rn(__fmul_rn(l, c), __fmul_rn(rr, s))
                            : __fadd_rn(__fmul_rn(l, s), __fmul_rn(rr, c));
        }
      }
      __syncthreads();
    }
    // per-head absmax over the 128 columns, scale = absmax/127, quantise
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float mx = warp_tree_max(fabsf(acc[m]));
      if (lane == 0) sRed[m][wid] = mx;
    }
    __syncthreads();
    for (int m = 0; m < mrows; ++m) {
      float mx = 0.0f;
#pragma unroll
      for (int b = 0; b < NT / 32; ++b) mx = fmaxf(mx, sRed[m][b]);
      const float scale = __fmul_rn(mx, kInv127);
      reinterpret_cast<int8_t *>(p.q8 + (long)(m0 + m) * p.q8_rb)[n] =
          static_cast<int8_t>(quant1(acc[m], scale));
      if (t == 0) *reinterpret_cast<float *>(p.qs + (long)(m0 + m) * p.qs_rb + (n0 / 128) * 4) = scale;
    }
  } else if (MODE == EPI_SWIGLU) {
    // silu(g)*u (ref_qwen3.py:194-200), per-256-column int8 quant (NT == 256)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float gt = acc[m];
      float e = exp_ref(__fmul_rn(gt, -1.0f));
      e = __fadd_rn(e, 1.0f);
      e = __frcp_rn(e);
      acc[m] = __fmul_rn(__fmul_rn(gt, e), acc2[DUAL ? m : 0]);
      const float mx = warp_tree_max(fabsf(acc[m]));
      if (lane == 0) sRed[m][wid] = mx;
    }
    __syncthreads();
    for (int m = 0; m < mrows; ++m) {
      float mx = 0.0f;
#pragma unroll
      for (int b = 0; b < NT / 32; ++b) mx = fmaxf(mx, sRed[m][b]);
      const float scale = __fmul_rn(mx, kInv127);
      reinterpret_cast<int8_t *>(p.q8 + (long)(m0 + m) * p.q8_rb)[n] =
          static_cast<int8_t>(quant1(acc[m], scale));
      if (t == 0) *reinterpret_cast<float *>(p.qs + (long)(m0 + m) * p.qs_rb + (n0 / 256) * 4) = scale;
    }
  } else if (MODE == EPI_ARGMAX) {
    // (max, first index) of each row over this CTA's columns -> atomicMax of a
    // packed key (monotone value << 32 | ~index): largest value, then smallest index
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[m] + 0.0f;   // -0 -> +0: equal maxima compare equal, as in `best < tmax`
      unsigned b = __float_as_uint(v);
      unsigned key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
      unsigned long long k =
          (static_cast<unsigned long long>(key) << 32) | (0xffffffffu - static_cast<unsigned>(n));
#pragma unroll
      for (int o = 16; o; o >>= 1) {
        const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
        k = ok > k ? ok : k;
      }
      if (lane == 0 && m < mrows) atomicMax(p.arg_keys + m0 + m, k);
    }
  }
}

__global__ void k_argmax_init(unsigned long long *keys, int rows) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < rows) keys[i] = 0ull;
}

// merge the row maxima into the caller's running (best, bidx): replace when
// best < max (lm_argmax.h:55-67 applied block by block has this net effect)
__global__ void k_argmax_finish(const unsigned long long *keys, float *best, int32_t *bidx,
                                int rows) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  const unsigned long long k = keys[i];
  const unsigned key = static_cast<unsigned>(k >> 32);
  const unsigned b = (key & 0x80000000u) ? (key & 0x7fffffffu) : ~key;
  const float v = __uint_as_float(b);
  const int idx = static_cast<int>(0xffffffffu - static_cast<unsigned>(k & 0xffffffffu));
  if (best[i] < v) {
    best[i] = v;
    bidx[i] = idx;
  }
}

template <int NT, int MT, int MODE>
static int launch_simt(const GemmArgs &p, cudaStream_t s) {
  dim3 grid(p.N / NT, (p.M + MT - 1) / MT);
  k_gemm_group_simt<NT, MT, MODE><<<grid, NT, 0, s>>>(p);
  return q3h::launch_status();
}

// the lm_head argmax keys: cleared before the row-max kernel, merged into
// (best, bidx) after it (whichever GEMM path ran)
int argmax_begin(const GemmArgs &p, cudaStream_t s) {
  k_argmax_init<<<(p.M + 127) / 128, 128, 0, s>>>(p.arg_keys, p.M);
  return q3h::launch_status();
}
int argmax_end(const GemmArgs &p, cudaStream_t s) {
  k_argmax_finish<<<(p.M + 127) / 128, 128, 0, s>>>(p.arg_keys, p.best, p.bidx, p.M);
  return q3h::launch_status();
}

int gemm_simt(const GemmArgs &p, cudaStream_t s) {
  switch (p.mode) {
    case EPI_STORE: return launch_simt<128, 8, EPI_STORE>(p, s);
    case EPI_ADD: return launch_simt<128, 8, EPI_ADD>(p, s);
    case EPI_QUANT: return launch_simt<128, 8, EPI_QUANT>(p, s);
    case EPI_NORMROPE: return launch_simt<128, 8, EPI_NORMROPE>(p, s);
    case EPI_SWIGLU: return launch_simt<256, 8, EPI_SWIGLU>(p, s);
    case EPI_ARGMAX: return launch_simt<128, 8, EPI_ARGMAX>(p, s);
  }
  return Q3_ERR_SHAPE;
}

}  // namespace q3
