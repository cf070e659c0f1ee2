// Group-ordered reductions of split-K GEMM partials with the path's epilogues
// fused in, for the batched decode step (one row per sequence).
//
// A partial buffer holds, per K-group g, the dequantised group product
// part[g][m][n] = (f32(A_g . W_g) * w_scale[n]) * a_scale[m][g]; the GEMM result
// is ((0 + part[0]) + part[1]) + ... in group order — the reference's sum
// (ref_qwen3.py:151-157).  The epilogues then follow:
//   k_red_qkv      Q heads: RMSNorm(nq) + RoPE + quant -> q8/qs;
//                  K heads: RMSNorm(nk) + RoPE + quant -> the KV page;
//                  V heads: quant -> the KV page (group_gemm.h:168-193,
//                  norm_rope_quant.h:17-86, main_big.cpp:183-209)
//   k_red_add_norm x += result (residual), then RMSNorm(w) + per-256 quant of
//                  the new x for the next GEMM (main_big.cpp:178-181, 258-259)
//   k_red_swiglu   silu(gate) * up, per-256 quant (swiglu_quant.h:164-255)
// Warp per (row, head) or (row, 256-group): a lane holds features l + 32k, so
// the reference's 32-column block trees are warp butterflies.  The kernels are
// launched as programmatic dependents of the GEMM before them and wait for it
// before touching memory.
#include "q3_common.cuh"

namespace q3 {

// every group's partial is loaded first (independent loads in flight
// together), then the partials are added in group order from 0
constexpr int kMaxGroups = 16;
__device__ __forceinline__ float group_sum(const float *part, size_t gstride, int G) {
  float v[kMaxGroups];
#pragma unroll
  for (int g = 0; g < kMaxGroups; ++g) v[g] = g < G ? part[g * gstride] : 0.0f;
  float acc = 0.0f;
#pragma unroll
  for (int g = 0; g < kMaxGroups; ++g)
    if (g < G) acc = __fadd_rn(acc, v[g]);
  return acc;
}

struct QkvArgs {
  const float *part;       // [G][B][QW + 2*KW]
  int G, B, heads, kv_heads;
  const float *nq, *nk;    // [128]
  const float *cos_t, *sin_t;  // [max_seq][64] tables
  const int32_t *pos;      // [B]
  float inv_hd;
  int8_t *q8;              // [B][QW]
  float *qs;               // [B][heads]
  char *pk, *pv, *pks, *pvs;   // this layer's page pools
  const uint16_t *tables;  // [B][max_pages]
  uint32_t max_pages;
};

// grid (heads + 2*kv_heads) / 4 x B, block 128: warp per (row, head)
__global__ void __launch_bounds__(128) k_red_qkv(QkvArgs a) {
  pdl_trigger();
  pdl_wait();     // the partials come from the kernel before
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.x * 4 + warp;
  const int m = blockIdx.y;
  const int nh = a.heads + 2 * a.kv_heads;
  if (h >= nh) return;
  const int N = nh * 128;
  const size_t gstride = static_cast<size_t>(a.B) * N;
  const float *pr = a.part + static_cast<size_t>(m) * N + h * 128;
  float v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = group_sum(pr + lane + 32 * k, gstride, a.G);
  const int p = a.pos[m];
  const bool is_v = h >= a.heads + a.kv_heads;
  if (!is_v) {
    const float *nw = h < a.heads ? a.nq : a.nk;
    float ss = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) ss = __fadd_rn(ss, warp_tree_sum(__fmul_rn(v[k], v[k])));
    ss = __fadd_rn(__fmul_rn(ss, a.inv_hd), kEps);
    const float r = rsqrt_ref(ss);
#pragma unroll
    for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(__fmul_rn(v[k], r), nw[lane + 32 * k]);
    const float *cr = a.cos_t + static_cast<size_t>(p) * 64;
    const float *sr = a.sin_t + static_cast<size_t>(p) * 64;
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const float cs = cr[lane + 32 * k], sn = sr[lane + 32 * k];
      const float l = v[k], rr = v[k + 2];
      v[k] = __fsub_rn(__fmul_rn(l, cs), __fmul_rn(rr, sn));
      v[k + 2] = __fadd_rn(__fmul_rn(l, sn), __fmul_rn(rr, cs));
    }
  }
  float mx = 0.0f;
#pragma unroll
  for (int k = 0; k < 4; ++k) mx = fmaxf(mx, fabsf(v[k]));
  mx = warp_tree_max(mx);
  const float scale = __fmul_rn(mx, kInv127);
  int8_t q[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) q[k] = static_cast<int8_t>(quant1(v[k], scale));
  if (h < a.heads) {
    int8_t *dst = a.q8 + static_cast<size_t>(m) * a.heads * 128 + h * 128;
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = q[k];
    if (lane == 0) a.qs[m * a.heads + h] = scale;
  } else {
    const int kvh = is_v ? h - a.heads - a.kv_heads : h - a.heads;
    const uint32_t page = a.tables[static_cast<size_t>(m) * a.max_pages + p / 32];
    const size_t row = static_cast<size_t>(page) * 32 + (p % 32);
    const int kw = a.kv_heads * 128;
    int8_t *dst = reinterpret_cast<int8_t *>(is_v ? a.pv : a.pk) + row * kw + kvh * 128;
#pragma unroll
    for (int k = 0; k < 4; ++k) dst[lane + 32 * k] = q[k];
    if (lane == 0) reinterpret_cast<float *>(is_v ? a.pvs : a.pks)[row * a.kv_heads + kvh] = scale;
  }
}

struct AddNormArgs {
  const float *part;       // [G][B][H]
  int G, B, H;
  float *x;                // [B][H] residual, updated in place
  const float *w;          // [H] RMSNorm weight of the next step (null: no norm)
  float inv;               // 1/H
  int8_t *h8;              // [B][H]
  float *hs;               // [B][H/256]
};

// CTA per row, 256 threads, H == 1024: thread t owns features t + 256k
__global__ void __launch_bounds__(256) k_red_add_norm(AddNormArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float blk[32];
  __shared__ float gmax[4][8];
  __shared__ float rsh;
  const int m = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const size_t gstride = static_cast<size_t>(a.B) * a.H;
  float xv[4], rv[4];
  // every load (partials, residual) before the first store: nothing to alias
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int n = t + 256 * k;
    rv[k] = group_sum(a.part + static_cast<size_t>(m) * a.H + n, gstride, a.G);
    xv[k] = a.x[static_cast<size_t>(m) * a.H + n];
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    xv[k] = __fadd_rn(xv[k], rv[k]);
    a.x[static_cast<size_t>(m) * a.H + t + 256 * k] = xv[k];
  }
  if (!a.w) return;
  // 32-column block b = warp + 8k: tree per block, blocks summed in order
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float s = warp_tree_sum(__fmul_rn(xv[k], xv[k]));
    if (lane == 0) blk[warp + 8 * k] = s;
  }
  __syncthreads();
  if (t == 0) {
    float ss = 0.0f;
    for (int b = 0; b < 32; ++b) ss = __fadd_rn(ss, blk[b]);
    ss = __fadd_rn(__fmul_rn(ss, a.inv), kEps);
    rsh = rsqrt_ref(ss);
  }
  __syncthreads();
  const float r = rsh;
  float hv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    hv[k] = __fmul_rn(__fmul_rn(xv[k], r), a.w[t + 256 * k]);
    const float mx = warp_tree_max(fabsf(hv[k]));
    if (lane == 0) gmax[k][warp] = mx;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; ++k) {   // group k = features [256k, 256k + 256)
    float mx = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) mx = fmaxf(mx, gmax[k][w]);
    const float scale = __fmul_rn(mx, kInv127);
    a.h8[static_cast<size_t>(m) * a.H + t + 256 * k] = static_cast<int8_t>(quant1(hv[k], scale));
    if (t == 0) a.hs[static_cast<size_t>(m) * (a.H / 256) + k] = scale;
  }
}

struct SwigluArgs {
  const float *part;       // [2][G][B][I]: gate then up
  int G, B, I;
  int8_t *s8;              // [B][I]
  float *ss;               // [B][I/256]
};

// grid (I/256)/4 x B, block 128: warp per (row, 256-column group)
__global__ void __launch_bounds__(128) k_red_swiglu(SwigluArgs a) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grp = blockIdx.x * 4 + warp, m = blockIdx.y;
  if (grp * 256 >= a.I) return;
  const size_t gstride = static_cast<size_t>(a.B) * a.I;
  const float *pg = a.part + static_cast<size_t>(m) * a.I + grp * 256;
  const float *pu = pg + static_cast<size_t>(a.G) * gstride;
  float sw[8];
  float mx = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float gt = group_sum(pg + lane + 32 * k, gstride, a.G);
    const float ut = group_sum(pu + lane + 32 * k, gstride, a.G);
    float e = exp_ref(__fmul_rn(gt, -1.0f));
    e = __fadd_rn(e, 1.0f);
    e = __fdiv_rn(1.0f, e);
    sw[k] = __fmul_rn(__fmul_rn(gt, e), ut);
    mx = fmaxf(mx, fabsf(sw[k]));
  }
  mx = warp_tree_max(mx);
  const float scale = __fmul_rn(mx, kInv127);
  int8_t *dst = a.s8 + static_cast<size_t>(m) * a.I + grp * 256;
#pragma unroll
  for (int k = 0; k < 8; ++k) dst[lane + 32 * k] = static_cast<int8_t>(quant1(sw[k], scale));
  if (lane == 0) a.ss[static_cast<size_t>(m) * (a.I / 256) + grp] = scale;
}

struct NormQuantArgs {
  const float *x;          // [B][H]
  const float *bsum;       // [B][H/32] tree sums of x^2 per 32-column block
  const float *w;          // [H] RMSNorm weight
  float inv;               // 1/H
  int B, H;
  int8_t *h8;              // [B][H]
  float *hs;               // [B][H/256]
};

// RMSNorm(w) + per-256 quant of x from its block sums (rmsnorm.h:34-81,
// quant.h:89-138): the block sums are added in block order.  CTA per row, 256
// threads, H == 1024: thread t owns features t + 256k.
__global__ void __launch_bounds__(256) k_norm_quant(NormQuantArgs a) {
  pdl_trigger();
  pdl_wait();
  __shared__ float gmax[4][8];
  const int m = blockIdx.x, t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const float *bs = a.bsum + static_cast<size_t>(m) * (a.H / 32);
  float ss = 0.0f;
  for (int b = 0; b < a.H / 32; ++b) ss = __fadd_rn(ss, bs[b]);
  ss = __fadd_rn(__fmul_rn(ss, a.inv), kEps);
  const float r = rsqrt_ref(ss);
  float hv[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int n = t + 256 * k;
    hv[k] = __fmul_rn(__fmul_rn(a.x[static_cast<size_t>(m) * a.H + n], r), a.w[n]);
    const float mx = warp_tree_max(fabsf(hv[k]));
    if (lane == 0) gmax[k][warp] = mx;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < 4; ++k) {   // group k = features [256k, 256k + 256)
    float mx = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) mx = fmaxf(mx, gmax[k][w]);
    const float scale = __fmul_rn(mx, kInv127);
    a.h8[static_cast<size_t>(m) * a.H + t + 256 * k] = static_cast<int8_t>(quant1(hv[k], scale));
    if (t == 0) a.hs[static_cast<size_t>(m) * (a.H / 256) + k] = scale;
  }
}

int norm_quant(const NormQuantArgs &a, cudaStream_t s) {
  if (a.H != 1024) return Q3_ERR_SHAPE;
  return q3h::launch_ex(true, k_norm_quant, dim3(a.B), dim3(256), 0, s, a);
}

int red_qkv(const QkvArgs &a, cudaStream_t s) {
  const int nh = a.heads + 2 * a.kv_heads;
  return q3h::launch_ex(true, k_red_qkv, dim3((nh + 3) / 4, a.B), dim3(128), 0, s, a);
}
int red_add_norm(const AddNormArgs &a, cudaStream_t s) {
  if (a.H != 1024) return Q3_ERR_SHAPE;
  return q3h::launch_ex(true, k_red_add_norm, dim3(a.B), dim3(256), 0, s, a);
}
int red_swiglu(const SwigluArgs &a, cudaStream_t s) {
  return q3h::launch_ex(true, k_red_swiglu, dim3((a.I / 256 + 3) / 4, a.B), dim3(128), 0, s, a);
}

}  // namespace q3
