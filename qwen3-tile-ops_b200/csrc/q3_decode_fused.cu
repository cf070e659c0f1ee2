// RMSNorm + per-256 quant of the residual stream for the batched decode step,
// from the per-32-column block sums of x^2 that the residual GEMM epilogues
// (q3_decode_gemm.cu) leave behind.  Launched as a programmatic dependent of
// the GEMM before it; waits for it before touching memory.
#include "q3_common.cuh"

namespace q3 {

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
  // the 32 block sums (H == 1024) loaded at once, then added in block order
  const float4 *bs = reinterpret_cast<const float4 *>(a.bsum + static_cast<size_t>(m) * 32);
  float4 b4[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) b4[i] = bs[i];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    ss = __fadd_rn(ss, b4[i].x);
    ss = __fadd_rn(ss, b4[i].y);
    ss = __fadd_rn(ss, b4[i].z);
    ss = __fadd_rn(ss, b4[i].w);
  }
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

}  // namespace q3
