// Internal GEMM interface shared by the SIMT and tensor-core paths.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

enum GemmEpilogue {
  EPI_STORE = 0,     // out = result                          (group_gemm.h:215-220)
  EPI_ADD = 1,       // out += result (residual)              (group_gemm.h:194-214)
  EPI_QUANT = 2,     // per-head int8 quant -> q8/qs          (group_gemm.h:173-193)
  EPI_NORMROPE = 3,  // per-head norm + rope + quant -> q8/qs (norm_rope_quant.h:17-86)
  EPI_SWIGLU = 4,    // gate/up, SwiGLU, per-256 quant        (swiglu_quant.h:164-255)
  EPI_ARGMAX = 5,    // running (max, first idx) per row      (lm_argmax.h:72-182)
};

struct GemmArgs {
  int mode;
  int M, N, K, group;
  const int8_t *a;            // [M][K], row stride a_rb
  long a_rb;
  const char *a_scale;        // [M][K/group] f32, row stride as_rb
  long as_rb;
  const int8_t *b;            // [N][K], row stride b_rb
  long b_rb;
  const float *b_scale;       // [N]
  const int8_t *b2;           // second weight (gate/up: up), same layout as b
  const float *b2_scale;
  char *out;                  // STORE/ADD: f32 [M][N]
  long out_rb;
  char *q8;                   // QUANT/NORMROPE/SWIGLU: i8 [M][N]
  long q8_rb;
  char *qs;                   // scales [M][N/head or N/256]
  long qs_rb;
  const float *nw;            // NORMROPE: [128]
  const char *cos, *sin;      // NORMROPE: [M][64] f32 rows at the absolute positions
  long cos_rb, sin_rb;
  float inv_hd;
  unsigned long long *arg_keys;  // ARGMAX: [M] workspace
  float *best;
  int32_t *bidx;
};

int gemm_simt(const GemmArgs &p, cudaStream_t s);
// CTA-pair tensor-core path for many-row GEMMs (q3_gemm_tc2.cu)
bool gemm_pair_eligible(const GemmArgs &p);
int gemm_pair(const GemmArgs &p, cudaStream_t s);
int gemm_tc(const GemmArgs &p, cudaStream_t s);
bool gemm_tc_eligible(const GemmArgs &p);
int argmax_begin(const GemmArgs &p, cudaStream_t s);
int argmax_end(const GemmArgs &p, cudaStream_t s);

// TMA map of an int8 [rows][cols] matrix (row stride `stride` bytes), 128-byte
// swizzle, box = 128 bytes x box_rows (q3_gemm_tc.cu)
namespace tc {
bool make_map(CUtensorMap *m, const void *base, uint64_t rows, uint64_t cols, uint64_t stride,
              uint32_t box_rows);
}

}  // namespace q3
