// Decode-sized GEMMs with the K-group reduction inside a thread-block cluster
// (q3_decode_gemm.cu).  Internal to the batched decode step.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

enum DgemmMode { DG_QKV = 0, DG_RESID = 1, DG_SWIGLU = 2, DG_PART = 3 };

constexpr int kTpMaxRanks = 8;

struct DgemmArgs {
  int M;                       // rows (sequences), <= 64
  int K, G;                    // set by dgemm_launch
  const char *a_scale;         // activation scales [M][K/group] f32, row stride as_rb
  long as_rb;
  const float *ws[3];          // weight scales per weight matrix
  int t1, t2;                  // QKV / RESID: 128-row tile boundaries between the matrices
  // QKV epilogue
  int heads, kv_heads;
  const float *nq, *nk;        // [128]
  const float *cos_t, *sin_t;  // [max_seq][64] tables
  const int32_t *pos;          // [M]
  float inv_hd;
  int8_t *q8;                  // [M][heads * 128]
  float *qs;                   // [M][heads]
  char *pk, *pv, *pks, *pvs;   // this layer's page pools
  const uint16_t *tables;      // [M][max_pages]
  uint32_t max_pages;
  // RESID epilogue
  float *x;                    // [M][H] residual, updated in place
  float *bsum;                 // [M][H / 32] tree sums of x^2 per 32-column block
  int H;
  // SWIGLU epilogue
  int8_t *s8;                  // [M][I]
  float *ss;                   // [M][I / 256]
  int I;
  // PART epilogue (tensor-parallel O / down): the dequantised partial of every
  // K group goes, unsummed, to slot slot0 + g of every rank's receive buffer
  // [slots][M][H] (peer pointers), after which each CTA adds 1 to its signal
  // counter at every rank
  float *dst[kTpMaxRanks];
  unsigned *sig[kTpMaxRanks];  // per rank: this rank's counter for this buffer
  unsigned *expect;            // this rank's expected counts [ranks] for this buffer
  int inc[kTpMaxRanks];        // CTAs each rank's producer launches per use
  int ndst, slot0;
};

// mode QKV: nmaps = 3 (Q, K, V weights), group 256; RESID: nmaps = 1, group 128
// or 256; SWIGLU: nmaps = 2 (gate, up), group 256; PART: nmaps = 1, group 128 or
// 256, any number of groups.  w[i]: [rows[i]][K] int8, row stride w_rb (0: K);
// a: [M][K] int8 (row stride a_rb).  Launched as a programmatic dependent of
// the kernel before it.
int dgemm_launch(int mode, int nmaps, const int8_t *const *w, const int *rows, const int8_t *a,
                 long a_rb, int K, int group, const DgemmArgs &args, cudaStream_t s,
                 long w_rb = 0);
// number of CTAs a PART launch of `rows` output features and `groups` K groups uses
inline int dgemm_part_ctas(int rows, int groups) { return (rows / 128) * groups; }
int dgemm_device_status_take();

}  // namespace q3
