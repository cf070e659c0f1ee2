// Tensor-parallel decode across the GPUs of one node (q3_tp.cu): the shard of
// the model each rank owns, the exchange region every rank maps from every
// other rank (CUDA IPC over NVLink), and the kernels that consume it.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "q3_decode_gemm.h"
#include "q3_ops.h"

namespace q3 {

constexpr int kTpMaxSlots = 16;   // K groups of O (heads) and down (I / 256)

// exchange buffers of the region
enum TpBuf { TP_O = 0, TP_DOWN = 1, TP_KEYS = 2, TP_NBUF = 3 };

struct TpComm {
  int rank, world;
  uint32_t max_seqs, hidden, heads, mlp_groups;
  char *local;                    // this rank's region (cudaMalloc)
  char *peer[kTpMaxRanks];        // every rank's region as mapped here (peer[rank] = local)
  bool opened[kTpMaxRanks];       // peer[q] came from cudaIpcOpenMemHandle
  size_t bytes;
  size_t off_sig, off_expect, off_orecv, off_drecv, off_keys, off_nccl;
  unsigned long long wait_ns;     // limit of every bounded wait on the peers' signals
  q3_tp_shard shard[kTpMaxRanks];
  int reduce_nccl;                // O/down reductions by ncclAllReduce (comparison variant)
  void *nccl;                     // ncclComm_t of the variant
};

// the comparison variant's reduction: this rank's group partials (slots
// 0..slots-1 of its receive buffer) summed in order, then summed over the
// ranks by ncclAllReduce (ring/tree order: not the reference's order)
int tp_nccl_reduce(const TpComm &c, const float *recv, int slots, int B, int H, float *out,
                   cudaStream_t s);

constexpr unsigned long long kTpDefaultWaitNs = 2000000000ull;

// per-buffer counters of a region: sig[buf][producer rank], expect[buf][producer rank]
inline unsigned *tp_sig(const TpComm &c, int q, int buf, int producer) {
  return reinterpret_cast<unsigned *>(c.peer[q] + c.off_sig) + buf * kTpMaxRanks + producer;
}
inline unsigned *tp_expect(const TpComm &c, int buf) {
  return reinterpret_cast<unsigned *>(c.local + c.off_expect) + buf * kTpMaxRanks;
}

// x += (((0 + p_0) + p_1) + ... + p_{slots-1}) row by row once every rank's
// producer has signalled, then RMSNorm(w) + per-256 quant of x -> h8/hs
struct TpReduceArgs {
  const float *recv;              // [slots][B][H] this rank's receive buffer
  int slots;
  const unsigned *sig;            // this rank's counters of the buffer [ranks]
  const unsigned *expect;         // [ranks]
  int world;
  float *x;                       // [B][H]
  const float *w;                 // [H]
  float inv;
  int B, H;
  int8_t *h8;                     // [B][H]
  float *hs;                      // [B][H/256]
  unsigned long long wait_ns;     // bounded wait on the signals
};
int tp_reduce_norm(const TpReduceArgs &a, cudaStream_t s);

// every rank's (best, first index) of its vocabulary slice -> the greedy id
int tp_argmax_exchange(const TpComm &c, const float *best, const int32_t *bidx, uint32_t v0,
                       int B, int32_t *next_ids, cudaStream_t s);

int tp_device_status_take();

// ---- tensor-parallel prefill (q3_tp_prefill_batch) --------------------------
// Exchanges of the prefill, all all-gathers: the attention output o8/os of
// each rank's q heads and the SwiGLU output s8/ss of its MLP groups; for each
// RMSNorm of the column-sharded residual, the 32-column block sums of x^2,
// the 128-column maxima of |h| and the quantised h8 of each rank's columns;
// the last rows' residual columns; the argmax keys.
enum PfEx { PF_O = 0, PF_S = 1, PF_NB = 2, PF_NA = 3, PF_NH = 4, PF_XL = 5, PF_KEYS = 6, PF_NEX = 7 };
constexpr int kPfPushCtas = 264;     // CTAs of every push (all ranks use the same count)

struct PfComm {
  int rank, world;
  uint32_t max_rows, max_seqs, hidden, heads, inter;
  char *local;                    // this rank's region (cudaMalloc)
  char *peer[kTpMaxRanks];
  bool opened[kTpMaxRanks];
  size_t bytes, off_sig, off_o8, off_os, off_x, off_s8, off_ss, off_keys;
  size_t off_h8, off_bsum, off_amax;   // [rows][H] i8, [rows][H/32] f32, [rows][H/128] f32
  unsigned gen[PF_NEX];           // rounds of each exchange so far (host count)
  unsigned long long wait_ns;
  q3_tp_shard shard[kTpMaxRanks];
  uint32_t col0[kTpMaxRanks], cols[kTpMaxRanks];   // residual columns of each rank
};

// a row slice [offset, offset + width) bytes of rows 0..rows-1 of a buffer with
// row stride row_bytes that every rank holds at the same region offset
struct PfSeg {
  size_t base;                    // region offset of the buffer
  uint32_t offset, width, row_bytes;
};
// copy this rank's segments into every other rank's region, then signal
// exchange `ex` at every rank (this one included); wait_pf blocks the stream
// until every rank's round `gen` of `ex` has arrived here
int pf_push(PfComm &c, int ex, const PfSeg *segs, int nseg, uint32_t rows, cudaStream_t s);
int pf_wait(const PfComm &c, int ex, cudaStream_t s);
// every rank's (best, index in its vocabulary slice) of each sequence -> the greedy id
int pf_argmax_exchange(PfComm &c, const float *best, int32_t *idx_then_ids, uint32_t v0, int B,
                       cudaStream_t s);

}  // namespace q3
