// Internal attention interface (single sequence or a batch of sequences).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace q3 {

struct AttnArgs {
  const char *q8;      // [n_seqs*q_rows][heads*128] i8
  long q_rb;
  const char *qs;      // [n_seqs*q_rows][heads] f32
  long qs_rb;
  char *o8;
  long o_rb;
  char *os;
  long os_rb;
  const char *k, *v, *ks, *vs;   // page pool (this layer)
  const uint16_t *table;         // [n_seqs][table_stride]
  long table_stride;
  uint32_t page_tokens, page_bytes, row_bytes, scale_page_bytes, scale_row_bytes;
  int heads, kv_heads, q_rows;
  int kv_len;                    // when kv_len_dev is null
  const int *kv_len_dev;         // [n_seqs] per-sequence kv length
  int causal;
  float qk_scale;
  // optional, a mixed batch: sequence s has item_rows[s] query rows (at most
  // q_rows) starting at row item_row0[s] of q8/qs/o8/os; null: q_rows rows
  // each, sequence s at row s * q_rows
  const int *item_rows, *item_row0;
};

int attention_launch(const AttnArgs &p, int n_seqs, cudaStream_t s);

// Decode attention: one query row per sequence, GQA group of 2, head_dim 128,
// 32-token pages of a page pool (q3_attention_decode.cu).
struct DecodeAttnArgs {
  const char *q8;      // [n_seqs][heads*128] i8
  long q_rb;
  const char *qs;      // [n_seqs][heads] f32
  long qs_rb;
  char *o8;
  long o_rb;
  char *os;
  long os_rb;
  const char *ks, *vs;           // per-head scale pools of this layer
  const uint16_t *table;         // [n_seqs][table_stride]
  long table_stride;
  uint32_t page_bytes, row_bytes, scale_page_bytes, scale_row_bytes;
  const int *kv_len;             // [n_seqs]
  float qk_scale;
  uint32_t num_pages;            // pages in the pool (page indices are checked)
};

// pdl: launched as a programmatic dependent of the kernel before it
// Causal prompt attention on the tensor cores (q3_attention_prefill.cu): query
// row t of sequence s is row s*T + t of q8/qs/o8/os, at position t; the keys
// are positions 0..t of the sequence's pages (32 tokens, head_dim 128).
struct PrefillAttnArgs {
  const char *qs;      // [n_seqs*T][heads] f32
  long qs_rb;
  char *o8;            // [n_seqs*T][heads*128] i8
  long o_rb;
  char *os;            // [n_seqs*T][heads] f32
  long os_rb;
  const char *ks, *vs;           // per-head scale pools of this layer
  const uint16_t *table;         // [n_seqs][table_stride]
  long table_stride;
  uint32_t scale_page_bytes, scale_row_bytes, num_pages;
  int heads, kv_heads, T;
  float qk_scale;
};
int attention_prefill_launch(const PrefillAttnArgs &p, const void *q8, long q_rb, int M,
                             const void *k_pool, const void *v_pool, uint32_t page_bytes,
                             uint32_t row_bytes, int n_seqs, cudaStream_t s);

int attention_decode_launch(const DecodeAttnArgs &p, const void *k_pool, const void *v_pool,
                            uint32_t num_pages, int kv_heads, int n_seqs, cudaStream_t s,
                            bool pdl = false);

}  // namespace q3
