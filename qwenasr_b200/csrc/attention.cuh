// attention.cuh -- host-side interface of the decode attention kernel.
#pragma once
#include "common.cuh"

namespace qasr {

constexpr int kAttnWarps = 4;
constexpr int kAttnPartStride = 132;  // floats per (split, head) partial: o[128], max, sum, pad
constexpr int kAttnMaxSplits = 64;

struct AttnDecodeParams {
  const float *q;        // [M, n_heads*128] normalised + rotated queries
  long q_stride;
  const float *k_cache;  // sequence m at k_cache + m*seq_stride, [n_layers, max_seq, kv_dim]
  const float *v_cache;
  long seq_stride;
  int layer, max_seq, kv_dim, n_kv_heads;
  const int32_t *positions;  // [M]: attend over rows 0..positions[m]
  float scale;
  int M, splits;
  float *partials;       // [M, n_kv, splits, G, kAttnPartStride]
  unsigned *counters;    // [M, n_kv], zero on entry, re-armed by the kernel
  float *out;            // [M, n_heads*128]
  long out_stride;
};

int attn_pick_splits(int M, int n_kv_heads, int max_len);
int attn_decode_launch(const AttnDecodeParams &p, int group, cudaStream_t st);

}  // namespace qasr
