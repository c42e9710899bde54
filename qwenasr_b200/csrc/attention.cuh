// attention.cuh -- host-side interface of the decode attention kernel.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace qasr {

// Warps per CTA: 8 for a batch of up to 3 sequences; 6 from 4 sequences on,
// where the smaller shared-memory footprint lets an attention CTA share an SM
// with the q/k/v kernel before it (measured: -3.5% step time at M=8, +2.5% at
// M=1, hence the split).
#ifndef QASR_ATTN_WIDE_WARPS
#define QASR_ATTN_WIDE_WARPS 6
#endif
constexpr int kAttnMaxWarps = 8, kAttnWideWarps = QASR_ATTN_WIDE_WARPS, kAttnWideFromM = 4;
// Decode-attention CTAs per SM (the grid is this many times the SM count).
#ifndef QASR_ATTN_CTAS_PER_SM
#define QASR_ATTN_CTAS_PER_SM 1
#endif
constexpr int kAttnCtasPerSm = QASR_ATTN_CTAS_PER_SM;
#ifndef QASR_ATTN_TILE
#define QASR_ATTN_TILE 8
#endif
#ifndef QASR_ATTN_STAGES
#define QASR_ATTN_STAGES 2
#endif
constexpr int kAttnTile = QASR_ATTN_TILE;      // keys per TMA tile (one warp's pipeline stage)
constexpr int kAttnStages = QASR_ATTN_STAGES;  // K+V tiles in flight per warp
constexpr int kAttnPartStride = 132;  // floats per (segment, head) partial: o[128], max, sum, pad
#ifndef QASR_ATTN_MIN_KEYS
#define QASR_ATTN_MIN_KEYS 256
#endif
constexpr int kAttnMinKeys = QASR_ATTN_MIN_KEYS;  // keys per CTA at least: short histories use fewer CTAs (fewer partials)
#ifndef QASR_ATTN_FLOOR_KEYS
#define QASR_ATTN_FLOOR_KEYS 64
#endif
// From kAttnWideFromM sequences on, when kAttnMinKeys keys per CTA would
// leave CTAs of the grid idle, down to kAttnFloorKeys keys per CTA (about one
// 8-key tile per warp).  Measured: -1.6 % step time at M=8 / KV 480, -2.7 %
// at M=4 / KV 700, unchanged at M=8 / KV 1024; at M=1 it costs +3.8 %, hence
// the batch threshold.
constexpr int kAttnFloorKeys = QASR_ATTN_FLOOR_KEYS;

struct AttnDecodeParams {
  CUtensorMap tm_k;      // 2D tensor maps over the whole cache: [rows = B*L*max_seq, kv_dim] f32,
  CUtensorMap tm_v;      // box [kAttnTile rows, 128 floats]
  const float *q;        // [M, n_heads*128] normalised + rotated queries
  long q_stride;
  int layer, n_layers, max_seq, n_kv_heads;
  const int32_t *positions;  // [M]: attend over rows 0..positions[m]
  float scale;
  int M;
  int floor_keys;        // keys per CTA at least when kAttnMinKeys leaves CTAs idle (set by attn_decode_launch)
  float *partials;       // [gridDim + M*n_kv, G, kAttnPartStride]
  unsigned *counters;    // [M*n_kv], zero on entry, re-armed by the kernel
  float *out;            // [M, n_heads*128]
  long out_stride;
  int *err;              // -QASR_ERR_TIMEOUT on a bounded-wait timeout
  unsigned long long *tstamp;  // optional [2]: first dependency-met and last exit %globaltimer (null = off)
};

// One segment of a batched causal attention: query rows q_row0 .. q_row0 +
// seq_q of q/out, keys/values at k/v + kv_off (floats), seq_k keys, the
// first query at position q_offset.
struct CaSeg {
  long q_row0;
  int seq_q, seq_k, q_offset;
  long kv_off;
};
int causal_attention_segments(float *out, const float *q, const float *k, const float *v, const CaSeg *segs, int n,
                              int max_seq_q, int n_heads, int n_kv_heads, int head_dim, float scale, cudaStream_t st);

// 2D tensor map over a KV cache [rows, kv_dim] f32 with box [kAttnTile, 128].
int attn_make_tensor_map(CUtensorMap *tm, const float *base, long rows, int kv_dim);
int attn_decode_launch(const AttnDecodeParams &p, int group, cudaStream_t st, bool pdl);
int attn_grid();         // SMs of the current device
int attn_decode_grid();  // CTAs of one decode-attention launch (size of the partials buffer)

}  // namespace qasr
