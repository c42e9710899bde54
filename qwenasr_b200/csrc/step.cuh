// step.cuh -- host interface of the persistent decode-step kernel
// (decode_step.cu): one launch runs decoder_forward_int8
// (crates/qwen-asr/src/decoder.rs:845-965) for up to 8 sequences, all
// layers, the final norm, the lm head and the argmax.
#pragma once
#include <cuda.h>

#include "common.cuh"

namespace qasr {

constexpr int kStepMaxM = 8;
constexpr int kStepMaxPairs = 64;    // sequences x kv heads
constexpr int kStepMaxSlots = 16;    // digit tiles staged per phase (hidden <= 2048)
constexpr int kStepSyncPerLayer = 32;
constexpr int kStepMaxLayers = 48;   // layer pointer table kept in shared memory

// Per-layer pointers the kernel reads (device array, one entry per layer).
struct StepLayerPtrs {
  const float *sqkv, *so, *sgu, *sdown;               // per-row INT8 scales
  const float *q_norm, *k_norm, *in_norm, *post_norm;  // norm weights
};

struct StepParams {
  // device array of tensor maps (64-byte aligned): [0] K cache, [1] V cache
  // (box 16 rows x 128 floats), [2] lm head, then per layer q|k|v, o,
  // gate/up, down (box 128 rows x 128 bytes, 128-byte swizzle)
  const CUtensorMap *maps;
  const StepLayerPtrs *layers;
  const float *final_norm, *lm_s;
  float *x;       // [M, H] residual stream (the embedding rows on entry)
  float *q_out;   // [M, n_heads*128]
  float *attn;    // [M, n_heads*128]
  float *h;       // [M, I]
  float *k_cache, *v_cache;
  long seq_stride;
  const float *rope_cos, *rope_sin;
  const int32_t *pos;  // [M]
  // scratch, all zero when the kernel starts (one memset before each launch)
  unsigned *sync;            // [n_layers * kStepSyncPerLayer]: per layer [0,8) kv-head flags, 8 attention
                             // pairs, 9 o-proj, 10 gate/up, 11 down row tiles done; [16,24) max|attn| and
                             // [24,32) max|h| per token (float bits)
  unsigned *tile_ctr;        // [256] split-K arrivals per row tile
  unsigned *pair_ctr;        // [kStepMaxPairs] attention contributors per pair
  unsigned long long *keys;  // [8] argmax keys
  unsigned *am_ctr;          // lm-head CTA arrivals
  long long *acc;            // [acc_rows][8 tokens] split-K sums (each finisher clears its rows again)
  float *part;               // attention partials [(grid + kStepMaxPairs) * 2 * 132] (not zeroed)
  float *logits;             // [M, V] or null
  int32_t *next;             // [M] greedy ids
  int *err;
  // optional phase timeline (null: off): CTA c writes %globaltimer stamps at
  // trace[c * step_trace_stride(L) + ...] (see step_trace_stride)
  unsigned long long *trace;
  int M, H, I, NQ, NKV, L, V, max_seq;
  float eps, scale;
  int S[4];                  // K chunks per row tile: q|k|v, o, gate/up, down
  int stages, kstages, slots;  // 16 KB stages of the weight and the K/V rings, digit tiles of 4 KB
};

// Stamps per CTA of the phase timeline: per layer five phases (q|k|v,
// attention, o-proj, gate/up, down) of four stamps each (entry, dependency
// met, digits staged / history streamed, results published), then four for
// the lm head.
__host__ __device__ inline int step_trace_stride(int n_layers) { return n_layers * 20 + 4; }

// Bytes of the zeroed scratch block and its layout for a decoder shape.
struct StepScratch {
  size_t sync, tile_ctr, pair_ctr, keys, am_ctr, acc, total;  // byte offsets, total size
};
StepScratch step_scratch_layout(int n_layers, long acc_rows);

// QASR_OK and a filled plan (S, stages, slots) when the kernel covers the
// shape, QASR_ERR_UNSUPPORTED otherwise.
int step_plan(StepParams &p, int grid);
// One decode step: the kernel on `grid` CTAs (one per SM, co-resident).
int step_launch(const StepParams &p, int grid, cudaStream_t st);
// 2D tensor map over a KV cache [rows, kv_dim] f32 with box [16 rows, 128 floats].
int step_kv_map(CUtensorMap *tm, const float *base, long rows, int kv_dim);

}  // namespace qasr
