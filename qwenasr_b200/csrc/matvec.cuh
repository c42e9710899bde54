// matvec.cuh -- host-side interface of the INT8 matvec family (int8_matvec.cu).
#pragma once
#include "common.cuh"

struct qasr_decoder;
struct qasr_encoder;

namespace qasr {

constexpr int kMvWarps = 4;  // warps per CTA

enum class MvEpi { Store, StoreBias, Residual, SwiGLU, Argmax, QkvPost };

// Per-head epilogue of the fused q|k|v projection (decoder.rs:888-895): when the
// last rows of a 128-wide head are written, that warp applies the q/k
// per-head RMSNorm and NeoX RoPE at positions[m] and appends K/V to the cache.
struct QkvPostParams {
  float *q_out;              // [M, n_heads*128]
  float *k_cache, *v_cache;  // per sequence m at + m*seq_stride, [n_layers, max_seq, kv_dim]
  long seq_stride;
  int layer, max_seq, n_heads, n_kv;
  const int32_t *positions;  // [M]
  const float *q_norm, *k_norm;      // [128]
  const float *cos_tab, *sin_tab;    // [max_seq, 128]
  unsigned *head_ctr;        // [n_heads + 2*n_kv], zero on entry, re-armed by the kernel
};

struct MvParams {
  const float *x;        // [M, K] activations, row stride x_stride
  const int8_t *w;       // [N, K] row-major int8
  const float *scales;   // [N]
  const float *bias;     // [N] (StoreBias)
  float *y;              // Store/Residual: [M, N]; SwiGLU: [M, N/2]; Argmax: logits [M, N] or null
  long x_stride, y_stride;
  int M, K, N;
  unsigned long long *keys;  // Argmax: [M] packed (value, index) keys, zero on entry
  unsigned *counter;         // Argmax: CTA completion counter, zero on entry
  int32_t *ids;              // Argmax: [M] result
};

// Weight-streaming matvec (matvec2.cu).
struct Mv2Params {
  const float *x;        // [M, K] activations, row stride x_stride (16-byte aligned rows)
  long x_stride;
  const float *norm_w;   // RMSNorm weights [K] applied to x while staging (S must be 1), or null
  float eps;
  const int8_t *w;       // [N, K] row-major int8, 16-byte aligned
  const float *scales;   // [N]
  const float *bias;     // [N] (StoreBias)
  float *y;              // as MvParams::y
  long y_stride;
  int M, K, N;
  int S, KS, KC;         // K slices, slice width, bytes of a row per pipeline stage
  float *partial;        // [S, M, N] split-K partial sums (S > 1)
  unsigned *rg_counter;  // [ceil(N/4)] split-K counters, zero on entry, re-armed by the kernel
  unsigned long long *keys;
  unsigned *counter;
  int32_t *ids;
  int *err;              // set to -QASR_ERR_TIMEOUT if a bounded wait gives up (may be null)
  QkvPostParams post;    // MvEpi::QkvPost only
  bool tiled;            // w is in the tiled layout of mv2_tile_weights (same S, KC)
};

int mv2_launch(const Mv2Params &p, MvEpi e, cudaStream_t st, bool pdl);
int mv2_pick_slices(int N, int K, int M, MvEpi e);
__host__ __device__ inline int mv2_chunk(int KS) { return KS % 1024 == 0 ? 1024 : 512; }  // tiled layout

// Tiled layout of an [N, K] INT8 matrix for a split into S slices of KS
// columns with pipeline chunks of KC columns and R = 4 rows per unit: items
// (slice, row group, chunk) stored one after another, each item the 4 row
// segments of KC bytes; inside every 512-byte block of a segment, byte
// 16L + 4q + e holds column 4L + 128q + e (L < 32, q < 4, e < 4), so that a
// warp's 16-byte weight reads and its 16-byte natural-layout x reads are both
// bank-conflict free.  The same bytes as the row-major matrix, permuted.
// Byte offset of element (row, k); n_rg = N / 4.
__host__ __device__ inline size_t mv2_tiled_offset(int row, int k, int KS, int KC, int n_rg) {
  const int slice = k / KS, ks = k % KS, c = ks / KC, kc = ks % KC;
  const int blk = kc >> 9, kk = kc & 511;
  const int pos = (blk << 9) + ((kk & 127) >> 2) * 16 + (kk >> 7) * 4 + (kk & 3);
  const int rg = row >> 2, r = row & 3;
  return ((((size_t)slice * n_rg + rg) * (KS / KC) + c) * 4 + r) * KC + pos;
}
// Re-tile an [N, K] row-major INT8 matrix for split S (device to device).
int mv2_tile_weights(int8_t *dst, const int8_t *src, int N, int K, int S, cudaStream_t st);
inline int mv2_rows(int M) { return 4; }  // rows per warp unit

// Enqueue one matvec.  R = rows per warp (1, 2, 4), 0 = automatic.
void mv_launch(const MvParams &p, MvEpi e, cudaStream_t st, int R);
int mv_pick_rows(int N, MvEpi e);

// Per-device scratch used by the kernel-level fused entry points (not
// re-entrant across concurrently running streams of one device).
int argmax_scratch(unsigned long long **keys, unsigned **counter);
int mv_norm_scratch(float **buf, size_t n_floats);

constexpr int kScratchPartial = 0, kScratchCounter = 1, kScratchDigits = 2, kScratchDigitScale = 3,
              kScratchWeightDigits = 4, kScratchWeightScale = 5, kScratchIm2col = 6, kScratchMelPower = 7,
              kScratchMelMax = 8, kScratchAudio = 9, kScratchMelOut = 10, kScratchEncOut = 11,
              kScratchPrompt = 12, kScratchDecode = 13, kScratchSlots = 14;
int dev_scratch(int slot, size_t bytes, void **out);

// Engine-owned scratch: while an ArenaScope is alive on a thread, dev_scratch
// calls on the arena's device use the arena's buffers.
struct ScratchArena;
ScratchArena *arena_create(int device);
void arena_free(ScratchArena *a);
struct ArenaScope {
  explicit ArenaScope(ScratchArena *a);
  ~ArenaScope();
  ArenaScope(const ArenaScope &) = delete;
  ArenaScope &operator=(const ArenaScope &) = delete;
  ScratchArena *prev;
};
// The engines' own arenas.
ScratchArena *decoder_arena(qasr_decoder *d);
ScratchArena *encoder_arena(qasr_encoder *e);

}  // namespace qasr
