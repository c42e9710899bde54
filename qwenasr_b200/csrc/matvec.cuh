// matvec.cuh -- host-side interface of the INT8 matvec family (int8_matvec.cu).
#pragma once
#include "common.cuh"

namespace qasr {

constexpr int kMvWarps = 4;  // warps per CTA

enum class MvEpi { Store, StoreBias, Residual, SwiGLU, Argmax };

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

// Enqueue one matvec.  R = rows per warp (1, 2, 4), 0 = automatic.
void mv_launch(const MvParams &p, MvEpi e, cudaStream_t st, int R);
int mv_pick_rows(int N, MvEpi e);

// Per-device scratch used by the kernel-level fused entry points (not
// re-entrant across concurrently running streams of one device).
int argmax_scratch(unsigned long long **keys, unsigned **counter);
int mv_norm_scratch(float **buf, size_t n_floats);

}  // namespace qasr
