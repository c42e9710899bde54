// umma.cuh -- host interface of the tcgen05 INT8 contraction (umma_matvec.cu).
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "matvec.cuh"

namespace qasr {

// y[m, o] = scales[o] * sum_k w[o, k] * x[m, k] for M <= 8 token rows, with
// the epilogues of the matvec family (MvEpi).  The weights are the
// reference's row-major [N, K] int8 matrix, read by TMA through `tmap`
// (umma_weight_map).  No scratch: split-K partials are reduced inside a
// thread-block cluster.
struct UmmaParams {
  CUtensorMap tmap;
  const float *x;       // [M, K], rows 16-byte aligned (x_stride % 4 == 0)
  long x_stride;
  const float *norm_w;  // RMSNorm weights [K] applied to x first (reference order), or null
  float eps;
  const float *scales;  // [N]
  const float *bias;    // [N] (StoreBias)
  float *y;             // as MvParams::y
  long y_stride;
  int M, K, N;
  unsigned long long *keys;  // Argmax: [M], zero on entry, re-armed
  unsigned *counter;         // Argmax: CTA counter, zero on entry, re-armed
  int32_t *ids;              // Argmax: [M]
  int *err;                  // -QASR_ERR_TIMEOUT if a bounded wait gives up (may be null)
  unsigned long long *tstamp;  // optional [2]: min over CTAs of %globaltimer after the dependency wait,
                               // max at exit (in-step timing of a graph-replayed step; null = off)
  QkvPostParams post;        // MvEpi::QkvPost (head_ctr unused)
  // filled in by umma_launch
  int stages, csize;
};

// Tensor map of an [N, K] int8 matrix: box 128 rows x 128 bytes, 128-byte swizzle.
int umma_weight_map(CUtensorMap *tm, const int8_t *w, int N, int K);
// QASR_ERR_UNSUPPORTED (nothing launched) for shapes it does not cover.
int umma_launch(UmmaParams p, MvEpi e, cudaStream_t st, bool pdl);

// y[t, o] = scales[o] * sum_k w[o, k] * x[t, k] (+ bias[o]) for T token rows on
// the tensor cores (umma_gemm.cu); QASR_ERR_UNSUPPORTED (nothing launched)
// for shapes it does not cover.
int int8_gemm(float *y, long y_stride, const float *x, long x_stride, const int8_t *w, const float *scales,
              const float *bias, int T, int K, int N, cudaStream_t st);

// y[t, o] = sum_k w[o, k] * x[t, k] (+ bias[o]) with f32 weights on the tensor
// cores (three digit planes per operand); QASR_ERR_UNSUPPORTED as above.
int f32_gemm(float *y, long y_stride, const float *x, long x_stride, const float *w, const float *bias, int T, int K,
             int N, cudaStream_t st);
// int8_gemm with a fused epilogue: 1 = add into y (residual), 2 = SwiGLU of
// interleaved (gate, up) row pairs into y [T, N/2].
int int8_gemm_epi(float *y, long y_stride, const float *x, long x_stride, const int8_t *w, const float *scales, int T,
                  int K, int N, int epi, cudaStream_t st);
// int8_gemm with the output rows split at n1 and n2 into three matrices.
int int8_gemm_split3(float *y0, long s0, float *y1, long s1, int n1, float *y2, long s2, int n2, const float *x,
                     long x_stride, const int8_t *w, const float *scales, int T, int K, int N, cudaStream_t st);
// f32 weights [N, K] held as their digit planes (built once).
struct F32Weight {
  int8_t *planes = nullptr;  // [3N, K]
  float *factors = nullptr;  // [N]
  int N = 0, K = 0;
  CUtensorMap tm;
};
// QASR_ERR_UNSUPPORTED for shapes the tensor-core GEMM does not take.
int f32_weight_prepare(F32Weight *pw, const float *w, int N, int K, cudaStream_t st);
void f32_weight_free(F32Weight *pw);
int f32_gemm_prepared(float *y, long y_stride, const float *x, long x_stride, const F32Weight &w, const float *bias,
                      int T, cudaStream_t st);
// A 3x3 / stride 2 / padding 1 convolution of a channel-last activation
// [B, h_in, w_in, C] as an implicit GEMM over w (channel-fastest patch order,
// K = 9*C): no im2col matrix is written.  QASR_ERR_UNSUPPORTED as above.
int f32_gemm_prepared_conv(float *y, long y_stride, const float *act, int C, int h_in, int w_in, int B, int h_out,
                           int w_out, const F32Weight &w, const float *bias, cudaStream_t st);
int f32_gemm_prepared_split3(float *y0, long s0, float *y1, long s1, int n1, float *y2, long s2, int n2,
                             const float *x, long x_stride, const F32Weight &w, const float *bias, int T,
                             cudaStream_t st);
// The same on CUDA cores, any shape.
int f32_gemm_fallback(float *y, const float *x, const float *w, const float *bias, int T, int K, int N,
                      cudaStream_t st);

// Driver entry point cuTensorMapEncodeTiled (resolved once).
void *tensor_map_encoder();

// kernels::bidirectional_attention with the longest window (keys) known on
// the host (encoder.cu).
int bidir_attention_launch(float *out, const float *q, const float *k, const float *v, int seq, int n_heads,
                           int head_dim, float scale, const int32_t *window_starts, int n_windows, int max_window,
                           cudaStream_t st);

}  // namespace qasr
