// rowops.cuh -- warp-level row reductions in the reference's summation order.
//
// The reference's x86_64 norms (crates/qwen-asr/src/kernels/avx.rs:377-481)
// accumulate a row in two 8-lane AVX registers: acc0 lane l sees elements
// 16j+l, acc1 lane l sees 16j+8+l, one more 8-block (if any) goes to acc0,
// then hsum_ps(acc0+acc1) and a scalar tail.  Here warp lanes 0..15 are those
// 16 accumulator lanes (lane L <-> element 16j+L), each running the same
// sequential chain, and shuffles rebuild hsum_ps's tree.  The result is the
// reference's f32 value bit for bit.  The row must already be in shared memory.
#pragma once
#include "common.cuh"

namespace qasr {

// Combine the 16 lane accumulators (lanes 0..15) as hsum_ps(acc0 + acc1).
// Every lane of the warp must call this; the result is valid in all lanes.
QASR_DEV float hsum16_avx_order(float acc) {
  const unsigned full = 0xffffffffu;
  float v = __fadd_rn(acc, __shfl_down_sync(full, acc, 8));  // lanes 0..7: acc0_l + acc1_l
  float s = __fadd_rn(v, __shfl_down_sync(full, v, 4));      // lanes 0..3: v_i + v_{i+4}
  float t = __fadd_rn(s, __shfl_down_sync(full, s, 1));      // lane 0: s0+s1, lane 2: s2+s3
  float r = __fadd_rn(t, __shfl_down_sync(full, t, 2));      // lane 0: (s0+s1)+(s2+s3)
  return __shfl_sync(full, r, 0);
}

// Number of elements covered by the vector loops of the AVX row kernels.
QASR_DEV int avx_vector_extent(int n) { return (n / 16) * 16 + ((n & 15) >= 8 ? 8 : 0); }

// 1/sqrt(sum(x^2)/n + eps) exactly as avx::rms_norm_row computes it.
QASR_DEV float rms_inv_ref(const float *xs, int n, float eps) {
  const int lane = threadIdx.x & 31;
  const int n16 = n / 16;
  float acc = 0.0f;
  if (lane < 16) {
    for (int j = 0; j < n16; ++j) {
      float v = xs[16 * j + lane];
      acc = fmaf(v, v, acc);
    }
    if ((n & 15) >= 8 && lane < 8) {
      float v = xs[16 * n16 + lane];
      acc = fmaf(v, v, acc);
    }
  }
  float sum = hsum16_avx_order(acc);
  if (lane == 0)
    for (int i = avx_vector_extent(n); i < n; ++i) sum = __fadd_rn(sum, __fmul_rn(xs[i], xs[i]));
  sum = __shfl_sync(0xffffffffu, sum, 0);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), eps)));
}

// Mean and 1/std exactly as avx::layer_norm_row computes them.
QASR_DEV void ln_stats_ref(const float *xs, int n, float eps, float &mean_out, float &inv_out) {
  const int lane = threadIdx.x & 31;
  const int n16 = n / 16;
  const bool has8 = (n & 15) >= 8;
  const int vext = avx_vector_extent(n);
  float acc = 0.0f;
  if (lane < 16) {
    for (int j = 0; j < n16; ++j) acc = __fadd_rn(acc, xs[16 * j + lane]);
    if (has8 && lane < 8) acc = __fadd_rn(acc, xs[16 * n16 + lane]);
  }
  float mean = hsum16_avx_order(acc);
  if (lane == 0)
    for (int i = vext; i < n; ++i) mean = __fadd_rn(mean, xs[i]);
  mean = __fdiv_rn(__shfl_sync(0xffffffffu, mean, 0), (float)n);

  acc = 0.0f;
  if (lane < 16) {
    for (int j = 0; j < n16; ++j) {
      float d = __fsub_rn(xs[16 * j + lane], mean);
      acc = fmaf(d, d, acc);
    }
    if (has8 && lane < 8) {
      float d = __fsub_rn(xs[16 * n16 + lane], mean);
      acc = fmaf(d, d, acc);
    }
  }
  float var = hsum16_avx_order(acc);
  if (lane == 0)
    for (int i = vext; i < n; ++i) {
      float d = __fsub_rn(xs[i], mean);
      var = __fadd_rn(var, __fmul_rn(d, d));
    }
  var = __shfl_sync(0xffffffffu, var, 0);
  mean_out = mean;
  inv_out = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(var, (float)n), eps)));
}

// Copy n floats global -> shared with the whole warp (16-byte vectors when
// both pointers allow it).
QASR_DEV void warp_load_row(float *dst, const float *src, int n) {
  const int lane = threadIdx.x & 31;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 && (n & 3) == 0) {
    const float4 *s4 = reinterpret_cast<const float4 *>(src);
    float4 *d4 = reinterpret_cast<float4 *>(dst);
    for (int i = lane; i < n / 4; i += 32) d4[i] = s4[i];
  } else {
    for (int i = lane; i < n; i += 32) dst[i] = src[i];
  }
  __syncwarp();
}

}  // namespace qasr
