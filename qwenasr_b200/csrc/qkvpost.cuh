// qkvpost.cuh -- the per-head epilogue of the fused q|k|v projection
// (crates/qwen-asr/src/decoder.rs:888-895), shared by the matvec kernels.
#pragma once
#include "common.cuh"
#include "matvec.cuh"

namespace qasr {

// q/k per-head RMSNorm (tree-order sum) + NeoX RoPE at positions[m], or the V
// copy, for one 128-wide head held as a float4 per lane (lane L = elements
// 4L..4L+3; the RoPE partner of a lane is lane^16).
QASR_DEV void qkv_head_post(const QkvPostParams &q, float eps, int h, int m, float4 v, int *err) {
  const int lane = threadIdx.x & 31;
  const int pos = q.positions[m];
  if (pos < 0 || pos >= q.max_seq) {
    if (lane == 0 && err) atomicExch(err, 2);
    return;
  }
  const int kv_dim = q.n_kv * 128;
  const size_t cache_row = (size_t)m * q.seq_stride + ((size_t)q.layer * q.max_seq + pos) * kv_dim;
  if (h >= q.n_heads + q.n_kv) {
    reinterpret_cast<float4 *>(q.v_cache + cache_row + (h - q.n_heads - q.n_kv) * 128)[lane] = v;
    return;
  }
  const float *nw = h < q.n_heads ? q.q_norm : q.k_norm;
  float ss = __fmul_rn(v.x, v.x);
  ss = fmaf(v.y, v.y, ss);
  ss = fmaf(v.z, v.z, ss);
  ss = fmaf(v.w, v.w, ss);
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), eps)));
  const float4 w4 = reinterpret_cast<const float4 *>(nw)[lane];
  v.x = __fmul_rn(__fmul_rn(v.x, inv), w4.x);
  v.y = __fmul_rn(__fmul_rn(v.y, inv), w4.y);
  v.z = __fmul_rn(__fmul_rn(v.z, inv), w4.z);
  v.w = __fmul_rn(__fmul_rn(v.w, inv), w4.w);
  float4 pr;
  pr.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
  pr.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
  pr.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
  pr.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
  const float4 c = reinterpret_cast<const float4 *>(q.cos_tab + (size_t)pos * 128)[lane];
  const float4 s = reinterpret_cast<const float4 *>(q.sin_tab + (size_t)pos * 128)[lane];
  const float sg = lane < 16 ? -1.0f : 1.0f;  // first half: x1*c - x2*s; second: x2*c + x1*s
  float4 o;
  o.x = __fadd_rn(__fmul_rn(v.x, c.x), __fmul_rn(sg * pr.x, s.x));
  o.y = __fadd_rn(__fmul_rn(v.y, c.y), __fmul_rn(sg * pr.y, s.y));
  o.z = __fadd_rn(__fmul_rn(v.z, c.z), __fmul_rn(sg * pr.z, s.z));
  o.w = __fadd_rn(__fmul_rn(v.w, c.w), __fmul_rn(sg * pr.w, s.w));
  if (h < q.n_heads)
    reinterpret_cast<float4 *>(q.q_out + (size_t)m * q.n_heads * 128 + h * 128)[lane] = o;
  else
    reinterpret_cast<float4 *>(q.k_cache + cache_row + (h - q.n_heads) * 128)[lane] = o;
}

}  // namespace qasr
