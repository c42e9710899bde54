// qkvpost.cuh -- the per-head epilogue of the fused q|k|v projection
// (crates/qwen-asr/src/decoder.rs:888-895), shared by the matvec kernels.
#pragma once
#include "common.cuh"
#include "matvec.cuh"

namespace qasr {

// Epilogue operands of one (head, token) that depend on nothing computed in
// the step: the token's position, its RoPE cos/sin elements and the head's
// norm weights (lane L: elements 4L..4L+3).  Loading them ahead of the
// accumulator keeps dependent loads off the epilogue's path.
struct QkvPostOperands {
  int pos;
  float4 c, s, w;
};

QASR_DEV QkvPostOperands qkv_post_operands(const QkvPostParams &q, int h, int m) {
  const int lane = threadIdx.x & 31;
  QkvPostOperands o;
  o.pos = q.positions[m];
  o.c = o.s = o.w = make_float4(0.f, 0.f, 0.f, 0.f);
  if (h < q.n_heads + q.n_kv && o.pos >= 0 && o.pos < q.max_seq) {
    o.c = reinterpret_cast<const float4 *>(q.cos_tab + (size_t)o.pos * 128)[lane];
    o.s = reinterpret_cast<const float4 *>(q.sin_tab + (size_t)o.pos * 128)[lane];
    o.w = reinterpret_cast<const float4 *>(h < q.n_heads ? q.q_norm : q.k_norm)[lane];
  }
  return o;
}

// q/k per-head RMSNorm (tree-order sum) + NeoX RoPE at positions[m], or the V
// copy, for one 128-wide head held as a float4 per lane (lane L = elements
// 4L..4L+3; the RoPE partner of a lane is lane^16), with its operands.
QASR_DEV void qkv_head_post(const QkvPostParams &q, float eps, int h, int m, float4 v, const QkvPostOperands &op,
                            int *err) {
  const int lane = threadIdx.x & 31;
  const int pos = op.pos;
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
  float ss = __fmul_rn(v.x, v.x);
  ss = fmaf(v.y, v.y, ss);
  ss = fmaf(v.z, v.z, ss);
  ss = fmaf(v.w, v.w, ss);
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), eps)));
  const float4 w4 = op.w;
  v.x = __fmul_rn(__fmul_rn(v.x, inv), w4.x);
  v.y = __fmul_rn(__fmul_rn(v.y, inv), w4.y);
  v.z = __fmul_rn(__fmul_rn(v.z, inv), w4.z);
  v.w = __fmul_rn(__fmul_rn(v.w, inv), w4.w);
  float4 pr;
  pr.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
  pr.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
  pr.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
  pr.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
  const float4 c = op.c, s = op.s;
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

QASR_DEV void qkv_head_post(const QkvPostParams &q, float eps, int h, int m, float4 v, int *err) {
  qkv_head_post(q, eps, h, m, v, qkv_post_operands(q, h, m), err);
}

}  // namespace qasr
