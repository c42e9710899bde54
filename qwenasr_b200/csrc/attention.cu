// attention.cu -- GQA causal attention (kernels::causal_attention,
// crates/qwen-asr/src/kernels/mod.rs:1124-1207).
//
// Two kernels:
//  * causal_attention_kernel: the general kernel-level entry (any seq_q,
//    e.g. prefill).  One warp per (query, head), lanes over head dims, the
//    reference's per-key online softmax update (mod.rs:1154-1164).
//  * attn_decode_kernel: the decode step of the engine.  Flash-decoding over
//    the f32 KV cache: the keys of one (sequence, kv head) are split across
//    CTAs, each CTA serves both query heads of the GQA group so every K/V row
//    is read from HBM exactly once, and the last CTA of a (sequence, kv head)
//    merges the partial softmax states (counter + threadfence, no spin).
#include "common.cuh"
#include "attention.cuh"

namespace qasr {

// ------------------------------------------------------------------ general
template <int EPL>  // elements per lane: head_dim / 32
__global__ void __launch_bounds__(256)
causal_attention_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ k,
                        const float *__restrict__ v, int seq_q, int seq_k, int n_heads, int n_kv_heads, float scale,
                        int q_offset) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long task = (long)blockIdx.x * 8 + warp;
  if (task >= (long)seq_q * n_heads) return;
  const int i = (int)(task / n_heads), h = (int)(task % n_heads);
  const int hd = EPL * 32;
  const int kv_h = h / (n_heads / n_kv_heads);
  const long q_hidden = (long)n_heads * hd, kv_hidden = (long)n_kv_heads * hd;
  float qv[EPL], o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qv[e] = q[i * q_hidden + (long)h * hd + lane * EPL + e];
    o[e] = 0.0f;
  }
  const int k_end = min(q_offset + i + 1, seq_k);
  float max_score = -1e30f, sum_exp = 0.0f;
  for (int j = 0; j < k_end; ++j) {
    const float *kr = k + j * kv_hidden + (long)kv_h * hd + lane * EPL;
    const float *vr = v + j * kv_hidden + (long)kv_h * hd + lane * EPL;
    float d = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) d = fmaf(qv[e], kr[e], d);
    const float score = __fmul_rn(warp_sum(d), scale);
    if (score > max_score) {
      const float corr = expf(__fsub_rn(max_score, score));
      sum_exp = __fadd_rn(__fmul_rn(sum_exp, corr), 1.0f);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(o[e], corr, vr[e]);
      max_score = score;
    } else {
      const float wt = expf(__fsub_rn(score, max_score));
      sum_exp = __fadd_rn(sum_exp, wt);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(vr[e], wt, o[e]);
    }
  }
  const float inv = sum_exp > 0.0f ? __fdiv_rn(1.0f, sum_exp) : 0.0f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[i * q_hidden + (long)h * hd + lane * EPL + e] = sum_exp > 0.0f ? __fmul_rn(o[e], inv) : o[e];
}

// ------------------------------------------------------------------- decode
// grid = (splits, n_kv_heads, M), 4 warps.  head_dim 128, GQA group size G.
template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32)
attn_decode_kernel(AttnDecodeParams p) {
  __shared__ float sp[kAttnWarps][G][32];          // per-warp softmax weights of a key group
  __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
  __shared__ float4 wo[kAttnWarps][G][32];
  __shared__ bool last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = blockIdx.x, kvh = blockIdx.y, m = blockIdx.z;
  // positions outside [0, max_seq) were flagged by the append kernel; clamp so
  // nothing here reads outside the cache
  const int len = max(1, min(p.positions[m] + 1, p.max_seq));
  const int chunk = ((len + p.splits - 1) / p.splits + 31) & ~31;
  const int begin = split * chunk, end = min(len, begin + chunk);
  const float *kc = p.k_cache + (size_t)m * p.seq_stride + (size_t)p.layer * p.max_seq * p.kv_dim + kvh * 128 + 4 * lane;
  const float *vc = p.v_cache + (size_t)m * p.seq_stride + (size_t)p.layer * p.max_seq * p.kv_dim + kvh * 128 + 4 * lane;

  float4 qv[G];
#pragma unroll
  for (int g = 0; g < G; ++g)
    qv[g] = *reinterpret_cast<const float4 *>(p.q + (size_t)m * p.q_stride + (kvh * G + g) * 128 + 4 * lane);
  float mx[G], sum[G];
  float4 o[G];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    mx[g] = -INFINITY;
    sum[g] = 0.0f;
    o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
  }

  for (int base = begin + warp * 32; base < end; base += kAttnWarps * 32) {
    const int nkeys = min(32, end - base);
    // Scores of this 32-key group: per half of 16 keys, each lane forms the
    // G*16 partial dots of its 4 dims, a reduce-scatter leaves one full dot
    // per lane group, and the owners park them in shared memory.
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      constexpr int V = G * 16;
      float part[V];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int key = half * 16 + j;
        float4 kv = make_float4(0.f, 0.f, 0.f, 0.f);
        if (key < nkeys) kv = *reinterpret_cast<const float4 *>(kc + (size_t)(base + key) * p.kv_dim);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float d = __fmul_rn(qv[g].x, kv.x);
          d = fmaf(qv[g].y, kv.y, d);
          d = fmaf(qv[g].z, kv.z, d);
          d = fmaf(qv[g].w, kv.w, d);
          part[g * 16 + j] = d;
        }
      }
      const float tot = warp_reduce_scatter<V>(part);
      const int idx = reduce_index<V>(lane);
      if ((lane & (32 / V - 1)) == 0) sp[warp][idx / 16][half * 16 + idx % 16] = __fmul_rn(tot, p.scale);
    }
    __syncwarp();
    float score[G];
#pragma unroll
    for (int g = 0; g < G; ++g) score[g] = lane < nkeys ? sp[warp][g][lane] : -INFINITY;
    __syncwarp();
    // online softmax over the group
    float corr[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float nmax = fmaxf(mx[g], warp_max(score[g]));
      corr[g] = mx[g] == -INFINITY ? 0.0f : expf(__fsub_rn(mx[g], nmax));
      const float pj = lane < nkeys ? expf(__fsub_rn(score[g], nmax)) : 0.0f;
      sum[g] = __fadd_rn(__fmul_rn(sum[g], corr[g]), warp_sum(pj));
      mx[g] = nmax;
      sp[warp][g][lane] = pj;
      o[g].x = __fmul_rn(o[g].x, corr[g]);
      o[g].y = __fmul_rn(o[g].y, corr[g]);
      o[g].z = __fmul_rn(o[g].z, corr[g]);
      o[g].w = __fmul_rn(o[g].w, corr[g]);
    }
    __syncwarp();
    for (int j = 0; j < nkeys; ++j) {
      const float4 vv = *reinterpret_cast<const float4 *>(vc + (size_t)(base + j) * p.kv_dim);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float w = sp[warp][g][j];
        o[g].x = fmaf(w, vv.x, o[g].x);
        o[g].y = fmaf(w, vv.y, o[g].y);
        o[g].z = fmaf(w, vv.z, o[g].z);
        o[g].w = fmaf(w, vv.w, o[g].w);
      }
    }
    __syncwarp();
  }

  // merge the warps of this CTA
#pragma unroll
  for (int g = 0; g < G; ++g) {
    if (lane == 0) {
      wm[warp][g] = mx[g];
      wl[warp][g] = sum[g];
    }
    wo[warp][g][lane] = o[g];
  }
  __syncthreads();
  float *part_base = p.partials + (((size_t)m * p.n_kv_heads + kvh) * p.splits + split) * (size_t)(G * kAttnPartStride);
  if (warp < G) {
    const int g = warp;
    float M = -INFINITY;
    for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int w = 0; w < kAttnWarps; ++w) {
      const float f = wm[w][g] == -INFINITY ? 0.0f : expf(__fsub_rn(wm[w][g], M));
      L = __fadd_rn(L, __fmul_rn(wl[w][g], f));
      const float4 ov = wo[w][g][lane];
      acc.x = fmaf(ov.x, f, acc.x);
      acc.y = fmaf(ov.y, f, acc.y);
      acc.z = fmaf(ov.z, f, acc.z);
      acc.w = fmaf(ov.w, f, acc.w);
    }
    float *pg = part_base + g * kAttnPartStride;
    reinterpret_cast<float4 *>(pg)[lane] = acc;
    if (lane == 0) {
      pg[128] = M;
      pg[129] = L;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned *ctr = p.counters + (size_t)m * p.n_kv_heads + kvh;
    last = atomicAdd(ctr, 1u) == (unsigned)p.splits - 1;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // last CTA of (m, kvh): merge all splits
  if (warp < G) {
    const int g = warp;
    const float *pb = p.partials + (((size_t)m * p.n_kv_heads + kvh) * p.splits) * (size_t)(G * kAttnPartStride) + g * kAttnPartStride;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(pb + (size_t)s * G * kAttnPartStride + 128));
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s = 0; s < p.splits; ++s) {
      const float *ps = pb + (size_t)s * G * kAttnPartStride;
      const float ms = __ldcg(ps + 128);
      const float f = ms == -INFINITY ? 0.0f : expf(__fsub_rn(ms, M));
      L = __fadd_rn(L, __fmul_rn(__ldcg(ps + 129), f));
      const float4 ov = __ldcg(reinterpret_cast<const float4 *>(ps) + lane);
      acc.x = fmaf(ov.x, f, acc.x);
      acc.y = fmaf(ov.y, f, acc.y);
      acc.z = fmaf(ov.z, f, acc.z);
      acc.w = fmaf(ov.w, f, acc.w);
    }
    const float inv = __fdiv_rn(1.0f, L);
    float4 r = make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
    *reinterpret_cast<float4 *>(p.out + (size_t)m * p.out_stride + (kvh * G + g) * 128 + 4 * lane) = r;
  }
  if (threadIdx.x == 0) p.counters[(size_t)m * p.n_kv_heads + kvh] = 0u;
}

int attn_pick_splits(int M, int n_kv_heads, int max_len) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int splits = (2 * sms + M * n_kv_heads - 1) / (M * n_kv_heads);
  const int max_splits = (max_len + 127) / 128;  // at least 128 keys per split
  splits = std::max(1, std::min(splits, max_splits));
  return std::min(splits, kAttnMaxSplits);
}

int attn_decode_launch(const AttnDecodeParams &p, int group, cudaStream_t st) {
  dim3 grid(p.splits, p.n_kv_heads, p.M);
  switch (group) {
    case 1: attn_decode_kernel<1><<<grid, kAttnWarps * 32, 0, st>>>(p); break;
    case 2: attn_decode_kernel<2><<<grid, kAttnWarps * 32, 0, st>>>(p); break;
    default:
      set_error("attention: GQA group size %d unsupported (1 or 2)", group);
      return QASR_ERR_UNSUPPORTED;
  }
  return QASR_OK;
}

}  // namespace qasr

using namespace qasr;

extern "C" int qasr_causal_attention(float *out, const float *q, const float *k, const float *v, int seq_q,
                                     int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset,
                                     void *stream) {
  if (!out || !q || !k || !v || seq_q < 0 || seq_k < 0 || n_heads <= 0 || n_kv_heads <= 0 ||
      n_heads % n_kv_heads || q_offset < 0) {
    set_error("qasr_causal_attention: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("qasr_causal_attention: head_dim %d unsupported (64 or 128)", head_dim);
    return QASR_ERR_UNSUPPORTED;
  }
  if (seq_q == 0) return QASR_OK;
  const long tasks = (long)seq_q * n_heads;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    causal_attention_kernel<4><<<ceil_div(tasks, 8), 256, 0, st>>>(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads,
                                                                   scale, q_offset);
  else
    causal_attention_kernel<2><<<ceil_div(tasks, 8), 256, 0, st>>>(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads,
                                                                   scale, q_offset);
  return launch_status("qasr_causal_attention");
}
