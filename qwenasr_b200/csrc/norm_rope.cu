// norm_rope.cu -- RMSNorm, LayerNorm(+PE), per-head norm, RoPE, KV append and
// the fused decoder pre-attention block, reproducing the reference's f32
// rounding sequence (crates/qwen-asr/src/kernels/avx.rs:377-481,
// kernels/mod.rs:866-935 and 1213-1267, decoder.rs:194-202, 253-289).
//
// All of these are HBM-bound row kernels: each row is read once with 16-byte
// vector loads into shared memory, reduced in the reference's order by one
// warp, and written once.
#include <algorithm>

#include "common.cuh"
#include "rowops.cuh"

namespace qasr {

constexpr int kRowWarps = 4;  // warps per CTA for one-warp-per-row kernels

// ---------------------------------------------------------------- rms_norm
__global__ void __launch_bounds__(kRowWarps * 32)
rms_norm_kernel(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w, int seq,
                int hidden, float eps) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= seq) return;
  float *xs = smem + (size_t)warp * hidden;
  warp_load_row(xs, x + (size_t)row * hidden, hidden);
  const float inv = rms_inv_ref(xs, hidden, eps);
  float *o = out + (size_t)row * hidden;
  for (int i = lane; i < hidden; i += 32) o[i] = __fmul_rn(__fmul_rn(xs[i], inv), w[i]);
}

// ------------------------------------------------------- rms_norm_per_head
// One warp per (row, head).  The reference sums the head sequentially
// (mod.rs:926-929), so lane 0 does exactly that; the scaling is parallel.
__global__ void __launch_bounds__(256)
rms_norm_per_head_kernel(float *__restrict__ x, const float *__restrict__ w, int seq, int n_heads, int head_dim,
                         float eps) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long task = (long)blockIdx.x * 8 + warp;
  if (task >= (long)seq * n_heads) return;
  float *hs = smem + (size_t)warp * head_dim;
  float *v = x + task * head_dim;
  warp_load_row(hs, v, head_dim);
  float inv = 0.0f;
  if (lane == 0) {
    float s = 0.0f;
    for (int d = 0; d < head_dim; ++d) s = __fadd_rn(s, __fmul_rn(hs[d], hs[d]));
    inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)head_dim), eps)));
  }
  inv = __shfl_sync(0xffffffffu, inv, 0);
  for (int d = lane; d < head_dim; d += 32) v[d] = __fmul_rn(__fmul_rn(hs[d], inv), w[d]);
}

// -------------------------------------------------------------- layer_norm
// out = layer_norm(x) (+ pe[row % n_pos] when pe != nullptr).
__global__ void __launch_bounds__(kRowWarps * 32)
layer_norm_kernel(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                  const float *__restrict__ b, const float *__restrict__ pe, int rows, int hidden, int n_pos,
                  float eps) {
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kRowWarps + warp;
  if (row >= rows) return;
  float *xs = smem + (size_t)warp * hidden;
  warp_load_row(xs, x + (size_t)row * hidden, hidden);
  float mean, inv;
  ln_stats_ref(xs, hidden, eps, mean, inv);
  // avx.rs:469-480: fma((x-mean)*inv, w, b) on the 8-aligned body, two
  // roundings more on the scalar tail.
  const int body = hidden - hidden % 8;
  float *o = out + (size_t)row * hidden;
  const float *p = pe ? pe + (size_t)(row % n_pos) * hidden : nullptr;
  for (int i = lane; i < hidden; i += 32) {
    float c = __fmul_rn(__fsub_rn(xs[i], mean), inv);
    float y = i < body ? fmaf(c, w[i], b[i]) : __fadd_rn(__fmul_rn(c, w[i]), b[i]);
    if (p) y = __fadd_rn(y, p[i]);
    o[i] = y;
  }
}

// --------------------------------------------------- LayerNorm+PE and GELU
// The encoder's elementwise steps in one launch: CTAs [0, ln_ctas) run
// out = layer_norm(x) + pe[row % n_pos] (one warp per row, the arithmetic of
// layer_norm_kernel), the remaining CTAs apply exact-erf GELU in place to the
// FFN activation `act`.  The LayerNorm CTAs are dispatched first, so their
// per-row reduction latency overlaps the GELU stream instead of forming a
// launch of its own.
constexpr int kLnGeluWarps = 8;
__global__ void __launch_bounds__(kLnGeluWarps * 32)
ln_pe_gelu_kernel(float *__restrict__ out, const float *__restrict__ x, const float *__restrict__ w,
                  const float *__restrict__ b, const float *__restrict__ pe, int rows, int hidden, int n_pos,
                  float eps, float *__restrict__ act, long n_act, int ln_ctas) {
  // launched with launch_pdl: no memory access before the previous kernel completed
  pdl_wait();
  pdl_launch_dependents();
  if ((int)blockIdx.x >= ln_ctas) {
    gelu_erf_pass(act, n_act, (long)blockIdx.x - ln_ctas, (long)gridDim.x - ln_ctas);
    return;
  }
  extern __shared__ float smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kLnGeluWarps + warp;
  if (row >= rows) return;
  float *xs = smem + (size_t)warp * hidden;
  warp_load_row(xs, x + (size_t)row * hidden, hidden);
  float mean, inv;
  ln_stats_ref(xs, hidden, eps, mean, inv);
  const int body = hidden - hidden % 8;
  float *o = out + (size_t)row * hidden;
  const float *p = pe + (size_t)(row % n_pos) * hidden;
  for (int i = lane; i < hidden; i += 32) {
    const float c = __fmul_rn(__fsub_rn(xs[i], mean), inv);
    const float y = i < body ? fmaf(c, w[i], b[i]) : __fadd_rn(__fmul_rn(c, w[i]), b[i]);
    o[i] = __fadd_rn(y, p[i]);
  }
}

// ------------------------------------------------------------------- RoPE
// cos/sin table rows.  The reference computes inv_freq[d] = 1/theta^(2d/D)
// once on the host with f32 powf (RopeCache::ensure, decoder.rs:258-262;
// compute_rope_neox mod.rs:1236) and then angle = pos*inv_freq in f32; the
// launchers below compute inv_freq the same way on the host (the same libm
// powf the Rust code calls) and pass it in.  cos/sin of the f32 angle are
// evaluated in double and rounded once (the correctly rounded f32 value).
// positions == nullptr means rows 0..seq-1.
struct InvFreq {
  float v[128];
};

__global__ void rope_table_kernel(float *__restrict__ cos_out, float *__restrict__ sin_out,
                                  const int32_t *__restrict__ positions, int seq, int head_dim,
                                  const __grid_constant__ InvFreq inv) {
  const int half = head_dim / 2;
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long)seq * half) return;
  const int s = (int)(t / half), d = (int)(t % half);
  const float pos = positions ? (float)positions[s] : (float)s;
  const float angle = __fmul_rn(pos, inv.v[d]);
  const float c = (float)cos((double)angle), sn = (float)sin((double)angle);
  const size_t r = (size_t)s * head_dim;
  cos_out[r + d] = c;
  cos_out[r + half + d] = c;
  sin_out[r + d] = sn;
  sin_out[r + half + d] = sn;
}

// Host: inv_freq of RopeCache::ensure (f32 powf, f32 reciprocal).
static InvFreq host_inv_freq(int head_dim, float theta) {
  InvFreq f{};
  const int half = head_dim / 2;
  for (int d = 0; d < half && d < 128; ++d) f.v[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
  return f;
}

// apply_rope_neox (mod.rs:1247-1267): one thread per (row, head, d < half).
__global__ void apply_rope_kernel(float *__restrict__ x, const float *__restrict__ cos_v,
                                  const float *__restrict__ sin_v, int seq, int n_heads, int head_dim) {
  const int half = head_dim / 2;
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long)seq * n_heads * half) return;
  const int d = (int)(t % half);
  const long sh = t / half;
  const int s = (int)(sh / n_heads);
  float *vec = x + sh * head_dim;
  const float *c = cos_v + (size_t)s * head_dim, *sn = sin_v + (size_t)s * head_dim;
  const float x1 = vec[d], x2 = vec[half + d];
  vec[d] = __fadd_rn(__fmul_rn(x1, c[d]), __fmul_rn(-x2, sn[d]));
  vec[half + d] = __fadd_rn(__fmul_rn(x2, c[half + d]), __fmul_rn(x1, sn[half + d]));
}

// KvCache row copies (decoder.rs:194-202): one float4 per thread.
__global__ void kv_append_kernel(float *__restrict__ k_cache, float *__restrict__ v_cache,
                                 const float *__restrict__ k_new, const float *__restrict__ v_new, int layer,
                                 int max_seq, int kv_dim, int start_pos, int seq) {
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = kv_dim / 4;
  if (t >= (long)seq * per_row) return;
  const int s = (int)(t / per_row), c = (int)(t % per_row);
  const size_t dst = ((size_t)layer * max_seq + start_pos + s) * kv_dim;
  reinterpret_cast<float4 *>(k_cache + dst)[c] = reinterpret_cast<const float4 *>(k_new + (size_t)s * kv_dim)[c];
  reinterpret_cast<float4 *>(v_cache + dst)[c] = reinterpret_cast<const float4 *>(v_new + (size_t)s * kv_dim)[c];
}

// --------------------------------------------------- fused pre-attn block
// One CTA per token row, 8 warps.  The row's x, q and k are staged in shared
// memory (q and k as n_heads + n_kv heads of 128 floats, each padded to 129
// so that lane h of a warp walking head h element by element hits bank
// (h + d) % 32: the 24 sequential sums run side by side without conflicts)
// and the V row goes straight to the cache.  Then warp 0 computes the x row's
// 1/rms in the reference's AVX order (rms_inv_ref) while warp 1 runs one
// per-head sequential sum per lane (mod.rs:926-929), and finally all threads
// write x_norm and the normalised, rotated q and k heads (4 elements and
// their RoPE partners per thread).  Every rounding step is the reference's,
// so all outputs are bit-exact.
#ifndef QASR_PRE_THREADS
#define QASR_PRE_THREADS 128
#endif
constexpr int kPreThreads = QASR_PRE_THREADS;  // threads per row of the configuration-1 block
constexpr int kHeadPad = 129;

// 16-byte global -> shared copy that completes asynchronously (waited for with
// cp_async_wait_all before a barrier).
QASR_DEV void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
QASR_DEV void cp_async_wait_all() { asm volatile("cp.async.commit_group;\n\tcp.async.wait_all;" ::: "memory"); }

__global__ void __launch_bounds__(kPreThreads)
pre_attn_block_kernel(float *__restrict__ x_norm, const float *__restrict__ x, const float *__restrict__ w_in,
                      int hidden, float *__restrict__ q, const float *__restrict__ k, const float *__restrict__ v,
                      float *__restrict__ k_out, const float *__restrict__ q_norm_w,
                      const float *__restrict__ k_norm_w, int n_heads, int n_kv_heads, float eps,
                      const float *__restrict__ cos_tab, const float *__restrict__ sin_tab, int start_pos,
                      float *__restrict__ k_cache, float *__restrict__ v_cache, int layer, int max_seq) {
  extern __shared__ __align__(16) float smem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int s = blockIdx.x, pos = start_pos + s;
  const int q_dim = n_heads * 128, kv_dim = n_kv_heads * 128, n_h = n_heads + n_kv_heads;
  // shared layout: x row | RoPE rows and norm weights (cp.async) | q|k heads (padded) | 1/rms values
  float *xs = smem;                                // [hidden]
  float *tab = xs + hidden;                        // cos[128] sin[128] qn[128] kn[128] w_in[hidden]
  float *hs = tab + 512 + hidden;                  // [n_h][kHeadPad]
  float *inv = hs + (size_t)n_h * kHeadPad;        // [0]: x row, [1 + h]: head h
  const size_t cache_row = ((size_t)layer * max_seq + pos) * kv_dim;
  // launched with launch_pdl: nothing is read or written before the previous
  // kernel of the stream has completed
  pdl_wait();
  pdl_launch_dependents();

  // ---- every global read of the row is issued before any of it is used: the
  // constant rows by cp.async straight into shared memory, the activations
  // into registers
  {
    const float *srcs[4] = {cos_tab + (size_t)pos * 128, sin_tab + (size_t)pos * 128, q_norm_w, k_norm_w};
    for (int i = tid; i < 128 + hidden / 4; i += kPreThreads) {
      if (i < 128)
        cp_async16(tab + 4 * i, srcs[i >> 5] + 4 * (i & 31));
      else
        cp_async16(tab + 512 + 4 * (i - 128), w_in + 4 * (i - 128));
    }
  }
  const float4 *x4 = reinterpret_cast<const float4 *>(x + (size_t)s * hidden);
  const float4 *q4 = reinterpret_cast<const float4 *>(q + (size_t)s * q_dim);
  const float4 *k4 = reinterpret_cast<const float4 *>(k + (size_t)s * kv_dim);
  const float4 *v4 = reinterpret_cast<const float4 *>(v + (size_t)s * kv_dim);
  // float4 per thread: x (hidden <= 2048), q|k (<= 3072 floats), v (<= 1024)
  constexpr int kVx = (512 + kPreThreads - 1) / kPreThreads, kVqk = (768 + kPreThreads - 1) / kPreThreads,
                kVv = (256 + kPreThreads - 1) / kPreThreads;
  float4 rx[kVx], rqk[kVqk], rv[kVv];
#pragma unroll
  for (int j = 0; j < kVx; ++j) {
    const int i = tid + j * kPreThreads;
    if (i < hidden / 4) rx[j] = x4[i];
  }
#pragma unroll
  for (int j = 0; j < kVv; ++j)
    if (tid + j * kPreThreads < kv_dim / 4) rv[j] = v4[tid + j * kPreThreads];
#pragma unroll
  for (int j = 0; j < kVqk; ++j) {
    const int i = tid + j * kPreThreads;
    if (i < (q_dim + kv_dim) / 4) rqk[j] = i < q_dim / 4 ? q4[i] : k4[i - q_dim / 4];
  }
  float4 *vc4 = reinterpret_cast<float4 *>(v_cache + cache_row);
#pragma unroll
  for (int j = 0; j < kVx; ++j) {
    const int i = tid + j * kPreThreads;
    if (i < hidden / 4) reinterpret_cast<float4 *>(xs)[i] = rx[j];
  }
#pragma unroll
  for (int j = 0; j < kVv; ++j)
    if (tid + j * kPreThreads < kv_dim / 4) vc4[tid + j * kPreThreads] = rv[j];
#pragma unroll
  for (int j = 0; j < kVqk; ++j) {
    const int i = tid + j * kPreThreads;
    if (i < (q_dim + kv_dim) / 4) {
      float *dst = hs + (size_t)(i >> 5) * kHeadPad + ((i & 31) << 2);  // head i/32, element 4*(i%32)
      dst[0] = rqk[j].x;
      dst[1] = rqk[j].y;
      dst[2] = rqk[j].z;
      dst[3] = rqk[j].w;
    }
  }
  cp_async_wait_all();
  __syncthreads();

  // ---- the sequential sums: warp 0 the x row (rms_inv_ref order), warp 1 one
  // head per lane (mod.rs:926-929)
  if (warp == 0) {
    const float r = rms_inv_ref(xs, hidden, eps);
    if (lane == 0) inv[0] = r;
  } else if (warp == 1 && lane < n_h) {
    const float *hp = hs + (size_t)lane * kHeadPad;
    float acc = 0.0f;
#pragma unroll 16
    for (int d = 0; d < 128; ++d) acc = __fadd_rn(acc, __fmul_rn(hp[d], hp[d]));
    inv[1 + lane] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(acc, 128.0f), eps)));
  }
  __syncthreads();

  // ---- outputs: x_norm, then the normalised and rotated q and k heads
  const float ix = inv[0];
  float4 *xo4 = reinterpret_cast<float4 *>(x_norm + (size_t)s * hidden);
  const float4 *w4 = reinterpret_cast<const float4 *>(tab + 512);
  for (int i = tid; i < hidden / 4; i += kPreThreads) {
    const float4 a = reinterpret_cast<const float4 *>(xs)[i], b = w4[i];
    xo4[i] = make_float4(__fmul_rn(__fmul_rn(a.x, ix), b.x), __fmul_rn(__fmul_rn(a.y, ix), b.y),
                         __fmul_rn(__fmul_rn(a.z, ix), b.z), __fmul_rn(__fmul_rn(a.w, ix), b.w));
  }
  const float *crow = tab, *srow = tab + 128;
  for (int it = tid; it < n_h * 16; it += kPreThreads) {
    const int h = it >> 4, d = (it & 15) << 2;  // elements d..d+3 and their partners d+64..d+67
    const float *hp = hs + (size_t)h * kHeadPad;
    const float ih = inv[1 + h];
    const float *nw = tab + (h < n_heads ? 256 : 384);
    float lo[4], hi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float x1 = __fmul_rn(__fmul_rn(hp[d + j], ih), nw[d + j]);
      const float x2 = __fmul_rn(__fmul_rn(hp[64 + d + j], ih), nw[64 + d + j]);
      lo[j] = __fadd_rn(__fmul_rn(x1, crow[d + j]), __fmul_rn(-x2, srow[d + j]));
      hi[j] = __fadd_rn(__fmul_rn(x2, crow[64 + d + j]), __fmul_rn(x1, srow[64 + d + j]));
    }
    const float4 l4 = make_float4(lo[0], lo[1], lo[2], lo[3]), h4 = make_float4(hi[0], hi[1], hi[2], hi[3]);
    float *dst;
    if (h < n_heads) {
      dst = q + (size_t)s * q_dim + h * 128;
    } else {
      dst = k_cache + cache_row + (h - n_heads) * 128;
      if (k_out) {
        float *ko = k_out + (size_t)s * kv_dim + (h - n_heads) * 128;
        *reinterpret_cast<float4 *>(ko + d) = l4;
        *reinterpret_cast<float4 *>(ko + 64 + d) = h4;
      }
    }
    *reinterpret_cast<float4 *>(dst + d) = l4;
    *reinterpret_cast<float4 *>(dst + 64 + d) = h4;
  }
}

// ---------------------------------------------------------- sinusoidal PE
// sinusoidal_pe (mod.rs:1213-1226): f32 steps in the reference's order, each
// transcendental evaluated in double and rounded once (see rope_table_kernel).
__global__ void sinusoidal_pe_kernel(float *__restrict__ pe, int n_pos, int d_model) {
  const int half = d_model / 2;
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long)n_pos * half) return;
  const int p = (int)(t / half), d = (int)(t % half);
  const float ln10k = (float)log(10000.0);
  const float log_ts = __fdiv_rn(ln10k, (float)(half - 1));
  const float arg = __fmul_rn(-(float)d, log_ts);
  const float inv_ts = (float)exp((double)arg);
  const float angle = __fmul_rn((float)p, inv_ts);
  pe[(size_t)p * d_model + d] = (float)sin((double)angle);
  pe[(size_t)p * d_model + half + d] = (float)cos((double)angle);
}

}  // namespace qasr

using namespace qasr;

static inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
static inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int qasr_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps,
                             void *stream) {
  if (!out || !x || !w || seq < 0 || hidden <= 0) {
    set_error("qasr_rms_norm: invalid arguments (seq=%d hidden=%d)", seq, hidden);
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const size_t smem = (size_t)kRowWarps * hidden * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("qasr_rms_norm: hidden=%d too large", hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(rms_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  rms_norm_kernel<<<ceil_div(seq, kRowWarps), kRowWarps * 32, smem, S(stream)>>>(out, x, w, seq, hidden, eps);
  return launch_status("qasr_rms_norm");
}

extern "C" int qasr_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim, float eps,
                                      void *stream) {
  if (!x || !w || seq < 0 || n_heads <= 0 || head_dim <= 0 || head_dim > 4096) {
    set_error("qasr_rms_norm_per_head: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const long tasks = (long)seq * n_heads;
  rms_norm_per_head_kernel<<<ceil_div(tasks, 8), 256, 8 * head_dim * sizeof(float), S(stream)>>>(
      x, w, seq, n_heads, head_dim, eps);
  return launch_status("qasr_rms_norm_per_head");
}

extern "C" int qasr_layer_norm(float *out, const float *x, const float *w, const float *b, int seq, int hidden,
                               float eps, void *stream) {
  if (!out || !x || !w || !b || seq < 0 || hidden <= 0) {
    set_error("qasr_layer_norm: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const size_t smem = (size_t)kRowWarps * hidden * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("qasr_layer_norm: hidden=%d too large", hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(layer_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  layer_norm_kernel<<<ceil_div(seq, kRowWarps), kRowWarps * 32, smem, S(stream)>>>(out, x, w, b, nullptr, seq,
                                                                                   hidden, 1, eps);
  return launch_status("qasr_layer_norm");
}

extern "C" int qasr_ln_pe(float *out, const float *x, const float *w, const float *b, const float *pe, int rows,
                          int hidden, int n_pos, float eps, void *stream) {
  if (!out || !x || !w || !b || !pe || rows < 0 || hidden <= 0 || n_pos <= 0) {
    set_error("qasr_ln_pe: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (rows == 0) return QASR_OK;
  const size_t smem = (size_t)kRowWarps * hidden * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("qasr_ln_pe: hidden=%d too large", hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(layer_norm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  layer_norm_kernel<<<ceil_div(rows, kRowWarps), kRowWarps * 32, smem, S(stream)>>>(out, x, w, b, pe, rows, hidden,
                                                                                    n_pos, eps);
  return launch_status("qasr_ln_pe");
}

extern "C" int qasr_ln_pe_gelu_erf(float *out, const float *x, const float *w, const float *b, const float *pe,
                                   int rows, int hidden, int n_pos, float eps, float *act, int64_t n_act,
                                   void *stream) {
  if (!out || !x || !w || !b || !pe || rows < 0 || hidden <= 0 || n_pos <= 0 || n_act < 0 || (n_act > 0 && !act) ||
      (act && !al16(act))) {
    set_error("qasr_ln_pe_gelu_erf: invalid arguments (act must be 16-byte aligned)");
    return QASR_ERR_INVALID;
  }
  const size_t smem = (size_t)kLnGeluWarps * hidden * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("qasr_ln_pe_gelu_erf: hidden=%d too large", hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if (rows == 0 && n_act == 0) return QASR_OK;
  static int sms = 0;
  if (!sms) {
    int dev = 0, v = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms = v > 0 ? v : 148;
  }
  const int ln_ctas = ceil_div(rows, kLnGeluWarps);
  const long gelu_items = (n_act / 4 + 4 * 256 - 1) / (4 * 256);  // 4 vectors per thread per round
  const long gelu_ctas = n_act > 0 ? std::max(1l, std::min(gelu_items, (long)sms * 8)) : 0;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(ln_pe_gelu_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cuda_status(launch_pdl(ln_pe_gelu_kernel, dim3((unsigned)(ln_ctas + gelu_ctas)), dim3(kLnGeluWarps * 32), smem,
                                S(stream), out, x, w, b, pe, rows, hidden, n_pos, eps, act, n_act, ln_ctas),
                     "qasr_ln_pe_gelu_erf");
}

extern "C" int qasr_compute_rope_neox(float *cos_out, float *sin_out, const int32_t *positions, int seq,
                                      int head_dim, float theta, void *stream) {
  if (!cos_out || !sin_out || !positions || seq < 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 256) {
    set_error("qasr_compute_rope_neox: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const long n = (long)seq * (head_dim / 2);
  rope_table_kernel<<<ceil_div(n, 256), 256, 0, S(stream)>>>(cos_out, sin_out, positions, seq, head_dim,
                                                              host_inv_freq(head_dim, theta));
  return launch_status("qasr_compute_rope_neox");
}

extern "C" int qasr_rope_cache_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta,
                                     void *stream) {
  if (!cos_out || !sin_out || n_pos < 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 256) {
    set_error("qasr_rope_cache_table: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n_pos == 0) return QASR_OK;
  const long n = (long)n_pos * (head_dim / 2);
  rope_table_kernel<<<ceil_div(n, 256), 256, 0, S(stream)>>>(cos_out, sin_out, nullptr, n_pos, head_dim,
                                                              host_inv_freq(head_dim, theta));
  return launch_status("qasr_rope_cache_table");
}

extern "C" int qasr_apply_rope_neox(float *x, const float *cos_v, const float *sin_v, int seq, int n_heads,
                                    int head_dim, void *stream) {
  if (!x || !cos_v || !sin_v || seq < 0 || n_heads <= 0 || head_dim <= 0 || (head_dim & 1)) {
    set_error("qasr_apply_rope_neox: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const long n = (long)seq * n_heads * (head_dim / 2);
  apply_rope_kernel<<<ceil_div(n, 256), 256, 0, S(stream)>>>(x, cos_v, sin_v, seq, n_heads, head_dim);
  return launch_status("qasr_apply_rope_neox");
}

extern "C" int qasr_kv_append(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                              int max_seq, int kv_dim, int start_pos, int seq, void *stream) {
  if (!k_cache || !v_cache || !k_new || !v_new || layer < 0 || max_seq <= 0 || kv_dim <= 0 || (kv_dim & 3) ||
      start_pos < 0 || seq < 0 || start_pos + seq > max_seq || !al16(k_cache) || !al16(v_cache) || !al16(k_new) ||
      !al16(v_new)) {
    set_error("qasr_kv_append: invalid arguments (start_pos=%d seq=%d max_seq=%d kv_dim=%d, 16-byte aligned "
              "pointers required)", start_pos, seq, max_seq, kv_dim);
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  const long n = (long)seq * (kv_dim / 4);
  kv_append_kernel<<<ceil_div(n, 256), 256, 0, S(stream)>>>(k_cache, v_cache, k_new, v_new, layer, max_seq, kv_dim,
                                                            start_pos, seq);
  return launch_status("qasr_kv_append");
}

extern "C" int qasr_pre_attn_block(float *x_norm, const float *x, const float *w_in, int seq, int hidden, float *q,
                                   const float *k, const float *v, float *k_out, const float *q_norm_w,
                                   const float *k_norm_w, int n_heads, int n_kv_heads, int head_dim, float eps,
                                   const float *cos_tab, const float *sin_tab, int start_pos, float *k_cache,
                                   float *v_cache, int layer, int max_seq, void *stream) {
  if (!x_norm || !x || !w_in || !q || !k || !v || !q_norm_w || !k_norm_w || !cos_tab || !sin_tab || !k_cache ||
      !v_cache || seq < 0 || hidden <= 0 || n_heads <= 0 || n_kv_heads <= 0 || start_pos < 0 || layer < 0 ||
      start_pos + seq > max_seq) {
    set_error("qasr_pre_attn_block: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (!al16(x) || !al16(q) || !al16(k) || !al16(v) || (k_out && !al16(k_out)) || !al16(q_norm_w) ||
      !al16(k_norm_w) || !al16(cos_tab) || !al16(sin_tab) || !al16(k_cache) || !al16(v_cache)) {
    set_error("qasr_pre_attn_block: all vector operands must be 16-byte aligned");
    return QASR_ERR_INVALID;
  }
  if (head_dim != 128 || (hidden & 3) || hidden > 2048 || (n_heads + n_kv_heads) * 128 > 3072 ||
      n_kv_heads * 128 > 1024 || !al16(w_in)) {
    set_error("qasr_pre_attn_block: head_dim must be 128 (got %d), hidden a multiple of 4 and <= 2048, q+k heads "
              "<= 24, kv heads <= 8, w_in 16-byte aligned", head_dim);
    return QASR_ERR_UNSUPPORTED;
  }
  if (seq == 0) return QASR_OK;
  const size_t smem =
      ((size_t)2 * hidden + 512 + (size_t)(n_heads + n_kv_heads) * kHeadPad + 33) * sizeof(float);
  if (smem > 200 * 1024) {
    set_error("qasr_pre_attn_block: hidden=%d too large", hidden);
    return QASR_ERR_UNSUPPORTED;
  }
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(pre_attn_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  return cuda_status(launch_pdl(pre_attn_block_kernel, dim3(seq), dim3(kPreThreads), smem, S(stream), x_norm, x, w_in,
                                hidden, q, k, v, k_out, q_norm_w, k_norm_w, n_heads, n_kv_heads, eps, cos_tab,
                                sin_tab, start_pos, k_cache, v_cache, layer, max_seq),
                     "qasr_pre_attn_block");
}

extern "C" int qasr_sinusoidal_pe(float *pe, int n_pos, int d_model, void *stream) {
  if (!pe || n_pos < 0 || d_model < 4 || (d_model & 1)) {
    set_error("qasr_sinusoidal_pe: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n_pos == 0) return QASR_OK;
  const long n = (long)n_pos * (d_model / 2);
  sinusoidal_pe_kernel<<<ceil_div(n, 256), 256, 0, S(stream)>>>(pe, n_pos, d_model);
  return launch_status("qasr_sinusoidal_pe");
}
