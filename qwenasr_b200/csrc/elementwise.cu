// elementwise.cu -- activations, SwiGLU, residual add, INT8 quantiser and the
// embedding gathers.  All HBM-bound streaming kernels: 16-byte loads/stores,
// grid sized to a multiple of the SM count with a grid-stride loop.
#include "common.cuh"

namespace qasr {

// Grid for a streaming kernel over n_vec work items: enough CTAs to fill the
// 148 SMs several times over, never more than the work.
static int stream_grid(long n_vec, int threads) {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  long want = (n_vec + threads - 1) / threads;
  long cap = (long)sms * 8;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

// Scalar tail of the same function (avx.rs:557-562), libm tanh.
QASR_DEV float gelu_tanh_tail(float val) {
  const float x3 = __fmul_rn(__fmul_rn(val, val), val);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(val, __fmul_rn(0.044715f, x3)));
  return __fmul_rn(__fmul_rn(0.5f, val), __fadd_rn(1.0f, tanhf(inner)));
}
__global__ void gelu_kernel(float *__restrict__ x, long n) {
  const long body = n - n % 8;
  const long nv = body / 4;
  float4 *x4 = reinterpret_cast<float4 *>(x);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    float4 v = x4[i];
    v.x = gelu_tanh_ref(v.x); v.y = gelu_tanh_ref(v.y); v.z = gelu_tanh_ref(v.z); v.w = gelu_tanh_ref(v.w);
    x4[i] = v;
  }
  if (blockIdx.x == 0 && threadIdx.x < n - body) x[body + threadIdx.x] = gelu_tanh_tail(x[body + threadIdx.x]);
}

__global__ void __launch_bounds__(256) gelu_erf_kernel(float *__restrict__ x, long n) {
  gelu_erf_pass(x, n, blockIdx.x, gridDim.x);
}

__global__ void silu_kernel(float *__restrict__ x, long n) {
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    const float v = x[i];
    x[i] = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
  }
}

// avx::swiglu_interleaved (avx.rs:568-599) per row: reference fast exp on the
// 8-aligned body, libm exp on the tail.  One thread per output pair.
__global__ void swiglu_kernel(float *__restrict__ out, const float *__restrict__ gu, int seq, int inter) {
  const int body = inter - inter % 8;
  const long n = (long)seq * inter;
  for (long t = (long)blockIdx.x * blockDim.x + threadIdx.x; t < n; t += (long)gridDim.x * blockDim.x) {
    const int j = (int)(t % inter);
    const float2 p = reinterpret_cast<const float2 *>(gu)[t];
    const float g = p.x, u = p.y;
    float silu;
    if (j < body) silu = __fdiv_rn(g, __fadd_rn(1.0f, fast_exp_ref(__fsub_rn(0.0f, g))));
    else silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
    out[t] = __fmul_rn(silu, u);
  }
}

__global__ void add_kernel(float *__restrict__ a, const float *__restrict__ b, long n) {
  const long nv = n / 4;
  float4 *a4 = reinterpret_cast<float4 *>(a);
  const float4 *b4 = reinterpret_cast<const float4 *>(b);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (long)gridDim.x * blockDim.x) {
    float4 x = a4[i];
    const float4 y = b4[i];
    x.x = __fadd_rn(x.x, y.x); x.y = __fadd_rn(x.y, y.y); x.z = __fadd_rn(x.z, y.z); x.w = __fadd_rn(x.w, y.w);
    a4[i] = x;
  }
  if (blockIdx.x == 0 && threadIdx.x < n - nv * 4) a[nv * 4 + threadIdx.x] = __fadd_rn(a[nv * 4 + threadIdx.x], b[nv * 4 + threadIdx.x]);
}

// quantize_f32_to_int8 (quantize.rs:633-662): one CTA per row; absmax is an
// exact max so the parallel order does not matter.
__global__ void __launch_bounds__(256) quantize_kernel(const float *__restrict__ data, long in_dim,
                                                       int8_t *__restrict__ q, float *__restrict__ scales) {
  __shared__ float red[8];
  const long row = blockIdx.x;
  const float *r = data + row * in_dim;
  float m = 0.0f;
  for (long k = threadIdx.x; k < in_dim; k += blockDim.x) m = fmaxf(m, fabsf(r[k]));
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  float absmax = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) absmax = fmaxf(absmax, red[i]);
  const float inv = absmax > 0.0f ? __fdiv_rn(127.0f, absmax) : 0.0f;
  if (threadIdx.x == 0) scales[row] = __fdiv_rn(absmax, 127.0f);
  int8_t *qr = q + row * in_dim;
  for (long k = threadIdx.x; k < in_dim; k += blockDim.x) {
    float v = roundf(__fmul_rn(r[k], inv));
    v = fminf(fmaxf(v, -128.0f), 127.0f);
    qr[k] = (int8_t)(int)v;
  }
}

// Embedding gathers: one CTA per id.  Bad ids flag and write zeros.
__global__ void embed_f32_kernel(float *__restrict__ dst, const float *__restrict__ table,
                                 const int32_t *__restrict__ ids, int dim, long vocab, int *bad) {
  const int i = blockIdx.x;
  const int32_t id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && bad && threadIdx.x == 0) atomicExch(bad, 1);
  const float4 *src = reinterpret_cast<const float4 *>(table + (size_t)(ok ? id : 0) * dim);
  float4 *d = reinterpret_cast<float4 *>(dst + (size_t)i * dim);
  for (int c = threadIdx.x; c < dim / 4; c += blockDim.x) d[c] = ok ? src[c] : make_float4(0.f, 0.f, 0.f, 0.f);
}

__global__ void embed_int8_kernel(float *__restrict__ dst, const int8_t *__restrict__ table,
                                  const float *__restrict__ scales, const int32_t *__restrict__ ids, int dim,
                                  long vocab, int *bad) {
  const int i = blockIdx.x;
  const int32_t id = ids[i];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && bad && threadIdx.x == 0) atomicExch(bad, 1);
  const float s = ok ? scales[id] : 0.0f;
  const uint32_t *src = reinterpret_cast<const uint32_t *>(table + (size_t)(ok ? id : 0) * dim);
  float4 *d = reinterpret_cast<float4 *>(dst + (size_t)i * dim);
  for (int c = threadIdx.x; c < dim / 4; c += blockDim.x) {
    float f[4];
    i8x4_to_f32(ok ? src[c] : 0u, f);
    d[c] = make_float4(__fmul_rn(f[0], s), __fmul_rn(f[1], s), __fmul_rn(f[2], s), __fmul_rn(f[3], s));
  }
}

}  // namespace qasr

using namespace qasr;
static inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }
static inline bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

extern "C" int qasr_gelu(float *x, int64_t n, void *stream) {
  if (!x || n < 0 || !al16(x)) {
    set_error("qasr_gelu: invalid arguments (null, negative n or pointer not 16-byte aligned)");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  gelu_kernel<<<stream_grid(n / 4, 256), 256, 0, S(stream)>>>(x, n);
  return launch_status("qasr_gelu");
}

extern "C" int qasr_gelu_erf(float *x, int64_t n, void *stream) {
  if (!x || n < 0 || !al16(x)) {
    set_error("qasr_gelu_erf: invalid arguments (null, negative n or pointer not 16-byte aligned)");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  gelu_erf_kernel<<<stream_grid((n / 4 + 3) / 4, 256), 256, 0, S(stream)>>>(x, n);  // 4 vectors per thread
  return launch_status("qasr_gelu_erf");
}

extern "C" int qasr_silu(float *x, int64_t n, void *stream) {
  if (!x || n < 0) {
    set_error("qasr_silu: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  silu_kernel<<<stream_grid(n, 256), 256, 0, S(stream)>>>(x, n);
  return launch_status("qasr_silu");
}

extern "C" int qasr_swiglu_multiply(float *out, const float *gate_up, int seq, int inter, void *stream) {
  if (!out || !gate_up || seq < 0 || inter <= 0 || (reinterpret_cast<uintptr_t>(gate_up) & 7)) {
    set_error("qasr_swiglu_multiply: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  swiglu_kernel<<<stream_grid((long)seq * inter, 256), 256, 0, S(stream)>>>(out, gate_up, seq, inter);
  return launch_status("qasr_swiglu_multiply");
}

extern "C" int qasr_add_inplace(float *a, const float *b, int64_t n, void *stream) {
  if (!a || !b || n < 0 || !al16(a) || !al16(b)) {
    set_error("qasr_add_inplace: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  add_kernel<<<stream_grid(n / 4, 256), 256, 0, S(stream)>>>(a, b, n);
  return launch_status("qasr_add_inplace");
}

extern "C" int qasr_quantize_f32_to_int8(const float *data, int64_t out_dim, int64_t in_dim, int8_t *q,
                                         float *scales, void *stream) {
  if (!data || !q || !scales || out_dim < 0 || in_dim <= 0 || out_dim > 0x7fffffff) {
    set_error("qasr_quantize_f32_to_int8: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (out_dim == 0) return QASR_OK;
  quantize_kernel<<<(unsigned)out_dim, 256, 0, S(stream)>>>(data, in_dim, q, scales);
  return launch_status("qasr_quantize_f32_to_int8");
}

extern "C" int qasr_embed_gather_f32(float *dst, const float *table, const int32_t *ids, int n, int dim,
                                     int64_t vocab, int *bad_id_flag, void *stream) {
  if (!dst || !table || !ids || n < 0 || dim <= 0 || (dim & 3) || vocab <= 0 || !al16(dst) || !al16(table)) {
    set_error("qasr_embed_gather_f32: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  embed_f32_kernel<<<n, 256, 0, S(stream)>>>(dst, table, ids, dim, vocab, bad_id_flag);
  return launch_status("qasr_embed_gather_f32");
}

extern "C" int qasr_embed_gather_int8(float *dst, const int8_t *table, const float *scales, const int32_t *ids,
                                      int n, int dim, int64_t vocab, int *bad_id_flag, void *stream) {
  if (!dst || !table || !scales || !ids || n < 0 || dim <= 0 || (dim & 3) || vocab <= 0 || !al16(dst) ||
      (reinterpret_cast<uintptr_t>(table) & 3)) {
    set_error("qasr_embed_gather_int8: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (n == 0) return QASR_OK;
  embed_int8_kernel<<<n, 256, 0, S(stream)>>>(dst, table, scales, ids, dim, vocab, bad_id_flag);
  return launch_status("qasr_embed_gather_int8");
}
