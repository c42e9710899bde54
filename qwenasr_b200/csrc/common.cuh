// common.cuh -- shared device helpers for the qwenasr_b200 kernels (sm_100a).
//
// The library is compiled with --fmad=false: nothing is contracted into an
// FMA unless the source says fmaf().  That is what lets the row kernels
// reproduce the reference's rounding sequence (Rust never contracts; the
// AVX2 code uses explicit _mm256_fmadd_ps).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qwenasr_cuda.h"

#define QASR_DEV __device__ __forceinline__

namespace qasr {

// Host-side error slot (thread-local); set by every failing entry point.
void set_error(const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);
// Returns QASR_ERR_CUDA if the last launch failed, else QASR_OK.
int launch_status(const char *what);

constexpr int kWarp = 32;

QASR_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

QASR_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Horizontal sum of an 8-lane AVX register in the order of the reference's
// hsum_ps (crates/qwen-asr/src/kernels/avx.rs:36-49):
// ((v0+v4)+(v1+v5)) + ((v2+v6)+(v3+v7)).
QASR_DEV float hsum8(const float v[8]) {
  float s0 = __fadd_rn(v[0], v[4]), s1 = __fadd_rn(v[1], v[5]);
  float s2 = __fadd_rn(v[2], v[6]), s3 = __fadd_rn(v[3], v[7]);
  return __fadd_rn(__fadd_rn(s0, s1), __fadd_rn(s2, s3));
}

// One lane of the reference's fast_exp_avx (avx.rs:487-514): clamp to
// [-126,126] in the base-2 domain, round-to-nearest-even integer part, degree
// 5 Taylor polynomial of e^f on the fractional part, scaled by 2^i.  These are
// the reference's own constants; restated so GELU/SwiGLU match it bit for bit.
QASR_DEV float fast_exp_ref(float x) {
  float val = __fmul_rn(x, 1.442695041f);
  val = fminf(val, 126.0f);
  val = fmaxf(val, -126.0f);
  int ip = __float2int_rn(val);
  float fp = __fsub_rn(val, __int2float_rn(ip));
  float exp_i = __int_as_float((ip + 127) << 23);
  float f = __fmul_rn(fp, 0.6931471806f);
  float p = fmaf(1.0f / 120.0f, f, 1.0f / 24.0f);
  p = fmaf(p, f, 1.0f / 6.0f);
  p = fmaf(p, f, 0.5f);
  p = fmaf(p, f, 1.0f);
  p = fmaf(p, f, 1.0f);
  return __fmul_rn(exp_i, p);
}

// tanh GELU of avx::gelu_inplace (avx.rs:536-555), one lane.
QASR_DEV float gelu_tanh_ref(float v) {
  const float v2 = __fmul_rn(v, v), v3 = __fmul_rn(v2, v);
  const float inner = __fmul_rn(0.7978845608028654f, fmaf(0.044715f, v3, v));
  const float e = fast_exp_ref(__fmul_rn(2.0f, inner));
  const float t = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(e, 1.0f)));
  return __fmul_rn(0.5f, __fmul_rn(v, __fadd_rn(1.0f, t)));
}

// Exact-erf GELU 0.5*x*(1+erf(x/sqrt(2))) (the Metal encoder's activation,
// encoder_gpu.rs:470), one lane.
QASR_DEV float gelu_erf_f(float v) {
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, erff(__fmul_rn(v, 0.70710678118654752f))));
}

// Exact-erf GELU over n floats in place, for the CTAs [0, n_ctas) of a
// grid-stride pass: four 16-byte vectors per thread per round, all loaded
// before any is computed, so each thread keeps 64 bytes in flight.
QASR_DEV void gelu_erf_pass(float *__restrict__ x, long n, long cta, long n_ctas) {
  const long nv = n / 4;
  float4 *x4 = reinterpret_cast<float4 *>(x);
  const long step = n_ctas * blockDim.x * 4;
  for (long base = cta * blockDim.x * 4 + threadIdx.x; base < nv; base += step) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (base + (long)u * blockDim.x < nv) v[u] = x4[base + (long)u * blockDim.x];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (base + (long)u * blockDim.x < nv) {
        float4 w = v[u];
        w.x = gelu_erf_f(w.x); w.y = gelu_erf_f(w.y); w.z = gelu_erf_f(w.z); w.w = gelu_erf_f(w.w);
        x4[base + (long)u * blockDim.x] = w;
      }
  }
  if (cta == 0 && threadIdx.x < n - nv * 4) x[nv * 4 + threadIdx.x] = gelu_erf_f(x[nv * 4 + threadIdx.x]);
}

// Four int8 values packed in a 32-bit word -> four exact floats.  Each byte
// (sign-flipped to excess-128) is placed in the mantissa of 2^23 with one
// byte permute; subtracting 2^23+128 recovers the signed value exactly.
QASR_DEV void i8x4_to_f32(uint32_t w, float out[4]) {
  uint32_t u = w ^ 0x80808080u;
  out[0] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7440)), 8388736.0f);
  out[1] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7441)), 8388736.0f);
  out[2] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7442)), 8388736.0f);
  out[3] = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7443)), 8388736.0f);
}

// Monotone u32 image of a float (for packed atomicMax argmax).
QASR_DEV uint32_t float_order(float f) {
  uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
QASR_DEV float float_unorder(uint32_t o) {
  uint32_t b = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
  return __uint_as_float(b);
}
// Key whose max is the largest value and, among equal values, the lowest
// index: the strict-'>' first-max rule of decoder.rs:942-947.
QASR_DEV unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)float_order(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}

// Streaming 128-bit load (no L1 allocation) for weights read exactly once per step.
QASR_DEV uint4 ldg_stream(const void *p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// prologue, and wait for the previous kernel's memory to be visible.
QASR_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
QASR_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Launch with programmatic stream serialization: the grid may be scheduled
// while the previous kernel of the stream is still running, so its launch
// and CTA set-up overlap that kernel's tail.  The kernel must call pdl_wait()
// before its first global-memory access (read or write): that wait returns
// once the previous grid has completed and its writes are visible, so the
// stream order of memory effects is unchanged.
template <typename... Params, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(Params...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<Params>(args)...);
}

// Warp reduce-scatter: V per-lane partial sums -> one full sum per lane group.
template <int V>
struct Log2 {
  static constexpr int value = 1 + Log2<V / 2>::value;
};
template <>
struct Log2<1> {
  static constexpr int value = 0;
};

// Sum each of the V per-lane values over the 32 lanes.  Afterwards lane l
// holds the total of value index reduce_index<V>(l) in v[0].
template <int V>
QASR_DEV float warp_reduce_scatter(float (&v)[V]) {
  const int lane = threadIdx.x & 31;
  constexpr int LOG = Log2<V>::value;
#pragma unroll
  for (int s = 0; s < LOG; ++s) {
    const int off = 16 >> s;
    const int n = V >> s;
    const bool upper = (lane & off) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, off));
    }
  }
#pragma unroll
  for (int off = 16 >> LOG; off >= 1; off >>= 1) v[0] = __fadd_rn(v[0], __shfl_xor_sync(0xffffffffu, v[0], off));
  return v[0];
}

template <int V>
QASR_DEV int reduce_index(int lane) {
  constexpr int LOG = Log2<V>::value;
  int idx = 0;
#pragma unroll
  for (int s = 0; s < LOG; ++s)
    if (lane & (16 >> s)) idx += V >> (s + 1);
  return idx;
}

inline int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

// Copies rows row0 .. row0+n-1, columns col0 .. col0+HD-1 of two row-major
// matrices (row stride `stride`) into shared memory (K rows padded by PADK
// floats, V rows dense).  Each thread issues eight independent loads before
// its stores, so a block has 8 x blockDim loads in flight instead of one.
template <int HD, int PADK>
QASR_DEV void stage_kv_rows(float *sK, float *sV, const float *__restrict__ k, const float *__restrict__ v, long row0,
                            long stride, long col0, int n) {
  const int total = n * HD;
  for (int base = threadIdx.x; base < total; base += blockDim.x * 8) {
    float kr[8], vr[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * (int)blockDim.x;
      if (idx < total) {
        const long g = (row0 + idx / HD) * stride + col0 + idx % HD;
        kr[u] = k[g];
        vr[u] = v[g];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int idx = base + u * (int)blockDim.x;
      if (idx < total) {
        const int j = idx / HD, d = idx % HD;
        sK[j * (HD + PADK) + d] = kr[u];
        sV[j * HD + d] = vr[u];
      }
    }
  }
}

}  // namespace qasr
