// int8_matvec.cu -- INT8 weight-only matvec family for M <= 8 tokens
// (generic::int8_matvec_fused, crates/qwen-asr/src/kernels/generic.rs:39-49,
// driven by linear_nobias_int8 / linear_int8, kernels/mod.rs:650-673).
//
// y[m,o] = scales[o] * sum_k f32(w[o,k]) * x[m,k], f32 accumulation.
//
// Layout and data movement: weights are the reference's row-major [N, K]
// int8.  A warp owns R rows and walks K in 512-element blocks; in block b,
// lane L covers elements b*512 + 128q + 4L + (0..3) for q = 0..3, so each
// weight load instruction of the warp reads 128 contiguous bytes of a row
// and each x load reads 512 contiguous bytes of a token -- every access is
// fully coalesced and x (M*K*4 bytes, shared by all warps) stays in L1/L2.
// The R*MT partial sums of a lane are reduced across the warp with a
// reduce-scatter (V-1 + log-steps shuffles for V values instead of 5V).
// Epilogues fuse the residual add, bias, SwiGLU of interleaved gate/up rows
// (decoder.rs:916-921) and the first-max argmax of the lm head
// (decoder.rs:936-947).
#include "common.cuh"
#include "matvec.cuh"
#include "umma.cuh"

namespace qasr {

QASR_DEV uint32_t ldg_w32(const int8_t *p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// -------------------------------------------------------------- kernel
template <int MT, int R, MvEpi E>
__global__ void __launch_bounds__(kMvWarps * 32)
int8_matvec_kernel(MvParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int V = R * MT;
  const int my_idx = reduce_index<V>(lane);
  const int my_r = my_idx / MT, my_m = my_idx % MT;
  const bool writer = (lane & ((32 / V) - 1)) == 0;
  const int K = p.K, N = p.N, M = p.M;
  const int nblk = K / 512;
  const int tail_q = (K % 512) / 128;  // 128-element quarters in a partial last block
  unsigned long long best = 0ull;      // argmax epilogue state (this lane's token my_m)

  const long n_groups = ((long)N + R - 1) / R;
  for (long g = (long)blockIdx.x * kMvWarps + warp; g < n_groups; g += (long)gridDim.x * kMvWarps) {
    const int row0 = (int)(g * R);
    float acc[R][MT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;
    const int8_t *wrow[R];
#pragma unroll
    for (int r = 0; r < R; ++r) wrow[r] = p.w + (size_t)min(row0 + r, N - 1) * K + 4 * lane;

    for (int b = 0; b <= nblk; ++b) {
      const int nq = b < nblk ? 4 : tail_q;
      if (nq == 0) break;
      uint32_t wv[R][4];
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int q = 0; q < 4; ++q) wv[r][q] = q < nq ? ldg_w32(wrow[r] + b * 512 + 128 * q) : 0u;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q >= nq) break;
        float4 xv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m)
          xv[m] = m < M ? *reinterpret_cast<const float4 *>(p.x + (size_t)m * p.x_stride + b * 512 + 128 * q + 4 * lane)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          float wf[4];
          i8x4_to_f32(wv[r][q], wf);
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            acc[r][m] = fmaf(wf[0], xv[m].x, acc[r][m]);
            acc[r][m] = fmaf(wf[1], xv[m].y, acc[r][m]);
            acc[r][m] = fmaf(wf[2], xv[m].z, acc[r][m]);
            acc[r][m] = fmaf(wf[3], xv[m].w, acc[r][m]);
          }
        }
      }
    }

    float flat[V];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) flat[r * MT + m] = acc[r][m];
    const float sum = warp_reduce_scatter<V>(flat);
    const int row = row0 + my_r;
    const bool valid = my_m < M && row < N;

    if constexpr (E == MvEpi::SwiGLU) {
      // partner value (same token, the other row of the gate/up pair)
      const float other = __shfl_xor_sync(0xffffffffu, sum, 32 / R);
      if (writer && valid && (my_r & 1) == 0) {
        const float g = __fmul_rn(sum, p.scales[row]);
        const float u = __fmul_rn(other, p.scales[row + 1]);
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        p.y[(size_t)my_m * p.y_stride + row / 2] = __fmul_rn(silu, u);
      }
    } else if constexpr (E == MvEpi::Argmax) {
      if (valid) {
        const float logit = __fmul_rn(sum, p.scales[row]);
        if (writer && p.y) p.y[(size_t)my_m * p.y_stride + row] = logit;
        const unsigned long long key = argmax_key(logit, (uint32_t)row);
        best = key > best ? key : best;
      }
    } else {
      if (writer && valid) {
        float v = __fmul_rn(sum, p.scales[row]);
        if constexpr (E == MvEpi::StoreBias) v = __fadd_rn(v, p.bias[row]);
        float *dst = p.y + (size_t)my_m * p.y_stride + row;
        if constexpr (E == MvEpi::Residual) v = __fadd_rn(*dst, v);
        *dst = v;
      }
    }
  }

  if constexpr (E == MvEpi::Argmax) {
    // per-token max over the CTA, one atomic per token, then the last CTA to
    // finish converts keys to ids and re-arms the keys/counter for next use.
    __shared__ unsigned long long sbest[kMvWarps * 32];
    __shared__ bool last;
    sbest[threadIdx.x] = best;
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int t = 0; t < kMvWarps * 32; ++t)
        if (reduce_index<V>(t & 31) % MT == (int)threadIdx.x && sbest[t] > b) b = sbest[t];
      if (b) atomicMax(p.keys + threadIdx.x, b);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (last && threadIdx.x < M) {
      __threadfence();
      const unsigned long long k = atomicExch(p.keys + threadIdx.x, 0ull);
      p.ids[threadIdx.x] = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    }
    if (last && threadIdx.x == 0) atomicExch(p.counter, 0u);
  }
}

// ------------------------------------------------------------ dispatch
static int sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

template <int MT, MvEpi E>
static void launch_mt(const MvParams &p, int R, cudaStream_t st) {
  const long warps_needed = ((long)p.N + R - 1) / R;
  long grid = (warps_needed + kMvWarps - 1) / kMvWarps;
  if (E == MvEpi::Argmax) grid = std::min<long>(grid, (long)sm_count() * 8);
  grid = std::max<long>(1, std::min<long>(grid, 1L << 30));
  switch (R) {
    case 1: int8_matvec_kernel<MT, 1, E><<<(unsigned)grid, kMvWarps * 32, 0, st>>>(p); break;
    case 2: int8_matvec_kernel<MT, 2, E><<<(unsigned)grid, kMvWarps * 32, 0, st>>>(p); break;
    default: int8_matvec_kernel<MT, 4, E><<<(unsigned)grid, kMvWarps * 32, 0, st>>>(p); break;
  }
}

template <MvEpi E>
static void launch_epi(const MvParams &p, int R, cudaStream_t st) {
  if (p.M <= 1) launch_mt<1, E>(p, R, st);
  else if (p.M <= 2) launch_mt<2, E>(p, R, st);
  else if (p.M <= 4) launch_mt<4, E>(p, R, st);
  else launch_mt<8, E>(p, R, st);
}

// Rows per warp: enough CTAs to cover the SMs twice when possible (R=4 gives
// the most reuse of each x load), R>=2 for the SwiGLU pair epilogue.
int mv_pick_rows(int N, MvEpi e) {
  const long target = (long)sm_count() * 2 * kMvWarps;  // warps
  int R = 4;
  while (R > 1 && (long)N / R < target) R >>= 1;
  if (e == MvEpi::SwiGLU && R < 2) R = 2;
  return R;
}

void mv_launch(const MvParams &p, MvEpi e, cudaStream_t st, int R) {
  if (R <= 0) R = mv_pick_rows(p.N, e);
  switch (e) {
    case MvEpi::Store: launch_epi<MvEpi::Store>(p, R, st); break;
    case MvEpi::StoreBias: launch_epi<MvEpi::StoreBias>(p, R, st); break;
    case MvEpi::Residual: launch_epi<MvEpi::Residual>(p, R, st); break;
    case MvEpi::SwiGLU: launch_epi<MvEpi::SwiGLU>(p, R, st); break;
    case MvEpi::Argmax: launch_epi<MvEpi::Argmax>(p, 4, st); break;
  }
}

// Per-device scratch for the argmax keys/counter of the kernel-level API.
struct ArgmaxScratch {
  unsigned long long *keys = nullptr;
  unsigned *counter = nullptr;
};
static ArgmaxScratch g_argmax_scratch[64];

int argmax_scratch(unsigned long long **keys, unsigned **counter) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return QASR_ERR_INVALID;
  ArgmaxScratch &s = g_argmax_scratch[dev];
  if (!s.keys) {
    void *buf = nullptr;
    if (cudaMalloc(&buf, 256) != cudaSuccess) {
      set_error("argmax scratch: cudaMalloc failed");
      return QASR_ERR_ALLOC;
    }
    cudaMemset(buf, 0, 256);
    s.keys = reinterpret_cast<unsigned long long *>(buf);
    s.counter = reinterpret_cast<unsigned *>(reinterpret_cast<char *>(buf) + 128);
  }
  *keys = s.keys;
  *counter = s.counter;
  return QASR_OK;
}

}  // namespace qasr

using namespace qasr;
static inline cudaStream_t S(void *s) { return reinterpret_cast<cudaStream_t>(s); }

static int check_mv(const char *fn, const float *y, const float *x, const int8_t *w, const float *scales, int seq,
                    int in_dim, int out_dim) {
  if (!y || !x || !w || !scales || seq < 0 || in_dim <= 0 || out_dim <= 0) {
    set_error("%s: invalid arguments", fn);
    return QASR_ERR_INVALID;
  }
  if (in_dim % 128 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 3)) {
    set_error("%s: in_dim must be a multiple of 128 with x 16-byte and w 4-byte aligned (in_dim=%d)", fn, in_dim);
    return QASR_ERR_UNSUPPORTED;
  }
  return QASR_OK;
}

// Try the tensor-core kernel (umma_matvec.cu) for M <= 8 tokens; returns
// QASR_ERR_UNSUPPORTED (nothing launched) for shapes it does not cover.
static int try_umma(const float *x, long xs, const float *nw, float eps, const int8_t *w, const float *scales,
                    const float *bias, float *y, long ys, int M, int K, int N, MvEpi e, int32_t *ids, cudaStream_t st) {
  if (K % 128 || N < 128 || (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (xs & 3) || (reinterpret_cast<uintptr_t>(nw) & 15) || M < 1 || M > 8 || (e == MvEpi::SwiGLU && (N & 1)))
    return QASR_ERR_UNSUPPORTED;
  UmmaParams p{};
  int rc = umma_weight_map(&p.tmap, w, N, K);
  if (rc) return rc;
  p.x = x; p.x_stride = xs; p.norm_w = nw; p.eps = eps; p.scales = scales; p.bias = bias;
  p.y = y; p.y_stride = ys; p.M = M; p.K = K; p.N = N;
  if (e == MvEpi::Argmax) {
    if ((rc = argmax_scratch(&p.keys, &p.counter))) return rc;
    p.ids = ids;
  }
  return umma_launch(p, e, st, false);
}

// Try the weight-streaming kernel (matvec2.cu) for M <= 8 tokens; returns
// QASR_ERR_UNSUPPORTED (nothing launched) for shapes it does not cover.
static int try_mv2(const float *x, long xs, const float *nw, float eps, const int8_t *w, const float *scales,
                   const float *bias, float *y, long ys, int M, int K, int N, MvEpi e, int32_t *ids, cudaStream_t st) {
  if (K % 512 || (reinterpret_cast<uintptr_t>(w) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) || (xs & 3) ||
      (reinterpret_cast<uintptr_t>(nw) & 15) ||
      M < 1 || M > 8)
    return QASR_ERR_UNSUPPORTED;
  Mv2Params p{};
  p.x = x; p.x_stride = xs; p.norm_w = nw; p.eps = eps; p.w = w; p.scales = scales; p.bias = bias;
  p.y = y; p.y_stride = ys; p.M = M; p.K = K; p.N = N;
  p.S = nw ? 1 : mv2_pick_slices(N, K, M, e);
  p.KS = K / p.S;
  p.KC = 512;  // row-major weights: one copy per 512-byte row segment
  if (p.S == 1 && (size_t)8 * K * 4 > 96 * 1024) return QASR_ERR_UNSUPPORTED;
  int rc;
  if (p.S > 1) {
    void *part, *ctr;
    if ((rc = dev_scratch(kScratchPartial, (size_t)p.S * M * N * 4, &part))) return rc;
    if ((rc = dev_scratch(kScratchCounter, (size_t)(N / 2 + 16) * 4, &ctr))) return rc;
    p.partial = static_cast<float *>(part);
    p.rg_counter = static_cast<unsigned *>(ctr);
  }
  if (e == MvEpi::Argmax) {
    if ((rc = argmax_scratch(&p.keys, &p.counter))) return rc;
    p.ids = ids;
  }
  return mv2_launch(p, e, st, false);
}

static int linear_int8_impl(const char *fn, float *y, const float *x, const int8_t *w, const float *scales,
                            const float *bias, int seq, int in_dim, int out_dim, void *stream) {
  int rc = check_mv(fn, y, x, w, scales, seq, in_dim, out_dim);
  if (rc) return rc;
  if (seq > 8) {  // prefill / encoder shapes: one tensor-core GEMM over all rows
    rc = int8_gemm(y, out_dim, x, in_dim, w, scales, bias, seq, in_dim, out_dim, S(stream));
    if (rc != QASR_ERR_UNSUPPORTED) return rc;
  }
  for (int s0 = 0; s0 < seq; s0 += 8) {
    const int m = std::min(8, seq - s0);
    rc = try_umma(x + (size_t)s0 * in_dim, in_dim, nullptr, 0.f, w, scales, bias, y + (size_t)s0 * out_dim, out_dim,
                  m, in_dim, out_dim, bias ? MvEpi::StoreBias : MvEpi::Store, nullptr, S(stream));
    if (rc == QASR_ERR_UNSUPPORTED)
      rc = try_mv2(x + (size_t)s0 * in_dim, in_dim, nullptr, 0.f, w, scales, bias, y + (size_t)s0 * out_dim, out_dim,
                   m, in_dim, out_dim, bias ? MvEpi::StoreBias : MvEpi::Store, nullptr, S(stream));
    if (rc == QASR_ERR_UNSUPPORTED) {
      MvParams p{};
      p.x = x + (size_t)s0 * in_dim;
      p.x_stride = in_dim;
      p.w = w;
      p.scales = scales;
      p.bias = bias;
      p.y = y + (size_t)s0 * out_dim;
      p.y_stride = out_dim;
      p.M = m;
      p.K = in_dim;
      p.N = out_dim;
      mv_launch(p, bias ? MvEpi::StoreBias : MvEpi::Store, S(stream), 0);
    } else if (rc) {
      return rc;
    }
  }
  return launch_status(fn);
}

extern "C" int qasr_linear_nobias_int8(float *y, const float *x, const int8_t *w, const float *scales, int seq,
                                       int in_dim, int out_dim, void *stream) {
  return linear_int8_impl("qasr_linear_nobias_int8", y, x, w, scales, nullptr, seq, in_dim, out_dim, stream);
}

extern "C" int qasr_linear_int8(float *y, const float *x, const int8_t *w, const float *scales, const float *bias,
                                int seq, int in_dim, int out_dim, void *stream) {
  return linear_int8_impl("qasr_linear_int8", y, x, w, scales, bias, seq, in_dim, out_dim, stream);
}

extern "C" int qasr_int8_matvec_residual(float *x, const float *a, const int8_t *w, const float *scales, int M,
                                         int in_dim, int out_dim, void *stream) {
  int rc = check_mv("qasr_int8_matvec_residual", x, a, w, scales, M, in_dim, out_dim);
  if (rc) return rc;
  if (M > 8) {
    set_error("qasr_int8_matvec_residual: M=%d > 8", M);
    return QASR_ERR_UNSUPPORTED;
  }
  if (M == 0) return QASR_OK;
  rc = try_umma(a, in_dim, nullptr, 0.f, w, scales, nullptr, x, out_dim, M, in_dim, out_dim, MvEpi::Residual, nullptr,
                S(stream));
  if (rc == QASR_ERR_UNSUPPORTED)
    rc = try_mv2(a, in_dim, nullptr, 0.f, w, scales, nullptr, x, out_dim, M, in_dim, out_dim, MvEpi::Residual, nullptr,
                 S(stream));
  if (rc != QASR_ERR_UNSUPPORTED) return rc ? rc : launch_status("qasr_int8_matvec_residual");
  MvParams p{};
  p.x = a;
  p.x_stride = in_dim;
  p.w = w;
  p.scales = scales;
  p.y = x;
  p.y_stride = out_dim;
  p.M = M;
  p.K = in_dim;
  p.N = out_dim;
  mv_launch(p, MvEpi::Residual, S(stream), 0);
  return launch_status("qasr_int8_matvec_residual");
}

extern "C" int qasr_int8_norm_gateup_swiglu(float *h, const float *x, const float *norm_w, const int8_t *w_gate_up,
                                            const float *scales, int M, int hidden, int inter, float eps,
                                            void *stream) {
  int rc = check_mv("qasr_int8_norm_gateup_swiglu", h, x, w_gate_up, scales, M, hidden, 2 * inter);
  if (rc) return rc;
  if (!norm_w || M > 8) {
    set_error("qasr_int8_norm_gateup_swiglu: norm_w missing or M=%d > 8", M);
    return QASR_ERR_INVALID;
  }
  if (M == 0) return QASR_OK;
  rc = try_umma(x, hidden, norm_w, eps, w_gate_up, scales, nullptr, h, inter, M, hidden, 2 * inter, MvEpi::SwiGLU,
                nullptr, S(stream));
  if (rc == QASR_ERR_UNSUPPORTED)
    rc = try_mv2(x, hidden, norm_w, eps, w_gate_up, scales, nullptr, h, inter, M, hidden, 2 * inter, MvEpi::SwiGLU,
                 nullptr, S(stream));
  if (rc != QASR_ERR_UNSUPPORTED) return rc ? rc : launch_status("qasr_int8_norm_gateup_swiglu");
  float *xn = nullptr;
  if ((rc = mv_norm_scratch(&xn, (size_t)M * hidden))) return rc;
  if ((rc = qasr_rms_norm(xn, x, norm_w, M, hidden, eps, stream))) return rc;
  MvParams p{};
  p.x = xn;
  p.x_stride = hidden;
  p.w = w_gate_up;
  p.scales = scales;
  p.y = h;
  p.y_stride = inter;
  p.M = M;
  p.K = hidden;
  p.N = 2 * inter;
  mv_launch(p, MvEpi::SwiGLU, S(stream), 0);
  return launch_status("qasr_int8_norm_gateup_swiglu");
}

extern "C" int qasr_final_norm_lmhead_argmax(int32_t *ids_out, float *logits_out, const float *x,
                                             const float *norm_w, const int8_t *w, const float *scales, int M,
                                             int hidden, int vocab, float eps, void *stream) {
  int rc = check_mv("qasr_final_norm_lmhead_argmax", logits_out ? logits_out : reinterpret_cast<float *>(ids_out),
                    x, w, scales, M, hidden, vocab);
  if (rc) return rc;
  if (!ids_out || !norm_w || M > 8) {
    set_error("qasr_final_norm_lmhead_argmax: ids_out/norm_w missing or M=%d > 8", M);
    return QASR_ERR_INVALID;
  }
  if (M == 0) return QASR_OK;
  rc = try_umma(x, hidden, norm_w, eps, w, scales, nullptr, logits_out, vocab, M, hidden, vocab, MvEpi::Argmax,
                ids_out, S(stream));
  if (rc == QASR_ERR_UNSUPPORTED)
    rc = try_mv2(x, hidden, norm_w, eps, w, scales, nullptr, logits_out, vocab, M, hidden, vocab, MvEpi::Argmax,
                 ids_out, S(stream));
  if (rc != QASR_ERR_UNSUPPORTED) return rc ? rc : launch_status("qasr_final_norm_lmhead_argmax");
  float *xn = nullptr;
  if ((rc = mv_norm_scratch(&xn, (size_t)M * hidden))) return rc;
  if ((rc = qasr_rms_norm(xn, x, norm_w, M, hidden, eps, stream))) return rc;
  unsigned long long *keys;
  unsigned *counter;
  if ((rc = argmax_scratch(&keys, &counter))) return rc;
  MvParams p{};
  p.x = xn;
  p.x_stride = hidden;
  p.w = w;
  p.scales = scales;
  p.y = logits_out;
  p.y_stride = vocab;
  p.M = M;
  p.K = hidden;
  p.N = vocab;
  p.keys = keys;
  p.counter = counter;
  p.ids = ids_out;
  mv_launch(p, MvEpi::Argmax, S(stream), 4);
  return launch_status("qasr_final_norm_lmhead_argmax");
}
