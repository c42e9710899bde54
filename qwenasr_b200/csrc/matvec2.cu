// matvec2.cu -- weight-streaming INT8 matvec for M <= 8 tokens (the decode
// projections and the lm head): y[m,o] = scales[o] * sum_k f32(w[o,k])*x[m,k]
// (generic::int8_matvec_fused, crates/qwen-asr/src/kernels/generic.rs:39-49).
//
// Design (HBM-bound: every weight byte is read exactly once per call):
//  * persistent grid, one 8-warp CTA per SM; the N x K weight matrix is cut
//    into units of R=4 rows x one K-slice (KS columns), numbered slice-major
//    and handed out to CTAs in contiguous ranges, warps round-robin;
//  * each warp streams its units' rows through its own 4-stage shared-memory
//    ring with 1D bulk copies (cp.async.bulk, completion on an mbarrier), so
//    up to 128 KB of weights per SM are in flight;
//  * x (<= 2 K-slices of all M tokens) is staged once per CTA in a permuted
//    layout in which both the 16-byte weight reads and the 16-byte x reads of
//    a warp are bank-conflict free; an optional RMSNorm (the reference's
//    exact summation order, rowops.cuh) is applied while staging;
//  * per unit a lane holds R*M partial sums, reduced with one warp
//    reduce-scatter; split-K units (S > 1) park partials and the last unit of
//    a row group (atomic counter) sums slices 0..S-1 in order, so results are
//    deterministic;
//  * epilogues: store, +bias, residual add, SwiGLU of interleaved gate/up rows
//    (decoder.rs:916-921), first-max argmax (decoder.rs:942-947);
//  * the weight prefetch is issued before griddepcontrol.wait, so under
//    programmatic dependent launch it overlaps the previous kernel.
// Every mbarrier wait is bounded (tma.cuh); a timeout sets *err and the kernel
// drains its copies and returns.
#include "common.cuh"
#include "matvec.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace qasr {

constexpr int kMv2Warps = 8;
constexpr int kMv2Stages = 4;
constexpr int kMv2R = 4;
constexpr int kMv2KCMax = 1024;  // largest bytes of one row per pipeline stage

// Position of element k (within a slice) in the permuted x layout.
QASR_DEV int xperm(int k) {
  const int blk = k >> 9, kk = k & 511;
  return (blk << 9) + (((kk & 15) >> 2) << 7) + ((kk >> 4) << 2) + (kk & 3);
}
// Inverse: slice-local element index of permuted slot idx.
QASR_DEV int xperm_inv(int idx) {
  const int blk = idx >> 9, r = idx & 511;
  return (blk << 9) + (((r & 127) >> 2) << 4) + ((r >> 7) << 2) + (r & 3);
}

struct Mv2Smem {
  uint64_t bar[kMv2Warps][kMv2Stages];
  float inv[8];
  int err;
  int last;
  unsigned long long best[kMv2Warps * 32];
};

template <int MT, MvEpi E, bool NORM>
__global__ void __launch_bounds__(kMv2Warps * 32, 1)
int8_mv2_kernel(const __grid_constant__ Mv2Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Mv2Smem &sm = *reinterpret_cast<Mv2Smem *>(smem_raw);
  const int KC = p.KC;
  int8_t *wbuf = reinterpret_cast<int8_t *>(smem_raw + ((sizeof(Mv2Smem) + 127) & ~size_t(127)));
  float *xs = reinterpret_cast<float *>(wbuf + (size_t)kMv2Warps * kMv2Stages * kMv2R * KC);

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int R = kMv2R;
  constexpr int V = R * MT;
  const int M = p.M, K = p.K, N = p.N, S = p.S, KS = p.KS;
  const int n_rg = (N + R - 1) / R;
  const long U = (long)n_rg * S;
  const long u0 = U * blockIdx.x / gridDim.x, u1 = U * (blockIdx.x + 1) / gridDim.x;
  const int slice_lo = (int)(u0 / n_rg);
  const int nchunk = KS / KC;
  const long my_units = u1 - u0 > warp ? (u1 - u0 - warp + kMv2Warps - 1) / kMv2Warps : 0;
  const long T = my_units * nchunk;  // pipeline items of this warp

  if (threadIdx.x < kMv2Warps * kMv2Stages) mbar_init(&sm.bar[threadIdx.x / kMv2Stages][threadIdx.x % kMv2Stages], 1);
  if (threadIdx.x == 0) sm.err = 0;
  mbar_fence_init();
  __syncthreads();

  int8_t *mybuf = wbuf + (size_t)warp * kMv2Stages * R * KC;
  auto issue = [&](long i) {  // lane 0 only
    const long j = i / nchunk;
    const int c = (int)(i % nchunk);
    const long u = u0 + warp + j * kMv2Warps;
    const int slice = (int)(u / n_rg), rg = (int)(u % n_rg);
    const int st = (int)(i % kMv2Stages);
    mbar_arrive_expect_tx(&sm.bar[warp][st], R * KC);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int row = min(rg * R + r, N - 1);
      bulk_g2s(mybuf + ((size_t)st * R + r) * KC, p.w + (size_t)row * K + (size_t)slice * KS + (size_t)c * KC, KC,
               &sm.bar[warp][st]);
    }
  };
  if (lane == 0)
    for (long i = 0; i < T && i < kMv2Stages; ++i) issue(i);

  // activations come from the previous kernel: wait for it only now
  pdl_wait();
  pdl_launch_dependents();

  // ---- stage x (slices slice_lo, slice_lo+1) in the permuted layout ----
  const int nsl = (u1 > u0) ? (int)((u1 - 1) / n_rg) - slice_lo + 1 : 0;
  for (int sl = 0; sl < nsl; ++sl) {
    const int n4 = M * KS / 4;
    for (int t = threadIdx.x; t < n4; t += blockDim.x) {
      const int m = t / (KS / 4), k = (t % (KS / 4)) * 4;
      const float4 v = *reinterpret_cast<const float4 *>(p.x + (size_t)m * p.x_stride + (size_t)(slice_lo + sl) * KS + k);
      *reinterpret_cast<float4 *>(xs + ((size_t)sl * MT + m) * KS + xperm(k)) = v;
    }
  }
  if constexpr (NORM) {  // S == 1: the slice is the whole row
    __syncthreads();
    if (warp < M) {
      const float *xr = xs + (size_t)warp * KS;
      const int n = K, n16 = n / 16, lane16 = lane;
      float acc = 0.0f;
      if (lane16 < 16) {
        for (int j = 0; j < n16; ++j) {
          const float v = xr[xperm(16 * j + lane16)];
          acc = fmaf(v, v, acc);
        }
        if ((n & 15) >= 8 && lane16 < 8) {
          const float v = xr[xperm(16 * n16 + lane16)];
          acc = fmaf(v, v, acc);
        }
      }
      float sum = hsum16_avx_order(acc);
      if (lane == 0)
        for (int i = avx_vector_extent(n); i < n; ++i) {
          const float v = xr[xperm(i)];
          sum = __fadd_rn(sum, __fmul_rn(v, v));
        }
      if (lane == 0) sm.inv[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), p.eps)));
    }
    __syncthreads();
    const int n4 = M * KS / 4;
    for (int t = threadIdx.x; t < n4; t += blockDim.x) {
      const int m = t / (KS / 4), slot = (t % (KS / 4)) * 4;
      float4 *v4 = reinterpret_cast<float4 *>(xs + (size_t)m * KS + slot);
      const int k = xperm_inv(slot);
      const float inv = sm.inv[m];
      const float4 wn = *reinterpret_cast<const float4 *>(p.norm_w + k);
      float4 v = *v4;
      v.x = __fmul_rn(__fmul_rn(v.x, inv), wn.x);
      v.y = __fmul_rn(__fmul_rn(v.y, inv), wn.y);
      v.z = __fmul_rn(__fmul_rn(v.z, inv), wn.z);
      v.w = __fmul_rn(__fmul_rn(v.w, inv), wn.w);
      *v4 = v;
    }
  }
  // rows m >= M of the staged x are never read (token loops stop at M)
  __syncthreads();

  const int my_idx = reduce_index<V>(lane);
  const int my_r = my_idx / MT, my_m = my_idx % MT;
  const bool writer = (lane & ((32 / V) - 1)) == 0;
  unsigned long long best = 0ull;
  bool failed = false;

  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;

  long fail_item = -1;
  for (long i = 0; i < T && !failed; ++i) {
    const int st = (int)(i % kMv2Stages);
    if (!mbar_wait(&sm.bar[warp][st], (unsigned)((i / kMv2Stages) & 1))) {
      failed = true;
      fail_item = i;
      break;
    }
    const long j = i / nchunk;
    const int c = (int)(i % nchunk);
    const long u = u0 + warp + j * kMv2Warps;
    const int slice = (int)(u / n_rg), rg = (int)(u % n_rg);
    const int8_t *wb = mybuf + (size_t)st * R * KC;
    const float *xb = xs + (size_t)(slice - slice_lo) * MT * KS + (size_t)c * KC + 4 * lane;
    for (int blk = 0; blk < KC; blk += 512) {
      uint4 wv[R];
#pragma unroll
      for (int r = 0; r < R; ++r) wv[r] = *reinterpret_cast<const uint4 *>(wb + (size_t)r * KC + blk + 16 * lane);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float4 xv[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m)
          xv[m] = m < M ? *reinterpret_cast<const float4 *>(xb + (size_t)m * KS + blk + 128 * q)
                        : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t word = q == 0 ? wv[r].x : q == 1 ? wv[r].y : q == 2 ? wv[r].z : wv[r].w;
          float wf[4];
          i8x4_to_f32(word, wf);
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
    __syncwarp();
    if (lane == 0 && i + kMv2Stages < T) {
      fence_proxy_async();
      issue(i + kMv2Stages);
    }
    if (c != nchunk - 1) continue;

    // ---- unit complete: reduce and finish ----
    float flat[V];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        flat[r * MT + m] = acc[r][m];
        acc[r][m] = 0.0f;
      }
    float sum = warp_reduce_scatter<V>(flat);
    const int row = rg * R + my_r;
    const bool valid = my_m < M && row < N;
    bool finish = true;
    if (S > 1) {
      if (writer && valid) p.partial[((size_t)slice * M + my_m) * N + row] = sum;
      __threadfence();
      __syncwarp();
      unsigned done = 0;
      if (lane == 0) done = atomicAdd(p.rg_counter + rg, 1u);
      done = __shfl_sync(0xffffffffu, done, 0);
      finish = done == (unsigned)S - 1;
      if (finish) {
        __threadfence();
        sum = 0.0f;
        if (valid)
          for (int s2 = 0; s2 < S; ++s2) sum = __fadd_rn(sum, __ldcg(p.partial + ((size_t)s2 * M + my_m) * N + row));
        if (lane == 0) p.rg_counter[rg] = 0u;
      }
    }
    if (!finish) continue;
    if constexpr (E == MvEpi::SwiGLU) {
      const float other = __shfl_xor_sync(0xffffffffu, sum, 32 / R);
      if (writer && valid && (my_r & 1) == 0) {
        const float g = __fmul_rn(sum, p.scales[row]);
        const float uu = __fmul_rn(other, p.scales[row + 1]);
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        p.y[(size_t)my_m * p.y_stride + row / 2] = __fmul_rn(silu, uu);
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

  if (failed) {
    // report, then let every copy this warp issued land before the CTA exits
    if (lane == 0) {
      sm.err = 1;
      if (p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
    }
    // items fail_item .. fail_item+kMv2Stages-1 (those < T) were issued and
    // not yet consumed: wait (bounded) for each of them
    for (long k = fail_item; k < T && k < fail_item + kMv2Stages; ++k)
      mbar_wait(&sm.bar[warp][k % kMv2Stages], (unsigned)((k / kMv2Stages) & 1));
  }

  if constexpr (E == MvEpi::Argmax) {
    int &last = sm.last;
    sm.best[threadIdx.x] = best;
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int t = 0; t < kMv2Warps * 32; ++t)
        if (reduce_index<V>(t & 31) % MT == (int)threadIdx.x && sm.best[t] > b) b = sm.best[t];
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

// ------------------------------------------------------------------- host --
static int mv2_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

size_t mv2_smem_bytes(int MT, int KS, int KC, int nsl) {
  return ((sizeof(Mv2Smem) + 127) & ~size_t(127)) + (size_t)kMv2Warps * kMv2Stages * kMv2R * KC +
         (size_t)nsl * MT * KS * sizeof(float);
}

// Pick the K split: the fewest slices (each a multiple of 512 columns,
// <= 1024 unless S = 1) giving about one unit per warp of the grid.
int mv2_pick_slices(int N, int K, int M, MvEpi e) {
  if (e == MvEpi::Argmax || K % 512) return 1;
  const long n_rg = (N + kMv2R - 1) / kMv2R;
  const long want = (long)mv2_sms() * kMv2Warps;
  int best = 1;
  for (int S = 1; S <= K / 512; ++S) {
    if (K % S || (K / S) % 512) continue;
    if (S > 1 && K / S > 1024) continue;
    best = S;
    if (n_rg * S >= want && (S > 1 || (size_t)M * K * 4 <= 96 * 1024)) break;
  }
  if (best == 1 && (size_t)8 * K * 4 > 96 * 1024) {
    for (int S = 2; S <= K / 512; ++S)
      if (K % S == 0 && (K / S) % 512 == 0 && K / S <= 1024) return S;
  }
  return best;
}

template <int MT, MvEpi E, bool NORM>
static int launch_t(const Mv2Params &p, cudaStream_t st, bool pdl) {
  const long n_rg = (p.N + kMv2R - 1) / kMv2R;
  const long U = n_rg * p.S;
  long G = std::min<long>(mv2_sms(), U);
  // each CTA must touch at most two K slices
  while (G > 1 && (U + G - 1) / G > n_rg) --G;
  const int nsl = p.S == 1 ? 1 : 2;
  const size_t smem = mv2_smem_bytes(MT, p.KS, p.KC, nsl);
  static bool attr_done = false;
  if (!attr_done) {
    int rc = cuda_status(cudaFuncSetAttribute(int8_mv2_kernel<MT, E, NORM>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                         "int8 matvec: shared memory opt-in");
    if (rc) return rc;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)G);
  cfg.blockDim = dim3(kMv2Warps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, int8_mv2_kernel<MT, E, NORM>, p), "int8 matvec launch");
}

template <MvEpi E, bool NORM>
static int launch_e(const Mv2Params &p, cudaStream_t st, bool pdl) {
  if (p.M <= 1) return launch_t<1, E, NORM>(p, st, pdl);
  if (p.M <= 2) return launch_t<2, E, NORM>(p, st, pdl);
  if (p.M <= 4) return launch_t<4, E, NORM>(p, st, pdl);
  return launch_t<8, E, NORM>(p, st, pdl);
}

int mv2_launch(const Mv2Params &p, MvEpi e, cudaStream_t st, bool pdl) {
  if (p.M < 1 || p.M > 8 || p.K % 512 || p.KS * p.S != p.K || (p.KC != 512 && p.KC != kMv2KCMax) || p.KS % p.KC ||
      (p.S > 1 && (!p.partial || !p.rg_counter)) || (p.norm_w && p.S != 1) ||
      (e == MvEpi::Argmax && (p.S != 1 || !p.keys || !p.counter || !p.ids)) ||
      mv2_smem_bytes(8, p.KS, p.KC, p.S == 1 ? 1 : 2) > 227 * 1024 || (reinterpret_cast<uintptr_t>(p.w) & 15) ||
      (reinterpret_cast<uintptr_t>(p.x) & 15) || (p.x_stride & 3)) {
    set_error("int8 matvec: unsupported configuration (M=%d K=%d N=%d S=%d)", p.M, p.K, p.N, p.S);
    return QASR_ERR_UNSUPPORTED;
  }
  const bool norm = p.norm_w != nullptr;
  switch (e) {
    case MvEpi::Store: return norm ? launch_e<MvEpi::Store, true>(p, st, pdl) : launch_e<MvEpi::Store, false>(p, st, pdl);
    case MvEpi::StoreBias: return launch_e<MvEpi::StoreBias, false>(p, st, pdl);
    case MvEpi::Residual: return launch_e<MvEpi::Residual, false>(p, st, pdl);
    case MvEpi::SwiGLU: return norm ? launch_e<MvEpi::SwiGLU, true>(p, st, pdl) : launch_e<MvEpi::SwiGLU, false>(p, st, pdl);
    case MvEpi::Argmax: return norm ? launch_e<MvEpi::Argmax, true>(p, st, pdl) : launch_e<MvEpi::Argmax, false>(p, st, pdl);
  }
  return QASR_ERR_INVALID;
}

}  // namespace qasr
