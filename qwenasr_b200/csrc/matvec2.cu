// matvec2.cu -- weight-streaming INT8 matvec for M <= 8 tokens (the decode
// projections and the lm head): y[m,o] = scales[o] * sum_k f32(w[o,k])*x[m,k]
// (generic::int8_matvec_fused, crates/qwen-asr/src/kernels/generic.rs:39-49).
//
// Design (HBM-bound: every weight byte is read exactly once per call):
//  * persistent grid, one 8-warp CTA per SM, sized (<= 128 registers, about
//    70 KB of shared memory) so that a CTA of the next kernel in the stream
//    fits beside it: under programmatic dependent launch the next kernel's
//    weight prefetch overlaps this kernel;
//  * the N x K weight matrix is cut into units of R rows x one K-slice (KS
//    columns), numbered slice-major and handed out to CTAs in contiguous
//    ranges, warps round-robin;
//  * each warp streams its units' rows through its own 4 KB shared-memory ring
//    with 1D bulk copies (cp.async.bulk, completion on an mbarrier);
//  * x (<= 2 K-slices of all M tokens) is staged once per CTA in a permuted
//    layout in which both the 16-byte weight reads and the 16-byte x reads of
//    a warp are bank-conflict free; an optional RMSNorm (the reference's
//    exact summation order, rowops.cuh) is applied while staging;
//  * per unit a lane holds R*M partial sums, reduced with one warp
//    reduce-scatter; split-K units (S > 1) park partials and the last unit of
//    a row group (atomic counter) sums slices 0..S-1 in order, so results are
//    deterministic;
//  * epilogues: store, +bias, residual add, SwiGLU of interleaved gate/up rows
//    (decoder.rs:916-921), first-max argmax (decoder.rs:942-947), and the
//    q/k per-head norm + RoPE + KV append of the fused QKV projection
//    (decoder.rs:888-895), run by the warp that completes a head;
//  * the weight prefetch is issued before griddepcontrol.wait.
// Every mbarrier wait is bounded (tma.cuh); a timeout sets *err and the kernel
// drains its copies and returns.
#include <atomic>

#include "common.cuh"
#include "matvec.cuh"
#include "qkvpost.cuh"
#include "rowops.cuh"
#include "tma.cuh"

namespace qasr {

constexpr int kMv2Warps = 8;
constexpr int kMv2R = 4;  // rows per unit (the engine tiles weights for it)
constexpr int kMv2KC = 512;          // bytes of one row per pipeline stage
constexpr int kMv2RingBytes = 8192;  // per-warp weight ring
constexpr int kMv2MaxStages = 8;
constexpr int kMv2MaxSlices = 12;  // largest split-K factor

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
  uint64_t bar[kMv2Warps][kMv2MaxStages];
  uint64_t nbar;  // norm weights copy
  uint64_t xbar;  // x staging copies (tiled layout)
  float inv[8];
  int last;
  unsigned long long best[kMv2Warps * 32];
};

// TILED: the weights are in the engine's tiled layout (mv2_tile_weights):
// every pipeline item is one contiguous bulk copy, and x is used in its
// natural layout (staged with one bulk copy per token row).  Otherwise the
// weights are the reference's row-major layout (one copy per row segment)
// and x is staged through registers into the permuted layout.
template <int MT, int R, MvEpi E, bool NORM, bool TILED>
__global__ void __launch_bounds__(kMv2Warps * 32, 2)
int8_mv2_kernel(const __grid_constant__ Mv2Params p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  Mv2Smem &sm = *reinterpret_cast<Mv2Smem *>(smem_raw);
  const int KC = p.KC;
  const int STAGES = kMv2RingBytes / (R * KC);
  int8_t *wbuf = reinterpret_cast<int8_t *>(smem_raw + ((sizeof(Mv2Smem) + 127) & ~size_t(127)));
  float *xs = reinterpret_cast<float *>(wbuf + (size_t)kMv2Warps * kMv2RingBytes);
  float *nws = xs + (size_t)(p.S == 1 ? 1 : 2) * MT * p.KS;  // NORM: norm weights [K]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int V = R * MT;
  const int M = p.M, K = p.K, N = p.N, S = p.S, KS = p.KS;
  const int n_rg = (N + R - 1) / R;
  const int U = n_rg * S;  // < 2^31 for every supported shape (checked on the host)
  const int u0 = (int)((long long)U * blockIdx.x / gridDim.x), u1 = (int)((long long)U * (blockIdx.x + 1) / gridDim.x);
  const int slice_lo = u0 / n_rg;
  const int nchunk = KS / KC;
  const int my_units = u1 - u0 > warp ? (u1 - u0 - warp + kMv2Warps - 1) / kMv2Warps : 0;
  const int T = my_units * nchunk;  // pipeline items of this warp

  if (threadIdx.x < kMv2Warps * STAGES) mbar_init(&sm.bar[threadIdx.x / STAGES][threadIdx.x % STAGES], 1);
  if (threadIdx.x == kMv2Warps * STAGES) mbar_init(&sm.nbar, 1);
  if (threadIdx.x == kMv2Warps * STAGES + 1) mbar_init(&sm.xbar, 1);
  mbar_fence_init();
  __syncthreads();
  if constexpr (NORM) {  // constant operand: fetch it before waiting for the previous kernel
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&sm.nbar, (unsigned)K * 4);
      bulk_g2s(nws, p.norm_w, (unsigned)K * 4, &sm.nbar);
    }
  }

  int8_t *mybuf = wbuf + (size_t)warp * kMv2RingBytes;
  // producer cursor (lane 0): unit (slice, row group) and chunk of the next item
  int pc = 0, pslice = (u0 + warp) / n_rg, prg = (u0 + warp) % n_rg;
  auto issue = [&](int i) {  // lane 0 only, called for i = 0, 1, 2, ... in order
    const int c = pc, slice = pslice, rg = prg;
    if (++pc == nchunk) {  // next unit of this warp: u += kMv2Warps
      pc = 0;
      prg += kMv2Warps;
      while (prg >= n_rg) {
        prg -= n_rg;
        ++pslice;
      }
    }
    const int st = i % STAGES;
    mbar_arrive_expect_tx(&sm.bar[warp][st], R * KC);
    if constexpr (TILED) {
      bulk_g2s(mybuf + (size_t)st * R * KC, p.w + (((size_t)slice * n_rg + rg) * nchunk + c) * R * KC, R * KC,
               &sm.bar[warp][st]);
    } else {
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = min(rg * R + r, N - 1);
        bulk_g2s(mybuf + ((size_t)st * R + r) * KC, p.w + (size_t)row * K + (size_t)slice * KS + (size_t)c * KC, KC,
                 &sm.bar[warp][st]);
      }
    }
  };
  if (lane == 0)
    for (int i = 0; i < T && i < STAGES; ++i) issue(i);

  // activations come from the previous kernel: wait for it only now
  pdl_wait();
  pdl_launch_dependents();

  // ---- stage x (slices slice_lo, slice_lo+1) in the permuted layout ----
  const int nsl = (u1 > u0) ? (int)((u1 - 1) / n_rg) - slice_lo + 1 : 0;
  if constexpr (TILED) {  // natural layout: one bulk copy per (slice, token) row
    if (threadIdx.x == 0 && nsl > 0) {
      mbar_arrive_expect_tx(&sm.xbar, (unsigned)(nsl * M * KS * 4));
      for (int sl = 0; sl < nsl; ++sl)
        for (int m = 0; m < M; ++m)
          bulk_g2s(xs + ((size_t)sl * MT + m) * KS, p.x + (size_t)m * p.x_stride + (size_t)(slice_lo + sl) * KS,
                   (unsigned)KS * 4, &sm.xbar);
    }
    if (nsl > 0 && !mbar_wait(&sm.xbar, 0) && p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
  }
  for (int sl = 0; sl < (TILED ? 0 : nsl); ++sl) {
    // per token: KS/4 float4s, four independent 16-byte loads in flight per thread
    for (int m = 0; m < M; ++m) {
      const float *src = p.x + (size_t)m * p.x_stride + (size_t)(slice_lo + sl) * KS;
      float *dst = xs + ((size_t)sl * MT + m) * KS;
      for (int k0 = 4 * threadIdx.x; k0 < KS; k0 += 16 * blockDim.x) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int k = k0 + 4 * u * blockDim.x;
          if (k < KS) v[u] = *reinterpret_cast<const float4 *>(src + k);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int k = k0 + 4 * u * blockDim.x;
          if (k < KS) *reinterpret_cast<float4 *>(dst + xperm(k)) = v[u];
        }
      }
    }
  }
  if constexpr (NORM) {  // S == 1: the slice is the whole row
    __syncthreads();
    if (warp < M) {
      const float *xr = xs + (size_t)warp * KS;
      const int n = K, n16 = n / 16;
      float acc = 0.0f;
      if (lane < 16) {
        // the chain must run in order; its operands are fetched 16 at a time
        // ahead of it so only the FMA latency is serial
        int j = 0;
        for (; j + 16 <= n16; j += 16) {
          float v[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) v[t] = xr[TILED ? 16 * (j + t) + lane : xperm(16 * (j + t) + lane)];
#pragma unroll
          for (int t = 0; t < 16; ++t) acc = fmaf(v[t], v[t], acc);
        }
        for (; j < n16; ++j) {
          const float v = xr[TILED ? 16 * j + lane : xperm(16 * j + lane)];
          acc = fmaf(v, v, acc);
        }
        if ((n & 15) >= 8 && lane < 8) {
          const float v = xr[TILED ? 16 * n16 + lane : xperm(16 * n16 + lane)];
          acc = fmaf(v, v, acc);
        }
      }
      float sum = hsum16_avx_order(acc);
      if (lane == 0)
        for (int i = avx_vector_extent(n); i < n; ++i) {
          const float v = xr[TILED ? i : xperm(i)];
          sum = __fadd_rn(sum, __fmul_rn(v, v));
        }
      if (lane == 0) sm.inv[warp] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)n), p.eps)));
    }
    if (!mbar_wait(&sm.nbar, 0) && threadIdx.x == 0 && p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
    __syncthreads();
    for (int slot = 4 * threadIdx.x; slot < KS; slot += 4 * blockDim.x) {
      const int k = TILED ? slot : xperm_inv(slot);
      const float4 wn = *reinterpret_cast<const float4 *>(nws + k);
      for (int m = 0; m < M; ++m) {
        float4 *v4 = reinterpret_cast<float4 *>(xs + (size_t)m * KS + slot);
        const float inv = sm.inv[m];
        float4 v = *v4;
        v.x = __fmul_rn(__fmul_rn(v.x, inv), wn.x);
        v.y = __fmul_rn(__fmul_rn(v.y, inv), wn.y);
        v.z = __fmul_rn(__fmul_rn(v.z, inv), wn.z);
        v.w = __fmul_rn(__fmul_rn(v.w, inv), wn.w);
        *v4 = v;
      }
    }
  }
  // rows m >= M of the staged x are never read (token loops stop at M)
  __syncthreads();

  const int my_idx = reduce_index<V>(lane);
  const int my_r = my_idx / MT, my_m = my_idx % MT;
  const bool writer = (lane & ((32 / V) - 1)) == 0;
  unsigned long long best = 0ull;
  bool failed = false;
  int fail_item = -1;
  int cc = 0, cslice = (u0 + warp) / n_rg, crg = (u0 + warp) % n_rg;  // consumer cursor

  float acc[R][MT];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[r][m] = 0.0f;

  for (int i = 0; i < T; ++i) {
    const int st = i % STAGES;
    if (!mbar_wait(&sm.bar[warp][st], (unsigned)((i / STAGES) & 1))) {
      failed = true;
      fail_item = i;
      break;
    }
    const int c = cc, slice = cslice, rg = crg;
    if (++cc == nchunk) {
      cc = 0;
      crg += kMv2Warps;
      while (crg >= n_rg) {
        crg -= n_rg;
        ++cslice;
      }
    }
    const int8_t *wb = mybuf + (size_t)st * R * KC;
    // epilogue operands of this lane's (row, token), loaded now so their
    // latency hides under the unit's arithmetic
    const int pre_row = min(rg * R + my_r, N - 1);
    const float pre_scale = p.scales[pre_row];
    float pre_aux = 0.0f;
    if constexpr (E == MvEpi::SwiGLU) pre_aux = p.scales[min(pre_row + 1, N - 1)];
    if constexpr (E == MvEpi::StoreBias) pre_aux = p.bias[pre_row];
    if constexpr (E == MvEpi::Residual)
      if (S == 1 && my_m < M) pre_aux = p.y[(size_t)my_m * p.y_stride + pre_row];
    const float *xb = xs + (size_t)(slice - slice_lo) * MT * KS + (size_t)c * KC + 4 * lane;
#pragma unroll 1
    for (int blk = 0; blk < KC; blk += 512) {  // 512-byte blocks of the chunk
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
    if (lane == 0 && i + STAGES < T) {
      fence_proxy_async();
      issue(i + STAGES);
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
        if (valid) {
          // all slice partials in flight at once, summed in slice order
          float part[kMv2MaxSlices];
#pragma unroll
          for (int s2 = 0; s2 < kMv2MaxSlices; ++s2)
            part[s2] = s2 < S ? __ldcg(p.partial + ((size_t)s2 * M + my_m) * N + row) : 0.0f;
#pragma unroll
          for (int s2 = 0; s2 < kMv2MaxSlices; ++s2)
            if (s2 < S) sum = __fadd_rn(sum, part[s2]);
        }
        if (lane == 0) p.rg_counter[rg] = 0u;
      }
    }
    if (!finish) continue;
    if constexpr (E == MvEpi::SwiGLU) {
      const float other = __shfl_xor_sync(0xffffffffu, sum, 32 / R);
      if (writer && valid && (my_r & 1) == 0) {
        const float g = __fmul_rn(sum, pre_scale);
        const float uu = __fmul_rn(other, pre_aux);
        const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        p.y[(size_t)my_m * p.y_stride + row / 2] = __fmul_rn(silu, uu);
      }
    } else if constexpr (E == MvEpi::Argmax) {
      if (valid) {
        const float logit = __fmul_rn(sum, pre_scale);
        if (writer && p.y) p.y[(size_t)my_m * p.y_stride + row] = logit;
        const unsigned long long key = argmax_key(logit, (uint32_t)row);
        best = key > best ? key : best;
      }
    } else {
      if (writer && valid) {
        float v = __fmul_rn(sum, pre_scale);
        if constexpr (E == MvEpi::StoreBias) v = __fadd_rn(v, pre_aux);
        float *dst = p.y + (size_t)my_m * p.y_stride + row;
        if constexpr (E == MvEpi::Residual) v = __fadd_rn(S == 1 ? pre_aux : *dst, v);
        *dst = v;
      }
      if constexpr (E == MvEpi::QkvPost) {
        // the warp completing the last rows of a head finishes the head
        const int head = (rg * R) / 128;
        __threadfence();
        __syncwarp();
        unsigned done = 0;
        if (lane == 0) done = atomicAdd(p.post.head_ctr + head, 1u);
        done = __shfl_sync(0xffffffffu, done, 0);
        if (done == 128 / R - 1) {
          __threadfence();
          float4 hv[MT];  // every token's head row in flight at once
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < M) hv[m] = __ldcg(reinterpret_cast<const float4 *>(p.y + (size_t)m * p.y_stride + head * 128) + lane);
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < M) qkv_head_post(p.post, p.eps, head, m, hv[m], p.err);
          if (lane == 0) p.post.head_ctr[head] = 0u;
        }
      }
    }
  }

  if (failed) {
    // report, then let every copy this warp issued land before the CTA exits
    if (lane == 0 && p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
    for (int k = fail_item; k < T && k < fail_item + STAGES; ++k)
      mbar_wait(&sm.bar[warp][k % STAGES], (unsigned)((k / STAGES) & 1));
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
      // a bounded wait that gave up anywhere in the grid leaves the keys
      // incomplete: report -1 (no token has that id) rather than a plausible id
      const bool timed_out = p.err && *reinterpret_cast<volatile int *>(p.err) != 0;
      p.ids[threadIdx.x] = timed_out ? -1 : (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    }
    if (last && threadIdx.x == 0) atomicExch(p.counter, 0u);
  }
}

// ------------------------------------------------------------ weight tiling --
__global__ void tile_weights_kernel(int8_t *__restrict__ dst, const int8_t *__restrict__ src, int N, int K, int KS,
                                    int KC) {
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;  // one 4-byte group
  if (t >= (long)N * K / 4) return;
  const int row = (int)(t / (K / 4)), k = (int)(t % (K / 4)) * 4;
  const uint32_t v = *reinterpret_cast<const uint32_t *>(src + (size_t)row * K + k);
  *reinterpret_cast<uint32_t *>(dst + mv2_tiled_offset(row, k, KS, KC, N / 4)) = v;
}

int mv2_tile_weights(int8_t *dst, const int8_t *src, int N, int K, int S, cudaStream_t st) {
  if (N % kMv2R || K % 512 || K % S || (K / S) % 512 || !dst || !src || dst == src) {
    set_error("mv2_tile_weights: unsupported shape N=%d K=%d S=%d", N, K, S);
    return QASR_ERR_INVALID;
  }
  const int KS = K / S, KC = mv2_chunk(KS);
  const long n = (long)N * K / 4;
  tile_weights_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(dst, src, N, K, KS, KC);
  return launch_status("mv2_tile_weights");
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

static size_t mv2_smem_bytes(int MT, int KS, int nsl, int K) {
  (void)0;
  return ((sizeof(Mv2Smem) + 127) & ~size_t(127)) + (size_t)kMv2Warps * kMv2RingBytes +
         (size_t)nsl * MT * KS * sizeof(float) + (size_t)K * sizeof(float);
}

// Pick the K split: the fewest slices (each a multiple of 512 columns,
// <= 1024 unless S = 1) giving about one unit per warp of the grid.
int mv2_pick_slices(int N, int K, int M, MvEpi e) {
  if (e == MvEpi::Argmax || e == MvEpi::QkvPost || K % 512) return 1;
  const long n_rg = (N + mv2_rows(M) - 1) / mv2_rows(M);
  const long want = (long)mv2_sms() * kMv2Warps;
  int best = 1;
  for (int S = 1; S <= K / 512 && S <= kMv2MaxSlices; ++S) {
    if (K % S || (K / S) % 512) continue;
    if (S > 1 && K / S > 1024) continue;
    best = S;
    if (n_rg * S >= want && (S > 1 || (size_t)8 * K * 4 <= 48 * 1024)) break;
  }
  if (best == 1 && (size_t)8 * K * 4 > 48 * 1024) {
    for (int S = 2; S <= K / 512; ++S)
      if (K % S == 0 && (K / S) % 512 == 0 && K / S <= 1024) return S;
  }
  return best;
}

template <int MT, int R, MvEpi E, bool NORM, bool TILED>
static int launch_t(const Mv2Params &p, cudaStream_t st, bool pdl) {
  const long n_rg = (p.N + R - 1) / R;
  const long U = n_rg * p.S;
  long G = std::min<long>(mv2_sms(), U);
  // each CTA must touch at most two K slices
  while (G > 1 && (U + G - 1) / G > n_rg) --G;
  const int nsl = p.S == 1 ? 1 : 2;
  const size_t smem = mv2_smem_bytes(MT, p.KS, nsl, NORM ? p.K : 0);
  // The shared-memory opt-in is a per-device property of the function: track
  // it per device (bit `dev` of a mask), so a call on a second device of the
  // same process opts in there too; concurrent first calls both set it.
  static std::atomic<unsigned long long> attr_done{0ull};
  int dev = 0;
  if (int rc = cuda_status(cudaGetDevice(&dev), "int8 matvec: cudaGetDevice")) return rc;
  const unsigned long long bit = dev >= 0 && dev < 64 ? 1ull << dev : 0ull;
  if (!bit || !(attr_done.load(std::memory_order_acquire) & bit)) {
    int rc = cuda_status(cudaFuncSetAttribute(int8_mv2_kernel<MT, R, E, NORM, TILED>,
                                              cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024),
                         "int8 matvec: shared memory opt-in");
    if (rc) return rc;
    attr_done.fetch_or(bit, std::memory_order_release);
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
  return cuda_status(cudaLaunchKernelEx(&cfg, int8_mv2_kernel<MT, R, E, NORM, TILED>, p), "int8 matvec launch");
}

template <MvEpi E, bool NORM, bool TILED>
static int launch_m(const Mv2Params &p, cudaStream_t st, bool pdl) {
  if (p.M <= 1) return launch_t<1, 4, E, NORM, TILED>(p, st, pdl);
  if (p.M <= 2) return launch_t<2, 4, E, NORM, TILED>(p, st, pdl);
  if (p.M <= 4) return launch_t<4, 4, E, NORM, TILED>(p, st, pdl);
  return launch_t<8, 4, E, NORM, TILED>(p, st, pdl);
}
template <MvEpi E, bool NORM>
static int launch_e(const Mv2Params &p, cudaStream_t st, bool pdl) {
  return p.tiled ? launch_m<E, NORM, true>(p, st, pdl) : launch_m<E, NORM, false>(p, st, pdl);
}

int mv2_launch(const Mv2Params &p, MvEpi e, cudaStream_t st, bool pdl) {
  if (p.M < 1 || p.M > 8 || p.K % 512 || p.KS * p.S != p.K || (p.KC != 512 && p.KC != 1024) || p.KS % p.KC ||
      (!p.tiled && p.KC != kMv2KC) || (p.tiled && p.N % kMv2R) ||
      (p.S > 1 && (!p.partial || !p.rg_counter)) || (p.norm_w && p.S != 1) ||
      (e == MvEpi::Argmax && (p.S != 1 || !p.keys || !p.counter || !p.ids)) ||
      (e == MvEpi::QkvPost && (p.S != 1 || !p.post.head_ctr || !p.post.positions)) ||
      mv2_smem_bytes(8, p.KS, p.S == 1 ? 1 : 2, p.K) > 227 * 1024 || (reinterpret_cast<uintptr_t>(p.w) & 15) ||
      (p.norm_w && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)) || p.S > kMv2MaxSlices ||
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
    case MvEpi::QkvPost: return norm ? launch_e<MvEpi::QkvPost, true>(p, st, pdl) : launch_e<MvEpi::QkvPost, false>(p, st, pdl);
  }
  return QASR_ERR_INVALID;
}

}  // namespace qasr
