// umma_matvec.cu -- INT8-weight contraction for up to 8 token rows on the
// 5th-generation tensor cores (tcgen05, kind::i8): the decode projections
// and the lm head (generic::int8_matvec_fused,
// crates/qwen-asr/src/kernels/generic.rs:39-49, applied per token as
// decoder_forward_int8 does, crates/qwen-asr/src/decoder.rs:870-964).
//
// Exact integer formulation.  Each activation row x[m] is scaled by a power
// of two 2^(22-E_m), where 2^E_m bounds max|x[m]|, and rounded to an integer
// X (|X| <= 2^22); X is split into three signed bytes, X = 65536*d0 + 256*d1
// + d2.  The tensor cores contract the int8 weights with the 24 digit rows
// (3 digits x 8 tokens, padded to N = 32) exactly in 32-bit integers, the
// three digit sums are recombined exactly in 64 bits, and only the final
// value is rounded: y = f32(V) * 2^(E_m-22) * scales[o].  The only
// approximation is rounding x to 23 significant bits relative to its row
// maximum, far below the f32 summation error of the reference's own path.
//
// Design (HBM-bound: every weight byte is read once per call):
//  * the N x K matrix is cut into 128-row x 128-byte tiles ("units"),
//    numbered row-tile-major; each CTA of a persistent grid takes an equal
//    contiguous range of units, so every SM streams the same bytes;
//  * one thread streams the CTA's weight tiles with 2D TMA loads
//    (SWIZZLE_128B, no multicast) into a ring of 16 KB stages, issuing the
//    first stages before griddepcontrol.wait (weights do not depend on the
//    previous kernel);
//  * all warps stage x: RMSNorm in the reference's summation order (NORM),
//    the per-row exponent, and the digit rows of the K tiles this CTA uses,
//    written in the canonical 128-byte-swizzled K-major layout;
//  * one thread issues tcgen05.mma (M=128, N=32, K=32) into a double-buffered
//    TMEM accumulator and frees each ring stage with tcgen05.commit;
//  * four epilogue warps read the accumulator with tcgen05.ld (thread = output
//    row), recombine the digits and apply the epilogue; a row tile shared
//    between CTAs is summed with 64-bit integer atomics (exact, so the result
//    does not depend on arrival order) and finished by the last contributor.
// Every wait is bounded (tma.cuh); a timeout sets *err, stops the roles,
// drains the copies and MMAs in flight and frees TMEM before returning.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "matvec.cuh"
#include "qkvpost.cuh"
#include "rowops.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kUWarps = 8;
constexpr int kUMaxStages = 6;
constexpr int kUTile = 128 * 128;        // bytes of one weight tile
constexpr int kUBSlot = 32 * 128;        // bytes of the digit rows of one K tile
constexpr int kUTmemCols = 64;           // two 32-column accumulators
constexpr int kUEpiThreads = 128;        // warps 0..3
constexpr int kUProducerWarp = 4, kUMmaWarp = 5;
constexpr uint32_t kUIdesc = umma_idesc_s8(128, 32);

struct alignas(16) USmem {
  uint64_t full[kUMaxStages], empty[kUMaxStages];
  uint64_t accfull[2], accempty[2];
  uint64_t xbar, nbar, done;
  uint32_t tmem;
  int abort;
  int fin;
  int last;
  float inv[8], qmul[8], dq[8];
  unsigned long long best[4][8];
  alignas(16) float hs[8][128];  // QkvPost: one head of every token (read as float4)
};

QASR_DEV bool u_aborted(const USmem &sm) { return *reinterpret_cast<const volatile int *>(&sm.abort) != 0; }

QASR_DEV void u_fail(USmem &sm, int *err) {
  atomicExch(&sm.abort, 1);
  if (err) atomicExch(err, -QASR_ERR_TIMEOUT);
}

QASR_DEV float pow2f(int e) {  // 2^e for -126 <= e <= 127
  return __int_as_float((127 + e) << 23);
}

template <MvEpi E, bool NORM>
__global__ void __launch_bounds__(kUWarps * 32, 1) int8_umma_kernel(const __grid_constant__ UmmaParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int STAGES = p.stages, NB = p.nb;
  unsigned char *a_ring = base;
  unsigned char *b_tiles = a_ring + (size_t)STAGES * kUTile;
  float *xs = reinterpret_cast<float *>(b_tiles + (size_t)NB * kUBSlot);  // NORM: [M, K]
  float *nws = xs + (NORM ? (size_t)p.M * p.K : 0);                         // NORM: [K]
  USmem &sm = *reinterpret_cast<USmem *>(nws + (NORM ? p.K : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = p.M, K = p.K, N = p.N;
  const int KT = K / 128, NT = (N + 127) / 128;
  const long long U = (long long)NT * KT;
  const int u0 = (int)(U * blockIdx.x / gridDim.x), u1 = (int)(U * (blockIdx.x + 1) / gridDim.x);
  const int nu = u1 - u0;
  const int kt_base = u0 % KT;
  auto slot_of = [&](int kt) { return nu >= KT ? kt : (kt - kt_base + KT) % KT; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUMaxStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.accfull[b], 1);
      mbar_init(&sm.accempty[b], 4);
    }
    mbar_init(&sm.xbar, 1);
    mbar_init(&sm.nbar, 1);
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == kUMmaWarp) tmem_alloc(&sm.tmem, kUTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;

  // ---- weight prefetch: constant operand, issued before waiting on the previous kernel
  int produced = 0;  // producer thread only
  auto produce = [&](int i) {
    const int u = u0 + i, st = i % STAGES;
    mbar_arrive_expect_tx(&sm.full[st], kUTile);
    tma_load_2d_u8(a_ring + (size_t)st * kUTile, &p.tmap, (u % KT) * 128, (u / KT) * 128, &sm.full[st]);
  };
  const bool producer = warp == kUProducerWarp && lane == 0;
  if (producer) {
    for (; produced < nu && produced < STAGES; ++produced) produce(produced);
  }
  if constexpr (NORM) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&sm.nbar, (unsigned)K * 4);
      bulk_g2s(nws, p.norm_w, (unsigned)K * 4, &sm.nbar);
    }
  }

  pdl_wait();
  pdl_launch_dependents();

  // ---- stage x: per-row exponent (and RMSNorm), then the digit rows
  if constexpr (NORM) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&sm.xbar, (unsigned)(M * K * 4));
      for (int m = 0; m < M; ++m) bulk_g2s(xs + (size_t)m * K, p.x + (size_t)m * p.x_stride, (unsigned)K * 4, &sm.xbar);
    }
  }
  if (warp < M) {
    const int m = warp;
    float bound;
    if constexpr (NORM) {
      bool ok = mbar_wait(&sm.xbar, 0);
      ok = mbar_wait(&sm.nbar, 0) && ok;
      if (!ok && lane == 0) u_fail(sm, p.err);
      const float *xr = xs + (size_t)m * K;
      // sum of squares in the reference's order (rowops.cuh): lanes 0..15 run
      // the sequential chains, operands fetched 16 at a time ahead of them
      const int n16 = K / 16;
      float acc = 0.0f;
      if (lane < 16) {
        int j = 0;
        for (; j + 16 <= n16; j += 16) {
          float v[16];
#pragma unroll
          for (int t = 0; t < 16; ++t) v[t] = xr[16 * (j + t) + lane];
#pragma unroll
          for (int t = 0; t < 16; ++t) acc = fmaf(v[t], v[t], acc);
        }
        for (; j < n16; ++j) {
          const float v = xr[16 * j + lane];
          acc = fmaf(v, v, acc);
        }
      }
      const float sum = hsum16_avx_order(acc);  // K % 128 == 0: no 8-block, no scalar tail
      const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), p.eps)));
      float mx = 0.0f, mw = 0.0f;
      for (int k = lane; k < K; k += 32) {
        mx = fmaxf(mx, fabsf(xr[k]));
        mw = fmaxf(mw, fabsf(nws[k]));
      }
      mx = warp_max(mx);
      mw = warp_max(mw);
      // rounding is monotonic, so this bounds every |rn(rn(x*inv)*w)|
      bound = __fmul_rn(__fmul_rn(mx, inv), mw);
      if (lane == 0) sm.inv[m] = inv;
    } else {
      const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.x_stride);
      float mx = 0.0f;
      for (int k4 = lane; k4 < K / 4; k4 += 32) {
        const float4 v = xr[k4];
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
      bound = warp_max(mx);
    }
    if (lane == 0) {
      int e = 0;
      if (bound > 0.0f && bound <= 3.0e38f) frexpf(bound, &e);  // bound < 2^e
      e = max(-100, min(e, 127));
      sm.qmul[m] = pow2f(22 - e);
      sm.dq[m] = pow2f(e - 22);
    }
  }
  __syncthreads();
  {
    const int nbu = min(KT, nu);
    // items: (slot, token row m in 0..7, 16-byte chunk c) -> digit rows m, 8+m, 16+m;
    // then the zero rows 24..31
    const int n_tok = nbu * 8 * 8;
    for (int it = threadIdx.x; it < 2 * n_tok; it += blockDim.x) {
      const int item = it < n_tok ? it : it - n_tok;
      const int slot = item >> 6, m = (item >> 3) & 7, c = item & 7;
      unsigned char *tile = b_tiles + (size_t)slot * kUBSlot;
      if (it >= n_tok) {  // padding row 24 + m
        const int n = 24 + m;
        *reinterpret_cast<uint4 *>(tile + (n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4)) =
            make_uint4(0u, 0u, 0u, 0u);
        continue;
      }
      uint32_t dg[3][4] = {{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
      if (m < M) {
        const int kt = nu >= KT ? slot : (kt_base + slot) % KT;
        const int k0 = kt * 128 + c * 16;
        const float qm = sm.qmul[m];
        float v[16];
        if constexpr (NORM) {
          const float inv = sm.inv[m];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = __fmul_rn(__fmul_rn(xs[(size_t)m * K + k0 + j], inv), nws[k0 + j]);
        } else {
          const float4 *src = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.x_stride + k0);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 t = src[j];
            v[4 * j] = t.x;
            v[4 * j + 1] = t.y;
            v[4 * j + 2] = t.z;
            v[4 * j + 3] = t.w;
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int X = __float2int_rn(__fmul_rn(v[j], qm));
          const int d2 = ((X + 128) & 255) - 128;
          const int t1 = (X - d2) >> 8;
          const int d1 = ((t1 + 128) & 255) - 128;
          const int d0 = (t1 - d1) >> 8;
          dg[0][j >> 2] |= (uint32_t)(d0 & 255) << (8 * (j & 3));
          dg[1][j >> 2] |= (uint32_t)(d1 & 255) << (8 * (j & 3));
          dg[2][j >> 2] |= (uint32_t)(d2 & 255) << (8 * (j & 3));
        }
      }
#pragma unroll
      for (int d = 0; d < 3; ++d) {
        const int n = 8 * d + m;
        *reinterpret_cast<uint4 *>(tile + (n >> 3) * 1024 + (n & 7) * 128 + ((c ^ (n & 7)) << 4)) =
            make_uint4(dg[d][0], dg[d][1], dg[d][2], dg[d][3]);
      }
    }
  }
  fence_proxy_async();  // digit rows written by threads -> visible to the tensor cores
  __syncthreads();

  unsigned long long best[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) best[m] = 0ull;

  if (producer) {
    // ---- TMA producer: refill each stage once the MMAs reading it completed
    for (; produced < nu; ++produced) {
      if (u_aborted(sm)) break;
      const int st = produced % STAGES;
      if (!mbar_wait(&sm.empty[st], (unsigned)((produced / STAGES - 1) & 1))) {
        u_fail(sm, p.err);
        break;
      }
      produce(produced);
    }
  } else if (warp == kUMmaWarp) {
    // ---- MMA issuer (one thread)
    if (lane == 0) {
      int pc = 0;
      bool first = true;
      for (int i = 0; i < nu; ++i) {
        const int u = u0 + i, kt = u % KT, st = i % STAGES, buf = pc & 1;
        if (first && pc >= 2 && !mbar_wait(&sm.accempty[buf], (unsigned)(((pc >> 1) - 1) & 1))) {
          u_fail(sm, p.err);
          break;
        }
        if (!mbar_wait(&sm.full[st], (unsigned)((i / STAGES) & 1))) {
          u_fail(sm, p.err);
          break;
        }
        if (u_aborted(sm)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_ring + (size_t)st * kUTile);
        const uint32_t b_addr = smem_u32(b_tiles + (size_t)slot_of(kt) * kUBSlot);
        const uint32_t d_addr = tmem + (uint32_t)(buf * 32);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_s8(d_addr, umma_desc_sw128(a_addr + 32 * s), umma_desc_sw128(b_addr + 32 * s), kUIdesc,
                  (first && s == 0) ? 0u : 1u);
        umma_commit(&sm.empty[st]);
        first = false;
        if (i == nu - 1 || kt == KT - 1) {  // piece (row tile within this CTA) complete
          umma_commit(&sm.accfull[buf]);
          ++pc;
          first = true;
        }
      }
      // every MMA issued so far has completed once `done` flips
      umma_commit(&sm.done);
      if (!mbar_wait(&sm.done, 0)) u_fail(sm, p.err);
    }
  } else if (warp < 4) {
    // ---- epilogue: thread = output row of the tile
    const int r_in_tile = warp * 32 + lane;
    int pc = 0;
    for (int i = 0; i < nu;) {
      const int u = u0 + i, t = u / KT, ka = u % KT;
      const int kb = min(KT, ka + (nu - i));  // this piece covers K tiles ka .. kb-1
      i += kb - ka;
      const int buf = pc & 1;
      if (!u_aborted(sm) && !mbar_wait(&sm.accfull[buf], (unsigned)((pc >> 1) & 1))) u_fail(sm, p.err);
      ++pc;
      named_bar(1, kUEpiThreads);  // the four epilogue warps decide together
      if (u_aborted(sm)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * 32), r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.accempty[buf])) : "memory");

      const int row = t * 128 + r_in_tile;
      const bool valid = row < N;
      long long V[8];
#pragma unroll
      for (int m = 0; m < 8; ++m)
        V[m] = ((long long)(int)r[m] << 16) + ((long long)(int)r[8 + m] << 8) + (long long)(int)r[16 + m];
      if (kb - ka != KT) {
        // row tile shared with other CTAs: exact 64-bit integer sum, last contributor finishes
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (valid && m < M) atomicAdd(p.acc + (size_t)row * 8 + m, (unsigned long long)V[m]);
        __threadfence();
        named_bar(1, kUEpiThreads);
        if (threadIdx.x == 0) {
          const unsigned old = atomicAdd(p.tile_ctr + t, (unsigned)(kb - ka));
          sm.fin = old + (unsigned)(kb - ka) == (unsigned)KT;
        }
        named_bar(1, kUEpiThreads);
        if (!sm.fin) continue;
        __threadfence();
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (valid && m < M) V[m] = (long long)atomicExch(p.acc + (size_t)row * 8 + m, 0ull);
        if (threadIdx.x == 0) atomicExch(p.tile_ctr + t, 0u);
      }
      const float sc = valid ? p.scales[row] : 0.0f;
      float yv[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) yv[m] = m < M ? __fmul_rn(__fmul_rn(__ll2float_rn(V[m]), sm.dq[m]), sc) : 0.0f;

      if constexpr (E == MvEpi::Store || E == MvEpi::StoreBias) {
        const float b = (E == MvEpi::StoreBias && valid) ? p.bias[row] : 0.0f;
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (valid && m < M) p.y[(size_t)m * p.y_stride + row] = E == MvEpi::StoreBias ? __fadd_rn(yv[m], b) : yv[m];
      } else if constexpr (E == MvEpi::Residual) {
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (valid && m < M) {
            float *dst = p.y + (size_t)m * p.y_stride + row;
            *dst = __fadd_rn(*dst, yv[m]);
          }
      } else if constexpr (E == MvEpi::SwiGLU) {
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          const float up = __shfl_xor_sync(0xffffffffu, yv[m], 1);
          if (m < M && valid && (row & 1) == 0) {
            const float g = yv[m];
            const float silu = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            p.y[(size_t)m * p.y_stride + row / 2] = __fmul_rn(silu, up);
          }
        }
      } else if constexpr (E == MvEpi::Argmax) {
#pragma unroll
        for (int m = 0; m < 8; ++m)
          if (valid && m < M) {
            if (p.y) p.y[(size_t)m * p.y_stride + row] = yv[m];
            const unsigned long long key = argmax_key(yv[m], (uint32_t)row);
            best[m] = key > best[m] ? key : best[m];
          }
      } else if constexpr (E == MvEpi::QkvPost) {
        // the tile is one 128-wide head: finish it here
#pragma unroll
        for (int m = 0; m < 8; ++m) sm.hs[m][r_in_tile] = yv[m];
        named_bar(2, kUEpiThreads);
        for (int m = warp; m < M; m += 4) {
          const float4 hv = reinterpret_cast<const float4 *>(sm.hs[m])[lane];
          qkv_head_post(p.post, p.eps, t, m, hv, p.err);
        }
        named_bar(2, kUEpiThreads);
      }
    }
  }
  __syncthreads();

  if constexpr (E == MvEpi::Argmax) {
    if (warp < 4) {
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        unsigned long long b = best[m];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const unsigned long long q = __shfl_xor_sync(0xffffffffu, b, o);
          b = q > b ? q : b;
        }
        if (lane == 0) sm.best[warp][m] = b;
      }
    }
    __syncthreads();
    if (threadIdx.x < M) {
      unsigned long long b = 0ull;
      for (int w = 0; w < 4; ++w) b = sm.best[w][threadIdx.x] > b ? sm.best[w][threadIdx.x] : b;
      if (b) atomicMax(p.keys + threadIdx.x, b);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) sm.last = atomicAdd(p.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (sm.last && threadIdx.x < M) {
      __threadfence();
      const unsigned long long k = atomicExch(p.keys + threadIdx.x, 0ull);
      p.ids[threadIdx.x] = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
    }
    if (sm.last && threadIdx.x == 0) atomicExch(p.counter, 0u);
  }

  // ---- teardown: copies in flight land, then TMEM is released
  if (producer) {
    for (int i = max(0, produced - STAGES); i < produced; ++i)
      mbar_wait(&sm.full[i % STAGES], (unsigned)((i / STAGES) & 1));
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kUMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kUTmemCols);
  }
}

// ------------------------------------------------------------------- host --
void *tensor_map_encoder() {
  static void *fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void *f = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = f;
  }
  return fn;
}

int umma_weight_map(CUtensorMap *tm, const int8_t *w, int N, int K) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  auto encode = reinterpret_cast<Encode>(tensor_map_encoder());
  if (!encode) {
    set_error("int8 tensor-core matvec: cuTensorMapEncodeTiled unavailable");
    return QASR_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(w) & 15) || K % 128 || N <= 0) {
    set_error("int8 tensor-core matvec: weights must be 16-byte aligned with K a multiple of 128");
    return QASR_ERR_UNSUPPORTED;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)N};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128, 128};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(w), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("int8 tensor-core matvec: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

static int umma_sms() {
  static int sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!sms[dev]) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    sms[dev] = v > 0 ? v : 148;
  }
  return sms[dev];
}

static size_t umma_smem_bytes(int stages, int nb, bool norm, int M, int K) {
  return 1024 + (size_t)stages * kUTile + (size_t)nb * kUBSlot + (norm ? (size_t)(M + 1) * K * 4 : 0) +
         sizeof(USmem);
}

template <MvEpi E, bool NORM>
static int umma_launch_t(const UmmaParams &p, int grid, size_t smem, cudaStream_t st, bool pdl) {
  static int attr_dev_mask = 0;  // devices on which the shared-memory opt-in was done
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 31 && !(attr_dev_mask & (1 << dev))) {
    int rc = cuda_status(cudaFuncSetAttribute(int8_umma_kernel<E, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              227 * 1024),
                         "int8 tensor-core matvec: shared memory opt-in");
    if (rc) return rc;
    attr_dev_mask |= 1 << dev;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kUWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, int8_umma_kernel<E, NORM>, p), "int8 tensor-core matvec launch");
}

int umma_launch(UmmaParams p, MvEpi e, cudaStream_t st, bool pdl) {
  const bool norm = p.norm_w != nullptr;
  if (p.M < 1 || p.M > 8 || p.K <= 0 || p.K % 128 || p.N <= 0 || !p.x || !p.scales || !p.acc || !p.tile_ctr ||
      (reinterpret_cast<uintptr_t>(p.x) & 15) || (p.x_stride & 3) ||
      (norm && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)) ||
      (e == MvEpi::Argmax && (!p.keys || !p.counter || !p.ids)) || (e == MvEpi::SwiGLU && (p.N & 1)) ||
      (e == MvEpi::QkvPost && (!p.post.positions || p.N != (p.post.n_heads + 2 * p.post.n_kv) * 128)) ||
      (e != MvEpi::Argmax && e != MvEpi::QkvPost && !p.y) || (e == MvEpi::StoreBias && !p.bias)) {
    set_error("int8 tensor-core matvec: unsupported configuration (M=%d K=%d N=%d)", p.M, p.K, p.N);
    return QASR_ERR_UNSUPPORTED;
  }
  const int KT = p.K / 128, NT = (p.N + 127) / 128;
  const long long U = (long long)NT * KT;
  if (U >= (1ll << 30)) {
    set_error("int8 tensor-core matvec: matrix too large");
    return QASR_ERR_UNSUPPORTED;
  }
  const int grid = (int)std::min<long long>(umma_sms(), U);
  const int nu_max = (int)((U + grid - 1) / grid);
  p.nb = std::min(KT, nu_max);
  p.stages = std::max(2, std::min(kUMaxStages, nu_max));
  while (p.stages > 2 && umma_smem_bytes(p.stages, p.nb, norm, p.M, p.K) > 227 * 1024) --p.stages;
  const size_t smem = umma_smem_bytes(p.stages, p.nb, norm, p.M, p.K);
  if (smem > 227 * 1024) {
    set_error("int8 tensor-core matvec: shared memory %zu too large (M=%d K=%d)", smem, p.M, p.K);
    return QASR_ERR_UNSUPPORTED;
  }
  switch (e) {
    case MvEpi::Store:
      return norm ? umma_launch_t<MvEpi::Store, true>(p, grid, smem, st, pdl)
                  : umma_launch_t<MvEpi::Store, false>(p, grid, smem, st, pdl);
    case MvEpi::StoreBias: return umma_launch_t<MvEpi::StoreBias, false>(p, grid, smem, st, pdl);
    case MvEpi::Residual: return umma_launch_t<MvEpi::Residual, false>(p, grid, smem, st, pdl);
    case MvEpi::SwiGLU:
      return norm ? umma_launch_t<MvEpi::SwiGLU, true>(p, grid, smem, st, pdl)
                  : umma_launch_t<MvEpi::SwiGLU, false>(p, grid, smem, st, pdl);
    case MvEpi::Argmax:
      return norm ? umma_launch_t<MvEpi::Argmax, true>(p, grid, smem, st, pdl)
                  : umma_launch_t<MvEpi::Argmax, false>(p, grid, smem, st, pdl);
    case MvEpi::QkvPost:
      return norm ? umma_launch_t<MvEpi::QkvPost, true>(p, grid, smem, st, pdl)
                  : umma_launch_t<MvEpi::QkvPost, false>(p, grid, smem, st, pdl);
  }
  return QASR_ERR_INVALID;
}

}  // namespace qasr
