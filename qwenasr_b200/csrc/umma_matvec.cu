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
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "matvec.cuh"
#include "qkvpost.cuh"
#include "rowops.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kUWarps = 8;
constexpr int kUMaxStages = 8;
// Ring depth of the gate/up kernel (the largest shared-memory user of the
// step): a shallower ring lets it share SMs with its neighbours in the step.
#ifndef QASR_SWIGLU_STAGES
#define QASR_SWIGLU_STAGES 3
#endif
constexpr int kUSwigluStages = QASR_SWIGLU_STAGES;
// Cluster sizes the planner must use per epilogue kind (0: its cost model).
#ifndef QASR_FORCE_C_RESIDUAL
#define QASR_FORCE_C_RESIDUAL 0
#endif
#ifndef QASR_FORCE_C_QKV
#define QASR_FORCE_C_QKV 0
#endif
#ifndef QASR_FORCE_C_SWIGLU
#define QASR_FORCE_C_SWIGLU 0
#endif
constexpr int kUForceCResidual = QASR_FORCE_C_RESIDUAL, kUForceCQkv = QASR_FORCE_C_QKV,
              kUForceCSwiglu = QASR_FORCE_C_SWIGLU;
constexpr int kUMaxCluster = 16;
constexpr int kUTile = 128 * 128;        // bytes of one weight tile
constexpr int kUBSlot = 32 * 128;        // bytes of the digit rows of one K tile
constexpr int kURed = 128 * 8 * 8;       // one tile's 64-bit partials [row][token]
constexpr int kUTmemCols = 64;           // two 32-column accumulators
constexpr int kUEpiThreads = 128;        // warps 0..3
constexpr int kUProducerWarp = 4, kUMmaWarp = 5;
constexpr uint32_t kUIdesc = umma_idesc_s8(128, 32);

struct alignas(16) USmem {
  uint64_t full[kUMaxStages], empty[kUMaxStages];
  uint64_t accfull[2], accempty[2];
  uint64_t redfull[2], redempty[2];  // cluster reduction of a tile's partials
  uint64_t xbar, nbar, done;
  uint32_t tmem;
  int abort;
  int last;
  float dq[8];
  unsigned long long best[4][8];
  alignas(16) float hs[8][128];  // QkvPost: one head of every token (read as float4)
};

// QkvPost: the first tile's RoPE rows and norm weights, copied into shared
// memory (cp.async) before the dependency wait; dynamic shared memory after USmem.
struct alignas(16) QkvStage {
  float c[8][128], s[8][128], w[128];
};

QASR_DEV void cp_async16_g2s(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}

QASR_DEV bool u_aborted(const USmem &sm) { return *reinterpret_cast<const volatile int *>(&sm.abort) != 0; }

QASR_DEV void u_fail(USmem &sm, int *err) {
  atomicExch(&sm.abort, 1);
  if (err) atomicExch(err, -QASR_ERR_TIMEOUT);
}

QASR_DEV float pow2f(int e) {  // 2^e for -126 <= e <= 127
  return __int_as_float((127 + e) << 23);
}

// Grid: clusters of C CTAs (C divides K/128).  Cluster c owns row tiles
// c, c + n_clusters, ...; CTA rank r of the cluster contracts K tiles
// [r*KC, (r+1)*KC) (KC = K/128/C) of each of them.  With C > 1 each rank
// parks its 64-bit partials in shared memory and finishes a share of the
// tile's rows by summing the partials of all ranks over distributed shared
// memory, in rank order.
template <MvEpi E, bool NORM>
__global__ void __launch_bounds__(kUWarps * 32, 1) int8_umma_kernel(const __grid_constant__ UmmaParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int STAGES = p.stages, C = p.csize;
  const int M = p.M, K = p.K, N = p.N;
  const int KT = K / 128, NT = (N + 127) / 128, KC = KT / C;
  unsigned char *a_ring = base;
  unsigned char *b_tiles = a_ring + (size_t)STAGES * kUTile;
  unsigned long long *red = reinterpret_cast<unsigned long long *>(b_tiles + (size_t)KC * kUBSlot);  // [2][128][8]
  float *xs = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(red) + (C > 1 ? 2 * kURed : 0));
  float *nws = xs + (NORM ? (size_t)M * K : 0);  // NORM: x rows [M, K], norm weights [K]
  USmem &sm = *reinterpret_cast<USmem *>(nws + (NORM ? K : 0));

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = C > 1 ? (int)cluster_ctarank() : 0;
  const int cid = C > 1 ? (int)cluster_id_x() : blockIdx.x;
  const int ncl = C > 1 ? (int)cluster_count_x() : gridDim.x;
  const int kt0 = rank * KC;
  const int ntiles = cid < NT ? (NT - 1 - cid) / ncl + 1 : 0;
  const int nu = ntiles * KC;  // pipeline items: (tile j, K tile kt0 + i % KC)

  if (threadIdx.x == 0) {
    for (int s = 0; s < kUMaxStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.accfull[b], 1);
      mbar_init(&sm.accempty[b], 4);
      mbar_init(&sm.redfull[b], C);
      mbar_init(&sm.redempty[b], C);
    }
    mbar_init(&sm.xbar, 1);
    mbar_init(&sm.nbar, 1);
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == kUMmaWarp) tmem_alloc(&sm.tmem, kUTmemCols);
  tc_fence_before();
  __syncwarp();
  if (C > 1)
    cluster_sync_all();  // every rank's barriers exist before any remote arrival
  else
    __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;

  // ---- weight prefetch: constant operand, issued before waiting on the previous kernel
  int produced = 0;  // producer thread only
  auto produce = [&](int i) {
    const int st = i % STAGES, t = cid + (i / KC) * ncl, kt = kt0 + i % KC;
    mbar_arrive_expect_tx(&sm.full[st], kUTile);
    tma_load_2d_u8(a_ring + (size_t)st * kUTile, &p.tmap, kt * 128, t * 128, &sm.full[st]);
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

  // Epilogue operands of this thread's first row (warps 0..3: thread = row of
  // the tile), loaded now so that no dependent load is left on the path from
  // the accumulator to the output: the row's scale (a constant, fetched before
  // the dependency wait) and, for the residual epilogue, the residual values.
  const int ri0 = (warp & 3) * 32 + lane;
  float sc_next = 0.0f;
  if (warp < 4 && ntiles > 0 && cid * 128 + ri0 < N) sc_next = __ldg(p.scales + cid * 128 + ri0);
  // QkvPost: the first tile's head operands for the two tokens this warp
  // finishes: positions (uploaded before the step) in registers, RoPE rows and
  // norm weights copied into shared memory
  int qpos[2] = {0, 0};
  QkvStage *qst = reinterpret_cast<QkvStage *>(reinterpret_cast<unsigned char *>(&sm) + sizeof(USmem));
  if constexpr (E == MvEpi::QkvPost) {
    const QkvPostParams &q = p.post;
    const bool rot = cid < q.n_heads + q.n_kv;  // a q or k head: normalised and rotated
    if (warp < 4 && ntiles > 0 && cid % C == rank) {
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int m = warp + 4 * i;
        if (m >= M) break;
        qpos[i] = q.positions[m];
        if (rot && qpos[i] >= 0 && qpos[i] < q.max_seq) {
          cp_async16_g2s(&qst->c[m][4 * lane], q.cos_tab + (size_t)qpos[i] * 128 + 4 * lane);
          cp_async16_g2s(&qst->s[m][4 * lane], q.sin_tab + (size_t)qpos[i] * 128 + 4 * lane);
        }
      }
      if (warp == 0 && rot) cp_async16_g2s(&qst->w[4 * lane], (cid < q.n_heads ? q.q_norm : q.k_norm) + 4 * lane);
      asm volatile("cp.async.commit_group;" ::: "memory");
    }
  }

  pdl_wait();
  pdl_launch_dependents();
  if (p.tstamp && threadIdx.x == 0) atomicMin(p.tstamp, globaltimer_ns());
  float res0[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) res0[m] = 0.0f;
  if constexpr (E == MvEpi::Residual) {
    const int row = cid * 128 + ri0;
    if (warp < 4 && ntiles > 0 && ri0 / (128 / C) == rank && row < N) {
#pragma unroll
      for (int m = 0; m < 8; ++m)
        if (m < M) res0[m] = p.y[(size_t)m * p.y_stride + row];
    }
  }

  // ---- stage x.  Warp m owns token row m: its exponent (after the RMSNorm
  // when NORM), then its three digit rows for every K tile this CTA uses.
  // Lane l covers floats 4l..4l+3 of a 128-float K tile, so every shared
  // access of the pass is a conflict-free 16-byte (or 4-byte) vector.
  if constexpr (NORM) {
    if (threadIdx.x == 0) {
      mbar_arrive_expect_tx(&sm.xbar, (unsigned)(M * K * 4));
      for (int m = 0; m < M; ++m) bulk_g2s(xs + (size_t)m * K, p.x + (size_t)m * p.x_stride, (unsigned)K * 4, &sm.xbar);
    }
  }
  {
    const int m = warp;  // 8 warps: one per token row (rows m >= M are zero)
    const int nbu = KC;
    auto kt_of = [&](int slot) { return kt0 + slot; };
    auto row_off = [&](int n) {  // byte offset of this lane's 4 bytes of digit row n in a slot
      return (n >> 3) * 1024 + (n & 7) * 128 + (((lane >> 2) ^ (n & 7)) << 4) + (lane & 3) * 4;
    };
    auto put_digits = [&](int slot, float4 v, float qm) {
      // X = rint(v * qm), |X| <= 2^22: v*qm is exact (power of two), and adding
      // 1.5*2^23 leaves X in the low mantissa bits, rounded to nearest even.
      // Balanced base-256 digits: d2 = low byte of X (as signed), X1 = (X+128)>>8,
      // d1 = low byte of X1, d0 = (X1+128)>>8 (|d0| <= 64).
      int X[4] = {__float_as_int(fmaf(v.x, qm, 12582912.0f)) - 0x4B400000,
                  __float_as_int(fmaf(v.y, qm, 12582912.0f)) - 0x4B400000,
                  __float_as_int(fmaf(v.z, qm, 12582912.0f)) - 0x4B400000,
                  __float_as_int(fmaf(v.w, qm, 12582912.0f)) - 0x4B400000};
      const uint32_t w2 = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
      for (int q = 0; q < 4; ++q) X[q] = (X[q] + 128) >> 8;
      const uint32_t w1 = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
      for (int q = 0; q < 4; ++q) X[q] = (X[q] + 128) >> 8;
      const uint32_t w0 = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
      unsigned char *tile = b_tiles + (size_t)slot * kUBSlot;
      *reinterpret_cast<uint32_t *>(tile + row_off(m)) = w0;
      *reinterpret_cast<uint32_t *>(tile + row_off(8 + m)) = w1;
      *reinterpret_cast<uint32_t *>(tile + row_off(16 + m)) = w2;
    };
    auto exponent = [&](float bound) {  // 2^e > bound (bound >= every |x| of the row)
      int e = 0;
      if (bound > 0.0f && bound <= 3.0e38f) frexpf(bound, &e);
      e = max(-100, min(e, 127));
      if (lane == 0) sm.dq[m] = pow2f(e - 22);
      return pow2f(22 - e);
    };
    if (m < M) {
      if constexpr (NORM) {
        bool ok = mbar_wait(&sm.xbar, 0);
        ok = mbar_wait(&sm.nbar, 0) && ok;
        if (!ok && lane == 0) u_fail(sm, p.err);
        const float *xr = xs + (size_t)m * K;
        // sum of squares in the reference's order (rowops.cuh): lanes 0..15 run
        // the sequential chains, operands fetched 16 at a time ahead of them
        const int n16 = K / 16;
        float acc = 0.0f, mx = 0.0f, mw = 0.0f;
        if (lane < 16) {
          for (int j = 0; j < n16; j += 16) {
            float v[16];
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = j + t < n16 ? xr[16 * (j + t) + lane] : 0.0f;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
              acc = j + t < n16 ? fmaf(v[t], v[t], acc) : acc;
              mx = fmaxf(mx, fabsf(v[t]));
            }
          }
        } else {
          for (int k4 = lane - 16; k4 < K / 4; k4 += 16) {
            const float4 b = reinterpret_cast<const float4 *>(nws)[k4];
            mw = fmaxf(mw, fmaxf(fmaxf(fabsf(b.x), fabsf(b.y)), fmaxf(fabsf(b.z), fabsf(b.w))));
          }
        }
        const float sum = hsum16_avx_order(acc);  // K % 128 == 0: no 8-block, no scalar tail
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)K), p.eps)));
        mx = warp_max(mx);
        mw = warp_max(mw);
        // rounding is monotonic, so this bounds every |rn(rn(x*inv)*w)|
        const float qm = exponent(__fmul_rn(__fmul_rn(mx, inv), mw));
        for (int slot = 0; slot < nbu; ++slot) {
          const int k = kt_of(slot) * 128 + 4 * lane;
          const float4 a = *reinterpret_cast<const float4 *>(xr + k);
          const float4 b = *reinterpret_cast<const float4 *>(nws + k);
          const float4 v = make_float4(__fmul_rn(__fmul_rn(a.x, inv), b.x), __fmul_rn(__fmul_rn(a.y, inv), b.y),
                                       __fmul_rn(__fmul_rn(a.z, inv), b.z), __fmul_rn(__fmul_rn(a.w, inv), b.w));
          put_digits(slot, v, qm);
        }
      } else {
        const float4 *xr = reinterpret_cast<const float4 *>(p.x + (size_t)m * p.x_stride);
        constexpr int kRegTiles = 24;
        if (KT <= kRegTiles) {  // the whole row in flight at once: one L2 round trip
          float4 v[kRegTiles];
#pragma unroll
          for (int i = 0; i < kRegTiles; ++i)
            if (i < KT) v[i] = xr[i * 32 + lane];
          float mx = 0.0f;
#pragma unroll
          for (int i = 0; i < kRegTiles; ++i)
            if (i < KT) mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
          const float qm = exponent(warp_max(mx));
          for (int slot = 0; slot < nbu; ++slot) put_digits(slot, xr[kt_of(slot) * 32 + lane], qm);
        } else {
          float mx = 0.0f;
          for (int k4 = lane; k4 < K / 4; k4 += 32) {
            const float4 a = xr[k4];
            mx = fmaxf(mx, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
          }
          const float qm = exponent(warp_max(mx));
          for (int slot = 0; slot < nbu; ++slot) put_digits(slot, xr[kt_of(slot) * 32 + lane], qm);
        }
      }
    } else {
      for (int slot = 0; slot < nbu; ++slot)
        for (int d = 0; d < 3; ++d)
          *reinterpret_cast<uint32_t *>(b_tiles + (size_t)slot * kUBSlot + row_off(8 * d + m)) = 0u;
    }
    for (int slot = 0; slot < nbu; ++slot)  // padding row 24 + warp
      *reinterpret_cast<uint32_t *>(b_tiles + (size_t)slot * kUBSlot + row_off(24 + warp)) = 0u;
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
    // ---- MMA issuer (one thread): one accumulator per tile, double-buffered
    if (lane == 0) {
      for (int i = 0; i < nu; ++i) {
        const int j = i / KC, kk = i % KC, st = i % STAGES, buf = j & 1;
        if (kk == 0 && j >= 2 && !mbar_wait(&sm.accempty[buf], (unsigned)(((j >> 1) - 1) & 1))) {
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
        const uint32_t b_addr = smem_u32(b_tiles + (size_t)kk * kUBSlot);
        const uint32_t d_addr = tmem + (uint32_t)(buf * 32);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_s8(d_addr, umma_desc_sw128(a_addr + 32 * s), umma_desc_sw128(b_addr + 32 * s), kUIdesc,
                  (kk == 0 && s == 0) ? 0u : 1u);
        umma_commit(&sm.empty[st]);
        if (kk == KC - 1) umma_commit(&sm.accfull[buf]);
      }
      // every MMA issued so far has completed once `done` flips
      umma_commit(&sm.done);
      if (!mbar_wait(&sm.done, 0)) u_fail(sm, p.err);
    }
  } else if (warp < 4) {
    // ---- epilogue: thread = row of the tile
    const int ri = warp * 32 + lane;
    // rows this rank finishes: a contiguous share (even-sized, so SwiGLU
    // pairs stay together), or the whole tile for the per-head QkvPost
    const int share = 128 / C;
    for (int j = 0; j < ntiles; ++j) {
      const int t = cid + j * ncl, buf = j & 1;
      if (!u_aborted(sm) && !mbar_wait(&sm.accfull[buf], (unsigned)((j >> 1) & 1))) u_fail(sm, p.err);
      named_bar(1, kUEpiThreads);  // the four epilogue warps decide together
      if (u_aborted(sm)) break;
      tc_fence_after();
      uint32_t r[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * 32), r);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.accempty[buf])) : "memory");

      long long V[8];
#pragma unroll
      for (int m = 0; m < 8; ++m)
        V[m] = ((long long)(int)r[m] << 16) + ((long long)(int)r[8 + m] << 8) + (long long)(int)r[16 + m];
      const int fin_rank = E == MvEpi::QkvPost ? t % C : ri / share;
      bool mine = fin_rank == rank;
      if (C > 1) {
        unsigned long long *rb = red + (size_t)buf * 128 * 8;
        // the ranks finished reading this buffer two tiles ago
        bool ok = j < 2 || mbar_wait_cluster(&sm.redempty[buf], (unsigned)(((j >> 1) - 1) & 1));
#pragma unroll
        for (int m = 0; m < 8; ++m) rb[ri * 8 + m] = (unsigned long long)V[m];
        named_bar(1, kUEpiThreads);
        if (threadIdx.x < C) {  // one arrival per rank, issued in parallel
          asm volatile("fence.acq_rel.cluster;" ::: "memory");
          mbar_arrive_remote(cluster_map(smem_u32(&sm.redfull[buf]), (uint32_t)threadIdx.x));
        }
        ok = mbar_wait_cluster(&sm.redfull[buf], (unsigned)((j >> 1) & 1)) && ok;
        if (!ok) u_fail(sm, p.err);
        if (mine) {
          const uint32_t local = smem_u32(rb + ri * 8);
#pragma unroll
          for (int m = 0; m < 8; ++m) V[m] = 0;
          for (int q = 0; q < C; ++q) {
            const uint32_t ra = cluster_map(local, (uint32_t)q);
            unsigned long long part[8];
#pragma unroll
            for (int h = 0; h < 4; ++h) ld_cluster_u64x2(ra + 16 * h, part[2 * h], part[2 * h + 1]);
#pragma unroll
            for (int m = 0; m < 8; ++m) V[m] += (long long)part[m];
          }
        }
        named_bar(1, kUEpiThreads);
        if (threadIdx.x < C)  // this rank is done reading every rank's partials
          mbar_arrive_remote(cluster_map(smem_u32(&sm.redempty[buf]), (uint32_t)threadIdx.x));
      }

      const int row = t * 128 + ri;
      const bool valid = mine && row < N;
      const float sc = valid ? sc_next : 0.0f;
      {  // the next tile's scale, in flight during this tile's epilogue
        const int nrow = (t + ncl) * 128 + ri;
        sc_next = j + 1 < ntiles && nrow < N ? __ldg(p.scales + nrow) : 0.0f;
      }
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
            *dst = __fadd_rn(j == 0 ? res0[m] : *dst, yv[m]);
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
        // the tile is one 128-wide head: its finishing rank completes it here
        if (fin_rank == rank) {
#pragma unroll
          for (int m = 0; m < 8; ++m) sm.hs[m][ri] = yv[m];
          if (j == 0) asm volatile("cp.async.wait_all;" ::: "memory");  // this thread's operand copies
          named_bar(2, kUEpiThreads);
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int m = warp + 4 * i;
            if (m >= M) break;
            const float4 hv = reinterpret_cast<const float4 *>(sm.hs[m])[lane];
            if (j == 0) {
              QkvPostOperands op;
              op.pos = qpos[i];
              op.c = reinterpret_cast<const float4 *>(qst->c[m])[lane];
              op.s = reinterpret_cast<const float4 *>(qst->s[m])[lane];
              op.w = reinterpret_cast<const float4 *>(qst->w)[lane];
              qkv_head_post(p.post, p.eps, t, m, hv, op, p.err);
            } else
              qkv_head_post(p.post, p.eps, t, m, hv, p.err);
          }
          named_bar(2, kUEpiThreads);
        }
      }
    }
  }
  if (C > 1) cluster_arrive_all();  // this thread touches no other rank's memory from here on
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

  // ---- teardown: copies in flight land, no rank leaves while a peer may
  // still read its partials or arrive on its barriers, then TMEM is released
  if (producer) {
    for (int i = max(0, produced - STAGES); i < produced; ++i)
      mbar_wait(&sm.full[i % STAGES], (unsigned)((i / STAGES) & 1));
  }
  tc_fence_before();
  __syncwarp();
  if (C > 1) cluster_wait_all();  // arrived after the role loops
  __syncthreads();
  if (warp == kUMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kUTmemCols);
  }
  if (p.tstamp && threadIdx.x == 0) atomicMax(p.tstamp + 1, globaltimer_ns());
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

static size_t umma_smem_bytes(int stages, int C, bool norm, int M, int K, bool qkv) {
  const int KC = K / 128 / C;
  return 1024 + (size_t)stages * kUTile + (size_t)KC * kUBSlot + (C > 1 ? 2 * kURed : 0) +
         (norm ? (size_t)(M + 1) * K * 4 : 0) + sizeof(USmem) + (qkv ? sizeof(QkvStage) : 0);
}

struct UmmaPlan {
  int C = 0, clusters = 0, stages = 0;
  size_t smem = 0;
};

// Shared-memory opt-in (and, for clusters above 8, the non-portable size) of
// one kernel instance on the current device; -1 if unavailable.
template <MvEpi E, bool NORM>
static int umma_prepare(int dev) {
  static int state[64] = {0};  // 0 unknown, 1 portable clusters only, 2 up to 16
  if (dev < 0 || dev >= 64) return -1;
  if (!state[dev]) {
    if (cudaFuncSetAttribute(int8_umma_kernel<E, NORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) !=
        cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    state[dev] = cudaFuncSetAttribute(int8_umma_kernel<E, NORM>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
                         cudaSuccess
                     ? 2
                     : 1;
    cudaGetLastError();
  }
  return state[dev];
}

// How many clusters of C CTAs with `smem` bytes each can be resident at once.
template <MvEpi E, bool NORM>
static int umma_max_clusters(int dev, int C, size_t smem) {
  static std::mutex mu;
  static std::map<std::tuple<int, int, size_t>, int> cache;
  std::lock_guard<std::mutex> lk(mu);
  const auto key = std::make_tuple(dev, C, smem);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)C);
  cfg.blockDim = dim3(kUWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = (unsigned)C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, int8_umma_kernel<E, NORM>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  cache[key] = n;
  return n;
}

// Pick the cluster size: the K tiles of a row tile are split over the C
// ranks of a cluster.  Cost model in units of one 16 KB weight tile streamed
// by one SM: the busiest cluster's row tiles x K tiles per rank, plus the
// exchange of partials when C > 1 (about three tiles' time, then one per
// further row tile); on a tie the larger cluster (more CTAs) wins.
template <MvEpi E, bool NORM>
static UmmaPlan umma_plan(const UmmaParams &p, bool norm) {
  UmmaPlan best;
  int dev = 0;
  cudaGetDevice(&dev);
  const int state = umma_prepare<E, NORM>(dev);
  if (state < 0) return best;
  const int KT = p.K / 128, NT = (p.N + 127) / 128;
  double best_cost = 1e30;
  int forced = E == MvEpi::Residual ? kUForceCResidual : E == MvEpi::QkvPost ? kUForceCQkv
               : E == MvEpi::SwiGLU   ? kUForceCSwiglu
                                      : 0;
  // Measured (M=8, 1.7B shapes): the fused q/k/v kernel over K = 2048 runs
  // the step 3.8 % faster in 2-CTA clusters than in the cost model's 4.
  if (!forced && E == MvEpi::QkvPost && p.K >= 2048 && KT % 2 == 0) forced = 2;
  for (int C = 1; C <= kUMaxCluster && C <= KT; ++C) {
    if (KT % C || (C > 8 && state < 2) || 128 % (2 * C) && C > 1) continue;  // even row shares
    if (forced && C != forced) continue;
    int stages = std::min(kUMaxStages, E == MvEpi::SwiGLU ? kUSwigluStages : kUMaxStages);
    while (stages > 2 && umma_smem_bytes(stages, C, norm, p.M, p.K, E == MvEpi::QkvPost) > 227 * 1024) --stages;
    const size_t smem = umma_smem_bytes(stages, C, norm, p.M, p.K, E == MvEpi::QkvPost);
    if (smem > 227 * 1024) continue;
    const int resident = C == 1 ? umma_max_clusters<E, NORM>(dev, 1, smem) * 1 : umma_max_clusters<E, NORM>(dev, C, smem);
    if (resident < 1) continue;
    const int clusters = std::min(NT, resident);
    const int tiles = (NT + clusters - 1) / clusters;
    const double cost = (double)tiles * (KT / C) + (C > 1 ? 3.0 + tiles : 0.0);
    if (cost < best_cost + 1e-9) {  // ties go to the larger cluster: more SMs stream the weights
      best_cost = cost;
      best.C = C;
      best.clusters = clusters;
      best.smem = smem;
      best.stages = std::max(2, std::min(stages, tiles * (KT / C)));
    }
  }
  return best;
}

template <MvEpi E, bool NORM>
static int umma_launch_t(UmmaParams p, cudaStream_t st, bool pdl) {
  const UmmaPlan plan = umma_plan<E, NORM>(p, NORM);
  if (!plan.C) {
    set_error("int8 tensor-core matvec: no launch configuration fits (M=%d K=%d N=%d)", p.M, p.K, p.N);
    return QASR_ERR_UNSUPPORTED;
  }
  p.csize = plan.C;
  p.stages = plan.stages;
  const size_t smem = umma_smem_bytes(p.stages, plan.C, NORM, p.M, p.K, E == MvEpi::QkvPost);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(plan.clusters * plan.C));
  cfg.blockDim = dim3(kUWarps * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (plan.C > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)plan.C;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cuda_status(cudaLaunchKernelEx(&cfg, int8_umma_kernel<E, NORM>, p), "int8 tensor-core matvec launch");
}

int umma_launch(UmmaParams p, MvEpi e, cudaStream_t st, bool pdl) {
  const bool norm = p.norm_w != nullptr;
  if (p.M < 1 || p.M > 8 || p.K <= 0 || p.K % 128 || p.N <= 0 || !p.x || !p.scales ||
      (reinterpret_cast<uintptr_t>(p.x) & 15) || (p.x_stride & 3) ||
      (norm && (reinterpret_cast<uintptr_t>(p.norm_w) & 15)) ||
      (e == MvEpi::Argmax && (!p.keys || !p.counter || !p.ids)) || (e == MvEpi::SwiGLU && (p.N & 1)) ||
      (e == MvEpi::QkvPost && (!p.post.positions || p.N != (p.post.n_heads + 2 * p.post.n_kv) * 128)) ||
      (e != MvEpi::Argmax && e != MvEpi::QkvPost && !p.y) || (e == MvEpi::StoreBias && !p.bias) ||
      (long long)((p.N + 127) / 128) * (p.K / 128) >= (1ll << 30)) {
    set_error("int8 tensor-core matvec: unsupported configuration (M=%d K=%d N=%d)", p.M, p.K, p.N);
    return QASR_ERR_UNSUPPORTED;
  }
  switch (e) {
    case MvEpi::Store:
      return norm ? umma_launch_t<MvEpi::Store, true>(p, st, pdl) : umma_launch_t<MvEpi::Store, false>(p, st, pdl);
    case MvEpi::StoreBias: return umma_launch_t<MvEpi::StoreBias, false>(p, st, pdl);
    case MvEpi::Residual: return umma_launch_t<MvEpi::Residual, false>(p, st, pdl);
    case MvEpi::SwiGLU:
      return norm ? umma_launch_t<MvEpi::SwiGLU, true>(p, st, pdl) : umma_launch_t<MvEpi::SwiGLU, false>(p, st, pdl);
    case MvEpi::Argmax:
      return norm ? umma_launch_t<MvEpi::Argmax, true>(p, st, pdl) : umma_launch_t<MvEpi::Argmax, false>(p, st, pdl);
    case MvEpi::QkvPost:
      return norm ? umma_launch_t<MvEpi::QkvPost, true>(p, st, pdl) : umma_launch_t<MvEpi::QkvPost, false>(p, st, pdl);
  }
  return QASR_ERR_INVALID;
}

}  // namespace qasr
