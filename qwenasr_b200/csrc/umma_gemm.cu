// umma_gemm.cu -- GEMMs for many token rows on the tcgen05 tensor cores:
//  * INT8 weights: the prefill and encoder projections,
//    kernels::linear_nobias_int8 / linear_int8 with seq_len > 8
//    (crates/qwen-asr/src/kernels/mod.rs:650-673; the reference runs seq_len
//    sequential matvecs of generic::int8_matvec_fused, generic.rs:39-49);
//  * f32 weights: kernels::linear / linear_nobias / matmul_t (mod.rs:503-568,
//    cblas_sgemm in the reference), the encoder projections of an f32 model.
//
// Exact integer formulation (as the decode contraction, umma_matvec.cu):
// every activation row t is scaled by 2^(22-E_t) (2^E_t bounds its largest
// magnitude), rounded to an integer X with |X| <= 2^22 and split into three
// balanced signed bytes X = 65536*d0 + 256*d1 + d2 ("digit rows").  INT8
// weights are used as they are.  f32 weights get the same treatment per
// weight row, giving three int8 "digit planes" W_a and a per-row factor; the
// product of two digit expansions is then sum_a sum_b 2^(8(2-a)) 2^(8(2-b))
// W_a . X_b.  The tensor cores compute every W_a . X_b exactly in 32-bit
// integers; the epilogue recombines them exactly in 64 bits and rounds once.
// The only approximation is the 23-bit rounding of each operand relative to
// its row maximum -- below the f32 summation error of the reference.
//
//  * digit_rows_kernel: one warp per row writes its three digit rows and its
//    dequantisation factor 2^(E-22).  Row r of digit d goes to
//    (r / B) * 3B + d * B + r % B: token blocks of B = 32 rows for
//    activations, one block of B = N rows (three planes) for weights.
//  * gemm_kernel<PLANES>: persistent; output tiles of 128 weight rows x one
//    32-token block, taken row-tile-major with the token block fastest so the
//    CTAs sharing a weight tile run together and it is read from HBM once.
//    One thread streams, for every 128-byte K step (and weight plane), the
//    weight tile and the digit tile with 2D TMA loads (128-byte swizzle, no
//    multicast) into a 4-stage ring; one thread issues tcgen05.mma kind::i8
//    (M=128, N=96, K=32) into a double-buffered TMEM accumulator (one per
//    weight plane); four epilogue warps read it with tcgen05.ld (thread =
//    output row), add the planes in 64-bit registers and write y (+bias),
//    coalesced over rows.
// Every wait is bounded; a timeout sets *err, stops the roles, drains the
// copies and MMAs in flight and frees TMEM.
#include <atomic>
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "matvec.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kGTok = 32;                 // tokens per block (the f32 three-plane GEMM; small INT8 grids)
constexpr int kGRows = 3 * kGTok;         // digit rows per block (MMA N)
constexpr int kGStages = 4;
constexpr int kGATile = 128 * 128;        // weight tile bytes

// Token block of TOK tokens: 3*TOK digit rows (the MMA's N), a digit tile of
// 3*TOK x 128 bytes per stage, two TMEM accumulators of 3*TOK columns (at
// column 0 and kBufCols).  TOK = 64 (N = 192) halves the MMA instructions
// and the weight-tile reads per token against TOK = 32.
template <int TOK>
struct GTile {
  static_assert(TOK == 32 || TOK == 64, "token block");
  static constexpr int kRows = 3 * TOK;
  static constexpr int kBTile = kRows * 128;
  static constexpr int kBufCols = TOK == 32 ? 128 : 256;
  static constexpr int kTmemCols = 2 * kBufCols;
  static constexpr uint32_t kIdesc = umma_idesc_s8(128, kRows);
  static constexpr size_t kSmem = 1024 + (size_t)kGStages * (kGATile + kBTile);
};
constexpr int kGemmStore = 0, kGemmResidual = 1, kGemmSwiGLU = 2;

// ---------------------------------------------------------------- digits --
// Four values of a row -> their balanced base-256 digits (X = rint(v*qm),
// |X| <= 2^22, X = 65536*d0 + 256*d1 + d2), written as bytes k..k+3 of the
// three digit rows at row0, row0 + dstep, row0 + 2*dstep.
QASR_DEV void put_digits4(int8_t *row0, size_t dstep, int k, float4 v, float qm) {
  // X = rint(v*qm) via the 1.5*2^23 magic constant; balanced base-256 digits
  int X[4] = {__float_as_int(fmaf(v.x, qm, 12582912.0f)) - 0x4B400000,
              __float_as_int(fmaf(v.y, qm, 12582912.0f)) - 0x4B400000,
              __float_as_int(fmaf(v.z, qm, 12582912.0f)) - 0x4B400000,
              __float_as_int(fmaf(v.w, qm, 12582912.0f)) - 0x4B400000};
  uint32_t w[3];
  w[2] = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
  for (int q = 0; q < 4; ++q) X[q] = (X[q] + 128) >> 8;
  w[1] = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
  for (int q = 0; q < 4; ++q) X[q] = (X[q] + 128) >> 8;
  w[0] = __byte_perm(__byte_perm(X[0], X[1], 0x0040), __byte_perm(X[2], X[3], 0x0040), 0x5410);
#pragma unroll
  for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t *>(row0 + d * dstep + k) = w[d];
}

// Exponent of a row from its largest magnitude: returns the scale qm that
// maps the row to |X| <= 2^22 and writes the row's factor 2^(e-22).
QASR_DEV float row_exponent(float mx, float *dq_slot, bool write) {
  int e = 0;
  if (mx > 0.0f && mx <= 3.0e38f) frexpf(mx, &e);  // mx < 2^e
  e = max(-100, min(e, 127));
  if (write) *dq_slot = __int_as_float((127 + e - 22) << 23);
  return __int_as_float((127 + 22 - e) << 23);
}

// The digit rows of a 3x3, stride-2, padding-1 convolution's patch matrix,
// read straight from the channel-last activation act [B, h_in, w_in, C]:
// row r = (b, oh, ow), column (ki*3 + kj)*C + ic = act[b, 2oh+ki-1, 2ow+kj-1,
// ic] (0 outside) -- the channel-fastest order the conv weights are permuted
// to.  The GEMM then reads the patches without a materialised im2col matrix;
// the digits equal digit_rows_kernel's on that matrix.  One warp per row.
__global__ void __launch_bounds__(256) conv_digit_rows_kernel(int8_t *__restrict__ D, float *__restrict__ dq,
                                                              const float *__restrict__ act, int C, int h_in,
                                                              int w_in, int h_out, int w_out, int rows, int rows_pad,
                                                              int B) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= rows_pad) return;
  const int K = 9 * C, C4 = C / 4;
  int8_t *row0 = D + ((size_t)(t / B) * 3 * B + t % B) * K;  // digit d at row0 + d*B*K
  const size_t dstep = (size_t)B * K;
  if (t >= rows) {  // rows past the end of the last block: zero digits
    for (int k = 4 * lane; k < K; k += 128)
      for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t *>(row0 + d * dstep + k) = 0u;
    if (lane == 0) dq[t] = 0.0f;
    return;
  }
  // 32-bit index math: the engine's stem passes keep B * h_in * w_in * C below 2^31
  const int ow = t % w_out, bt = t / w_out, oh = bt % h_out, b = bt / h_out;
  const float4 *src = reinterpret_cast<const float4 *>(act);
  auto tap = [&](int kk) -> const float4 * {  // the tap's C channels, or null in the padding
    const int ih = 2 * oh + kk / 3 - 1, iw = 2 * ow + kk % 3 - 1;
    return (ih >= 0 && ih < h_in && iw >= 0 && iw < w_in) ? src + ((b * h_in + ih) * w_in + iw) * C4 : nullptr;
  };
  float mx = 0.0f;
  for (int kk = 0; kk < 9; ++kk) {
    const float4 *tp = tap(kk);
    if (!tp) continue;
    for (int c4 = lane; c4 < C4; c4 += 32) {
      const float4 v = tp[c4];
      mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
  mx = warp_max(mx);
  const float qm = row_exponent(mx, dq + t, lane == 0);
  for (int kk = 0; kk < 9; ++kk) {
    const float4 *tp = tap(kk);
    for (int c4 = lane; c4 < C4; c4 += 32)
      put_digits4(row0, dstep, kk * C + 4 * c4, tp ? tp[c4] : make_float4(0.f, 0.f, 0.f, 0.f), qm);
  }
}

__global__ void __launch_bounds__(256) digit_rows_kernel(int8_t *__restrict__ D, float *__restrict__ dq,
                                                         const float *__restrict__ x, long x_stride, int rows, int K,
                                                         int rows_pad, int B) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= rows_pad) return;
  int8_t *row0 = D + ((size_t)(t / B) * 3 * B + t % B) * K;  // digit d at row0 + d*B*K
  const size_t dstep = (size_t)B * K;
  if (t >= rows) {  // rows past the end of the last block: zero digits
    for (int k = 4 * lane; k < K; k += 128)
      for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t *>(row0 + d * dstep + k) = 0u;
    if (lane == 0) dq[t] = 0.0f;
    return;
  }
  const float4 *xr = reinterpret_cast<const float4 *>(x + (size_t)t * x_stride);
  float mx = 0.0f;
  for (int k4 = lane; k4 < K / 4; k4 += 32) {
    const float4 v = xr[k4];
    mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  mx = warp_max(mx);
  const float qm = row_exponent(mx, dq + t, lane == 0);
  for (int k4 = lane; k4 < K / 4; k4 += 32) put_digits4(row0, dstep, 4 * k4, xr[k4], qm);  // L1 hit: read above
}

// ------------------------------------------------------------------ GEMM --
struct GemmParams {
  CUtensorMap tm_w;  // [PLANES*N, K] int8, box 128 x 128, SW128 (plane a at rows a*N..)
  CUtensorMap tm_d;  // [blocks*96, K] int8 digit rows, box 96 x 128, SW128
  const float *dq;   // [blocks*32] per token row
  const float *scales, *bias;  // per weight row: INT8 scales, or the f32 weights' factors
  float *y;          // [T, N], row stride y_stride
  long y_stride;
  // optional split of the output by weight row: rows >= n1 go to y1 (column
  // row - n1, stride y1_stride), rows >= n2 to y2 (n1, n2 multiples of 128)
  float *y1, *y2;
  long y1_stride, y2_stride;
  int n1, n2;
  int epi;  // kGemmStore, kGemmResidual (y += result), kGemmSwiGLU (rows g,u interleaved -> y[t, row/2])
  int T, K, N;
  int *err;
};

struct alignas(16) GSmem {
  uint64_t full[kGStages], empty[kGStages];
  uint64_t accfull[2], accempty[2];
  uint64_t done;
  uint32_t tmem;
  int abort;
};

QASR_DEV bool g_aborted(const GSmem &sm) { return *reinterpret_cast<const volatile int *>(&sm.abort) != 0; }
QASR_DEV void g_fail(GSmem &sm, int *err) {
  atomicExch(&sm.abort, 1);
  if (err) atomicExch(err, -QASR_ERR_TIMEOUT);
}

template <int PLANES, int TOK>
__global__ void __launch_bounds__(256, 1) gemm_kernel(const __grid_constant__ GemmParams p) {
  using G = GTile<TOK>;
  static_assert(PLANES == 1 || TOK == 32, "the plane sums of the f32 GEMM stay in registers: 32-token blocks");
  constexpr int kHalves = TOK / 32;  // the epilogue reads TMEM 32 tokens at a time
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  unsigned char *a_ring = base;
  unsigned char *b_ring = a_ring + (size_t)kGStages * kGATile;
  GSmem &sm = *reinterpret_cast<GSmem *>(b_ring + (size_t)kGStages * G::kBTile);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = (p.K + 127) / 128, NT = (p.N + 127) / 128, NB = (p.T + TOK - 1) / TOK;
  const int tiles = NT * NB;
  const int my_tiles = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  // pipeline items: (output tile j, weight plane a, K step kt); one accumulator per (j, a) "piece"
  const int per_tile = PLANES * KT;
  const int nu = my_tiles * per_tile;
  auto tile_of = [&](int j) { return (int)blockIdx.x + j * (int)gridDim.x; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.accfull[b], 1);
      mbar_init(&sm.accempty[b], 4);
    }
    mbar_init(&sm.done, 1);
    sm.abort = 0;
    mbar_fence_init();
  }
  if (warp == 5) tmem_alloc(&sm.tmem, G::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  pdl_wait();
  pdl_launch_dependents();

  int produced = 0;
  auto produce = [&](int i) {
    const int st = i % kGStages, tile = tile_of(i / per_tile), a = (i / KT) % PLANES, kt = i % KT;
    const int rt = tile / NB, tb = tile % NB;
    mbar_arrive_expect_tx(&sm.full[st], kGATile + G::kBTile);
    tma_load_2d_u8(a_ring + (size_t)st * kGATile, &p.tm_w, kt * 128, a * p.N + rt * 128, &sm.full[st]);
    tma_load_2d_u8(b_ring + (size_t)st * G::kBTile, &p.tm_d, kt * 128, tb * G::kRows, &sm.full[st]);
  };
  const bool producer = warp == 4 && lane == 0;
  if (producer) {
    for (; produced < nu; ++produced) {
      if (g_aborted(sm)) break;
      const int st = produced % kGStages;
      if (produced >= kGStages && !mbar_wait(&sm.empty[st], (unsigned)((produced / kGStages - 1) & 1))) {
        g_fail(sm, p.err);
        break;
      }
      produce(produced);
    }
  } else if (warp == 5) {
    if (lane == 0) {
      for (int i = 0; i < nu; ++i) {
        const int piece = i / KT, kt = i % KT, st = i % kGStages, buf = piece & 1;
        if (kt == 0 && piece >= 2 && !mbar_wait(&sm.accempty[buf], (unsigned)(((piece >> 1) - 1) & 1))) {
          g_fail(sm, p.err);
          break;
        }
        if (!mbar_wait(&sm.full[st], (unsigned)((i / kGStages) & 1))) {
          g_fail(sm, p.err);
          break;
        }
        if (g_aborted(sm)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(a_ring + (size_t)st * kGATile);
        const uint32_t b_addr = smem_u32(b_ring + (size_t)st * G::kBTile);
        const uint32_t d_addr = tmem + (uint32_t)(buf * G::kBufCols);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_s8(d_addr, umma_desc_sw128(a_addr + 32 * s), umma_desc_sw128(b_addr + 32 * s), G::kIdesc,
                  (kt == 0 && s == 0) ? 0u : 1u);
        umma_commit(&sm.empty[st]);
        if (kt == KT - 1) umma_commit(&sm.accfull[buf]);
      }
      umma_commit(&sm.done);
      if (!mbar_wait(&sm.done, 0)) g_fail(sm, p.err);
    }
  } else if (warp < 4) {
    const int ri = warp * 32 + lane;
    long long V[kGTok];
#pragma unroll
    for (int t = 0; t < kGTok; ++t) V[t] = 0;
    for (int piece = 0; piece < my_tiles * PLANES; ++piece) {
      const int j = piece / PLANES, a = piece % PLANES, buf = piece & 1;
      const int tile = tile_of(j), rt = tile / NB, tb = tile % NB;
      if (!g_aborted(sm) && !mbar_wait(&sm.accfull[buf], (unsigned)((piece >> 1) & 1))) g_fail(sm, p.err);
      named_bar(1, 128);  // the four epilogue warps decide together
      if (g_aborted(sm)) break;
      tc_fence_after();
      // plane a carries weight digit a: weight 2^(8*(PLANES-1-a)) within the plane sum
      const int wshift = 8 * (PLANES - 1 - a);
      const int row = rt * 128 + ri;
      const bool row_ok = row < p.N;
      for (int h = 0; h < kHalves; ++h) {
        uint32_t a0[32], a1[32], a2[32];
        // digit d of token tl sits in column d*TOK + tl of the accumulator
        const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * G::kBufCols + 32 * h);
        tmem_ld32(taddr, a0);
        tmem_ld32(taddr + TOK, a1);
        tmem_ld32(taddr + 2 * TOK, a2);
        if (h == kHalves - 1) {  // the accumulator is free for the MMA warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0)
            asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.accempty[buf])) : "memory");
        }
#pragma unroll
        for (int tl = 0; tl < kGTok; ++tl)
          V[tl] += (((long long)(int)a0[tl] << 16) + ((long long)(int)a1[tl] << 8) + (long long)(int)a2[tl]) << wshift;
        if (a != PLANES - 1) continue;  // PLANES > 1 implies one half: on to the next plane
        const float sc = row_ok ? p.scales[row] : 0.0f;
        const float b = (row_ok && p.bias) ? p.bias[row] : 0.0f;
        const int t0 = tb * TOK + 32 * h;
#pragma unroll
        for (int tl = 0; tl < kGTok; ++tl) {
          const int t = t0 + tl;  // dq holds the padded block: defined past T
          float v = __fmul_rn(__fmul_rn(__ll2float_rn(V[tl]), __ldg(p.dq + t)), sc);
          if (p.bias) v = __fadd_rn(v, b);
          if (p.epi == kGemmSwiGLU) {
            // avx::swiglu_interleaved (avx.rs:568-599) on the (gate, up) row pair
            const float u = __shfl_xor_sync(0xffffffffu, v, 1);
            if (t < p.T && row_ok && !(ri & 1)) {
              const int j = row >> 1, body = (p.N >> 1) - (p.N >> 1) % 8;
              const float silu = j < body ? __fdiv_rn(v, __fadd_rn(1.0f, fast_exp_ref(__fsub_rn(0.0f, v))))
                                          : __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
              p.y[(size_t)t * p.y_stride + j] = __fmul_rn(silu, u);
            }
          } else if (t < p.T && row_ok) {
            float *dst;
            if (row >= p.n2)
              dst = p.y2 + (size_t)t * p.y2_stride + (row - p.n2);
            else if (row >= p.n1)
              dst = p.y1 + (size_t)t * p.y1_stride + (row - p.n1);
            else
              dst = p.y + (size_t)t * p.y_stride + row;
            *dst = p.epi == kGemmResidual ? __fadd_rn(*dst, v) : v;
          }
        }
#pragma unroll
        for (int t = 0; t < kGTok; ++t) V[t] = 0;
      }
    }
  }
  __syncthreads();
  if (producer)
    for (int i = max(0, produced - kGStages); i < produced; ++i)
      mbar_wait(&sm.full[i % kGStages], (unsigned)((i / kGStages) & 1));
  tc_fence_before();
  __syncwarp();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem, G::kTmemCols);
  }
}

static int gemm_sms() {
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

// 2D map over an int8 [rows, K] matrix, box `box_rows` x 128 bytes, 128-byte swizzle.
static int int8_map(CUtensorMap *tm, const int8_t *base, long rows, int K, int box_rows) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  auto encode = reinterpret_cast<Encode>(tensor_map_encoder());
  if (!encode) {
    set_error("tensor-core GEMM: cuTensorMapEncodeTiled unavailable");
    return QASR_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("tensor-core GEMM: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

static int digit_rows(int8_t *D, float *dq, const float *x, long x_stride, int rows, int rows_pad, int K, int B,
                      cudaStream_t st) {
  digit_rows_kernel<<<(rows_pad + 7) / 8, 256, 0, st>>>(D, dq, x, x_stride, rows, K, rows_pad, B);
  return launch_status("tensor-core GEMM: digit rows");
}

template <int PLANES, int TOK>
static int gemm_launch(GemmParams &p, cudaStream_t st) {
  using G = GTile<TOK>;
  if (!p.y1) p.n1 = p.n2 = 0x7fffffff;  // no split
  static std::atomic<unsigned> attr_mask{0};  // engines on several host threads reach here
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = G::kSmem + sizeof(GSmem);
  if (dev < 31 && !(attr_mask.load() & (1u << dev))) {
    int rc = cuda_status(cudaFuncSetAttribute(gemm_kernel<PLANES, TOK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)smem),
                         "tensor-core GEMM: shared memory opt-in");
    if (rc) return rc;
    attr_mask.fetch_or(1u << dev);
  }
  const long tiles = (long)((p.N + 127) / 128) * ((p.T + TOK - 1) / TOK);
  const int grid = (int)std::min<long>(gemm_sms(), tiles);
  gemm_kernel<PLANES, TOK><<<grid, 256, smem, st>>>(p);
  return launch_status("tensor-core GEMM");
}

// Token block of an INT8 GEMM: the one with fewer rounds of tiles over the
// SMs, a 64-token tile counted as kGTok64Cost / 10 of a 32-token one (fewer
// MMA instructions and weight-tile reads per token, more work per tile).
#ifndef QASR_GEMM_TOK64_COST
#define QASR_GEMM_TOK64_COST 16
#endif
constexpr int kGTok64Cost = QASR_GEMM_TOK64_COST;
static int int8_gemm_tok(int T, int N) {
  const long sms = gemm_sms(), nt = (N + 127) / 128;
  const long waves32 = (nt * ((T + 31) / 32) + sms - 1) / sms, waves64 = (nt * ((T + 63) / 64) + sms - 1) / sms;
  return waves64 * kGTok64Cost < waves32 * 10 ? 64 : 32;
}

// The activation digits of x (token blocks of TOK) and the launch, for an
// INT8 GEMM whose weight map, scales and outputs p already holds.
static int int8_gemm_run(GemmParams &p, const float *x, long x_stride, cudaStream_t st) {
  const int T = p.T, K = p.K, TOK = int8_gemm_tok(T, p.N);
  const int NB = (T + TOK - 1) / TOK, T_pad = NB * TOK, rows = 3 * TOK;
  void *dbuf = nullptr, *qbuf = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * rows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  if ((rc = int8_map(&p.tm_d, static_cast<int8_t *>(dbuf), (long)NB * rows, K, rows))) return rc;
  p.dq = static_cast<float *>(qbuf);
  if ((rc = digit_rows(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), x, x_stride, T, T_pad, K, TOK, st)))
    return rc;
  return TOK == 64 ? gemm_launch<1, 64>(p, st) : gemm_launch<1, 32>(p, st);
}

// Shapes the tensor-core GEMMs take: K a multiple of 16 (TMA row pitch) and
// at least one 128-byte tile, at least one 128-row weight tile, 16-byte
// aligned rows.
static bool gemm_shape_ok(const float *x, long x_stride, int T, int K, int N) {
  return T > 0 && K >= 128 && K % 16 == 0 && N >= 128 && !(reinterpret_cast<uintptr_t>(x) & 15) && !(x_stride & 3) &&
         (long)((N + 127) / 128) * ((T + kGTok - 1) / kGTok) < (1l << 30);
}

int int8_gemm(float *y, long y_stride, const float *x, long x_stride, const int8_t *w, const float *scales,
              const float *bias, int T, int K, int N, cudaStream_t st) {
  if (!gemm_shape_ok(x, x_stride, T, K, N) || (reinterpret_cast<uintptr_t>(w) & 15)) return QASR_ERR_UNSUPPORTED;
  GemmParams p{};
  if (int rc = int8_map(&p.tm_w, w, N, K, 128)) return rc;
  p.scales = scales;
  p.bias = bias;
  p.y = y;
  p.y_stride = y_stride;
  p.T = T;
  p.K = K;
  p.N = N;
  return int8_gemm_run(p, x, x_stride, st);
}

// int8_gemm with a fused epilogue: kGemmResidual adds the result to y (the
// residual stream: add_inplace of the projection), kGemmSwiGLU turns each
// interleaved (gate, up) row pair into silu(g) * u at y[t, row / 2].
int int8_gemm_epi(float *y, long y_stride, const float *x, long x_stride, const int8_t *w, const float *scales, int T,
                  int K, int N, int epi, cudaStream_t st) {
  if (!gemm_shape_ok(x, x_stride, T, K, N) || (reinterpret_cast<uintptr_t>(w) & 15) || (epi == kGemmSwiGLU && N % 128))
    return QASR_ERR_UNSUPPORTED;
  GemmParams p{};
  if (int rc = int8_map(&p.tm_w, w, N, K, 128)) return rc;
  p.scales = scales;
  p.y = y;
  p.y_stride = y_stride;
  p.T = T;
  p.K = K;
  p.N = N;
  p.epi = epi;
  return int8_gemm_run(p, x, x_stride, st);
}

// int8_gemm over one weight matrix whose row ranges [0, n1), [n1, n2),
// [n2, N) are written to three outputs (the fused q|k|v projection of the
// prefill: the activation digits are made once).
int int8_gemm_split3(float *y0, long s0, float *y1, long s1, int n1, float *y2, long s2, int n2, const float *x,
                     long x_stride, const int8_t *w, const float *scales, int T, int K, int N, cudaStream_t st) {
  if (!gemm_shape_ok(x, x_stride, T, K, N) || (reinterpret_cast<uintptr_t>(w) & 15) || n1 % 128 || n2 % 128 ||
      !(0 < n1 && n1 <= n2 && n2 <= N))
    return QASR_ERR_UNSUPPORTED;
  GemmParams p{};
  if (int rc = int8_map(&p.tm_w, w, N, K, 128)) return rc;
  p.scales = scales;
  p.y = y0;
  p.y_stride = s0;
  p.y1 = y1;
  p.y1_stride = s1;
  p.n1 = n1;
  p.y2 = y2;
  p.y2_stride = s2;
  p.n2 = n2;
  p.T = T;
  p.K = K;
  p.N = N;
  return int8_gemm_run(p, x, x_stride, st);
}

int f32_gemm(float *y, long y_stride, const float *x, long x_stride, const float *w, const float *bias, int T, int K,
             int N, cudaStream_t st) {
  if (!gemm_shape_ok(x, x_stride, T, K, N) || (reinterpret_cast<uintptr_t>(w) & 15)) return QASR_ERR_UNSUPPORTED;
  const int NB = (T + kGTok - 1) / kGTok, T_pad = NB * kGTok;
  void *dbuf = nullptr, *qbuf = nullptr, *wbuf = nullptr, *wq = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * kGRows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  if ((rc = dev_scratch(kScratchWeightDigits, (size_t)3 * N * K, &wbuf))) return rc;
  if ((rc = dev_scratch(kScratchWeightScale, (size_t)N * 4, &wq))) return rc;
  GemmParams p{};
  if ((rc = int8_map(&p.tm_w, static_cast<int8_t *>(wbuf), 3l * N, K, 128))) return rc;
  if ((rc = int8_map(&p.tm_d, static_cast<int8_t *>(dbuf), (long)NB * kGRows, K, kGRows))) return rc;
  p.dq = static_cast<float *>(qbuf);
  p.scales = static_cast<float *>(wq);
  p.bias = bias;
  p.y = y;
  p.y_stride = y_stride;
  p.T = T;
  p.K = K;
  p.N = N;
  // weight digit planes: rows of plane a at a*N (one block of N rows)
  if ((rc = digit_rows(static_cast<int8_t *>(wbuf), static_cast<float *>(wq), w, K, N, N, K, N, st))) return rc;
  if ((rc = digit_rows(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), x, x_stride, T, T_pad, K, kGTok, st)))
    return rc;
  return gemm_launch<3, kGTok>(p, st);
}

// f32 weights [N, K] converted once into their three digit planes (rows of
// plane a at a*N) and per-row factors, with the tensor map: the constant
// operand of f32_gemm_prepared.
int f32_weight_prepare(F32Weight *pw, const float *w, int N, int K, cudaStream_t st) {
  *pw = F32Weight{};
  if (!w || N < 128 || K < 128 || K % 16 || (reinterpret_cast<uintptr_t>(w) & 15)) return QASR_ERR_UNSUPPORTED;
  int rc = cuda_status(cudaMalloc(&pw->planes, (size_t)3 * N * K), "f32 weight digits");
  if (!rc) rc = cuda_status(cudaMalloc(&pw->factors, (size_t)N * 4), "f32 weight factors");
  if (!rc) rc = int8_map(&pw->tm, pw->planes, 3l * N, K, 128);
  if (!rc) rc = digit_rows(pw->planes, pw->factors, w, K, N, N, K, N, st);
  if (rc) {
    f32_weight_free(pw);
    return rc;
  }
  pw->N = N;
  pw->K = K;
  return QASR_OK;
}

void f32_weight_free(F32Weight *pw) {
  if (pw->planes) cudaFree(pw->planes);
  if (pw->factors) cudaFree(pw->factors);
  *pw = F32Weight{};
}

// f32_gemm with the weight operand prepared: only the activation rows are
// converted per call.
int f32_gemm_prepared(float *y, long y_stride, const float *x, long x_stride, const F32Weight &w, const float *bias,
                      int T, cudaStream_t st) {
  if (!w.planes || !gemm_shape_ok(x, x_stride, T, w.K, w.N)) return QASR_ERR_UNSUPPORTED;
  const int K = w.K, NB = (T + kGTok - 1) / kGTok, T_pad = NB * kGTok;
  void *dbuf = nullptr, *qbuf = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * kGRows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  GemmParams p{};
  p.tm_w = w.tm;
  if ((rc = int8_map(&p.tm_d, static_cast<int8_t *>(dbuf), (long)NB * kGRows, K, kGRows))) return rc;
  p.dq = static_cast<float *>(qbuf);
  p.scales = w.factors;
  p.bias = bias;
  p.y = y;
  p.y_stride = y_stride;
  p.T = T;
  p.K = K;
  p.N = w.N;
  if ((rc = digit_rows(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), x, x_stride, T, T_pad, K, kGTok, st)))
    return rc;
  return gemm_launch<3, kGTok>(p, st);
}

// A 3x3, stride-2, padding-1 convolution of the channel-last activation act
// [B, h_in, w_in, C] as an implicit GEMM: the digit rows of its patches come
// straight from act (conv_digit_rows_kernel), y [B*h_out*w_out, w.N] = patches
// x w^T (+ bias), with w the weights in the channel-fastest patch order.
int f32_gemm_prepared_conv(float *y, long y_stride, const float *act, int C, int h_in, int w_in, int B, int h_out,
                           int w_out, const F32Weight &w, const float *bias, cudaStream_t st) {
  const long T = (long)B * h_out * w_out;
  if (!w.planes || C % 4 || w.K != 9 * C || T <= 0 || T >= (1l << 30) || (long)B * h_in * w_in * C >= (1l << 31) ||
      (reinterpret_cast<uintptr_t>(act) & 15) || !gemm_shape_ok(act, w.K, (int)T, w.K, w.N))
    return QASR_ERR_UNSUPPORTED;
  const int K = w.K, NB = (int)((T + kGTok - 1) / kGTok), T_pad = NB * kGTok;
  void *dbuf = nullptr, *qbuf = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * kGRows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  GemmParams p{};
  p.tm_w = w.tm;
  if ((rc = int8_map(&p.tm_d, static_cast<int8_t *>(dbuf), (long)NB * kGRows, K, kGRows))) return rc;
  p.dq = static_cast<float *>(qbuf);
  p.scales = w.factors;
  p.bias = bias;
  p.y = y;
  p.y_stride = y_stride;
  p.T = (int)T;
  p.K = K;
  p.N = w.N;
  conv_digit_rows_kernel<<<(T_pad + 7) / 8, 256, 0, st>>>(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), act,
                                                          C, h_in, w_in, h_out,
                                                          w_out, (int)T, T_pad, kGTok);
  if ((rc = launch_status("tensor-core GEMM: conv digit rows"))) return rc;
  return gemm_launch<3, kGTok>(p, st);
}

// f32_gemm_prepared over a weight whose row ranges [0, n1), [n1, n2),
// [n2, N) go to three outputs (the encoder's fused q|k|v projection: one
// activation digit pass and one launch for the three).
int f32_gemm_prepared_split3(float *y0, long s0, float *y1, long s1, int n1, float *y2, long s2, int n2,
                             const float *x, long x_stride, const F32Weight &w, const float *bias, int T,
                             cudaStream_t st) {
  if (!w.planes || !gemm_shape_ok(x, x_stride, T, w.K, w.N) || n1 % 128 || n2 % 128 || !(0 < n1 && n1 <= n2 && n2 <= w.N))
    return QASR_ERR_UNSUPPORTED;
  const int K = w.K, NB = (T + kGTok - 1) / kGTok, T_pad = NB * kGTok;
  void *dbuf = nullptr, *qbuf = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * kGRows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  GemmParams p{};
  p.tm_w = w.tm;
  if ((rc = int8_map(&p.tm_d, static_cast<int8_t *>(dbuf), (long)NB * kGRows, K, kGRows))) return rc;
  p.dq = static_cast<float *>(qbuf);
  p.scales = w.factors;
  p.bias = bias;
  p.y = y0;
  p.y_stride = s0;
  p.y1 = y1;
  p.y1_stride = s1;
  p.n1 = n1;
  p.y2 = y2;
  p.y2_stride = s2;
  p.n2 = n2;
  p.T = T;
  p.K = K;
  p.N = w.N;
  if ((rc = digit_rows(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), x, x_stride, T, T_pad, K, kGTok, st)))
    return rc;
  return gemm_launch<3, kGTok>(p, st);
}

// ------------------------------------------------- CUDA-core fallback SGEMM --
// y[t, o] = sum_k x[t, k] w[o, k] (+ b[o]) for shapes the tensor-core GEMM
// does not take (K not a multiple of 16, unaligned rows): 32x32 output tiles,
// K staged through shared memory, f32 accumulation in k order.
__global__ void __launch_bounds__(256) sgemm_nt_kernel(float *__restrict__ y, const float *__restrict__ x,
                                                       const float *__restrict__ w, const float *__restrict__ b,
                                                       int T, int K, int N) {
  __shared__ float xs[32][33], ws[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows of 4 outputs per thread
  const int t0 = blockIdx.y * 32, o0 = blockIdx.x * 32;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < K; k0 += 32) {
    for (int i = ty; i < 32; i += 8) {
      xs[i][tx] = (t0 + i < T && k0 + tx < K) ? x[(size_t)(t0 + i) * K + k0 + tx] : 0.0f;
      ws[i][tx] = (o0 + i < N && k0 + tx < K) ? w[(size_t)(o0 + i) * K + k0 + tx] : 0.0f;
    }
    __syncthreads();
    for (int kk = 0; kk < 32; ++kk)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[r] = fmaf(xs[ty + 8 * r][kk], ws[tx][kk], acc[r]);
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int t = t0 + ty + 8 * r, o = o0 + tx;
    if (t < T && o < N) y[(size_t)t * N + o] = b ? __fadd_rn(acc[r], b[o]) : acc[r];
  }
}

int f32_gemm_fallback(float *y, const float *x, const float *w, const float *bias, int T, int K, int N,
                      cudaStream_t st) {
  dim3 grid((N + 31) / 32, (T + 31) / 32);
  sgemm_nt_kernel<<<grid, 256, 0, st>>>(y, x, w, bias, T, K, N);
  return launch_status("f32 GEMM (CUDA cores)");
}

}  // namespace qasr

using namespace qasr;

static int linear_f32_impl(const char *fn, float *y, const float *x, const float *w, const float *b, int seq,
                           int in_dim, int out_dim, void *stream) {
  if (!y || !x || !w || seq < 0 || in_dim <= 0 || out_dim <= 0) {
    set_error("%s: invalid arguments", fn);
    return QASR_ERR_INVALID;
  }
  if (seq == 0) return QASR_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = f32_gemm(y, out_dim, x, in_dim, w, b, seq, in_dim, out_dim, st);
  if (rc != QASR_ERR_UNSUPPORTED) return rc;
  return f32_gemm_fallback(y, x, w, b, seq, in_dim, out_dim, st);
}

extern "C" int qasr_linear(float *y, const float *x, const float *w, const float *b, int seq, int in_dim,
                           int out_dim, void *stream) {
  return linear_f32_impl("qasr_linear", y, x, w, b, seq, in_dim, out_dim, stream);
}

extern "C" int qasr_linear_nobias(float *y, const float *x, const float *w, int seq, int in_dim, int out_dim,
                                  void *stream) {
  return linear_f32_impl("qasr_linear_nobias", y, x, w, nullptr, seq, in_dim, out_dim, stream);
}

extern "C" int qasr_matmul_t(float *c, const float *a, const float *b, int m, int k, int n, void *stream) {
  return linear_f32_impl("qasr_matmul_t", c, a, b, nullptr, m, k, n, stream);
}
