// umma_gemm.cu -- INT8-weight GEMM for many token rows on the tcgen05 tensor
// cores: the prefill and encoder projections, kernels::linear_nobias_int8 /
// linear_int8 with seq_len > 8 (crates/qwen-asr/src/kernels/mod.rs:650-673,
// which the reference runs as seq_len sequential matvecs of
// generic::int8_matvec_fused, generic.rs:39-49).
//
// Same exact integer formulation as the decode contraction (umma_matvec.cu):
// every activation row t is scaled by 2^(22-E_t) (2^E_t bounds its largest
// magnitude), rounded to an integer X with |X| <= 2^22 and split into three
// balanced signed bytes X = 65536*d0 + 256*d1 + d2.  The tensor cores contract
// the int8 weights with the digit rows exactly in 32-bit integers; the
// epilogue recombines the digits in 64 bits and rounds once.
//
//  * digit_rows_kernel: one warp per token row writes its three digit rows
//    into token blocks of 32: block b holds rows d*32 + t (d = digit, t =
//    token in block), 96 rows of K bytes, plus the row's dequantisation
//    factor 2^(E-22).
//  * int8_gemm_kernel: persistent; output tiles of 128 weight rows x one token
//    block, taken row-tile-major with the token block fastest so the CTAs
//    sharing a weight tile run together and the tile is read from HBM once.
//    One thread streams the weight tile and the digit tile of every 128-byte
//    K step with 2D TMA loads (128-byte swizzle, no multicast) into a 4-stage
//    ring; one thread issues tcgen05.mma kind::i8 (M=128, N=96, K=32) into a
//    double-buffered TMEM accumulator; four epilogue warps read it with
//    tcgen05.ld (thread = output row) and write y (+bias), coalesced over rows.
// Every wait is bounded; a timeout sets *err, stops the roles, drains the
// copies and MMAs in flight and frees TMEM.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "matvec.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kGTok = 32;                 // tokens per block
constexpr int kGRows = 3 * kGTok;         // digit rows per block (MMA N)
constexpr int kGStages = 4;
constexpr int kGATile = 128 * 128;        // weight tile bytes
constexpr int kGBTile = kGRows * 128;     // digit tile bytes
constexpr int kGTmemCols = 256;           // two 96-column accumulators
constexpr uint32_t kGIdesc = umma_idesc_s8(128, kGRows);

// ---------------------------------------------------------------- digits --
__global__ void __launch_bounds__(256) digit_rows_kernel(int8_t *__restrict__ D, float *__restrict__ dq,
                                                         const float *__restrict__ x, long x_stride, int T, int K,
                                                         int T_pad) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T_pad) return;
  const int b = t / kGTok, tl = t % kGTok;
  int8_t *row0 = D + ((size_t)b * kGRows + tl) * K;  // digit d at row0 + d*kGTok*K
  const size_t dstep = (size_t)kGTok * K;
  if (t >= T) {  // tokens past the end of the last block: zero digits
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
  int e = 0;
  if (mx > 0.0f && mx <= 3.0e38f) frexpf(mx, &e);  // mx < 2^e
  e = max(-100, min(e, 127));
  const float qm = __int_as_float((127 + 22 - e) << 23);
  if (lane == 0) dq[t] = __int_as_float((127 + e - 22) << 23);
  for (int k4 = lane; k4 < K / 4; k4 += 32) {
    const float4 v = xr[k4];  // L1 hit: read just above
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
    for (int d = 0; d < 3; ++d) *reinterpret_cast<uint32_t *>(row0 + d * dstep + 4 * k4) = w[d];
  }
}

// ------------------------------------------------------------------ GEMM --
struct GemmParams {
  CUtensorMap tm_w;  // [N, K] int8, box 128 x 128, SW128
  CUtensorMap tm_d;  // [blocks*96, K] int8 digit rows, box 96 x 128, SW128
  const float *dq;   // [blocks*32]
  const float *scales, *bias;
  float *y;          // [T, N], row stride y_stride
  long y_stride;
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

__global__ void __launch_bounds__(256, 1) int8_gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  unsigned char *a_ring = base;
  unsigned char *b_ring = a_ring + (size_t)kGStages * kGATile;
  GSmem &sm = *reinterpret_cast<GSmem *>(b_ring + (size_t)kGStages * kGBTile);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = p.K / 128, NT = (p.N + 127) / 128, NB = (p.T + kGTok - 1) / kGTok;
  const int tiles = NT * NB;
  const int my_tiles = (int)blockIdx.x < tiles ? (tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int nu = my_tiles * KT;  // pipeline items (tile j, K step kt)
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
  if (warp == 5) tmem_alloc(&sm.tmem, kGTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  pdl_wait();
  pdl_launch_dependents();

  int produced = 0;
  auto produce = [&](int i) {
    const int st = i % kGStages, tile = tile_of(i / KT), kt = i % KT;
    const int rt = tile / NB, tb = tile % NB;
    mbar_arrive_expect_tx(&sm.full[st], kGATile + kGBTile);
    tma_load_2d_u8(a_ring + (size_t)st * kGATile, &p.tm_w, kt * 128, rt * 128, &sm.full[st]);
    tma_load_2d_u8(b_ring + (size_t)st * kGBTile, &p.tm_d, kt * 128, tb * kGRows, &sm.full[st]);
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
        const int j = i / KT, kt = i % KT, st = i % kGStages, buf = j & 1;
        if (kt == 0 && j >= 2 && !mbar_wait(&sm.accempty[buf], (unsigned)(((j >> 1) - 1) & 1))) {
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
        const uint32_t b_addr = smem_u32(b_ring + (size_t)st * kGBTile);
        const uint32_t d_addr = tmem + (uint32_t)(buf * 128);
#pragma unroll
        for (int s = 0; s < 4; ++s)
          umma_s8(d_addr, umma_desc_sw128(a_addr + 32 * s), umma_desc_sw128(b_addr + 32 * s), kGIdesc,
                  (kt == 0 && s == 0) ? 0u : 1u);
        umma_commit(&sm.empty[st]);
        if (kt == KT - 1) umma_commit(&sm.accfull[buf]);
      }
      umma_commit(&sm.done);
      if (!mbar_wait(&sm.done, 0)) g_fail(sm, p.err);
    }
  } else if (warp < 4) {
    const int ri = warp * 32 + lane;
    for (int j = 0; j < my_tiles; ++j) {
      const int tile = tile_of(j), buf = j & 1;
      const int rt = tile / NB, tb = tile % NB;
      if (!g_aborted(sm) && !mbar_wait(&sm.accfull[buf], (unsigned)((j >> 1) & 1))) g_fail(sm, p.err);
      named_bar(1, 128);  // the four epilogue warps decide together
      if (g_aborted(sm)) break;
      tc_fence_after();
      uint32_t a0[32], a1[32], a2[32];
      const uint32_t taddr = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(buf * 128);
      tmem_ld32(taddr, a0);
      tmem_ld32(taddr + 32, a1);
      tmem_ld32(taddr + 64, a2);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.accempty[buf])) : "memory");
      const int row = rt * 128 + ri;
      if (row < p.N) {
        const float sc = p.scales[row];
        const float b = p.bias ? p.bias[row] : 0.0f;
        const int t0 = tb * kGTok;
#pragma unroll
        for (int tl = 0; tl < kGTok; ++tl) {
          const int t = t0 + tl;
          if (t < p.T) {
            const long long V = ((long long)(int)a0[tl] << 16) + ((long long)(int)a1[tl] << 8) + (long long)(int)a2[tl];
            float v = __fmul_rn(__fmul_rn(__ll2float_rn(V), __ldg(p.dq + t)), sc);
            if (p.bias) v = __fadd_rn(v, b);
            p.y[(size_t)t * p.y_stride + row] = v;
          }
        }
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
    tmem_dealloc(tmem, kGTmemCols);
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

static int digit_map(CUtensorMap *tm, const int8_t *D, int rows, int K) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  auto encode = reinterpret_cast<Encode>(tensor_map_encoder());
  if (!encode) {
    set_error("int8 tensor-core GEMM: cuTensorMapEncodeTiled unavailable");
    return QASR_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K};
  const cuuint32_t box[2] = {128, (cuuint32_t)kGRows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<int8_t *>(D), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("int8 tensor-core GEMM: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

// y[t, o] = scales[o] * sum_k w[o, k] * x[t, k] (+ bias[o]) for T token rows.
// QASR_ERR_UNSUPPORTED (nothing launched) for shapes it does not cover.
int int8_gemm(float *y, long y_stride, const float *x, long x_stride, const int8_t *w, const float *scales,
              const float *bias, int T, int K, int N, cudaStream_t st) {
  if (T <= 0 || K <= 0 || K % 128 || N <= 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (x_stride & 3) ||
      (reinterpret_cast<uintptr_t>(w) & 15))
    return QASR_ERR_UNSUPPORTED;
  const int NB = (T + kGTok - 1) / kGTok, T_pad = NB * kGTok;
  void *dbuf = nullptr, *qbuf = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchDigits, (size_t)NB * kGRows * K, &dbuf))) return rc;
  if ((rc = dev_scratch(kScratchDigitScale, (size_t)T_pad * 4, &qbuf))) return rc;
  GemmParams p{};
  if ((rc = umma_weight_map(&p.tm_w, w, N, K))) return rc;
  if ((rc = digit_map(&p.tm_d, static_cast<int8_t *>(dbuf), NB * kGRows, K))) return rc;
  p.dq = static_cast<float *>(qbuf);
  p.scales = scales;
  p.bias = bias;
  p.y = y;
  p.y_stride = y_stride;
  p.T = T;
  p.K = K;
  p.N = N;
  digit_rows_kernel<<<(T_pad + 7) / 8, 256, 0, st>>>(static_cast<int8_t *>(dbuf), static_cast<float *>(qbuf), x,
                                                      x_stride, T, K, T_pad);
  if ((rc = launch_status("int8 tensor-core GEMM: digit rows"))) return rc;
  static int attr_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  const size_t smem = 1024 + (size_t)kGStages * (kGATile + kGBTile) + sizeof(GSmem);
  if (dev < 31 && !(attr_mask & (1 << dev))) {
    if ((rc = cuda_status(cudaFuncSetAttribute(int8_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                          "int8 tensor-core GEMM: shared memory opt-in")))
      return rc;
    attr_mask |= 1 << dev;
  }
  const long tiles = (long)((N + 127) / 128) * NB;
  const int grid = (int)std::min<long>(gemm_sms(), tiles);
  int8_gemm_kernel<<<grid, 256, smem, st>>>(p);
  return launch_status("int8 tensor-core GEMM");
}

}  // namespace qasr
