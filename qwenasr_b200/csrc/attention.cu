// attention.cu -- GQA causal attention (kernels::causal_attention,
// crates/qwen-asr/src/kernels/mod.rs:1124-1207).
//
// Two kernels:
//  * causal_attention_kernel: the general kernel-level entry (any seq_q,
//    e.g. prefill).  One warp per (query, head), lanes over head dims, the
//    reference's per-key online softmax update (mod.rs:1154-1164).
//  * attn_decode_kernel: the decode step of the engine.  Flash-decoding over
//    the f32 KV cache: the keys of one (sequence, kv head) are split across
//    CTAs, each CTA serves both query heads of the GQA group so every K/V row
//    is read from HBM exactly once, and the last CTA of a (sequence, kv head)
//    merges the partial softmax states (counter + threadfence, no spin).
#include <cudaTypedefs.h>

#include "attention.cuh"
#include "common.cuh"
#include "tma.cuh"

namespace qasr {

// ------------------------------------------------------------------ general
template <int EPL>  // elements per lane: head_dim / 32
__global__ void __launch_bounds__(256)
causal_attention_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ k,
                        const float *__restrict__ v, int seq_q, int seq_k, int n_heads, int n_kv_heads, float scale,
                        int q_offset) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long task = (long)blockIdx.x * 8 + warp;
  if (task >= (long)seq_q * n_heads) return;
  const int i = (int)(task / n_heads), h = (int)(task % n_heads);
  const int hd = EPL * 32;
  const int kv_h = h / (n_heads / n_kv_heads);
  const long q_hidden = (long)n_heads * hd, kv_hidden = (long)n_kv_heads * hd;
  float qv[EPL], o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qv[e] = q[i * q_hidden + (long)h * hd + lane * EPL + e];
    o[e] = 0.0f;
  }
  const int k_end = min(q_offset + i + 1, seq_k);
  float max_score = -1e30f, sum_exp = 0.0f;
  for (int j = 0; j < k_end; ++j) {
    const float *kr = k + j * kv_hidden + (long)kv_h * hd + lane * EPL;
    const float *vr = v + j * kv_hidden + (long)kv_h * hd + lane * EPL;
    float d = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) d = fmaf(qv[e], kr[e], d);
    const float score = __fmul_rn(warp_sum(d), scale);
    if (score > max_score) {
      const float corr = expf(__fsub_rn(max_score, score));
      sum_exp = __fadd_rn(__fmul_rn(sum_exp, corr), 1.0f);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(o[e], corr, vr[e]);
      max_score = score;
    } else {
      const float wt = expf(__fsub_rn(score, max_score));
      sum_exp = __fadd_rn(sum_exp, wt);
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(vr[e], wt, o[e]);
    }
  }
  const float inv = sum_exp > 0.0f ? __fdiv_rn(1.0f, sum_exp) : 0.0f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) out[i * q_hidden + (long)h * hd + lane * EPL + e] = sum_exp > 0.0f ? __fmul_rn(o[e], inv) : o[e];
}

// ------------------------------------------------------------------- decode
// Persistent flash-decoding.  The keys of all (sequence, kv head) pairs are
// laid end to end and cut into gridDim equal ranges, so every SM streams the
// same number of K/V bytes whatever the batch and lengths.  A CTA walks its
// range as segments (one per pair it touches) of 64-key tiles; thread 0 keeps
// kAttnStages K+V tile pairs in flight with 2D TMA loads (box: 64 rows x one
// 128-float head slice, no multicast).  Each of the 4 warps scores 16 keys of
// a tile for both query heads of the GQA group (every K/V byte is read from
// HBM once), keeps an online-softmax state, and the CTA merges its warps at
// the end of a segment.  A pair split over several CTAs is merged by the last
// one to finish (counter + threadfence, slots in CTA order: deterministic).
struct AttnSmall {
  uint64_t bar[kAttnStages];
  int nseg;
  int seg_pair[128], seg_a[128], seg_b[128];
};

QASR_DEV void tma_load_2d(float *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <int G>
__global__ void __launch_bounds__(kAttnWarps * 32, 1)
attn_decode_kernel(const __grid_constant__ AttnDecodeParams p) {
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int TILE_F = kAttnTile * 128;  // floats per K (or V) tile
  float *tiles = reinterpret_cast<float *>(smem_raw);
  AttnSmall &sm = *reinterpret_cast<AttnSmall *>(smem_raw + (size_t)kAttnStages * 2 * TILE_F * 4);
  // warp w serves query head (w % G) of the group on key group (w / G) of
  // each tile: KPW keys per warp
  constexpr int KPW = kAttnTile * G / kAttnWarps;
  __shared__ float sp[kAttnWarps][KPW];
  __shared__ float wm[kAttnWarps], wl[kAttnWarps];
  __shared__ float4 wo[kAttnWarps][32];
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = p.n_kv_heads, n_pairs = p.M * n_kv;
  auto len_of = [&](int pair) { return max(1, min(p.positions[pair / n_kv] + 1, p.max_seq)); };
  long long Tk = 0;
  for (int pr = 0; pr < n_pairs; ++pr) Tk += len_of(pr);
  // Virtual grid: with fewer keys than CTAs, only the first Tk CTAs take part,
  // so every participating CTA owns at least one key and the CTAs covering a
  // pair are exactly c_of(first key) .. c_of(last key).
  const long long Gd = min((long long)gridDim.x, Tk), c = blockIdx.x;
  if (c >= Gd) return;
  const long long t0 = c * Tk / Gd, t1 = (c + 1) * Tk / Gd;

  if (threadIdx.x == 0) {
    int ns = 0;
    long long off = 0;
    for (int pr = 0; pr < n_pairs && ns < 128; ++pr) {
      const long long len = len_of(pr);
      const long long a = max(off, t0), b = min(off + len, t1);
      if (a < b) {
        sm.seg_pair[ns] = pr;
        sm.seg_a[ns] = (int)(a - off);
        sm.seg_b[ns] = (int)(b - off);
        ++ns;
      }
      off += len;
    }
    sm.nseg = ns;
    for (int st = 0; st < kAttnStages; ++st) mbar_init(&sm.bar[st], 1);
  }
  mbar_fence_init();
  __syncthreads();
  const int nseg = sm.nseg;

  // tile cursor shared by producer and consumers (advanced in the same order)
  auto tiles_of = [&](int sg) { return (sm.seg_b[sg] - sm.seg_a[sg] + kAttnTile - 1) / kAttnTile; };
  int total = 0;
  for (int sg = 0; sg < nseg; ++sg) total += tiles_of(sg);

  int is = 0, it = 0;  // producer cursor (thread 0)
  auto issue_next = [&](int item) {
    while (it >= tiles_of(is)) {
      it = 0;
      ++is;
    }
    const int pr = sm.seg_pair[is], m = pr / n_kv, kvh = pr % n_kv;
    const int row = (m * p.n_layers + p.layer) * p.max_seq + sm.seg_a[is] + it * kAttnTile;
    const int st = item % kAttnStages;
    mbar_arrive_expect_tx(&sm.bar[st], 2 * TILE_F * 4);
    tma_load_2d(tiles + (size_t)(2 * st) * TILE_F, &p.tm_k, kvh * 128, row, &sm.bar[st]);
    tma_load_2d(tiles + (size_t)(2 * st + 1) * TILE_F, &p.tm_v, kvh * 128, row, &sm.bar[st]);
    ++it;
  };
  // q and the newest K/V row are written by the previous kernel: wait for it
  // before the first tile load (the tile holding the newest row may be any)
  pdl_wait();
  pdl_launch_dependents();
  if (threadIdx.x == 0)
    for (int i = 0; i < total && i < kAttnStages; ++i) issue_next(i);

  const int hg = warp % G, kgrp = warp / G;  // this warp's head in the group, key group
  float mx = -INFINITY, sum = 0.0f;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f), qv = o;
  int cs = 0, ct = 0;  // consumer cursor
  int cur_pair = -1;
  const int my_key = reduce_index<KPW>(lane);
  const bool writer = (lane & (32 / KPW - 1)) == 0;
  for (int i = 0; i < total; ++i) {
    while (ct >= tiles_of(cs)) {
      ct = 0;
      ++cs;
    }
    const int pr = sm.seg_pair[cs], m = pr / n_kv, kvh = pr % n_kv;
    if (pr != cur_pair) {  // new segment: load q, reset state
      cur_pair = pr;
      qv = *reinterpret_cast<const float4 *>(p.q + (size_t)m * p.q_stride + (kvh * G + hg) * 128 + 4 * lane);
      mx = -INFINITY;
      sum = 0.0f;
      o = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const int st = i % kAttnStages;
    const bool ok = mbar_wait(&sm.bar[st], (unsigned)((i / kAttnStages) & 1));
    if (__syncthreads_or(!ok)) {
      if (threadIdx.x == 0 && p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
      for (int k2 = i; k2 < total && k2 < i + kAttnStages; ++k2)
        mbar_wait(&sm.bar[k2 % kAttnStages], (unsigned)((k2 / kAttnStages) & 1));
      return;
    }
    const float *kt = tiles + (size_t)(2 * st) * TILE_F;
    const float *vt = tiles + (size_t)(2 * st + 1) * TILE_F;
    const int nk = min(kAttnTile, sm.seg_b[cs] - sm.seg_a[cs] - ct * kAttnTile);
    const int k0 = kgrp * KPW;
    const int nkw = max(0, min(KPW, nk - k0));  // keys of this warp in the tile
    if (nkw > 0) {
      float part[KPW];
#pragma unroll
      for (int j = 0; j < KPW; ++j) {
        const float4 kv = *reinterpret_cast<const float4 *>(kt + (size_t)(k0 + j) * 128 + 4 * lane);
        float d = __fmul_rn(qv.x, kv.x);
        d = fmaf(qv.y, kv.y, d);
        d = fmaf(qv.z, kv.z, d);
        d = fmaf(qv.w, kv.w, d);
        part[j] = d;
      }
      const float tot = warp_reduce_scatter<KPW>(part);
      const bool live = my_key < nkw;
      const float sc = live ? __fmul_rn(tot, p.scale) : -INFINITY;
      const float nmax = fmaxf(mx, warp_max(sc));
      const float corr = mx == -INFINITY ? 0.0f : expf(__fsub_rn(mx, nmax));
      const float pj = live ? expf(__fsub_rn(sc, nmax)) : 0.0f;
      sum = __fadd_rn(__fmul_rn(sum, corr), warp_sum(writer ? pj : 0.0f));
      mx = nmax;
      if (writer) sp[warp][my_key] = pj;
      __syncwarp();
      o.x = __fmul_rn(o.x, corr);
      o.y = __fmul_rn(o.y, corr);
      o.z = __fmul_rn(o.z, corr);
      o.w = __fmul_rn(o.w, corr);
#pragma unroll
      for (int j = 0; j < KPW; ++j) {
        if (j < nkw) {
          const float4 vv = *reinterpret_cast<const float4 *>(vt + (size_t)(k0 + j) * 128 + 4 * lane);
          const float w = sp[warp][j];
          o.x = fmaf(w, vv.x, o.x);
          o.y = fmaf(w, vv.y, o.y);
          o.z = fmaf(w, vv.z, o.z);
          o.w = fmaf(w, vv.w, o.w);
        }
      }
      __syncwarp();
    }
    __syncthreads();  // every warp is done with stage st
    if (threadIdx.x == 0 && i + kAttnStages < total) {
      fence_proxy_async();
      issue_next(i + kAttnStages);
    }
    ++ct;
    if (ct < tiles_of(cs)) continue;

    // ---- end of segment: merge the warps of each head ----
    if (lane == 0) {
      wm[warp] = mx;
      wl[warp] = sum;
    }
    wo[warp][lane] = o;
    __syncthreads();
    // CTAs covering this pair: c_of(t) = floor(((t+1)*Gd - 1) / Tk)
    long long off = 0;
    for (int q2 = 0; q2 < pr; ++q2) off += len_of(q2);
    const long long len = len_of(pr);
    const long long c_first = ((off + 1) * Gd - 1) / Tk, c_last = ((off + len) * Gd - 1) / Tk;
    const bool alone = c_first == c_last;
    if (warp < G) {
      const int g = warp;
      float Mx = -INFINITY;
      for (int w = g; w < kAttnWarps; w += G) Mx = fmaxf(Mx, wm[w]);
      float L = 0.0f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = g; w < kAttnWarps; w += G) {
        const float f = wm[w] == -INFINITY ? 0.0f : expf(__fsub_rn(wm[w], Mx));
        L = __fadd_rn(L, __fmul_rn(wl[w], f));
        const float4 ov = wo[w][lane];
        acc.x = fmaf(ov.x, f, acc.x);
        acc.y = fmaf(ov.y, f, acc.y);
        acc.z = fmaf(ov.z, f, acc.z);
        acc.w = fmaf(ov.w, f, acc.w);
      }
      float *dst_out = p.out + (size_t)m * p.out_stride + (kvh * G + g) * 128;
      if (alone) {
        const float inv = __fdiv_rn(1.0f, L);
        reinterpret_cast<float4 *>(dst_out)[lane] =
            make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
      } else {
        float *slot = p.partials + ((size_t)(c + pr) * G + g) * kAttnPartStride;
        reinterpret_cast<float4 *>(slot)[lane] = acc;
        if (lane == 0) {
          slot[128] = Mx;
          slot[129] = L;
        }
      }
    }
    if (!alone) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) s_last = atomicAdd(p.counters + pr, 1u) == (unsigned)(c_last - c_first);
      __syncthreads();
      if (s_last) {
        __threadfence();
        if (warp < G) {
          const int g = warp;
          float Mx = -INFINITY;
          for (long long c2 = c_first; c2 <= c_last; ++c2)
            Mx = fmaxf(Mx, __ldcg(p.partials + ((size_t)(c2 + pr) * G + g) * kAttnPartStride + 128));
          float L = 0.0f;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (long long c2 = c_first; c2 <= c_last; ++c2) {
            const float *ps = p.partials + ((size_t)(c2 + pr) * G + g) * kAttnPartStride;
            const float ms = __ldcg(ps + 128);
            const float f = ms == -INFINITY ? 0.0f : expf(__fsub_rn(ms, Mx));
            L = __fadd_rn(L, __fmul_rn(__ldcg(ps + 129), f));
            const float4 ov = __ldcg(reinterpret_cast<const float4 *>(ps) + lane);
            acc.x = fmaf(ov.x, f, acc.x);
            acc.y = fmaf(ov.y, f, acc.y);
            acc.z = fmaf(ov.z, f, acc.z);
            acc.w = fmaf(ov.w, f, acc.w);
          }
          const float inv = __fdiv_rn(1.0f, L);
          *reinterpret_cast<float4 *>(p.out + (size_t)m * p.out_stride + (kvh * G + g) * 128 + 4 * lane) =
              make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv),
                          __fmul_rn(acc.w, inv));
        }
        if (threadIdx.x == 0) p.counters[pr] = 0u;
      }
    }
    __syncthreads();
  }
}

int attn_grid() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int attn_make_tensor_map(CUtensorMap *tm, const float *base, long rows, int kv_dim) {
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  if (!encode) {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn) {
      set_error("attention: cuTensorMapEncodeTiled unavailable");
      return QASR_ERR_CUDA;
    }
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || kv_dim % 128 || rows <= 0) {
    set_error("attention: KV cache must be 16-byte aligned with kv_dim a multiple of 128");
    return QASR_ERR_INVALID;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)kv_dim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kv_dim * 4};
  const cuuint32_t box[2] = {128, (cuuint32_t)kAttnTile};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

static size_t attn_smem() {
  return (size_t)kAttnStages * 2 * kAttnTile * 128 * 4 + sizeof(AttnSmall);
}

template <int G>
static int attn_launch_t(const AttnDecodeParams &p, cudaStream_t st, bool pdl) {
  static bool attr_done = false;
  if (!attr_done) {
    int rc = cuda_status(cudaFuncSetAttribute(attn_decode_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)attn_smem()),
                         "attention: shared memory opt-in");
    if (rc) return rc;
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)attn_grid());
  cfg.blockDim = dim3(kAttnWarps * 32);
  cfg.dynamicSmemBytes = attn_smem();
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, attn_decode_kernel<G>, p), "attention launch");
}

int attn_decode_launch(const AttnDecodeParams &p, int group, cudaStream_t st, bool pdl) {
  if (p.M * p.n_kv_heads > 128) {
    set_error("attention: M*n_kv_heads = %d > 128", p.M * p.n_kv_heads);
    return QASR_ERR_UNSUPPORTED;
  }
  switch (group) {
    case 1: return attn_launch_t<1>(p, st, pdl);
    case 2: return attn_launch_t<2>(p, st, pdl);
    default:
      set_error("attention: GQA group size %d unsupported (1 or 2)", group);
      return QASR_ERR_UNSUPPORTED;
  }
}

}  // namespace qasr

using namespace qasr;

extern "C" int qasr_causal_attention(float *out, const float *q, const float *k, const float *v, int seq_q,
                                     int seq_k, int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset,
                                     void *stream) {
  if (!out || !q || !k || !v || seq_q < 0 || seq_k < 0 || n_heads <= 0 || n_kv_heads <= 0 ||
      n_heads % n_kv_heads || q_offset < 0) {
    set_error("qasr_causal_attention: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("qasr_causal_attention: head_dim %d unsupported (64 or 128)", head_dim);
    return QASR_ERR_UNSUPPORTED;
  }
  if (seq_q == 0) return QASR_OK;
  const long tasks = (long)seq_q * n_heads;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    causal_attention_kernel<4><<<ceil_div(tasks, 8), 256, 0, st>>>(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads,
                                                                   scale, q_offset);
  else
    causal_attention_kernel<2><<<ceil_div(tasks, 8), 256, 0, st>>>(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads,
                                                                   scale, q_offset);
  return launch_status("qasr_causal_attention");
}
