// decode_step.cu -- one greedy decode step of the INT8 decoder
// (decoder_forward_int8, crates/qwen-asr/src/decoder.rs:845-965, as driven by
// QwenCtx::decoder_forward_token, context.rs:311) for up to 8 independent
// sequences, as ONE persistent kernel: every layer's RMSNorm + q|k|v
// projection + q/k norm + RoPE + KV append, attention, o-proj + residual,
// RMSNorm + gate/up + SwiGLU, down + residual, then the final norm, the lm
// head and the first-max argmax.
//
// Why one kernel.  A decode step moves its weights and KV history once
// (HBM-bound), but as a chain of ~140 dependent launches each projection
// pays a fixed cost (launch, grid drain, activation staging, exit) that is
// larger than its streaming time.  Here one CTA runs on every SM for the
// whole step and the dependencies become device-side counters:
//  * the weights and the K/V history depend on nothing computed in the step,
//    so one thread per CTA streams them with 2D TMA loads (no multicast) into
//    a ring of 16 KB stages in exactly the order the CTA consumes them,
//    running ahead across phase and layer boundaries while the rest of the
//    CTA waits for the previous phase's results;
//  * each projection is cut into units (a 128-row tile x a chunk of its K
//    tiles) dealt round-robin to the CTAs.  A unit is contracted on the
//    tensor cores with the exact integer scheme of umma_matvec.cu (int8
//    weights x three signed-byte digit rows per token, tcgen05.mma kind::i8
//    into TMEM, recombined exactly in 64 bits); units of one row tile add
//    their 64-bit sums into a global accumulator (integer atomics: the
//    result does not depend on arrival order) and the last one to arrive
//    applies the epilogue (per-head q/k norm + RoPE + KV append, residual
//    add, or SwiGLU) and counts the row tile as done;
//  * attention is flash-decoding over the K/V history split evenly over the
//    CTAs (keys of all (sequence, kv head) pairs end to end), 16-key K and V
//    tiles from the same ring, both query heads of a GQA group per warp; the
//    pair's newest row (written in this step) is read after its head is
//    counted done; pairs split over CTAs are merged by the last contributor.
// Consumers wait on counters with acquire loads; producers publish with a
// fence and an atomic add.  Every wait is bounded by %globaltimer; a timeout
// (or another CTA's) sets *err, stops every role and drains the copies and
// MMAs in flight before the CTA exits.
//
// Numerics: the contractions are the exact integer scheme of the per-kernel
// path; the input RMSNorms sum the squares in a fixed warp-tree order (not
// the reference's AVX lane order: a difference of about one ulp in the norm
// factor, far inside the 2e-3 bar); SwiGLU, q/k norm and RoPE as in the
// per-kernel path.
#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#include "matvec.cuh"
#include "qkvpost.cuh"
#include "step.cuh"
#include "tcgen05.cuh"
#include "tma.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kSWorkerWarps = 8, kSProducerWarp = 8, kSMmaWarp = 9, kSKvWarp = 10, kSThreads = 352;
constexpr int kSStage = 16384;     // bytes of a ring stage: one 128x128 weight tile, or 16 K + 16 V rows
constexpr int kSMaxStages = 12;
constexpr int kSKeys = 16;         // keys per attention stage
constexpr int kSSlot = 32 * 128;   // bytes of the digit rows of one K tile
constexpr int kSMaxSeg = 80, kSMaxGroups = 11;
constexpr int kSPart = 132;        // floats of an attention partial: o[128], max, sum, pad
constexpr int kSTmemCols = 64;
constexpr uint32_t kSIdesc = umma_idesc_s8(128, 32);
enum { kQKV = 0, kO = 1, kGU = 2, kDOWN = 3, kLM = 4 };
// named barriers: 1 = the eight worker warps, 2 and 3 = the four epilogue warps
constexpr int kBarWorkers = 1, kBarEpi = 2, kBarHead = 3;

struct alignas(16) StepSmem {
  uint64_t full[kSMaxStages], empty[kSMaxStages];    // weight ring
  uint64_t kfull[kSMaxStages], kempty[kSMaxStages];  // K/V ring
  int kv_issued;  // K/V ring items issued so far (written by the K/V producer only)
  uint64_t accfull[2], accempty[2];
  uint64_t dready, dfree, mdone;
  uint32_t tmem;
  int abort;
  int flag;
  int nseg, ngroups, att_items;
  float dq[8];
  unsigned long long best[4][8];
  int seg_pair[kSMaxSeg], seg_a[kSMaxSeg], seg_b[kSMaxSeg], seg_new[kSMaxSeg], seg_cf[kSMaxSeg], seg_cl[kSMaxSeg];
  int g_first[kSMaxGroups], g_n[kSMaxGroups], g_items[kSMaxGroups];
  int wseg[kSMaxGroups][8], wa[kSMaxGroups][8], wb[kSMaxGroups][8], wt[kSMaxGroups][8];
  int merge[kSWorkerWarps];  // per segment of a group: this CTA merges the pair's partials
  StepLayerPtrs lp[kStepMaxLayers];  // the layer pointer table
  alignas(16) float nws[kStepMaxSlots * 128];  // norm weights of the current phase
  alignas(16) float qkn[2][128];               // q and k per-head norm weights of the current layer
  alignas(16) float hs[8][128];
  alignas(16) float slot[8][2][kSPart];
  float sp[8][2][kSKeys];
};

// ---------------------------------------------------------------- geometry
struct Geo {
  int N, K, NT, KT, S, KC, U, off;
};

QASR_DEV Geo step_geo(const StepParams &p, int k, int G) {
  Geo g;
  const int q = p.NQ * 128, kv = p.NKV * 128;
  int S = 1;
  switch (k) {
    case kQKV: g.N = q + 2 * kv; g.K = p.H; S = p.S[0]; break;
    case kO: g.N = p.H; g.K = q; S = p.S[1]; break;
    case kGU: g.N = 2 * p.I; g.K = p.H; S = p.S[2]; break;
    case kDOWN: g.N = p.H; g.K = p.I; S = p.S[3]; break;
    default: g.N = p.V; g.K = p.H; break;
  }
  g.S = S;
  g.NT = (g.N + 127) / 128;
  g.KT = g.K / 128;
  g.KC = g.KT / S;
  g.U = g.NT * S;
  // deal the phases of a layer one after another around the CTAs, so that the
  // CTAs left without a unit in one phase get the first units of the next
  int off = 0;
  if (k >= kO && k <= kDOWN) {
    const int uq = ((q + 2 * kv + 127) / 128) * p.S[0];
    const int uo = ((p.H + 127) / 128) * p.S[1];
    const int ug = ((2 * p.I + 127) / 128) * p.S[2];
    off = k == kO ? uq : k == kGU ? uq + uo : uq + uo + ug;
  }
  g.off = off % G;
  return g;
}
QASR_DEV int first_unit(const Geo &g, int c, int G) { return (c - g.off + G) % G; }
QASR_DEV int unit_count(const Geo &g, int first, int G) { return first < g.U ? (g.U - 1 - first) / G + 1 : 0; }
// K tiles [k0, k0 + KC) of unit u
QASR_DEV int unit_k0(const Geo &g, int u) { return (u % g.S) * g.KC; }
// union of the K tiles of this CTA's units in a phase
QASR_DEV void unit_krange(const Geo &g, int first, int n, int G, int &kmin, int &kmax) {
  kmin = g.KT;
  kmax = 0;
  for (int j = 0; j < n; ++j) {
    const int k0 = unit_k0(g, first + j * G);
    kmin = min(kmin, k0);
    kmax = max(kmax, k0 + g.KC);
  }
}

// ------------------------------------------------------------ primitives
QASR_DEV bool s_aborted(const StepSmem &sm) { return *reinterpret_cast<const volatile int *>(&sm.abort) != 0; }
QASR_DEV void s_fail(StepSmem &sm, int *err) {
  atomicExch(&sm.abort, 1);
  if (err) atomicExch(err, -QASR_ERR_TIMEOUT);
}
// Bounded mbarrier wait that also gives up once the CTA has aborted.
QASR_DEV bool s_wait(StepSmem &sm, uint64_t *bar, unsigned parity, int *err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (s_aborted(sm)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      s_fail(sm, err);
      return false;
    }
  }
  return true;
}
// Named barrier that also ORs a predicate over the participating threads:
// every thread gets the same answer, so an abort decided here is uniform and
// no thread is left waiting at a later barrier.
QASR_DEV bool bar_any(int id, int count, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(count)
      : "memory");
  return r != 0;
}
// Bounded wait until the K/V producer has issued ring item `item`.
QASR_DEV bool s_wait_issued(StepSmem &sm, int item, int *err) {
  const volatile int *v = reinterpret_cast<const volatile int *>(&sm.kv_issued);
  if (*v > item) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (*v <= item) {
    if (s_aborted(sm)) return false;
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      s_fail(sm, err);
      return false;
    }
  }
  return true;
}
QASR_DEV unsigned ld_acquire(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Wait until *ctr >= target (another CTA's release); false on timeout, on a
// failure reported by any CTA (*err) or once this CTA has aborted.
QASR_DEV bool s_wait_count(StepSmem &sm, const unsigned *ctr, unsigned target, int *err) {
  if (ld_acquire(ctr) >= target) return true;
  const unsigned long long t0 = globaltimer_ns();
  for (;;) {
    __nanosleep(32);
    if (ld_acquire(ctr) >= target) return true;
    if (s_aborted(sm) || *reinterpret_cast<volatile int *>(err) == -QASR_ERR_TIMEOUT) {
      atomicExch(&sm.abort, 1);
      return false;
    }
    if (globaltimer_ns() - t0 > kWaitLimitNs) {
      s_fail(sm, err);
      return false;
    }
  }
}
// Publish: every write before this call (by any thread of the group that
// synchronised with the caller) is visible before the counter moves.

// Publish without waiting for a reply: writes before this (by any thread that
// synchronised with the caller) become visible before the counter moves.
QASR_DEV void s_release_add(unsigned *ctr) {
  asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}
// Fetch a 2D box into L2 only (no shared memory, no completion to wait for).
QASR_DEV void s_prefetch_l2(const CUtensorMap *tm, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(tm), "r"(x), "r"(y) : "memory");
}
QASR_DEV void s_signal(unsigned *ctr) { s_release_add(ctr); }
QASR_DEV void s_red_add(long long *a, long long v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(a), "l"((unsigned long long)v) : "memory");
}
QASR_DEV void s_tma_f32(void *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
QASR_DEV float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
QASR_DEV float s_pow2(int e) { return __int_as_float((127 + e) << 23); }

// Digit rows of one token's 4 floats (lane L: elements 4L..4L+3 of a K tile)
// into the 128-byte-swizzled K-major digit tile (rows m, 8+m, 16+m).
QASR_DEV void s_put_digits(unsigned char *tile, int m, float4 v, float qm) {
  const int lane = threadIdx.x & 31;
  auto row_off = [&](int n) { return (n >> 3) * 1024 + (n & 7) * 128 + (((lane >> 2) ^ (n & 7)) << 4) + (lane & 3) * 4; };
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
  *reinterpret_cast<uint32_t *>(tile + row_off(m)) = w0;
  *reinterpret_cast<uint32_t *>(tile + row_off(8 + m)) = w1;
  *reinterpret_cast<uint32_t *>(tile + row_off(16 + m)) = w2;
}
// 2^(22-e) with 2^e > bound; the token's dequantisation factor 2^(e-22) goes to *dq.
QASR_DEV float s_exponent(float bound, float *dq) {
  int e = 0;
  if (bound > 0.0f && bound <= 3.0e38f) frexpf(bound, &e);
  e = max(-100, min(e, 127));
  *dq = s_pow2(e - 22);
  return s_pow2(22 - e);
}

// Phase timeline stamp (worker thread 0 only; phase 0..4 of layer l, or the
// lm head as layer L phase 0).
QASR_DEV void s_stamp(const StepParams &p, int l, int phase, int e) {
  if (p.trace && threadIdx.x == 0)
    p.trace[(size_t)blockIdx.x * step_trace_stride(p.L) + (size_t)l * 20 + phase * 4 + e] = globaltimer_ns();
}

QASR_DEV unsigned *sync_at(const StepParams &p, int l, int i) { return p.sync + (size_t)l * kStepSyncPerLayer + i; }

// Which counter a phase waits on before staging its input, and its target.
QASR_DEV void phase_dep(const StepParams &p, int k, int l, int G, const unsigned **ctr, unsigned *target) {
  const int P = p.M * p.NKV;
  *ctr = nullptr;
  *target = 0;
  switch (k) {
    case kQKV:
      if (l > 0) {
        *ctr = sync_at(p, l - 1, 11);
        *target = (unsigned)step_geo(p, kDOWN, G).NT;
      }
      break;
    case kO: *ctr = sync_at(p, l, 8); *target = (unsigned)P; break;
    case kGU: *ctr = sync_at(p, l, 9); *target = (unsigned)step_geo(p, kO, G).NT; break;
    case kDOWN: *ctr = sync_at(p, l, 10); *target = (unsigned)step_geo(p, kGU, G).NT; break;
    default: *ctr = sync_at(p, p.L - 1, 11); *target = (unsigned)step_geo(p, kDOWN, G).NT; break;
  }
}

QASR_DEV const CUtensorMap *phase_map(const StepParams &p, int k, int l) {
  return k == kLM ? p.maps + 2 : p.maps + 3 + 4 * l + k;
}


// The q|k|v finisher's per-head epilogue (decoder.rs:888-895): q/k per-head
// RMSNorm (warp-tree sum) + NeoX RoPE at the token's position into q_out or
// the K cache row, or the V copy; one 128-wide head held as a float4 per lane
// (lane L = elements 4L..4L+3, RoPE partner lane L^16).  The arithmetic of
// qkv_head_post with this layer's norm weights from shared memory.
QASR_DEV void s_head_post(const StepParams &p, const StepSmem &sm, int l, int h, int m, float4 v) {
  const int lane = threadIdx.x & 31;
  const int pos = p.pos[m];
  if (pos < 0 || pos >= p.max_seq) {
    if (lane == 0) atomicExch(p.err, 2);
    return;
  }
  const int kv_dim = p.NKV * 128;
  const size_t cache_row = (size_t)m * p.seq_stride + ((size_t)l * p.max_seq + pos) * kv_dim;
  if (h >= p.NQ + p.NKV) {
    reinterpret_cast<float4 *>(p.v_cache + cache_row + (h - p.NQ - p.NKV) * 128)[lane] = v;
    return;
  }
  const float *nw = sm.qkn[h < p.NQ ? 0 : 1];
  float ss = __fmul_rn(v.x, v.x);
  ss = fmaf(v.y, v.y, ss);
  ss = fmaf(v.z, v.z, ss);
  ss = fmaf(v.w, v.w, ss);
  ss = warp_sum(ss);
  const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, 128.0f), p.eps)));
  const float4 w4 = reinterpret_cast<const float4 *>(nw)[lane];
  v.x = __fmul_rn(__fmul_rn(v.x, inv), w4.x);
  v.y = __fmul_rn(__fmul_rn(v.y, inv), w4.y);
  v.z = __fmul_rn(__fmul_rn(v.z, inv), w4.z);
  v.w = __fmul_rn(__fmul_rn(v.w, inv), w4.w);
  float4 pr;
  pr.x = __shfl_xor_sync(0xffffffffu, v.x, 16);
  pr.y = __shfl_xor_sync(0xffffffffu, v.y, 16);
  pr.z = __shfl_xor_sync(0xffffffffu, v.z, 16);
  pr.w = __shfl_xor_sync(0xffffffffu, v.w, 16);
  const float4 c = __ldg(reinterpret_cast<const float4 *>(p.rope_cos + (size_t)pos * 128) + lane);
  const float4 s = __ldg(reinterpret_cast<const float4 *>(p.rope_sin + (size_t)pos * 128) + lane);
  const float sg = lane < 16 ? -1.0f : 1.0f;  // first half: x1*c - x2*s; second: x2*c + x1*s
  float4 o;
  o.x = __fadd_rn(__fmul_rn(v.x, c.x), __fmul_rn(sg * pr.x, s.x));
  o.y = __fadd_rn(__fmul_rn(v.y, c.y), __fmul_rn(sg * pr.y, s.y));
  o.z = __fadd_rn(__fmul_rn(v.z, c.z), __fmul_rn(sg * pr.z, s.z));
  o.w = __fadd_rn(__fmul_rn(v.w, c.w), __fmul_rn(sg * pr.w, s.w));
  if (h < p.NQ)
    reinterpret_cast<float4 *>(p.q_out + (size_t)m * p.NQ * 128 + h * 128)[lane] = o;
  else
    reinterpret_cast<float4 *>(p.k_cache + cache_row + (h - p.NQ) * 128)[lane] = o;
}

// ------------------------------------------------------- attention plan
// Keys before each pair's newest row are laid end to end and cut into equal
// ranges, one per CTA; the newest row of a pair is taken by the CTA owning the
// pair's last history key (pair p % G when it has none).  Segments of this
// CTA are handled in groups of up to eight, warps shared in proportion to
// their keys (as in attention.cu).
// Only the first Gd CTAs take history keys, at least kSMinKeys each, so no
// CTA range inside a pair is empty; CTA of key t: floor(((t+1)*Gd - 1) / Th).
constexpr int kSMinKeys = 64;
QASR_DEV long long att_cta_of(long long t, long long Th, long long Gd) { return ((t + 1) * Gd - 1) / Th; }

QASR_DEV void build_att_plan(const StepParams &p, StepSmem &sm, int c, int G) {
  const int P = p.M * p.NKV;
  long long off[kStepMaxPairs + 1];
  off[0] = 0;
  for (int pr = 0; pr < P; ++pr) off[pr + 1] = off[pr] + max(0, min(p.pos[pr / p.NKV], p.max_seq - 1));
  const long long Th = off[P];
  const long long Gd = max(1ll, min((long long)G, Th / kSMinKeys));
  const long long t0 = c < Gd ? (long long)c * Th / Gd : Th, t1 = c < Gd ? (long long)(c + 1) * Th / Gd : Th;
  int ns = 0;
  for (int pr = 0; pr < P && ns < kSMaxSeg; ++pr) {
    const long long len = off[pr + 1] - off[pr];
    int cf, cl;
    if (len > 0) {
      cf = (int)att_cta_of(off[pr], Th, Gd);
      cl = (int)att_cta_of(off[pr] + len - 1, Th, Gd);
    } else {
      cf = cl = pr % G;
    }
    const long long a = max(off[pr], t0), b = min(off[pr + 1], t1);
    const bool hist = a < b;
    const bool newest = cl == c;
    if (!hist && !newest) continue;
    sm.seg_pair[ns] = pr;
    sm.seg_a[ns] = hist ? (int)(a - off[pr]) : (int)len;
    sm.seg_b[ns] = hist ? (int)(b - off[pr]) : (int)len;
    sm.seg_new[ns] = newest;
    sm.seg_cf[ns] = cf;
    sm.seg_cl[ns] = cl;
    ++ns;
  }
  sm.nseg = ns;
  int ng = 0, items = 0;
  for (int s0 = 0; s0 < ns && ng < kSMaxGroups; s0 += kSWorkerWarps, ++ng) {
    const int gn = min(kSWorkerWarps, ns - s0);
    int cnt[kSWorkerWarps];
    long long len[kSWorkerWarps];
    for (int s = 0; s < gn; ++s) {
      cnt[s] = 1;
      len[s] = sm.seg_b[s0 + s] - sm.seg_a[s0 + s];
    }
    for (int extra = kSWorkerWarps - gn; extra > 0; --extra) {
      int best = 0;
      for (int s = 1; s < gn; ++s)
        if (len[s] * cnt[best] > len[best] * cnt[s]) best = s;
      ++cnt[best];
    }
    int w = 0, gi = 0;
    for (int s = 0; s < gn; ++s) {
      const int a = sm.seg_a[s0 + s], n = sm.seg_b[s0 + s] - a;
      for (int i = 0; i < cnt[s]; ++i, ++w) {
        sm.wseg[ng][w] = s0 + s;
        sm.wa[ng][w] = a + (int)((long long)n * i / cnt[s]);
        sm.wb[ng][w] = a + (int)((long long)n * (i + 1) / cnt[s]);
        sm.wt[ng][w] = (sm.wb[ng][w] - sm.wa[ng][w] + kSKeys - 1) / kSKeys;
        gi += sm.wt[ng][w];
      }
    }
    for (; w < kSWorkerWarps; ++w) {
      sm.wseg[ng][w] = -1;
      sm.wa[ng][w] = sm.wb[ng][w] = sm.wt[ng][w] = 0;
    }
    sm.g_first[ng] = s0;
    sm.g_n[ng] = gn;
    sm.g_items[ng] = items;
    items += gi;
  }
  sm.ngroups = ng;
  sm.att_items = items;
  if (ns >= kSMaxSeg || ng * kSWorkerWarps < ns) s_fail(sm, p.err);  // unreachable within the host's limits
}

// ============================================================= the kernel
__global__ void __launch_bounds__(kSThreads, 1) decode_step_kernel(const __grid_constant__ StepParams p) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  unsigned char *base = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  const int STG = p.stages, KSTG = p.kstages;
  unsigned char *ring = base;                              // weight tiles
  unsigned char *kring = ring + (size_t)STG * kSStage;     // K/V history tiles
  unsigned char *dig = kring + (size_t)KSTG * kSStage;
  StepSmem &sm = *reinterpret_cast<StepSmem *>(dig + (size_t)p.slots * kSSlot);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int c = blockIdx.x, G = gridDim.x;
  const int M = p.M, H = p.H;
  const int GQ = p.NQ / p.NKV;

  if (tid == 0) {
    for (int s = 0; s < kSMaxStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
      mbar_init(&sm.kfull[s], 1);
      mbar_init(&sm.kempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.accfull[b], 1);
      mbar_init(&sm.accempty[b], 4);
    }
    mbar_init(&sm.dready, 1);
    mbar_init(&sm.dfree, 1);
    mbar_init(&sm.mdone, 1);
    sm.abort = 0;
    sm.kv_issued = 0;
    mbar_fence_init();
    build_att_plan(p, sm, c, G);
  }
  for (int i = tid; i < p.L * (int)(sizeof(StepLayerPtrs) / 8); i += kSThreads)
    reinterpret_cast<unsigned long long *>(sm.lp)[i] = reinterpret_cast<const unsigned long long *>(p.layers)[i];
  // digit tiles start at zero: rows of tokens >= M and the padding rows 24..31
  // are never written again
  for (int i = tid; i < p.slots * kSSlot / 16; i += kSThreads) reinterpret_cast<uint4 *>(dig)[i] = make_uint4(0, 0, 0, 0);
  if (warp == kSMmaWarp) tmem_alloc(&sm.tmem, kSTmemCols);
  fence_proxy_async();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem;
  // items of one layer in the ring, by phase (the same for every layer)
  const int n_att = sm.att_items;  // K/V stages of one layer

  if (warp == kSProducerWarp) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      auto slot_for = [&](int &st) {
        st = it % STG;
        if (it >= STG && !s_wait(sm, &sm.empty[st], (unsigned)(((it / STG) - 1) & 1), p.err)) return false;
        return !s_aborted(sm);
      };
      auto push_w = [&](const CUtensorMap *tm, int kt, int t) {
        int st;
        if (!slot_for(st)) return false;
        mbar_arrive_expect_tx(&sm.full[st], kSStage);
        tma_load_2d_u8(ring + (size_t)st * kSStage, tm, kt * 128, t * 128, &sm.full[st]);
        ++it;
        return true;
      };
      auto push_phase = [&](int k, int l) {
        const Geo g = step_geo(p, k, G);
        const int f = first_unit(g, c, G), n = unit_count(g, f, G);
        const CUtensorMap *tm = phase_map(p, k, l);
        for (int j = 0; j < n; ++j) {
          const int u = f + j * G, t = u / g.S, k0 = unit_k0(g, u);
          for (int q = 0; q < g.KC; ++q)
            if (!push_w(tm, k0 + q, t)) return false;
        }
        return true;
      };
      for (int l = 0; l < p.L && ok; ++l)
        ok = push_phase(kQKV, l) && push_phase(kO, l) && push_phase(kGU, l) && push_phase(kDOWN, l);
      if (ok) push_phase(kLM, 0);
      // copies still in flight (only after an abort) land before the CTA exits
      for (int i = max(0, it - STG); i < it; ++i) mbar_wait(&sm.full[i % STG], (unsigned)((i / STG) & 1));
    }
  } else if (warp == kSKvWarp) {
    // ------------------------------------------- K/V history producer
    // the attention stages of every layer, in the order the workers take them
    // (round-robin over the warps of each group); its own ring, so the weight
    // tiles of the phases after attention stream in while attention runs
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int l = 0; l < p.L && ok; ++l)
        for (int gi = 0; gi < sm.ngroups && ok; ++gi) {
          int maxT = 0;
          for (int w = 0; w < kSWorkerWarps; ++w) maxT = max(maxT, sm.wt[gi][w]);
          for (int r = 0; r < maxT && ok; ++r)
            for (int w = 0; w < kSWorkerWarps && ok; ++w) {
              if (r >= sm.wt[gi][w]) continue;
              const int pr = sm.seg_pair[sm.wseg[gi][w]], m = pr / p.NKV, kvh = pr % p.NKV;
              const int row = (m * p.L + l) * p.max_seq + sm.wa[gi][w] + r * kSKeys;
              const int st = it % KSTG;
              if (it >= KSTG && !s_wait(sm, &sm.kempty[st], (unsigned)(((it / KSTG) - 1) & 1), p.err)) ok = false;
              if (!ok || s_aborted(sm)) {
                ok = false;
                break;
              }
              unsigned char *dst = kring + (size_t)st * kSStage;
              mbar_arrive_expect_tx(&sm.kfull[st], kSStage);
              s_tma_f32(dst, p.maps + 0, kvh * 128, row, &sm.kfull[st]);
              s_tma_f32(dst + kSStage / 2, p.maps + 1, kvh * 128, row, &sm.kfull[st]);
              ++it;
              *reinterpret_cast<volatile int *>(&sm.kv_issued) = it;
            }
        }
      for (int i = max(0, it - KSTG); i < it; ++i) mbar_wait(&sm.kfull[i % KSTG], (unsigned)((i / KSTG) & 1));
    }
  } else if (warp == kSMmaWarp) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      int it = 0, j = 0, sp = 0;
      bool ok = true;
      auto run_phase = [&](int k, int l) {
        const Geo g = step_geo(p, k, G);
        const int f = first_unit(g, c, G), n = unit_count(g, f, G);
        if (!n) return true;
        int kmin, kmax;
        unit_krange(g, f, n, G, kmin, kmax);
        if (!s_wait(sm, &sm.dready, (unsigned)(sp & 1), p.err)) return false;
        tc_fence_after();
        for (int jj = 0; jj < n; ++jj) {
          const int u = f + jj * G, k0 = unit_k0(g, u), buf = j & 1;
          if (j >= 2 && !s_wait(sm, &sm.accempty[buf], (unsigned)(((j >> 1) - 1) & 1), p.err)) return false;
          tc_fence_after();
          for (int q = 0; q < g.KC; ++q) {
            const int st = it % STG;
            if (!s_wait(sm, &sm.full[st], (unsigned)((it / STG) & 1), p.err)) return false;
            tc_fence_after();
            const uint32_t a_addr = smem_u32(ring + (size_t)st * kSStage);
            const uint32_t b_addr = smem_u32(dig + (size_t)(k0 + q - kmin) * kSSlot);
#pragma unroll
            for (int s = 0; s < 4; ++s)
              umma_s8(tmem + (uint32_t)(buf * 32), umma_desc_sw128(a_addr + 32 * s), umma_desc_sw128(b_addr + 32 * s),
                      kSIdesc, (q == 0 && s == 0) ? 0u : 1u);
            umma_commit(&sm.empty[st]);
            ++it;
          }
          umma_commit(&sm.accfull[buf]);
          ++j;
        }
        umma_commit(&sm.dfree);  // the digit tiles may be rewritten once these MMAs complete
        ++sp;
        return true;
      };
      for (int l = 0; l < p.L && ok; ++l) {
        ok = run_phase(kQKV, l) && run_phase(kO, l) && run_phase(kGU, l) && run_phase(kDOWN, l);
      }
      if (ok) run_phase(kLM, 0);
      umma_commit(&sm.mdone);
      mbar_wait(&sm.mdone, 0);
    }
  } else {
    // -------------------------------------------------------------- workers
    int j = 0, sp = 0;
    bool ok = true;
    unsigned long long best[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) best[m] = 0ull;

    // Stage the digit rows of phase k's input for this CTA's units, then run
    // the epilogue of each unit (warps 0..3).  Returns false on abort.
    auto contraction = [&](int k, int l) -> bool {
      const Geo g = step_geo(p, k, G);
      const int f = first_unit(g, c, G), n = unit_count(g, f, G);
      const int tl = k == kLM ? p.L : l, tp = k == kLM ? 0 : k == kQKV ? 0 : k + 1;  // timeline slot
      s_stamp(p, tl, tp, 0);
      if (!n) return true;
      const StepLayerPtrs *Lp = &sm.lp[l];
      const bool norm = k == kQKV || k == kGU || k == kLM;
      // the phase's constant vectors, fetched while its input is still being produced
      if (norm) {
        const float4 *nw4 = reinterpret_cast<const float4 *>(k == kQKV ? Lp->in_norm : k == kGU ? Lp->post_norm
                                                                                             : p.final_norm);
        for (int i = tid; i < H / 4; i += kSWorkerWarps * 32) reinterpret_cast<float4 *>(sm.nws)[i] = __ldg(nw4 + i);
      }
      if (k == kQKV && tid < 64)
        reinterpret_cast<float4 *>(&sm.qkn[0][0])[tid] =
            __ldg(reinterpret_cast<const float4 *>(tid < 32 ? Lp->q_norm : Lp->k_norm) + (tid & 31));
      const float *scales = k == kQKV ? Lp->sqkv : k == kO ? Lp->so : k == kGU ? Lp->sgu : k == kDOWN ? Lp->sdown
                                                                                                      : p.lm_s;
      const int ri = warp * 32 + (threadIdx.x & 31);
      auto row_scale = [&](int jj) {  // this thread's row scale in unit jj (0 past the end)
        if (warp >= 4 || jj >= n) return 0.0f;
        const int row = (f + jj * G) / g.S * 128 + ri;
        return row < g.N ? __ldg(scales + row) : 0.0f;
      };
      float sc_next = row_scale(0);
      const unsigned *dctr;
      unsigned dtarget;
      phase_dep(p, k, l, G, &dctr, &dtarget);
      bool fail = false;
      if (tid == 0) fail = (dctr && !s_wait_count(sm, dctr, dtarget, p.err)) || s_aborted(sm);
      if (bar_any(kBarWorkers, kSWorkerWarps * 32, fail)) return false;
      s_stamp(p, tl, tp, 1);
      int kmin, kmax;
      unit_krange(g, f, n, G, kmin, kmax);
      if (sp > 0) fail = !s_wait(sm, &sm.dfree, (unsigned)((sp - 1) & 1), p.err);
      // ---- stage: warp m owns token m
      if (warp < M && !__any_sync(0xffffffffu, fail)) {
        const int m = warp;
        if (norm) {
          const float *xr = p.x + (size_t)m * H;
          float4 v[kStepMaxSlots];
          float ss = 0.0f;
#pragma unroll
          for (int i = 0; i < kStepMaxSlots; ++i)
            if (i < g.KT) v[i] = ldcg4(xr + i * 128 + 4 * lane);
#pragma unroll
          for (int i = 0; i < kStepMaxSlots; ++i)
            if (i < g.KT) {
              ss = fmaf(v[i].x, v[i].x, ss);
              ss = fmaf(v[i].y, v[i].y, ss);
              ss = fmaf(v[i].z, v[i].z, ss);
              ss = fmaf(v[i].w, v[i].w, ss);
            }
          ss = warp_sum(ss);
          const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps)));
          float mx = 0.0f;
#pragma unroll
          for (int i = 0; i < kStepMaxSlots; ++i)
            if (i < g.KT) {
              const float4 w4 = *reinterpret_cast<const float4 *>(sm.nws + i * 128 + 4 * lane);
              v[i] = make_float4(__fmul_rn(__fmul_rn(v[i].x, inv), w4.x), __fmul_rn(__fmul_rn(v[i].y, inv), w4.y),
                                 __fmul_rn(__fmul_rn(v[i].z, inv), w4.z), __fmul_rn(__fmul_rn(v[i].w, inv), w4.w));
              mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w))));
            }
          mx = warp_max(mx);
          float dq;
          const float qm = s_exponent(mx, &dq);
          if (lane == 0) sm.dq[m] = dq;
#pragma unroll
          for (int i = 0; i < kStepMaxSlots; ++i)
            if (i >= kmin && i < kmax) s_put_digits(dig + (size_t)(i - kmin) * kSSlot, m, v[i], qm);
        } else {
          const float *src = k == kO ? p.attn : p.h;
          const float bound = __uint_as_float(__ldcg(sync_at(p, l, (k == kO ? 16 : 24) + m)));
          float dq;
          const float qm = s_exponent(bound, &dq);
          if (lane == 0) sm.dq[m] = dq;
          for (int i = kmin; i < kmax; ++i)
            s_put_digits(dig + (size_t)(i - kmin) * kSSlot, m, ldcg4(src + (size_t)m * g.K + i * 128 + 4 * lane), qm);
        }
      }
      fence_proxy_async();  // digit rows written by threads -> visible to the tensor cores
      if (bar_any(kBarWorkers, kSWorkerWarps * 32, fail)) return false;
      if (tid == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.dready)) : "memory");
      s_stamp(p, tl, tp, 2);
      ++sp;
      // ---- epilogue (warps 0..3): thread = row of the unit's tile; then all
      // eight warps meet, so a failure reaches every worker at one barrier
      bool efail = false;
      for (int jj = 0; jj < n && warp < 4; ++jj, ++j) {
        const int u = f + jj * G, t = u / g.S, buf = j & 1;
        if (bar_any(kBarEpi, 128, !s_wait(sm, &sm.accfull[buf], (unsigned)((j >> 1) & 1), p.err))) {
          efail = true;
          break;
        }
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
        const int row = t * 128 + ri;
        const bool valid = row < g.N;
        const float sc = sc_next;
        sc_next = row_scale(jj + 1);
        if (g.S > 1) {
          // split K: every unit adds its exact sums into the tile's accumulator
          // (integer atomics, fire and forget); the unit holding the first K
          // chunk waits for the other chunks to count in and then takes the
          // totals, clearing the accumulator for the next phase
          long long *acc = p.acc + ((size_t)t * 128 + ri) * 8;
          if (valid)
            for (int m = 0; m < M; ++m) s_red_add(acc + m, V[m]);
          named_bar(kBarEpi, 128);
          if (u % g.S != 0) {
            if (tid == 0) s_release_add(p.tile_ctr + t);
            continue;
          }
          bool wfail = false;
          if (tid == 0) wfail = !s_wait_count(sm, p.tile_ctr + t, (unsigned)(g.S - 1), p.err);
          if (bar_any(kBarEpi, 128, wfail)) {
            efail = true;
            break;
          }
          if (valid)
            for (int m = 0; m < M; ++m)
              V[m] = (long long)atomicExch(reinterpret_cast<unsigned long long *>(acc + m), 0ull);
          if (tid == 0) p.tile_ctr[t] = 0u;  // re-armed for the next phase (published with this tile)
        }
        // ---- finish the row tile
        float y[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) y[m] = m < M ? __fmul_rn(__fmul_rn(__ll2float_rn(V[m]), sm.dq[m]), sc) : 0.0f;
        if (k == kQKV) {
#pragma unroll
          for (int m = 0; m < 8; ++m) sm.hs[m][ri] = y[m];
          named_bar(kBarHead, 128);
          for (int m = warp; m < M; m += 4)
            s_head_post(p, sm, l, t, m, reinterpret_cast<const float4 *>(sm.hs[m])[lane]);
          named_bar(kBarHead, 128);
          const int kvh = t < p.NQ ? t / GQ : t < p.NQ + p.NKV ? t - p.NQ : t - p.NQ - p.NKV;
          if (tid == 0) s_signal(sync_at(p, l, kvh));
        } else if (k == kO || k == kDOWN) {
          if (valid)
            for (int m = 0; m < M; ++m) {
              float *dst = p.x + (size_t)m * H + row;
              *dst = __fadd_rn(__ldcg(dst), y[m]);
            }
          named_bar(kBarEpi, 128);
          if (tid == 0) s_signal(sync_at(p, l, k == kO ? 9 : 11));
        } else if (k == kGU) {
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            const float up = __shfl_xor_sync(0xffffffffu, y[m], 1);
            float hv = 0.0f;
            if (m < M && valid && (row & 1) == 0) {
              const float gt = y[m];
              hv = __fmul_rn(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))), up);
              p.h[(size_t)m * p.I + row / 2] = hv;
            }
            const float amx = warp_max(fabsf(hv));
            if (lane == 0 && m < M) atomicMax(sync_at(p, l, 24 + m), __float_as_uint(amx));
          }
          named_bar(kBarEpi, 128);
          if (tid == 0) s_signal(sync_at(p, l, 10));
        } else {  // lm head
#pragma unroll
          for (int m = 0; m < 8; ++m)
            if (valid && m < M) {
              if (p.logits) p.logits[(size_t)m * p.V + row] = y[m];
              const unsigned long long key = argmax_key(y[m], (uint32_t)row);
              best[m] = key > best[m] ? key : best[m];
            }
        }
      }
      const bool good = !bar_any(kBarWorkers, kSWorkerWarps * 32, efail);
      s_stamp(p, tl, tp, 3);
      return good;
    };

    // Bring this CTA's K/V history tiles of layer l into L2 (fire and forget),
    // so that the layer's attention streams them from L2 instead of HBM.
    auto prefetch_kv = [&](int l) {
      if (lane != 0) return;
      for (int gi = 0; gi < sm.ngroups; ++gi) {
        const int seg = sm.wseg[gi][warp];
        if (seg < 0) continue;
        const int pr = sm.seg_pair[seg], m = pr / p.NKV, kvh = pr % p.NKV;
        const int row0 = (m * p.L + l) * p.max_seq + sm.wa[gi][warp];
        for (int r = 0; r < sm.wt[gi][warp]; ++r) {
          s_prefetch_l2(p.maps + 0, kvh * 128, row0 + r * kSKeys);
          s_prefetch_l2(p.maps + 1, kvh * 128, row0 + r * kSKeys);
        }
      }
    };

    // One layer's attention for this CTA's segments.
    auto attention = [&](int l) -> bool {
      const int att0 = l * n_att;  // K/V ring index of this layer's first stage
      s_stamp(p, l, 1, 0);
      for (int gi = 0; gi < sm.ngroups; ++gi) {
        const int seg = sm.wseg[gi][warp];
        bool fail = false;
        if (seg >= 0) do {
          const int pr = sm.seg_pair[seg], m = pr / p.NKV, kvh = pr % p.NKV;
          const int wa = sm.wa[gi][warp], wb = sm.wb[gi][warp], T = sm.wt[gi][warp];
          const bool has_new = sm.seg_new[seg] && wb == sm.seg_b[seg];
          bool good = true;
          if (lane == 0) good = s_wait_count(sm, sync_at(p, l, kvh), (unsigned)(GQ + 2), p.err);
          if (gi == 0) s_stamp(p, l, 1, 1);
          good = __shfl_sync(0xffffffffu, good ? 1 : 0, 0) != 0;
          if (!good) {
            fail = true;
            break;
          }
          float4 qv[2];
          float mx[2], sum[2];
          float4 o[2];
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            qv[g] = ldcg4(p.q_out + (size_t)m * p.NQ * 128 + (kvh * 2 + g) * 128 + 4 * lane);
            mx[g] = -INFINITY;
            sum[g] = 0.0f;
            o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
          const int my_idx = reduce_index<32>(lane), my_g = my_idx / kSKeys, my_key = my_idx % kSKeys;
          // ring index of tile r of this warp: stages are dealt round-robin over the warps
          int rbase = att0 + sm.g_items[gi];
          for (int r = 0; r < T; ++r) {
            int before = 0, in_round = 0;
            for (int w = 0; w < kSWorkerWarps; ++w)
              if (sm.wt[gi][w] > r) {
                before += w < warp;
                ++in_round;
              }
            const int item = rbase + before;
            rbase += in_round;
            const int st = item % KSTG;
            // The warps take the stages round-robin and a warp's next item can
            // lie more than one lap of the ring ahead; waiting for the item to
            // be issued first keeps the parity wait within one lap (an mbarrier
            // parity cannot tell phase n from phase n + 2).
            const bool ready = s_wait_issued(sm, item, p.err) &&
                               s_wait(sm, &sm.kfull[st], (unsigned)((item / KSTG) & 1), p.err);
            if (!__all_sync(0xffffffffu, ready)) {
              fail = true;
              break;
            }
            const float *kt = reinterpret_cast<const float *>(kring + (size_t)st * kSStage);
            const float *vt = kt + kSKeys * 128;
            const int nk = min(kSKeys, wb - wa - r * kSKeys);
            float part[32];
#pragma unroll
            for (int jk = 0; jk < kSKeys; ++jk) {
              const float4 kv = *reinterpret_cast<const float4 *>(kt + jk * 128 + 4 * lane);
#pragma unroll
              for (int g = 0; g < 2; ++g) {
                float d = __fmul_rn(qv[g].x, kv.x);
                d = fmaf(qv[g].y, kv.y, d);
                d = fmaf(qv[g].z, kv.z, d);
                d = fmaf(qv[g].w, kv.w, d);
                part[g * kSKeys + jk] = d;
              }
            }
            const float tot = warp_reduce_scatter<32>(part);
            const bool live = my_key < nk;
            const float sc = live ? __fmul_rn(tot, p.scale) : -INFINITY;
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              const float nmax = fmaxf(mx[g], warp_max(my_g == g ? sc : -INFINITY));
              const float corr = mx[g] == -INFINITY ? 0.0f : __expf(__fsub_rn(mx[g], nmax));
              const float pj = (my_g == g && live) ? __expf(__fsub_rn(sc, nmax)) : 0.0f;
              sum[g] = __fadd_rn(__fmul_rn(sum[g], corr), warp_sum(pj));
              mx[g] = nmax;
              if (my_g == g) sm.sp[warp][g][my_key] = pj;
              o[g].x = __fmul_rn(o[g].x, corr);
              o[g].y = __fmul_rn(o[g].y, corr);
              o[g].z = __fmul_rn(o[g].z, corr);
              o[g].w = __fmul_rn(o[g].w, corr);
            }
            __syncwarp();
            for (int jk = 0; jk < nk; ++jk) {
              const float4 vv = *reinterpret_cast<const float4 *>(vt + jk * 128 + 4 * lane);
#pragma unroll
              for (int g = 0; g < 2; ++g) {
                const float w = sm.sp[warp][g][jk];
                o[g].x = fmaf(w, vv.x, o[g].x);
                o[g].y = fmaf(w, vv.y, o[g].y);
                o[g].z = fmaf(w, vv.z, o[g].z);
                o[g].w = fmaf(w, vv.w, o[g].w);
              }
            }
            __syncwarp();  // the stage and sp are free
            if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&sm.kempty[st])) : "memory");
          }
          if (fail) break;
          if (has_new) {
            // the pair's newest row, appended by this step's q|k|v finisher
            const int pos = max(0, min(p.pos[m], p.max_seq - 1));
            const size_t row_off = (size_t)m * p.seq_stride + ((size_t)l * p.max_seq + pos) * p.NKV * 128 + kvh * 128;
            const float4 kv = ldcg4(p.k_cache + row_off + 4 * lane), vv = ldcg4(p.v_cache + row_off + 4 * lane);
#pragma unroll
            for (int g = 0; g < 2; ++g) {
              float d = __fmul_rn(qv[g].x, kv.x);
              d = fmaf(qv[g].y, kv.y, d);
              d = fmaf(qv[g].z, kv.z, d);
              d = fmaf(qv[g].w, kv.w, d);
              const float sc = __fmul_rn(warp_sum(d), p.scale);
              const float nmax = fmaxf(mx[g], sc);
              const float corr = mx[g] == -INFINITY ? 0.0f : __expf(__fsub_rn(mx[g], nmax));
              const float pj = __expf(__fsub_rn(sc, nmax));
              sum[g] = __fadd_rn(__fmul_rn(sum[g], corr), pj);
              mx[g] = nmax;
              o[g].x = fmaf(pj, vv.x, __fmul_rn(o[g].x, corr));
              o[g].y = fmaf(pj, vv.y, __fmul_rn(o[g].y, corr));
              o[g].z = fmaf(pj, vv.z, __fmul_rn(o[g].z, corr));
              o[g].w = fmaf(pj, vv.w, __fmul_rn(o[g].w, corr));
            }
          }
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            reinterpret_cast<float4 *>(sm.slot[warp][g])[lane] = o[g];
            if (lane == 0) {
              sm.slot[warp][g][128] = mx[g];
              sm.slot[warp][g][129] = sum[g];
            }
          }
        } while (false);
        if (bar_any(kBarWorkers, kSWorkerWarps * 32, fail)) return false;
        if (gi == 0) s_stamp(p, l, 1, 2);
        // ---- merge the warps of each segment; pairs split over CTAs via partials
        const int s0 = sm.g_first[gi], gn = sm.g_n[gi];
        for (int task = warp; task < gn * 2; task += kSWorkerWarps) {
          const int s = s0 + task / 2, g = task % 2;
          const int prs = sm.seg_pair[s], ms = prs / p.NKV, kvs = prs % p.NKV;
          float Mx = -INFINITY;
          for (int w = 0; w < kSWorkerWarps; ++w)
            if (sm.wseg[gi][w] == s) Mx = fmaxf(Mx, sm.slot[w][g][128]);
          float L = 0.0f;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int w = 0; w < kSWorkerWarps; ++w) {
            if (sm.wseg[gi][w] != s) continue;
            const float *ws = sm.slot[w][g];
            const float fct = ws[128] == -INFINITY ? 0.0f : expf(__fsub_rn(ws[128], Mx));
            L = __fadd_rn(L, __fmul_rn(ws[129], fct));
            const float4 ov = reinterpret_cast<const float4 *>(ws)[lane];
            acc.x = fmaf(ov.x, fct, acc.x);
            acc.y = fmaf(ov.y, fct, acc.y);
            acc.z = fmaf(ov.z, fct, acc.z);
            acc.w = fmaf(ov.w, fct, acc.w);
          }
          if (sm.seg_cf[s] == sm.seg_cl[s]) {
            const float inv = __fdiv_rn(1.0f, L);
            const float4 res = make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv),
                                           __fmul_rn(acc.w, inv));
            reinterpret_cast<float4 *>(p.attn + (size_t)ms * p.NQ * 128 + (kvs * 2 + g) * 128)[lane] = res;
            const float amx = warp_max(fmaxf(fmaxf(fabsf(res.x), fabsf(res.y)), fmaxf(fabsf(res.z), fabsf(res.w))));
            if (lane == 0) atomicMax(sync_at(p, l, 16 + ms), __float_as_uint(amx));
          } else {
            float *slot = p.part + ((size_t)(c + prs) * 2 + g) * kSPart;
            reinterpret_cast<float4 *>(slot)[lane] = acc;
            if (lane == 0) {
              slot[128] = Mx;
              slot[129] = L;
            }
          }
        }
        named_bar(kBarWorkers, kSWorkerWarps * 32);
        // one arrival per segment: a single-contributor pair is done; of a split
        // pair, the CTA holding its newest row merges once the others counted in
        if (tid < gn) {
          const int s = s0 + tid;
          sm.merge[tid] = 0;
          if (sm.seg_cf[s] == sm.seg_cl[s])
            s_signal(sync_at(p, l, 8));
          else if (c != sm.seg_cl[s])
            s_release_add(p.pair_ctr + sm.seg_pair[s]);
          else
            sm.merge[tid] = 1;
        }
        named_bar(kBarWorkers, kSWorkerWarps * 32);
        bool mfail = false;
        for (int task = warp; task < gn * 2 && !mfail; task += kSWorkerWarps) {
          if (!sm.merge[task / 2]) continue;
          const int s = s0 + task / 2, g = task % 2;
          const int prs = sm.seg_pair[s], ms = prs / p.NKV, kvs = prs % p.NKV;
          const int pcf = sm.seg_cf[s], pcl = sm.seg_cl[s];
          bool good = true;
          if (lane == 0) good = s_wait_count(sm, p.pair_ctr + prs, (unsigned)(pcl - pcf), p.err);
          if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) {
            mfail = true;
            break;
          }
          auto part = [&](int c2) { return p.part + ((size_t)(c2 + prs) * 2 + g) * kSPart; };
          float Mx = -INFINITY;
          for (int c2 = pcf + lane; c2 <= pcl; c2 += 32) Mx = fmaxf(Mx, __ldcg(part(c2) + 128));
          Mx = warp_max(Mx);
          float L = 0.0f;
          for (int c2 = pcf + lane; c2 <= pcl; c2 += 32) {
            const float m2 = __ldcg(part(c2) + 128);
            L = __fadd_rn(L, __fmul_rn(__ldcg(part(c2) + 129), m2 == -INFINITY ? 0.0f : expf(__fsub_rn(m2, Mx))));
          }
          L = warp_sum(L);
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int c2 = pcf; c2 <= pcl; ++c2) {
            const float m2 = __ldcg(part(c2) + 128);
            const float fct = m2 == -INFINITY ? 0.0f : expf(__fsub_rn(m2, Mx));
            const float4 ov = ldcg4(part(c2) + 4 * lane);
            acc.x = fmaf(ov.x, fct, acc.x);
            acc.y = fmaf(ov.y, fct, acc.y);
            acc.z = fmaf(ov.z, fct, acc.z);
            acc.w = fmaf(ov.w, fct, acc.w);
          }
          const float inv = __fdiv_rn(1.0f, L);
          const float4 res = make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv),
                                         __fmul_rn(acc.w, inv));
          reinterpret_cast<float4 *>(p.attn + (size_t)ms * p.NQ * 128 + (kvs * 2 + g) * 128)[lane] = res;
          const float amx = warp_max(fmaxf(fmaxf(fabsf(res.x), fabsf(res.y)), fmaxf(fabsf(res.z), fabsf(res.w))));
          if (lane == 0) atomicMax(sync_at(p, l, 16 + ms), __float_as_uint(amx));
        }
        if (bar_any(kBarWorkers, kSWorkerWarps * 32, mfail)) return false;
        if (tid < gn && sm.merge[tid]) {
          p.pair_ctr[sm.seg_pair[s0 + tid]] = 0u;  // re-armed for the next layer (published below)
          s_signal(sync_at(p, l, 8));
        }
        named_bar(kBarWorkers, kSWorkerWarps * 32);  // slots and flags are rewritten by the next group
      }
      s_stamp(p, l, 1, 3);
      if (l + 1 < p.L) prefetch_kv(l + 1);
      return true;
    };

    prefetch_kv(0);
    // one call site per phase kind (the code is inlined once: a single copy of
    // each phase's instructions keeps the kernel small enough for the
    // instruction caches)
    for (int q = 0; q <= 5 * p.L && ok; ++q) {
      const int l = q / 5, ph = q % 5;
      if (q == 5 * p.L) {
        ok = contraction(kLM, p.L - 1);
      } else if (ph == 1) {
        ok = attention(l);
      } else {
        ok = contraction(ph == 0 ? kQKV : ph - 1, l);
      }
    }
    if (ok && warp < 4) {
      // ---- argmax over the CTA, then over the grid (the last CTA writes the ids)
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        unsigned long long b = best[m];
#pragma unroll
        for (int o2 = 16; o2 > 0; o2 >>= 1) {
          const unsigned long long q = __shfl_xor_sync(0xffffffffu, b, o2);
          b = q > b ? q : b;
        }
        if (lane == 0) sm.best[warp][m] = b;
      }
      named_bar(kBarEpi, 128);
      if (tid < M) {
        unsigned long long b = 0ull;
        for (int w = 0; w < 4; ++w) b = sm.best[w][tid] > b ? sm.best[w][tid] : b;
        if (b) atomicMax(p.keys + tid, b);
      }
      named_bar(kBarEpi, 128);
      if (tid == 0) {
        __threadfence();
        sm.flag = atomicAdd(p.am_ctr, 1u) == (unsigned)(G - 1);
      }
      named_bar(kBarEpi, 128);
      if (sm.flag && tid < M) {
        __threadfence();
        const unsigned long long key = atomicExch(p.keys + tid, 0ull);
        p.next[tid] = (int32_t)(0xffffffffu - (uint32_t)(key & 0xffffffffull));
      }
    }
  }

  // ---- teardown: no copy or MMA in flight, then TMEM is released
  tc_fence_before();
  __syncthreads();
  if (warp == kSMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kSTmemCols);
  }
}

// =================================================================== host
StepScratch step_scratch_layout(int n_layers, long acc_rows) {
  StepScratch s{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = (o + bytes + 255) & ~size_t(255);
    return at;
  };
  s.sync = take((size_t)n_layers * kStepSyncPerLayer * 4);
  s.tile_ctr = take(256 * 4);
  s.pair_ctr = take(kStepMaxPairs * 4);
  s.keys = take(8 * 8);
  s.am_ctr = take(4);
  s.acc = take((size_t)acc_rows * 8 * 8);
  s.total = o;
  return s;
}

// Cost of a K split in tile-MMA units (measured phase timelines: a split phase
// pays a wait for the other chunks plus a read of their partials).
#ifndef QASR_STEP_SPLIT_COST
#define QASR_STEP_SPLIT_COST 3.0
#endif
constexpr double kStepSplitCost = QASR_STEP_SPLIT_COST;

static size_t step_smem_bytes(int stages, int slots) {  // stages: both rings together
  return 1024 + (size_t)stages * kSStage + (size_t)slots * kSSlot + sizeof(StepSmem);
}

int step_plan(StepParams &p, int grid) {
  const int q = p.NQ * 128, kv = p.NKV * 128;
  if (p.M < 1 || p.M > kStepMaxM || p.NKV < 1 || p.NKV > 8 || p.NQ != 2 * p.NKV || p.M * p.NKV > kStepMaxPairs ||
      p.H % 128 || p.H / 128 > kStepMaxSlots || p.I % 128 || p.L < 1 || p.L > kStepMaxLayers || p.V < 128 ||
      grid < 1 ||
      (2 * p.I + 127) / 128 > 256 || (q + 2 * kv) / 128 > 256 || p.H / 128 > 256) {
    set_error("decode step kernel: unsupported shape");
    return QASR_ERR_UNSUPPORTED;
  }
  const int N[4] = {q + 2 * kv, p.H, 2 * p.I, p.H}, K[4] = {p.H, q, p.H, p.I};
  int slots = p.H / 128;  // the lm head stages every K tile of the final norm
  for (int k = 0; k < 4; ++k) {
    const int NT = (N[k] + 127) / 128, KT = K[k] / 128;
    // Latency model of a phase in units of one weight tile per CTA (fetch and
    // MMAs, about 0.4 us; a CTA's tiles of a phase are only partly prefetched):
    // a unit takes KC tiles; splitting K adds the finisher's wait for the
    // other chunks and its read of the accumulated sums.  A split keeps at
    // most one unit per CTA, so no CTA waits on itself.
    int S = 0;
    double best = 1e30;
    for (int s = 1; s <= KT; ++s) {
      if (KT % s || KT / s > kStepMaxSlots || (s > 1 && NT * s > grid)) continue;
      const double cost = (double)(KT / s) * ((NT * s + grid - 1) / grid) + (s > 1 ? kStepSplitCost : 0.0);
      if (cost < best - 1e-9) {
        best = cost;
        S = s;
      }
    }
    if (!S) {
      set_error("decode step kernel: K=%d too large for one unit", K[k]);
      return QASR_ERR_UNSUPPORTED;
    }
    p.S[k] = S;
    slots = std::max(slots, KT / S);
  }
  p.slots = slots;
  int stages = kSMaxStages;
  while (stages > 2 && step_smem_bytes(stages, slots) > 227 * 1024) --stages;
  if (step_smem_bytes(stages, slots) > 227 * 1024) {
    set_error("decode step kernel: shared memory");
    return QASR_ERR_UNSUPPORTED;
  }
  // the K/V ring takes up to half of the stages (at least 2 each)
  if (stages < 4) {
    set_error("decode step kernel: shared memory");
    return QASR_ERR_UNSUPPORTED;
  }
  p.kstages = std::min(5, stages / 2);
  p.stages = stages - p.kstages;
  return QASR_OK;
}

int step_kv_map(CUtensorMap *tm, const float *base, long rows, int kv_dim) {
  using Encode = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                              const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
  auto encode = reinterpret_cast<Encode>(tensor_map_encoder());
  if (!encode) {
    set_error("decode step kernel: cuTensorMapEncodeTiled unavailable");
    return QASR_ERR_CUDA;
  }
  if ((reinterpret_cast<uintptr_t>(base) & 15) || kv_dim % 128 || rows <= 0) {
    set_error("decode step kernel: KV cache must be 16-byte aligned with kv_dim a multiple of 128");
    return QASR_ERR_INVALID;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)kv_dim, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kv_dim * 4};
  const cuuint32_t box[2] = {128, (cuuint32_t)kSKeys};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float *>(base), dims, strides, box, estr,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("decode step kernel: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return QASR_ERR_CUDA;
  }
  return QASR_OK;
}

int step_launch(const StepParams &p, int grid, cudaStream_t st) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return QASR_ERR_INVALID;
  const size_t smem = step_smem_bytes(p.stages + p.kstages, p.slots);
  if (!attr_done[dev]) {
    int rc = cuda_status(cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              227 * 1024),
                         "decode step kernel: shared memory opt-in");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kSThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA co-resident: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, decode_step_kernel, p), "decode step kernel launch");
}

}  // namespace qasr
