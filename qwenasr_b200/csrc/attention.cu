// attention.cu -- GQA causal attention (kernels::causal_attention,
// crates/qwen-asr/src/kernels/mod.rs:1124-1207).
//
// Two kernels:
//  * causal_attention_kernel: the general kernel-level entry (any seq_q,
//    e.g. prefill, kernels::causal_attention mod.rs:1124-1207).  K/V tiles of
//    32 keys staged in shared memory serve the block's queries and every
//    query head of their GQA group; scores one key per lane, merged tile by
//    tile (flash-style) instead of the reference's per-key update -- the same
//    softmax up to f32 rounding.
//  * attn_decode_kernel: the decode step of the engine.  Flash-decoding over
//    the f32 KV cache: the keys of one (sequence, kv head) are split across
//    CTAs, each CTA serves both query heads of the GQA group so every K/V row
//    is read from HBM exactly once, and the last CTA of a (sequence, kv head)
//    merges the partial softmax states (counter + threadfence, no spin).
#include <cudaTypedefs.h>

#include <algorithm>

#include "attention.cuh"
#include "common.cuh"
#include "tma.cuh"

namespace qasr {

// ------------------------------------------------------------------ general
constexpr int kCaTile = 32;   // keys per shared-memory tile (one per lane for the scores)
constexpr int kCaTasks = 16;  // (query, head) tasks per block: two per warp

// Block (query block qb, kv head kvh): queries qb*QB .. +QB, every query head of
// the GQA group (task = query * G + head-in-group); warp w takes tasks w and
// w + 8 together, so every K and V value it reads from shared memory serves
// both.  K/V tiles of kCaTile keys are staged in shared memory (K rows padded
// by 4 floats: 16-byte rows whose float4 reads, one key per lane, are
// conflict-free) and shared by all tasks; each task keeps a running (max, sum,
// o) merged tile by tile (flash-style), its causal limit masking the keys
// after q_offset + query.
template <int EPL>  // elements per lane: head_dim / 32
__global__ void __launch_bounds__(256, 2)
causal_attention_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ k,
                        const float *__restrict__ v, CaSeg one, const CaSeg *__restrict__ many, int n_heads,
                        int n_kv_heads, float scale) {
  // segment blockIdx.z: its query rows, its keys / values and causal offset
  const CaSeg sg = many ? many[blockIdx.z] : one;
  const int seq_q = sg.seq_q, seq_k = sg.seq_k, q_offset = sg.q_offset;
  q += sg.q_row0 * (long)n_heads * (EPL * 32);
  out += sg.q_row0 * (long)n_heads * (EPL * 32);
  k += sg.kv_off;
  v += sg.kv_off;
  constexpr int HD = EPL * 32, KP = HD + 4;
  __shared__ __align__(16) float sK[kCaTile][KP];
  __shared__ __align__(16) float sV[kCaTile][HD];
  __shared__ __align__(16) float sQ[kCaTasks][HD];
  __shared__ float sP[8][2][kCaTile];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = n_heads / n_kv_heads, QB = max(1, kCaTasks / G), n_tasks = QB * G;
  const int kvh = blockIdx.y, i0 = blockIdx.x * QB;
  if (i0 >= seq_q) return;  // block-uniform: the grid covers the longest segment
  const long q_hidden = (long)n_heads * HD, kv_hidden = (long)n_kv_heads * HD;
  const int i_last = min(seq_q, i0 + QB) - 1;
  const int k_end = min(q_offset + i_last + 1, seq_k);  // keys any task of the block needs
  // q rows of the block's tasks (zero for the unused ones)
  for (int idx = threadIdx.x; idx < kCaTasks * HD; idx += blockDim.x) {
    const int t = idx / HD, d = idx % HD, i = i0 + t / G, h = kvh * G + t % G;
    sQ[t][d] = (t < n_tasks && i < seq_q) ? q[(long)i * q_hidden + (long)h * HD + d] : 0.0f;
  }
  bool act[2];
  int lim[2];
  float m[2], l[2], o[2][EPL];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int t = warp + 8 * u, i = i0 + t / G;
    act[u] = t < n_tasks && i < seq_q;
    lim[u] = act[u] ? min(q_offset + i + 1, seq_k) : 0;  // keys < lim are visible
    m[u] = -INFINITY;
    l[u] = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[u][e] = 0.0f;
  }
  const float4 *q0 = reinterpret_cast<const float4 *>(sQ[warp]), *q1 = reinterpret_cast<const float4 *>(sQ[warp + 8]);
  for (int t0 = 0; t0 < k_end; t0 += kCaTile) {
    const int nk = min(kCaTile, k_end - t0);
    __syncthreads();  // the previous tile is consumed (and sQ written, first time)
    stage_kv_rows<HD, 4>(&sK[0][0], &sV[0][0], k, v, t0, kv_hidden, (long)kvh * HD, nk);
    __syncthreads();
    if (!act[0] && !act[1]) continue;  // warp-uniform, no barrier before the next tile
    // scores of both tasks, one key per lane, two partial sums each
    float sc[2] = {-INFINITY, -INFINITY};
    if (lane < nk) {
      const float4 *kr = reinterpret_cast<const float4 *>(sK[lane]);
      float a0 = 0.0f, a1 = 0.0f, b0 = 0.0f, b1 = 0.0f;
#pragma unroll 8
      for (int e4 = 0; e4 < HD / 4; ++e4) {
        const float4 kk = kr[e4], x = q0[e4], y = q1[e4];
        a0 = fmaf(x.x, kk.x, a0);
        a1 = fmaf(x.y, kk.y, a1);
        b0 = fmaf(y.x, kk.x, b0);
        b1 = fmaf(y.y, kk.y, b1);
        a0 = fmaf(x.z, kk.z, a0);
        a1 = fmaf(x.w, kk.w, a1);
        b0 = fmaf(y.z, kk.z, b0);
        b1 = fmaf(y.w, kk.w, b1);
      }
      const int key = t0 + lane;
      if (key < lim[0]) sc[0] = __fmul_rn(__fadd_rn(a0, a1), scale);
      if (key < lim[1]) sc[1] = __fmul_rn(__fadd_rn(b0, b1), scale);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      float pj = 0.0f, corr = 1.0f;
      if (act[u]) {  // warp-uniform
        const float mn = fmaxf(m[u], warp_max(sc[u]));
        if (mn != -INFINITY) {  // some key of this task visible so far
          corr = m[u] == -INFINITY ? 0.0f : expf(__fsub_rn(m[u], mn));
          pj = sc[u] == -INFINITY ? 0.0f : expf(__fsub_rn(sc[u], mn));
          l[u] = __fadd_rn(__fmul_rn(l[u], corr), warp_sum(pj));
          m[u] = mn;
        }
      }
      sP[warp][u][lane] = pj;  // zero for masked keys, skipped and unused tasks
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[u][e] = __fmul_rn(o[u][e], corr);
    }
    __syncwarp();
    for (int j = 0; j < nk; ++j) {
      const float p0 = sP[warp][0][j], p1 = sP[warp][1][j];
      float vv[EPL];
      if constexpr (EPL == 4) {
        const float4 t4 = *reinterpret_cast<const float4 *>(&sV[j][lane * 4]);
        vv[0] = t4.x;
        vv[1] = t4.y;
        vv[2] = t4.z;
        vv[3] = t4.w;
      } else {
        const float2 t2 = *reinterpret_cast<const float2 *>(&sV[j][lane * 2]);
        vv[0] = t2.x;
        vv[1] = t2.y;
      }
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        o[0][e] = fmaf(p0, vv[e], o[0][e]);
        o[1][e] = fmaf(p1, vv[e], o[1][e]);
      }
    }
    __syncwarp();  // sP is rewritten by the next tile
  }
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    if (!act[u]) continue;
    const int t = warp + 8 * u, i = i0 + t / G, h = kvh * G + t % G;
    const float inv = l[u] > 0.0f ? __fdiv_rn(1.0f, l[u]) : 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      out[(long)i * q_hidden + (long)h * HD + lane * EPL + e] = l[u] > 0.0f ? __fmul_rn(o[u][e], inv) : o[u][e];
  }
}

// ------------------------------------------------------------------- decode
// Persistent flash-decoding.  The keys of all (sequence, kv head) pairs are
// laid end to end and cut into equal ranges, one per CTA, so every SM streams
// the same number of K/V bytes whatever the batch and lengths.  The pairs a
// CTA touches ("segments", usually one or two) share its 8 warps in
// proportion to their key counts, so they stream at the same time; each warp
// streams its contiguous key range of one segment through its own 2-stage
// ring of 8-key K and V tiles (2D TMA, box 8 rows x one 128-float head slice,
// no multicast), scores its keys for both query heads of the GQA group (each
// K/V byte is read from HBM once and used twice) and keeps an online-softmax
// state whose maximum is raised only when a score exceeds it by more than 8
// (the common tile pays no rescale), with the tile's V rows loaded while its
// scores are reduced.  The CTA then merges the warps of each segment; a pair split over
// several CTAs is merged by the last one to finish (counter + threadfence,
// partials in CTA order: deterministic).  History tiles are fetched before
// griddepcontrol.wait; only a tile holding the pair's newest row (appended by
// the previous kernel) waits for it.  More than 8 segments (very short
// pairs) are taken 8 at a time.
struct AttnSmall {
  uint64_t bar[kAttnMaxWarps][kAttnStages];
  int nseg;
  int seg_pair[128], seg_a[128], seg_b[128];
  long long off[129];  // prefix sums of the pair lengths (off[n_pairs] = total keys)
  int wseg[kAttnMaxWarps], wa[kAttnMaxWarps], wb[kAttnMaxWarps];  // per group: warp -> segment, key range
  int last[kAttnMaxWarps];
};

QASR_DEV void tma_load_2d(float *dst, const CUtensorMap *tm, int x, int y, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
          "r"(smem_u32(dst)),
      "l"(tm), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

constexpr int kMergeRegs = 4;  // partials a cross-CTA merge takes in one round of loads

template <int G, int W>
__global__ void __launch_bounds__(W * 32, kAttnCtasPerSm)
attn_decode_kernel(const __grid_constant__ AttnDecodeParams p) {
  static_assert(W <= kAttnMaxWarps, "warps per CTA");
  extern __shared__ __align__(128) unsigned char smem_raw[];
  constexpr int TILE_F = kAttnTile * 128;  // floats per K (or V) tile
  constexpr int KPW = kAttnTile;           // keys per tile
  float *tiles = reinterpret_cast<float *>(smem_raw);
  float *slots = tiles + (size_t)W * kAttnStages * 2 * TILE_F;  // [warp][G][kAttnPartStride]
  AttnSmall &sm = *reinterpret_cast<AttnSmall *>(slots + (size_t)W * G * kAttnPartStride);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kv = p.n_kv_heads, n_pairs = p.M * n_kv;
  // pair lengths -> prefix offsets, one warp-parallel scan (<= 128 pairs)
  if (warp == 0) {
    long long carry = 0;
    for (int base = 0; base < n_pairs; base += 32) {
      const int pr = base + lane;
      long long v = pr < n_pairs ? (long long)max(1, min(p.positions[pr / n_kv] + 1, p.max_seq)) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const long long t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (pr < n_pairs) sm.off[pr + 1] = carry + v;
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
    if (lane == 0) sm.off[0] = 0;
  }
  __syncthreads();
  const long long Tk = sm.off[n_pairs];
  // Virtual grid: only the first Gd CTAs take part, each owning at least
  // kAttnMinKeys keys -- or, when that would leave CTAs of the grid idle,
  // at least p.floor_keys -- (one when Tk is smaller), so the CTAs covering
  // a pair are exactly c_of(first key) .. c_of(last key) and short histories
  // are split into few partials.
  const long long per_cta = max((long long)max(1, p.floor_keys), min((long long)kAttnMinKeys, Tk / gridDim.x));
  const long long Gd = max(1ll, min((long long)gridDim.x, Tk / per_cta)), c = blockIdx.x;
  if (c >= Gd) return;
  const long long t0 = c * Tk / Gd, t1 = (c + 1) * Tk / Gd;

  if (threadIdx.x == 0) {
    int ns = 0;
    for (int pr = 0; pr < n_pairs && ns < 128; ++pr) {
      const long long off = sm.off[pr], len = sm.off[pr + 1] - off;
      const long long a = max(off, t0), b = min(off + len, t1);
      if (a < b) {
        sm.seg_pair[ns] = pr;
        sm.seg_a[ns] = (int)(a - off);
        sm.seg_b[ns] = (int)(b - off);
        ++ns;
      }
    }
    sm.nseg = ns;
  }
  if (lane < kAttnStages) mbar_init(&sm.bar[warp][lane], 1);
  mbar_fence_init();
  __syncthreads();
  const int nseg = sm.nseg;
  float *mytiles = tiles + (size_t)warp * kAttnStages * 2 * TILE_F;
  // CTAs covering a pair: c_of(t) = floor(((t+1)*Gd - 1) / Tk) of its first and last key
  auto c_first = [&](int s) { return ((sm.off[sm.seg_pair[s]] + 1) * Gd - 1) / Tk; };
  auto c_last = [&](int s) { return (sm.off[sm.seg_pair[s] + 1] * Gd - 1) / Tk; };

  int issued = 0, waited = 0;  // this warp's ring items, over all groups
  bool failed = false;
  constexpr int V = G * KPW;
  const int my_idx = reduce_index<V>(lane);  // value (head my_idx/KPW, key my_idx%KPW)
  const bool writer = (lane & (32 / V - 1)) == 0;
  const int my_g = my_idx / KPW, my_key = my_idx % KPW;

  for (int g0 = 0; g0 < nseg; g0 += W) {
    const int gn = min(W, nseg - g0);
    if (threadIdx.x == 0) {
      // warps per segment in proportion to its keys (each segment gets >= 1)
      int cnt[W];
      long long len[W];
      for (int s = 0; s < gn; ++s) {
        cnt[s] = 1;
        len[s] = sm.seg_b[g0 + s] - sm.seg_a[g0 + s];
      }
      for (int extra = W - gn; extra > 0; --extra) {
        int best = 0;
        for (int s = 1; s < gn; ++s)  // largest keys per warp gets the next warp
          if (len[s] * cnt[best] > len[best] * cnt[s]) best = s;
        ++cnt[best];
      }
      int w = 0;
      for (int s = 0; s < gn; ++s) {
        const int a = sm.seg_a[g0 + s], n = sm.seg_b[g0 + s] - a;
        for (int i = 0; i < cnt[s]; ++i, ++w) {
          sm.wseg[w] = g0 + s;
          sm.wa[w] = a + (int)((long long)n * i / cnt[s]);
          sm.wb[w] = a + (int)((long long)n * (i + 1) / cnt[s]);
        }
      }
    }
    __syncthreads();
    const int sg = sm.wseg[warp], wa = sm.wa[warp], wb = sm.wb[warp];
    const int pr = sm.seg_pair[sg], m = pr / n_kv, kvh = pr % n_kv;
    const int T = (wb - wa + KPW - 1) / KPW;  // tiles of this warp in this group
    const int newest = p.positions[m];         // row appended by the previous kernel
    const int row0 = (m * p.n_layers + p.layer) * p.max_seq;
    const int first_item = issued;             // ring index of this group's tile 0
    auto issue = [&](int i) {  // lane 0: tile i of this group
      const int st = issued % kAttnStages;
      mbar_arrive_expect_tx(&sm.bar[warp][st], 2 * TILE_F * 4);
      tma_load_2d(mytiles + (size_t)(2 * st) * TILE_F, &p.tm_k, kvh * 128, row0 + wa + i * KPW, &sm.bar[warp][st]);
      tma_load_2d(mytiles + (size_t)(2 * st + 1) * TILE_F, &p.tm_v, kvh * 128, row0 + wa + i * KPW, &sm.bar[warp][st]);
      ++issued;
    };
    int next_issue = 0;  // next tile of this group to issue (lane 0)
    if (g0 == 0) {
      // history tiles before the dependency wait, in order, up to the first
      // tile that holds the newest row
      if (lane == 0)
        while (next_issue < T && next_issue < kAttnStages && wa + next_issue * KPW + KPW - 1 < newest) issue(next_issue++);
      // q and the newest K/V rows come from the previous kernel
      pdl_wait();
      pdl_launch_dependents();
      if (p.tstamp && threadIdx.x == 0) atomicMin(p.tstamp, globaltimer_ns());
    }
    if (lane == 0)
      while (next_issue < T && next_issue < kAttnStages) issue(next_issue++);
    issued = __shfl_sync(0xffffffffu, issued, 0);
    __syncwarp();

    float mx[G], sum[G];
    float4 o[G], qv[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      qv[g] = *reinterpret_cast<const float4 *>(p.q + (size_t)m * p.q_stride + (kvh * G + g) * 128 + 4 * lane);
      mx[g] = -INFINITY;
      sum[g] = 0.0f;
      o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int i = 0; i < T; ++i) {
      const int item = first_item + i, st = item % kAttnStages;
      if (!failed) {  // warp-uniform outcome: the tile math below is warp-collective
        if (__all_sync(0xffffffffu, mbar_wait(&sm.bar[warp][st], (unsigned)((item / kAttnStages) & 1))))
          ++waited;
        else
          failed = true;
      }
      if (!failed) {
        const float *kt = mytiles + (size_t)(2 * st) * TILE_F;
        const float *vt = mytiles + (size_t)(2 * st + 1) * TILE_F;
        const int nk = min(KPW, wb - wa - i * KPW);
        float part[V];
#pragma unroll
        for (int j = 0; j < KPW; ++j) {
          const float4 kv = *reinterpret_cast<const float4 *>(kt + (size_t)j * 128 + 4 * lane);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float d = __fmul_rn(qv[g].x, kv.x);
            d = fmaf(qv[g].y, kv.y, d);
            d = fmaf(qv[g].z, kv.z, d);
            d = fmaf(qv[g].w, kv.w, d);
            part[g * KPW + j] = d;
          }
        }
        // the V rows do not depend on the scores: in flight during the softmax
        float4 vr[KPW];
#pragma unroll
        for (int j = 0; j < KPW; ++j) {
          vr[j] = *reinterpret_cast<const float4 *>(vt + (size_t)j * 128 + 4 * lane);
          if (j >= nk) vr[j] = make_float4(0.f, 0.f, 0.f, 0.f);  // rows past the range may hold anything
        }
        const float tot = warp_reduce_scatter<V>(part);
        const bool live = my_key < nk;
        const float sc = live ? __fmul_rn(tot, p.scale) : -INFINITY;
        // Each lane carries one (head, key) score, the key in lane bits KB ..
        // KB+LOGK-1 (lane (g*KPW + j) << KB holds head g, key j).
        constexpr int LOGK = Log2<KPW>::value, KB = 5 - Log2<V>::value;
        float mine = -INFINITY;
#pragma unroll
        for (int g = 0; g < G; ++g)
          if (my_g == g) mine = mx[g];
        // Online softmax with a lazy maximum: while no score exceeds its
        // head's running maximum by more than 8 (e^8 bounds the terms), the
        // maximum, the sums and the output keep their scale; only a tile that
        // does raise it pays for the tile maximum and the rescale.
        if (__any_sync(0xffffffffu, live && sc > __fadd_rn(mine, 8.0f))) {
          float hm = sc;
#pragma unroll
          for (int b = LOGK - 1; b >= 0; --b) hm = fmaxf(hm, __shfl_xor_sync(0xffffffffu, hm, 1 << (KB + b)));
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float nmax = fmaxf(mx[g], __shfl_sync(0xffffffffu, hm, g << (KB + LOGK)));
            const float corr = mx[g] == -INFINITY ? 0.0f : __expf(__fsub_rn(mx[g], nmax));
            mx[g] = nmax;
            sum[g] = __fmul_rn(sum[g], corr);
            o[g].x = __fmul_rn(o[g].x, corr);
            o[g].y = __fmul_rn(o[g].y, corr);
            o[g].z = __fmul_rn(o[g].z, corr);
            o[g].w = __fmul_rn(o[g].w, corr);
            if (my_g == g) mine = nmax;
          }
        }
        const float pj = live ? __expf(__fsub_rn(sc, mine)) : 0.0f;
        // per-lane exp-sums (one lane per (head, key)), reduced after the loop
#pragma unroll
        for (int g = 0; g < G; ++g) sum[g] = __fadd_rn(sum[g], (writer && my_g == g) ? pj : 0.0f);
        // o += p_j * V_j with p_j broadcast from the lane that holds it
#pragma unroll
        for (int j = 0; j < KPW; ++j) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float w = __shfl_sync(0xffffffffu, pj, (g * KPW + j) << KB);
            o[g].x = fmaf(w, vr[j].x, o[g].x);
            o[g].y = fmaf(w, vr[j].y, o[g].y);
            o[g].z = fmaf(w, vr[j].z, o[g].z);
            o[g].w = fmaf(w, vr[j].w, o[g].w);
          }
        }
      }
      __syncwarp();  // every lane is done with stage st
      if (lane == 0 && !failed && next_issue < T) {
        fence_proxy_async();
        issue(next_issue++);
      }
      issued = __shfl_sync(0xffffffffu, issued, 0);
    }
#pragma unroll
    for (int g = 0; g < G; ++g) sum[g] = warp_sum(sum[g]);  // the per-lane exp-sums
    // park this warp's state (an empty range leaves max = -inf, sum = 0)
    float *sl = slots + (size_t)warp * G * kAttnPartStride;
#pragma unroll
    for (int g = 0; g < G; ++g) {
      reinterpret_cast<float4 *>(sl + g * kAttnPartStride)[lane] = o[g];
      if (lane == 0) {
        sl[g * kAttnPartStride + 128] = mx[g];
        sl[g * kAttnPartStride + 129] = sum[g];
      }
    }
    __syncthreads();

    // ---- merge the warps of each segment of the group (task s*G+g: segment s, head g)
    bool any_split = false;
    for (int s = g0; s < g0 + gn; ++s) any_split |= c_first(s) != c_last(s);
    for (int task = warp; task < gn * G; task += W) {
      const int s = g0 + task / G, g = task % G;
      const int prs = sm.seg_pair[s], ms = prs / n_kv, kvs = prs % n_kv;
      float Mx = -INFINITY;
      for (int w = 0; w < W; ++w)
        if (sm.wseg[w] == s) Mx = fmaxf(Mx, slots[((size_t)w * G + g) * kAttnPartStride + 128]);
      float L = 0.0f;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
      for (int w = 0; w < W; ++w) {
        if (sm.wseg[w] != s) continue;
        const float *ws = slots + ((size_t)w * G + g) * kAttnPartStride;
        const float f = ws[128] == -INFINITY ? 0.0f : expf(__fsub_rn(ws[128], Mx));
        L = __fadd_rn(L, __fmul_rn(ws[129], f));
        const float4 ov = reinterpret_cast<const float4 *>(ws)[lane];
        acc.x = fmaf(ov.x, f, acc.x);
        acc.y = fmaf(ov.y, f, acc.y);
        acc.z = fmaf(ov.z, f, acc.z);
        acc.w = fmaf(ov.w, f, acc.w);
      }
      if (c_first(s) == c_last(s)) {
        const float inv = __fdiv_rn(1.0f, L);
        reinterpret_cast<float4 *>(p.out + (size_t)ms * p.out_stride + (kvs * G + g) * 128)[lane] =
            make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
      } else {
        float *slot = p.partials + ((size_t)(c + prs) * G + g) * kAttnPartStride;
        reinterpret_cast<float4 *>(slot)[lane] = acc;
        if (lane == 0) {
          slot[128] = Mx;
          slot[129] = L;
        }
      }
    }
    if (any_split) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x < gn) {
        const int s = g0 + threadIdx.x;
        const long long cf = c_first(s), cl = c_last(s);
        sm.last[threadIdx.x] = cf != cl && atomicAdd(p.counters + sm.seg_pair[s], 1u) == (unsigned)(cl - cf);
      }
      __syncthreads();
      for (int task = warp; task < gn * G; task += W) {
        if (!sm.last[task / G]) continue;
        __threadfence();
        const int s = g0 + task / G, g = task % G;
        const int prs = sm.seg_pair[s], ms = prs / n_kv, kvs = prs % n_kv;
        const long long cf = c_first(s), cl = c_last(s);
        auto part = [&](long long c2) { return p.partials + ((size_t)(c2 + prs) * G + g) * kAttnPartStride; };
        float Mx = -INFINITY, L = 0.0f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (cl - cf < kMergeRegs) {
          // up to kMergeRegs partials (the usual case): every load of the
          // merge in one round, then max, weights, sum and vector on registers
          float4 ov[kMergeRegs];
          float mp[kMergeRegs], lp[kMergeRegs];
#pragma unroll
          for (int u = 0; u < kMergeRegs; ++u) {
            ov[u] = make_float4(0.f, 0.f, 0.f, 0.f);
            mp[u] = -INFINITY;
            lp[u] = 0.0f;
            if (cf + u <= cl) {
              ov[u] = __ldcg(reinterpret_cast<const float4 *>(part(cf + u)) + lane);
              mp[u] = __ldcg(part(cf + u) + 128);
              lp[u] = __ldcg(part(cf + u) + 129);
            }
          }
#pragma unroll
          for (int u = 0; u < kMergeRegs; ++u)
            if (cf + u <= cl) Mx = fmaxf(Mx, mp[u]);
#pragma unroll
          for (int u = 0; u < kMergeRegs; ++u) {
            const float f = (cf + u > cl || mp[u] == -INFINITY) ? 0.0f : expf(__fsub_rn(mp[u], Mx));
            L = __fadd_rn(L, __fmul_rn(lp[u], f));
            acc.x = fmaf(ov[u].x, f, acc.x);
            acc.y = fmaf(ov[u].y, f, acc.y);
            acc.z = fmaf(ov[u].z, f, acc.z);
            acc.w = fmaf(ov[u].w, f, acc.w);
          }
        } else {
          // max and sum: one partial per lane, then a warp reduction
          for (long long c2 = cf + lane; c2 <= cl; c2 += 32) Mx = fmaxf(Mx, __ldcg(part(c2) + 128));
          Mx = warp_max(Mx);
          for (long long c2 = cf + lane; c2 <= cl; c2 += 32) {
            const float ms2 = __ldcg(part(c2) + 128);
            L = __fadd_rn(L, __fmul_rn(__ldcg(part(c2) + 129), ms2 == -INFINITY ? 0.0f : expf(__fsub_rn(ms2, Mx))));
          }
          L = warp_sum(L);
          // the vectors: independent loads, four partials per round
          for (long long c0 = cf; c0 <= cl; c0 += 4) {
            float4 ov[4];
            float f[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const long long c2 = min(c0 + u, cl);
              ov[u] = __ldcg(reinterpret_cast<const float4 *>(part(c2)) + lane);
              const float ms2 = __ldcg(part(c2) + 128);
              f[u] = (c0 + u > cl || ms2 == -INFINITY) ? 0.0f : expf(__fsub_rn(ms2, Mx));
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              acc.x = fmaf(ov[u].x, f[u], acc.x);
              acc.y = fmaf(ov[u].y, f[u], acc.y);
              acc.z = fmaf(ov[u].z, f[u], acc.z);
              acc.w = fmaf(ov[u].w, f[u], acc.w);
            }
          }
        }
        const float inv = __fdiv_rn(1.0f, L);
        *reinterpret_cast<float4 *>(p.out + (size_t)ms * p.out_stride + (kvs * G + g) * 128 + 4 * lane) =
            make_float4(__fmul_rn(acc.x, inv), __fmul_rn(acc.y, inv), __fmul_rn(acc.z, inv), __fmul_rn(acc.w, inv));
        if (lane == 0 && g == 0) p.counters[prs] = 0u;
      }
    }
    __syncthreads();  // slots and the warp map are rewritten by the next group
  }
  if (failed && lane == 0 && p.err) atomicExch(p.err, -QASR_ERR_TIMEOUT);
  // copies still in flight (only after a timeout) land before the CTA exits
  for (int k2 = waited; k2 < issued; ++k2)
    mbar_wait(&sm.bar[warp][k2 % kAttnStages], (unsigned)((k2 / kAttnStages) & 1));
  if (p.tstamp) {
    __syncthreads();
    if (threadIdx.x == 0) atomicMax(p.tstamp + 1, globaltimer_ns());
  }
}

// kernels::causal_attention for n segments in one launch (blockIdx.z):
// segs (device) give each segment's query rows in q/out, its key/value
// offset into k/v, its lengths and causal offset.
int causal_attention_segments(float *out, const float *q, const float *k, const float *v, const CaSeg *segs, int n,
                              int max_seq_q, int n_heads, int n_kv_heads, int head_dim, float scale,
                              cudaStream_t st) {
  const int G = n_heads / n_kv_heads;
  if (G > kCaTasks || n_heads % n_kv_heads || (head_dim != 64 && head_dim != 128) || n <= 0 || n > 65535) {
    set_error("causal attention: unsupported shape");
    return QASR_ERR_UNSUPPORTED;
  }
  const int QB = std::max(1, kCaTasks / G);
  const dim3 grid((unsigned)((max_seq_q + QB - 1) / QB), (unsigned)n_kv_heads, (unsigned)n);
  const CaSeg none{};
  if (head_dim == 128)
    causal_attention_kernel<4><<<grid, 256, 0, st>>>(out, q, k, v, none, segs, n_heads, n_kv_heads, scale);
  else
    causal_attention_kernel<2><<<grid, 256, 0, st>>>(out, q, k, v, none, segs, n_heads, n_kv_heads, scale);
  return launch_status("causal attention (segments)");
}

int attn_decode_grid() { return attn_grid() * kAttnCtasPerSm; }

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

static size_t attn_smem(int G, int W) {
  return (size_t)W * kAttnStages * 2 * kAttnTile * 128 * 4 + (size_t)W * G * kAttnPartStride * 4 + sizeof(AttnSmall);
}

template <int G, int W>
static int attn_launch_t(const AttnDecodeParams &p, cudaStream_t st, bool pdl) {
  static bool attr_done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return QASR_ERR_INVALID;
  if (!attr_done[dev]) {
    int rc = cuda_status(cudaFuncSetAttribute(attn_decode_kernel<G, W>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)attn_smem(G, W)),
                         "attention: shared memory opt-in");
    if (rc) return rc;
    attr_done[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)attn_decode_grid());
  cfg.blockDim = dim3(W * 32);
  cfg.dynamicSmemBytes = attn_smem(G, W);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, attn_decode_kernel<G, W>, p), "attention launch");
}

int attn_decode_launch(const AttnDecodeParams &p, int group, cudaStream_t st, bool pdl) {
  if (p.M * p.n_kv_heads > 128) {
    set_error("attention: M*n_kv_heads = %d > 128", p.M * p.n_kv_heads);
    return QASR_ERR_UNSUPPORTED;
  }
  const bool wide = p.M >= kAttnWideFromM;
  AttnDecodeParams q = p;
  q.floor_keys = wide ? kAttnFloorKeys : kAttnMinKeys;
  switch (group) {
    case 1: return wide ? attn_launch_t<1, kAttnWideWarps>(q, st, pdl) : attn_launch_t<1, kAttnMaxWarps>(q, st, pdl);
    case 2: return wide ? attn_launch_t<2, kAttnWideWarps>(q, st, pdl) : attn_launch_t<2, kAttnMaxWarps>(q, st, pdl);
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
  const int G = n_heads / n_kv_heads;
  if (G > kCaTasks) {
    set_error("qasr_causal_attention: %d query heads per kv head unsupported (at most %d)", G, kCaTasks);
    return QASR_ERR_UNSUPPORTED;
  }
  const int QB = std::max(1, kCaTasks / G);
  const dim3 grid((unsigned)((seq_q + QB - 1) / QB), (unsigned)n_kv_heads);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const CaSeg one{0, seq_q, seq_k, q_offset, 0};
  if (head_dim == 128)
    causal_attention_kernel<4><<<grid, 256, 0, st>>>(out, q, k, v, one, nullptr, n_heads, n_kv_heads, scale);
  else
    causal_attention_kernel<2><<<grid, 256, 0, st>>>(out, q, k, v, one, nullptr, n_heads, n_kv_heads, scale);
  return launch_status("qasr_causal_attention");
}
