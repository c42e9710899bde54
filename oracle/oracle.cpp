// oracle.cpp -- CPU restatement of the QwenASR x86_64 kernel path.
//
// TEST INFRASTRUCTURE ONLY (parity checker + timed CPU baseline); see oracle.h
// for what is restated and how it is pinned.  Reference paths are relative to
// crates/qwen-asr/src/ of ZhaoChaoqun/QwenASR.
//
// Build: oracle/Makefile (g++ -O3 -march=native -ffp-contract=off).  The
// no-contraction flag matters: Rust evaluates `a * b + c` as two roundings.
#include "oracle.h"

#include <cmath>
#include <cstring>
#include <vector>
#include <thread>
#include <mutex>
#include <condition_variable>
#include <functional>
#include <algorithm>
#include <atomic>

namespace {

// --------------------------------------------------------------------------
// Thread pool.  Semantics of kernels::parallel_for (mod.rs:316-361): the
// caller runs tid 0, workers run tids 1..n-1, work is split by the closure
// itself (output rows in ceil(out/nt) chunks).  Capped at 16 (mod.rs:177).
// --------------------------------------------------------------------------
class Pool {
 public:
  void set_threads(int n) {
    n = std::max(1, std::min(16, n));
    std::unique_lock<std::mutex> lk(mu_);
    while ((int)workers_.size() < n - 1) {
      int tid = (int)workers_.size() + 1;
      workers_.emplace_back([this, tid] { worker(tid); });
    }
    n_threads_ = n;
  }
  int threads() const { return n_threads_; }

  void run(const std::function<void(int, int)> &fn) {
    int nt = n_threads_;
    if (nt <= 1) { fn(0, 1); return; }
    {
      std::unique_lock<std::mutex> lk(mu_);
      job_ = &fn;
      job_nt_ = nt;
      n_done_ = 0;
      ++generation_;
    }
    work_cv_.notify_all();
    fn(0, nt);
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return n_done_ >= nt - 1; });
    job_ = nullptr;
  }

  ~Pool() {
    {
      std::unique_lock<std::mutex> lk(mu_);
      shutdown_ = true;
    }
    work_cv_.notify_all();
    for (auto &t : workers_) t.join();
  }

 private:
  void worker(int tid) {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void(int, int)> *job;
      int nt;
      {
        std::unique_lock<std::mutex> lk(mu_);
        work_cv_.wait(lk, [&] { return shutdown_ || generation_ != seen; });
        if (shutdown_) return;
        seen = generation_;
        job = job_;
        nt = job_nt_;
      }
      if (job && tid < nt) (*job)(tid, nt);
      {
        std::unique_lock<std::mutex> lk(mu_);
        if (job && tid < nt) ++n_done_;
      }
      done_cv_.notify_one();
    }
  }
  std::mutex mu_;
  std::condition_variable work_cv_, done_cv_;
  std::vector<std::thread> workers_;
  const std::function<void(int, int)> *job_ = nullptr;
  int job_nt_ = 1;
  int n_threads_ = 1;
  int n_done_ = 0;
  uint64_t generation_ = 0;
  bool shutdown_ = false;
};

Pool &pool() {
  static Pool p;
  return p;
}

// Row-range split used by every threaded kernel in mod.rs (e.g. 606-618).
inline void chunk_range(int total, int tid, int nt, int &s, int &e) {
  int chunk = (total + nt - 1) / nt;
  s = tid * chunk;
  e = std::min(s + chunk, total);
}

// --------------------------------------------------------------------------
// 8-lane emulation of the AVX2 helpers in avx.rs.
// --------------------------------------------------------------------------
struct F8 {
  float v[8];
};
inline F8 f8_zero() { F8 r; for (int l = 0; l < 8; ++l) r.v[l] = 0.0f; return r; }
inline F8 f8_load(const float *p) { F8 r; for (int l = 0; l < 8; ++l) r.v[l] = p[l]; return r; }
inline F8 f8_add(F8 a, F8 b) { F8 r; for (int l = 0; l < 8; ++l) r.v[l] = a.v[l] + b.v[l]; return r; }
inline F8 f8_fma(F8 a, F8 b, F8 c) { F8 r; for (int l = 0; l < 8; ++l) r.v[l] = fmaf(a.v[l], b.v[l], c.v[l]); return r; }

// hsum_ps (avx.rs:36-49): (v0+v4 + v1+v5) + (v2+v6 + v3+v7) in that tree.
inline float hsum8(F8 v) {
  float s0 = v.v[0] + v.v[4], s1 = v.v[1] + v.v[5], s2 = v.v[2] + v.v[6], s3 = v.v[3] + v.v[7];
  return (s0 + s1) + (s2 + s3);
}

// fast_exp_avx (avx.rs:487-514), one lane.  _mm256_cvtps_epi32 rounds to
// nearest-even under the default MXCSR, which is nearbyintf here.
inline float fast_exp_lane(float x) {
  const float log2e = 1.442695041f;
  const float ln2 = 0.6931471806f;
  float val = x * log2e;
  val = std::min(val, 126.0f);   // _mm256_min_ps(val, 126)
  val = std::max(val, -126.0f);  // _mm256_max_ps(val, -126)
  int32_t ip = (int32_t)nearbyintf(val);
  float fp = val - (float)ip;
  uint32_t bits = (uint32_t)(ip + 127) << 23;
  float exp_i;
  std::memcpy(&exp_i, &bits, 4);
  float f = fp * ln2;
  const float c2 = 0.5f, c3 = 1.0f / 6.0f, c4 = 1.0f / 24.0f, c5 = 1.0f / 120.0f;
  float p = fmaf(c5, f, c4);
  p = fmaf(p, f, c3);
  p = fmaf(p, f, c2);
  p = fmaf(p, f, 1.0f);
  p = fmaf(p, f, 1.0f);
  return exp_i * p;
}

// avx::rms_norm_row (avx.rs:377-415).
void rms_norm_row(float *out, const float *x, const float *w, int hidden, float eps) {
  int i = 0;
  F8 acc0 = f8_zero(), acc1 = f8_zero();
  for (; i + 16 <= hidden; i += 16) {
    F8 x0 = f8_load(x + i), x1 = f8_load(x + i + 8);
    acc0 = f8_fma(x0, x0, acc0);
    acc1 = f8_fma(x1, x1, acc1);
  }
  for (; i + 8 <= hidden; i += 8) {
    F8 xv = f8_load(x + i);
    acc0 = f8_fma(xv, xv, acc0);
  }
  float sum_sq = hsum8(f8_add(acc0, acc1));
  for (; i < hidden; ++i) sum_sq += x[i] * x[i];
  float rms_inv = 1.0f / sqrtf(sum_sq / (float)hidden + eps);
  for (int j = 0; j < hidden; ++j) out[j] = (x[j] * rms_inv) * w[j];
}

// avx::layer_norm_row (avx.rs:420-481).
void layer_norm_row(float *out, const float *x, const float *w, const float *b, int hidden, float eps) {
  int i = 0;
  F8 s0 = f8_zero(), s1 = f8_zero();
  for (; i + 16 <= hidden; i += 16) {
    s0 = f8_add(s0, f8_load(x + i));
    s1 = f8_add(s1, f8_load(x + i + 8));
  }
  for (; i + 8 <= hidden; i += 8) s0 = f8_add(s0, f8_load(x + i));
  float mean = hsum8(f8_add(s0, s1));
  for (; i < hidden; ++i) mean += x[i];
  mean /= (float)hidden;

  i = 0;
  F8 v0 = f8_zero(), v1 = f8_zero();
  for (; i + 16 <= hidden; i += 16) {
    F8 d0, d1;
    for (int l = 0; l < 8; ++l) { d0.v[l] = x[i + l] - mean; d1.v[l] = x[i + 8 + l] - mean; }
    v0 = f8_fma(d0, d0, v0);
    v1 = f8_fma(d1, d1, v1);
  }
  for (; i + 8 <= hidden; i += 8) {
    F8 d;
    for (int l = 0; l < 8; ++l) d.v[l] = x[i + l] - mean;
    v0 = f8_fma(d, d, v0);
  }
  float var = hsum8(f8_add(v0, v1));
  for (; i < hidden; ++i) { float d = x[i] - mean; var += d * d; }
  float inv_std = 1.0f / sqrtf(var / (float)hidden + eps);

  int vec_end = hidden - hidden % 8;
  for (int j = 0; j < vec_end; ++j) out[j] = fmaf((x[j] - mean) * inv_std, w[j], b[j]);
  for (int j = vec_end; j < hidden; ++j) out[j] = (x[j] - mean) * inv_std * w[j] + b[j];
}

// avx::dot_f32 (avx.rs:247-299): 4 x 8-lane accumulators over 32-blocks, then
// 8-blocks into acc0, hsum((a0+a1)+(a2+a3)), scalar tail.
float dot_avx(const float *a, const float *b, int n) {
  int i = 0;
  F8 a0 = f8_zero(), a1 = f8_zero(), a2 = f8_zero(), a3 = f8_zero();
  for (; i + 32 <= n; i += 32) {
    a0 = f8_fma(f8_load(a + i), f8_load(b + i), a0);
    a1 = f8_fma(f8_load(a + i + 8), f8_load(b + i + 8), a1);
    a2 = f8_fma(f8_load(a + i + 16), f8_load(b + i + 16), a2);
    a3 = f8_fma(f8_load(a + i + 24), f8_load(b + i + 24), a3);
  }
  for (; i + 8 <= n; i += 8) a0 = f8_fma(f8_load(a + i), f8_load(b + i), a0);
  float sum = hsum8(f8_add(f8_add(a0, a1), f8_add(a2, a3)));
  for (; i < n; ++i) sum += a[i] * b[i];
  return sum;
}

// avx::vec_scale_add (avx.rs:346-370): dst = fma(dst, c, src) on 8-lane
// blocks, dst*c + src on the tail.
void scale_add_avx(float *dst, const float *src, float c, int n) {
  int vec_end = n - n % 8;
  for (int i = 0; i < vec_end; ++i) dst[i] = fmaf(dst[i], c, src[i]);
  for (int i = vec_end; i < n; ++i) dst[i] = dst[i] * c + src[i];
}
// avx::vec_axpy_inplace (avx.rs:322-343): dst = fma(src, a, dst).
void axpy_avx(float *dst, const float *src, float a, int n) {
  int vec_end = n - n % 8;
  for (int i = 0; i < vec_end; ++i) dst[i] = fmaf(src[i], a, dst[i]);
  for (int i = vec_end; i < n; ++i) dst[i] += a * src[i];
}
// avx::vec_scale_inplace (avx.rs:301-320).
void scale_avx(float *dst, float s, int n) {
  for (int i = 0; i < n; ++i) dst[i] *= s;
}

// generic::int8_matvec_fused (generic.rs:39-49): sequential f32 sum of
// f32(w)*x, scaled once at the end.
void int8_matvec_rows(float *y, const float *x, const int8_t *w, const float *scales, int in_dim,
                      int row_begin, int row_end) {
  for (int o = row_begin; o < row_end; ++o) {
    const int8_t *wr = w + (size_t)o * in_dim;
    float sum = 0.0f;
    for (int k = 0; k < in_dim; ++k) sum += (float)wr[k] * x[k];
    y[o] = sum * scales[o];
  }
}

// int8_matvec_threaded (mod.rs:622-647).
void int8_matvec_threaded(float *y, const float *x, const int8_t *w, const float *scales, int in_dim, int out_dim) {
  pool().run([&](int tid, int nt) {
    int s, e;
    chunk_range(out_dim, tid, nt, s, e);
    if (s < e) int8_matvec_rows(y, x, w, scales, in_dim, s, e);
  });
}

// causal_attention_heads (mod.rs:1124-1172).
void causal_heads(float *out, const float *q, const float *k, const float *v, int seq_q, int seq_k,
                  int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, int h0, int h1) {
  int heads_per_kv = n_heads / n_kv_heads;
  size_t q_hidden = (size_t)n_heads * head_dim, kv_hidden = (size_t)n_kv_heads * head_dim;
  for (int h = h0; h < h1; ++h) {
    int kv_h = h / heads_per_kv;
    for (int i = 0; i < seq_q; ++i) {
      const float *q_row = q + i * q_hidden + (size_t)h * head_dim;
      float *o_row = out + i * q_hidden + (size_t)h * head_dim;
      int global_pos = q_offset + i;
      int k_end = std::min(global_pos + 1, seq_k);
      float max_score = -1e30f, sum_exp = 0.0f;
      for (int d = 0; d < head_dim; ++d) o_row[d] = 0.0f;
      for (int j = 0; j < k_end; ++j) {
        const float *k_row = k + j * kv_hidden + (size_t)kv_h * head_dim;
        const float *v_row = v + j * kv_hidden + (size_t)kv_h * head_dim;
        float score = dot_avx(q_row, k_row, head_dim) * scale;
        if (score > max_score) {
          float corr = expf(max_score - score);
          sum_exp = sum_exp * corr + 1.0f;
          scale_add_avx(o_row, v_row, corr, head_dim);
          max_score = score;
        } else {
          float wt = expf(score - max_score);
          sum_exp += wt;
          axpy_avx(o_row, v_row, wt, head_dim);
        }
      }
      if (sum_exp > 0.0f) scale_avx(o_row, 1.0f / sum_exp, head_dim);
    }
  }
}

}  // namespace

extern "C" {

void orc_set_threads(int n) { pool().set_threads(n); }
int orc_get_threads(void) { return pool().threads(); }

// kernels::rms_norm (mod.rs:897-918) on x86_64 -> avx::rms_norm_row.
void orc_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps) {
  for (int s = 0; s < seq; ++s) rms_norm_row(out + (size_t)s * hidden, x + (size_t)s * hidden, w, hidden, eps);
}

// kernels::rms_norm_per_head (mod.rs:920-935): scalar sequential sum.
void orc_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim, float eps) {
  size_t hidden = (size_t)n_heads * head_dim;
  for (int s = 0; s < seq; ++s)
    for (int h = 0; h < n_heads; ++h) {
      float *vec = x + s * hidden + (size_t)h * head_dim;
      float sum_sq = 0.0f;
      for (int d = 0; d < head_dim; ++d) sum_sq += vec[d] * vec[d];
      float rms_inv = 1.0f / sqrtf(sum_sq / (float)head_dim + eps);
      for (int d = 0; d < head_dim; ++d) vec[d] = vec[d] * rms_inv * w[d];
    }
}

// kernels::layer_norm (mod.rs:866-895) on x86_64 -> avx::layer_norm_row.
void orc_layer_norm(float *out, const float *x, const float *w, const float *b, int seq, int hidden, float eps) {
  for (int s = 0; s < seq; ++s)
    layer_norm_row(out + (size_t)s * hidden, x + (size_t)s * hidden, w, b, hidden, eps);
}

// kernels::compute_rope_neox (mod.rs:1228-1245).
void orc_compute_rope_neox(float *cos_out, float *sin_out, const int32_t *positions, int seq, int head_dim, float theta) {
  int half = head_dim / 2;
  for (int s = 0; s < seq; ++s) {
    float pos = (float)positions[s];
    for (int d = 0; d < half; ++d) {
      float freq = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
      float angle = pos * freq;
      float c = cosf(angle), sn = sinf(angle);
      cos_out[s * head_dim + d] = c;
      cos_out[s * head_dim + half + d] = c;
      sin_out[s * head_dim + d] = sn;
      sin_out[s * head_dim + half + d] = sn;
    }
  }
}

// RopeCache::ensure (decoder.rs:253-289): rows 0..n_pos of the cos/sin table,
// inv_freq computed once, angle = p * inv_freq[d].
void orc_rope_cache_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta) {
  int half = head_dim / 2;
  std::vector<float> inv_freq(half);
  for (int d = 0; d < half; ++d) inv_freq[d] = 1.0f / powf(theta, (float)(2 * d) / (float)head_dim);
  for (int p = 0; p < n_pos; ++p) {
    float pf = (float)p;
    for (int d = 0; d < half; ++d) {
      float angle = pf * inv_freq[d];
      float c = cosf(angle), sn = sinf(angle);
      cos_out[(size_t)p * head_dim + d] = c;
      cos_out[(size_t)p * head_dim + half + d] = c;
      sin_out[(size_t)p * head_dim + d] = sn;
      sin_out[(size_t)p * head_dim + half + d] = sn;
    }
  }
}

// kernels::apply_rope_neox (mod.rs:1247-1267).
void orc_apply_rope_neox(float *x, const float *cos_v, const float *sin_v, int seq, int n_heads, int head_dim) {
  int half = head_dim / 2;
  size_t hidden = (size_t)n_heads * head_dim;
  for (int s = 0; s < seq; ++s) {
    const float *c = cos_v + (size_t)s * head_dim;
    const float *sn = sin_v + (size_t)s * head_dim;
    for (int h = 0; h < n_heads; ++h) {
      float *vec = x + s * hidden + (size_t)h * head_dim;
      for (int d = 0; d < half; ++d) {
        float x1 = vec[d], x2 = vec[half + d];
        vec[d] = x1 * c[d] + (-x2) * sn[d];
        vec[half + d] = x2 * c[half + d] + x1 * sn[half + d];
      }
    }
  }
}

// kernels::sinusoidal_pe (mod.rs:1213-1226).
void orc_sinusoidal_pe(float *pe, int n_pos, int d_model) {
  int half = d_model / 2;
  float log_timescale = logf(10000.0f) / (float)(half - 1);
  for (int p = 0; p < n_pos; ++p) {
    float *row = pe + (size_t)p * d_model;
    for (int d = 0; d < half; ++d) {
      float inv_ts = expf(-(float)d * log_timescale);
      float angle = (float)p * inv_ts;
      row[d] = sinf(angle);
      row[half + d] = cosf(angle);
    }
  }
}

// avx::gelu_inplace (avx.rs:536-563): fast_exp tanh on 8-blocks, libm tanhf tail.
void orc_gelu(float *x, long n) {
  long vec_end = n - n % 8;
  const float coeff = 0.7978845608028654f, c3 = 0.044715f;
  for (long i = 0; i < vec_end; ++i) {
    float v = x[i];
    float v2 = v * v, v3 = v2 * v;
    float inner = coeff * fmaf(c3, v3, v);
    float e = fast_exp_lane(2.0f * inner);
    float t = 1.0f - 2.0f / (e + 1.0f);
    x[i] = 0.5f * (v * (1.0f + t));
  }
  for (long i = vec_end; i < n; ++i) {
    float val = x[i];
    float x3 = val * val * val;
    float inner = 0.7978845608028654f * (val + 0.044715f * x3);
    x[i] = 0.5f * val * (1.0f + tanhf(inner));
  }
}

// Exact-erf GELU, 0.5*x*(1+erf(x/sqrt(2))): the encoder activation of the
// reference's Metal path (encoder_gpu.rs:470,480) and of the BASELINE encoder config.
void orc_gelu_erf(float *x, long n) {
  const float inv_sqrt2 = 0.70710678118654752f;
  for (long i = 0; i < n; ++i) {
    float v = x[i];
    x[i] = 0.5f * v * (1.0f + erff(v * inv_sqrt2));
  }
}

// kernels::silu (mod.rs:941-946).
void orc_silu(float *x, long n) {
  for (long i = 0; i < n; ++i) { float v = x[i]; x[i] = v / (1.0f + expf(-v)); }
}

// kernels::swiglu_multiply (mod.rs:965-985) -> avx::swiglu_interleaved (avx.rs:568-599).
void orc_swiglu_multiply(float *out, const float *gate_up, int seq, int inter) {
  int vec_end = inter - inter % 8;
  for (int s = 0; s < seq; ++s) {
    const float *gu = gate_up + (size_t)s * 2 * inter;
    float *o = out + (size_t)s * inter;
    for (int j = 0; j < vec_end; ++j) {
      float g = gu[2 * j], u = gu[2 * j + 1];
      float e = fast_exp_lane(0.0f - g);
      float silu_g = g / (1.0f + e);
      o[j] = silu_g * u;
    }
    for (int j = vec_end; j < inter; ++j) {
      float g = gu[2 * j], u = gu[2 * j + 1];
      float gs = g / (1.0f + expf(-g));
      o[j] = gs * u;
    }
  }
}

// Decode-path SwiGLU, scalar with libm exp (decoder.rs:916-921).
void orc_swiglu_decode(float *out, const float *gate_up, int inter) {
  for (int j = 0; j < inter; ++j) {
    float g = gate_up[2 * j], u = gate_up[2 * j + 1];
    float gs = g / (1.0f + expf(-g));
    out[j] = gs * u;
  }
}

// kernels::softmax (mod.rs:996-1032) on x86_64 (avx::exp_inplace).
void orc_softmax(float *x, int rows, int cols) {
  int vec_end = cols - cols % 8;
  for (int r = 0; r < rows; ++r) {
    float *row = x + (size_t)r * cols;
    float mx = -INFINITY;
    for (int c = 0; c < cols; ++c) mx = std::max(mx, row[c]);
    for (int c = 0; c < cols; ++c) row[c] -= mx;
    for (int c = 0; c < vec_end; ++c) row[c] = fast_exp_lane(row[c]);
    for (int c = vec_end; c < cols; ++c) row[c] = expf(row[c]);
    float sum = 0.0f;
    for (int c = 0; c < cols; ++c) sum += row[c];
    float inv = 1.0f / sum;
    for (int c = 0; c < cols; ++c) row[c] *= inv;
  }
}

float orc_fast_exp(float x) { return fast_exp_lane(x); }
float orc_dot_f32(const float *a, const float *b, int n) { return dot_avx(a, b, n); }
float orc_dot_f32_generic(const float *a, const float *b, int n) {
  float s = 0.0f;
  for (int i = 0; i < n; ++i) s += a[i] * b[i];
  return s;
}
void orc_vec_scale_inplace(float *dst, float s, int n) { scale_avx(dst, s, n); }
void orc_vec_axpy_inplace(float *dst, const float *src, float alpha, int n) { axpy_avx(dst, src, alpha, n); }
void orc_vec_scale_add(float *dst, const float *src, float c, int n) { scale_add_avx(dst, src, c, n); }
void orc_add_inplace(float *a, const float *b, long n) { for (long i = 0; i < n; ++i) a[i] += b[i]; }

// kernels::linear_nobias_int8 (mod.rs:650-661): seq_len > 1 is a loop of matvecs.
void orc_linear_nobias_int8(float *y, const float *x, const int8_t *w, const float *scales,
                            int seq, int in_dim, int out_dim) {
  for (int s = 0; s < seq; ++s)
    int8_matvec_threaded(y + (size_t)s * out_dim, x + (size_t)s * in_dim, w, scales, in_dim, out_dim);
}

// kernels::linear_int8 (mod.rs:664-673).
void orc_linear_int8(float *y, const float *x, const int8_t *w, const float *scales,
                     const float *bias, int seq, int in_dim, int out_dim) {
  orc_linear_nobias_int8(y, x, w, scales, seq, in_dim, out_dim);
  if (bias)
    for (int s = 0; s < seq; ++s)
      for (int o = 0; o < out_dim; ++o) y[(size_t)s * out_dim + o] += bias[o];
}

// kernels::linear (mod.rs:531-565) calls cblas_sgemm, whose summation order is
// the BLAS library's own (unpinned).  This stand-in accumulates in double and
// rounds once, i.e. it is the exact product to f32 precision; bias is added
// afterwards in f32 like the reference.
void orc_linear(float *y, const float *x, const float *w, const float *bias, int seq, int in_dim, int out_dim) {
  pool().run([&](int tid, int nt) {
    int s0, s1;
    chunk_range(out_dim, tid, nt, s0, s1);
    for (int s = 0; s < seq; ++s) {
      const float *xr = x + (size_t)s * in_dim;
      for (int o = s0; o < s1; ++o) {
        const float *wr = w + (size_t)o * in_dim;
        double acc = 0.0;
        for (int k = 0; k < in_dim; ++k) acc += (double)xr[k] * (double)wr[k];
        float r = (float)acc;
        if (bias) r += bias[o];
        y[(size_t)s * out_dim + o] = r;
      }
    }
  });
}

static inline float bf16f(uint16_t b) {
  uint32_t u = (uint32_t)b << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

// generic::bf16_matvec_fused (generic.rs:8-17).
void orc_bf16_matvec_generic(float *y, const float *x, const uint16_t *w, const float *bias, int in_dim, int out_dim) {
  for (int o = 0; o < out_dim; ++o) {
    float sum = bias ? bias[o] : 0.0f;
    for (int k = 0; k < in_dim; ++k) sum += bf16f(w[(size_t)o * in_dim + k]) * x[k];
    y[o] = sum;
  }
}

// avx::bf16_matvec_fused (avx.rs:55-163), single-row form: two 8-lane
// accumulators over 16-blocks, 8-block into acc0, sum += hsum(acc0+acc1), tail.
// (The two-rows-at-a-time loop in the reference uses identical per-row order.)
void orc_bf16_matvec(float *y, const float *x, const uint16_t *w, const float *bias, int in_dim, int out_dim) {
  for (int o = 0; o < out_dim; ++o) {
    const uint16_t *wr = w + (size_t)o * in_dim;
    float sum = bias ? bias[o] : 0.0f;
    F8 a0 = f8_zero(), a1 = f8_zero();
    int k = 0;
    for (; k + 16 <= in_dim; k += 16) {
      F8 wl, wh;
      for (int l = 0; l < 8; ++l) { wl.v[l] = bf16f(wr[k + l]); wh.v[l] = bf16f(wr[k + 8 + l]); }
      a0 = f8_fma(wl, f8_load(x + k), a0);
      a1 = f8_fma(wh, f8_load(x + k + 8), a1);
    }
    for (; k + 8 <= in_dim; k += 8) {
      F8 wv;
      for (int l = 0; l < 8; ++l) wv.v[l] = bf16f(wr[k + l]);
      a0 = f8_fma(wv, f8_load(x + k), a0);
    }
    sum += hsum8(f8_add(a0, a1));
    for (; k < in_dim; ++k) sum += bf16f(wr[k]) * x[k];
    y[o] = sum;
  }
}

// kernels::causal_attention (mod.rs:1174-1207): heads split over the pool.
void orc_causal_attention(float *out, const float *q, const float *k, const float *v,
                          int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim,
                          float scale, int q_offset) {
  pool().run([&](int tid, int nt) {
    int h0, h1;
    chunk_range(n_heads, tid, nt, h0, h1);
    if (h0 < h1) causal_heads(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset, h0, h1);
  });
}

// kernels::bidirectional_attention (mod.rs:1038-1122).
void orc_bidirectional_attention(float *out, const float *q, const float *k, const float *v,
                                 int seq, int n_heads, int head_dim, float scale,
                                 const int32_t *window_starts, int n_windows) {
  (void)seq;
  size_t hidden = (size_t)n_heads * head_dim;
  pool().run([&](int tid, int nt) {
    int h0, h1;
    chunk_range(n_heads, tid, nt, h0, h1);
    for (int h = h0; h < h1; ++h)
      for (int w = 0; w < n_windows; ++w) {
        int ws = window_starts[w], we = window_starts[w + 1];
        for (int i = ws; i < we; ++i) {
          const float *q_row = q + i * hidden + (size_t)h * head_dim;
          float *o_row = out + i * hidden + (size_t)h * head_dim;
          float max_score = -1e30f, sum_exp = 0.0f;
          for (int d = 0; d < head_dim; ++d) o_row[d] = 0.0f;
          for (int j = ws; j < we; ++j) {
            const float *k_row = k + j * hidden + (size_t)h * head_dim;
            const float *v_row = v + j * hidden + (size_t)h * head_dim;
            float score = dot_avx(q_row, k_row, head_dim) * scale;
            if (score > max_score) {
              float corr = expf(max_score - score);
              sum_exp = sum_exp * corr + 1.0f;
              scale_add_avx(o_row, v_row, corr, head_dim);
              max_score = score;
            } else {
              float wt = expf(score - max_score);
              sum_exp += wt;
              axpy_avx(o_row, v_row, wt, head_dim);
            }
          }
          if (sum_exp > 0.0f) scale_avx(o_row, 1.0f / sum_exp, head_dim);
        }
      }
  });
}

// quantize_f32_to_int8 (quantize.rs:633-662): symmetric per-row, Rust
// f32::round = round half away from zero = roundf.
void orc_quantize_f32_to_int8(const float *data, int64_t out_dim, int64_t in_dim, int8_t *q, float *scales) {
  for (int64_t o = 0; o < out_dim; ++o) {
    const float *row = data + o * in_dim;
    float absmax = 0.0f;
    for (int64_t k = 0; k < in_dim; ++k) {
      float a = fabsf(row[k]);
      if (a > absmax) absmax = a;
    }
    scales[o] = absmax / 127.0f;
    float inv = absmax > 0.0f ? 127.0f / absmax : 0.0f;
    for (int64_t k = 0; k < in_dim; ++k) {
      float r = roundf(row[k] * inv);
      r = std::min(std::max(r, -128.0f), 127.0f);
      q[o * in_dim + k] = (int8_t)r;
    }
  }
}

// tok_embed_int8_to_f32 (decoder.rs:639-646).
void orc_embed_int8(float *dst, const int8_t *table, const float *scales, int token, int dim) {
  const int8_t *row = table + (size_t)token * dim;
  float s = scales[token];
  for (int i = 0; i < dim; ++i) dst[i] = (float)row[i] * s;
}

// tok_embed_bf16_to_f32 (decoder.rs:631-636).
void orc_embed_bf16(float *dst, const uint16_t *table, int token, int dim) {
  for (int i = 0; i < dim; ++i) dst[i] = bf16f(table[(size_t)token * dim + i]);
}

// First-max argmax with strict '>' (decoder.rs:942-947).
int orc_argmax_first(const float *x, int n) {
  int best = 0;
  float bv = x[0];
  for (int i = 1; i < n; ++i)
    if (x[i] > bv) { bv = x[i]; best = i; }
  return best;
}

// Gate/up row interleave of DecoderInt8::load (decoder.rs:699-719).
void orc_interleave_gate_up(const int8_t *gate, const float *gate_s, const int8_t *up, const float *up_s,
                            int inter, int hidden, int8_t *fused, float *fused_s) {
  for (int r = 0; r < inter; ++r) {
    std::memcpy(fused + (size_t)(2 * r) * hidden, gate + (size_t)r * hidden, hidden);
    std::memcpy(fused + (size_t)(2 * r + 1) * hidden, up + (size_t)r * hidden, hidden);
    fused_s[2 * r] = gate_s[r];
    fused_s[2 * r + 1] = up_s[r];
  }
}

// decoder_forward_int8 (decoder.rs:845-965) for one sequence at position pos.
// Returns the greedy token; logits_out (optional, [vocab]) and x_out
// (optional, [hidden], the final-normed hidden state) expose intermediates.
int orc_decoder_forward_int8(const orc_decoder *dec, float *k_cache, float *v_cache, int max_seq,
                             int pos, const float *input_embed, float *logits_out, float *x_out) {
  const int dim = dec->hidden, nh = dec->n_heads, nkv = dec->n_kv_heads, hd = dec->head_dim;
  const int inter = dec->inter, q_dim = nh * hd, kv_dim = nkv * hd;
  const float eps = dec->eps;
  std::vector<float> x(input_embed, input_embed + dim), x_norm(dim), q(q_dim), k(kv_dim), v(kv_dim);
  std::vector<float> attn(q_dim), proj(dim), gate_buf(2 * inter), ffn(inter);
  std::vector<float> cosr(hd), sinr(hd);
  int32_t p32 = pos;
  // RopeCache::cos_at(pos) == row pos of the ensure() table.
  {
    int half = hd / 2;
    for (int d = 0; d < half; ++d) {
      float inv_freq = 1.0f / powf(dec->theta, (float)(2 * d) / (float)hd);
      float angle = (float)p32 * inv_freq;
      cosr[d] = cosr[half + d] = cosf(angle);
      sinr[d] = sinr[half + d] = sinf(angle);
    }
  }
  float scale = 1.0f / sqrtf((float)hd);
  for (int l = 0; l < dec->n_layers; ++l) {
    const orc_dec_layer &L = dec->layers[l];
    orc_rms_norm(x_norm.data(), x.data(), L.input_norm, 1, dim, eps);
    int8_matvec_threaded(q.data(), x_norm.data(), L.wq, L.wq_s, dim, q_dim);
    int8_matvec_threaded(k.data(), x_norm.data(), L.wk, L.wk_s, dim, kv_dim);
    int8_matvec_threaded(v.data(), x_norm.data(), L.wv, L.wv_s, dim, kv_dim);
    orc_rms_norm_per_head(q.data(), L.q_norm, 1, nh, hd, eps);
    orc_rms_norm_per_head(k.data(), L.k_norm, 1, nkv, hd, eps);
    orc_apply_rope_neox(q.data(), cosr.data(), sinr.data(), 1, nh, hd);
    orc_apply_rope_neox(k.data(), cosr.data(), sinr.data(), 1, nkv, hd);
    size_t off = ((size_t)l * max_seq + pos) * kv_dim;
    std::memcpy(k_cache + off, k.data(), kv_dim * 4);
    std::memcpy(v_cache + off, v.data(), kv_dim * 4);
    const float *fk = k_cache + (size_t)l * max_seq * kv_dim;
    const float *fv = v_cache + (size_t)l * max_seq * kv_dim;
    orc_causal_attention(attn.data(), q.data(), fk, fv, 1, pos + 1, nh, nkv, hd, scale, pos);
    int8_matvec_threaded(proj.data(), attn.data(), L.wo, L.wo_s, q_dim, dim);
    orc_add_inplace(x.data(), proj.data(), dim);
    orc_rms_norm(x_norm.data(), x.data(), L.post_attn_norm, 1, dim, eps);
    int8_matvec_threaded(gate_buf.data(), x_norm.data(), L.gate_up, L.gate_up_s, dim, 2 * inter);
    orc_swiglu_decode(ffn.data(), gate_buf.data(), inter);
    int8_matvec_threaded(gate_buf.data(), ffn.data(), L.down, L.down_s, inter, dim);
    orc_add_inplace(x.data(), gate_buf.data(), dim);
  }
  std::vector<float> tmp(x);
  orc_rms_norm(x.data(), tmp.data(), dec->norm, 1, dim, eps);
  if (x_out) std::memcpy(x_out, x.data(), dim * 4);
  std::vector<float> logits(dec->vocab);
  int8_matvec_threaded(logits.data(), x.data(), dec->lm_head, dec->lm_head_s, dim, dec->vocab);
  if (logits_out) std::memcpy(logits_out, logits.data(), (size_t)dec->vocab * 4);
  return orc_argmax_first(logits.data(), dec->vocab);
}

// decoder_prefill_int8 (decoder.rs:751-842).  x_out (optional) receives the
// final residual stream [seq_len, hidden] before the final norm.
void orc_decoder_prefill_int8(const orc_decoder *dec, float *k_cache, float *v_cache, int max_seq,
                              int start_pos, const float *input_embeds, int seq_len, float *x_out) {
  const int dim = dec->hidden, nh = dec->n_heads, nkv = dec->n_kv_heads, hd = dec->head_dim;
  const int inter = dec->inter, q_dim = nh * hd, kv_dim = nkv * hd;
  const float eps = dec->eps;
  size_t S = seq_len;
  std::vector<float> x(input_embeds, input_embeds + S * dim), x_norm(S * dim), q(S * q_dim), k(S * kv_dim), v(S * kv_dim);
  std::vector<float> attn(S * q_dim), proj(S * dim), gu(S * 2 * inter), gate(S * inter), ffn(S * dim);
  std::vector<float> cos_t((size_t)(start_pos + seq_len) * hd), sin_t((size_t)(start_pos + seq_len) * hd);
  orc_rope_cache_table(cos_t.data(), sin_t.data(), start_pos + seq_len, hd, dec->theta);
  const float *rc = cos_t.data() + (size_t)start_pos * hd, *rs = sin_t.data() + (size_t)start_pos * hd;
  float scale = 1.0f / sqrtf((float)hd);
  for (int l = 0; l < dec->n_layers; ++l) {
    const orc_dec_layer &L = dec->layers[l];
    orc_rms_norm(x_norm.data(), x.data(), L.input_norm, seq_len, dim, eps);
    orc_linear_nobias_int8(q.data(), x_norm.data(), L.wq, L.wq_s, seq_len, dim, q_dim);
    orc_linear_nobias_int8(k.data(), x_norm.data(), L.wk, L.wk_s, seq_len, dim, kv_dim);
    orc_linear_nobias_int8(v.data(), x_norm.data(), L.wv, L.wv_s, seq_len, dim, kv_dim);
    orc_rms_norm_per_head(q.data(), L.q_norm, seq_len, nh, hd, eps);
    orc_rms_norm_per_head(k.data(), L.k_norm, seq_len, nkv, hd, eps);
    orc_apply_rope_neox(q.data(), rc, rs, seq_len, nh, hd);
    orc_apply_rope_neox(k.data(), rc, rs, seq_len, nkv, hd);
    for (int s = 0; s < seq_len; ++s) {
      size_t off = ((size_t)l * max_seq + start_pos + s) * kv_dim;
      std::memcpy(k_cache + off, k.data() + (size_t)s * kv_dim, kv_dim * 4);
      std::memcpy(v_cache + off, v.data() + (size_t)s * kv_dim, kv_dim * 4);
    }
    int total = start_pos + seq_len;
    const float *fk = k_cache + (size_t)l * max_seq * kv_dim;
    const float *fv = v_cache + (size_t)l * max_seq * kv_dim;
    orc_causal_attention(attn.data(), q.data(), fk, fv, seq_len, total, nh, nkv, hd, scale, start_pos);
    orc_linear_nobias_int8(proj.data(), attn.data(), L.wo, L.wo_s, seq_len, q_dim, dim);
    orc_add_inplace(x.data(), proj.data(), S * dim);
    orc_rms_norm(x_norm.data(), x.data(), L.post_attn_norm, seq_len, dim, eps);
    orc_linear_nobias_int8(gu.data(), x_norm.data(), L.gate_up, L.gate_up_s, seq_len, dim, 2 * inter);
    orc_swiglu_multiply(gate.data(), gu.data(), seq_len, inter);
    orc_linear_nobias_int8(ffn.data(), gate.data(), L.down, L.down_s, seq_len, inter, dim);
    orc_add_inplace(x.data(), ffn.data(), S * dim);
  }
  if (x_out) std::memcpy(x_out, x.data(), S * dim * 4);
}

// The BASELINE config-1 block in the prefill order of decoder.rs:770-810.
void orc_pre_attn_block(float *x_norm, const float *x, const float *w_in, int seq, int hidden,
                        float *q, float *k, const float *v, const float *q_norm_w, const float *k_norm_w,
                        int n_heads, int n_kv_heads, int head_dim, float eps,
                        const float *cos_tab, const float *sin_tab, int start_pos,
                        float *k_cache, float *v_cache) {
  orc_rms_norm(x_norm, x, w_in, seq, hidden, eps);
  orc_rms_norm_per_head(q, q_norm_w, seq, n_heads, head_dim, eps);
  orc_rms_norm_per_head(k, k_norm_w, seq, n_kv_heads, head_dim, eps);
  const float *rc = cos_tab + (size_t)start_pos * head_dim, *rs = sin_tab + (size_t)start_pos * head_dim;
  orc_apply_rope_neox(q, rc, rs, seq, n_heads, head_dim);
  orc_apply_rope_neox(k, rc, rs, seq, n_kv_heads, head_dim);
  size_t kv_dim = (size_t)n_kv_heads * head_dim;
  for (int s = 0; s < seq; ++s) {
    std::memcpy(k_cache + (size_t)(start_pos + s) * kv_dim, k + s * kv_dim, kv_dim * 4);
    std::memcpy(v_cache + (size_t)(start_pos + s) * kv_dim, v + s * kv_dim, kv_dim * 4);
  }
}

// --------------------------------------------------------------------------
// Log-mel front end (audio.rs:202-385).  Every table is built with the same
// f32 expression order and the same libm calls (logf, expf, cosf, sinf,
// log10f) as the reference; sums are sequential (Rust does not reassociate
// or contract them).
// --------------------------------------------------------------------------
static float orc_hz_to_mel(float hz) {  // audio.rs:202-213 (Slaney scale)
  const float log_step = 27.0f / logf(6.4f);
  if (hz >= 1000.0f) return 15.0f + logf(hz / 1000.0f) * log_step;
  return 3.0f * hz / 200.0f;
}

static float orc_mel_to_hz(float mel) {  // audio.rs:215-224
  const float log_step = logf(6.4f) / 27.0f;
  if (mel >= 15.0f) return 1000.0f * expf(log_step * (mel - 15.0f));
  return 200.0f * mel / 3.0f;
}

// filters [128, 201]: triangular Slaney-normalised filters (audio.rs:226-263).
void orc_mel_filters(float *filters) {
  const int nf = ORC_MEL_FREQS, nm = ORC_MEL_BINS;
  std::vector<float> bin_hz(nf), edge_hz(nm + 2), width(nm + 1);
  for (int f = 0; f < nf; ++f) bin_hz[f] = (float)f * (16000.0f / 2.0f) / (float)(nf - 1);
  const float lo = orc_hz_to_mel(0.0f), hi = orc_hz_to_mel(8000.0f);
  for (int i = 0; i < nm + 2; ++i) edge_hz[i] = orc_mel_to_hz(lo + (hi - lo) * (float)i / (float)(nm + 1));
  for (int i = 0; i < nm + 1; ++i) {
    width[i] = edge_hz[i + 1] - edge_hz[i];
    if (width[i] == 0.0f) width[i] = 1e-6f;
  }
  for (int m = 0; m < nm; ++m) {
    const float norm = 2.0f / (edge_hz[m + 2] - edge_hz[m]);
    for (int f = 0; f < nf; ++f) {
      const float rise = (bin_hz[f] - edge_hz[m]) / width[m];
      const float fall = (edge_hz[m + 2] - bin_hz[f]) / width[m + 1];
      filters[(size_t)m * nf + f] = std::max(std::min(rise, fall), 0.0f) * norm;
    }
  }
}

// window [400] (periodic Hann), cos_t / sin_t [201, 400] DFT rows (audio.rs:303-325).
void orc_mel_tables(float *window, float *cos_t, float *sin_t) {
  const float two_pi = 2.0f * 3.14159265358979323846f;
  for (int i = 0; i < ORC_MEL_NFFT; ++i) window[i] = 0.5f * (1.0f - cosf(two_pi * (float)i / (float)ORC_MEL_NFFT));
  for (int k = 0; k < ORC_MEL_FREQS; ++k)
    for (int n = 0; n < ORC_MEL_NFFT; ++n) {
      const float angle = two_pi * (float)k * (float)n / (float)ORC_MEL_NFFT;
      cos_t[(size_t)k * ORC_MEL_NFFT + n] = cosf(angle);
      sin_t[(size_t)k * ORC_MEL_NFFT + n] = sinf(angle);
    }
}

int orc_mel_frames(int n_samples) { return n_samples > 0 ? n_samples / ORC_MEL_HOP : 0; }

// Sample g of the reflect-padded signal (audio.rs:277-287): 200 samples
// mirrored about samples[0] in front, 200 mirrored about samples[n-1] behind,
// zero where the mirror runs off a short input.
static float orc_padded_sample(const float *s, int n, long g) {
  const int pad = ORC_MEL_NFFT / 2;
  if (g < pad) {
    const long src = pad - g;
    return src < n ? s[src] : 0.0f;
  }
  if (g < pad + n) return s[g - pad];
  const long src = (long)n - 2 - (g - pad - n);
  return src >= 0 ? s[src] : 0.0f;
}

// mel [128, n_frames] = (max(log10(mel power), global max - 8) + 4) / 4.
// Returns n_frames, 0 if the input is too short for one frame.
int orc_mel_spectrogram(float *mel, const float *samples, int n_samples) {
  const int n_frames = orc_mel_frames(n_samples);
  if (n_frames <= 0) return 0;
  const int NF = ORC_MEL_NFFT, NK = ORC_MEL_FREQS, NM = ORC_MEL_BINS;
  std::vector<float> filt((size_t)NM * NK), win(NF), ct((size_t)NK * NF), st((size_t)NK * NF);
  orc_mel_filters(filt.data());
  orc_mel_tables(win.data(), ct.data(), st.data());
  std::vector<float> logmel((size_t)n_frames * NM), frame(NF), power(NK);
  float top = -1e30f;
  for (int t = 0; t < n_frames; ++t) {
    for (int i = 0; i < NF; ++i) frame[i] = orc_padded_sample(samples, n_samples, (long)t * ORC_MEL_HOP + i) * win[i];
    for (int k = 0; k < NK; ++k) {
      float re = 0.0f, im = 0.0f;
      const float *c = &ct[(size_t)k * NF], *s = &st[(size_t)k * NF];
      for (int i = 0; i < NF; ++i) {
        re += frame[i] * c[i];
        im += frame[i] * s[i];
      }
      power[k] = re * re + im * im;
    }
    for (int m = 0; m < NM; ++m) {
      const float *f = &filt[(size_t)m * NK];
      float acc = 0.0f;
      for (int k = 0; k < NK; ++k) acc += f[k] * power[k];
      if (acc < 1e-10f) acc = 1e-10f;
      const float v = log10f(acc);
      logmel[(size_t)t * NM + m] = v;
      if (v > top) top = v;
    }
  }
  const float floor_v = top - 8.0f;
  for (int t = 0; t < n_frames; ++t)
    for (int m = 0; m < NM; ++m) {
      const float v = std::max(logmel[(size_t)t * NM + m], floor_v);
      mel[(size_t)m * n_frames + t] = (v + 4.0f) / 4.0f;
    }
  return n_frames;
}

}  // extern "C"
