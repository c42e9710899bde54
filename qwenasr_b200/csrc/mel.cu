// mel.cu -- audio::mel_spectrogram (crates/qwen-asr/src/audio.rs:202-385) on
// the device: 16 kHz samples -> [128, n_frames] normalised log-mel.
//
// The constant tables (periodic Hann window, the 201 x 400 DFT cos/sin rows,
// the 128 x 201 Slaney filter bank) are built once per device on the host
// with the reference's f32 expression order and the same libm calls (logf,
// expf, cosf, sinf), then uploaded, as the reference caches them in
// OnceLocks.  The device work is three kernels:
//   1. mel_power_kernel: reflect padding, windowing and the 400-point DFT of
//      32 frames per block, one frame per lane, with the reference's
//      sequential f32 sums (explicit __fmul_rn / __fadd_rn, so the power
//      spectrum is bit-identical to the reference's);
//   2. mel_log_kernel: the filter-bank sums (sequential over the 201 bins),
//      the 1e-10 floor and log10, written straight into the [128, frames]
//      output layout, and the global maximum (ordered-integer atomicMax);
//   3. mel_norm_kernel: clamp at max - 8, then (v + 4) / 4, in place.
// log10 is evaluated in double and rounded once, i.e. correctly rounded;
// glibc's log10f, which the reference calls, differs from that by one ulp on
// a few percent of inputs.
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"

namespace qasr {
namespace {

constexpr int kFft = 400, kFreqs = 201, kHop = 160, kBins = 128;
constexpr int kFramesPerBlock = 32, kFramePitch = 404;  // 404: float4 rows, conflict-free lanes
constexpr int kBinsPerWarp = 4, kBinsPerBlock = 8 * kBinsPerWarp;

struct MelTables {
  float *window = nullptr, *cos_t = nullptr, *sin_t = nullptr, *filters = nullptr;
};
MelTables g_tables[64];
std::mutex g_tables_mu;

float hz_to_mel(float hz) {  // audio.rs:202-213
  const float log_step = 27.0f / logf(6.4f);
  if (hz >= 1000.0f) return 15.0f + logf(hz / 1000.0f) * log_step;
  return 3.0f * hz / 200.0f;
}

float mel_to_hz(float mel) {  // audio.rs:215-224
  const float log_step = logf(6.4f) / 27.0f;
  if (mel >= 15.0f) return 1000.0f * expf(log_step * (mel - 15.0f));
  return 200.0f * mel / 3.0f;
}

void host_tables(std::vector<float> &window, std::vector<float> &cos_t, std::vector<float> &sin_t,
                 std::vector<float> &filters) {
  const float two_pi = 2.0f * 3.14159265358979323846f;  // 2 * f32 PI, exact
  window.resize(kFft);
  for (int i = 0; i < kFft; ++i) window[i] = 0.5f * (1.0f - cosf(two_pi * (float)i / (float)kFft));
  cos_t.resize((size_t)kFreqs * kFft);
  sin_t.resize((size_t)kFreqs * kFft);
  for (int k = 0; k < kFreqs; ++k)
    for (int n = 0; n < kFft; ++n) {
      const float angle = two_pi * (float)k * (float)n / (float)kFft;
      cos_t[(size_t)k * kFft + n] = cosf(angle);
      sin_t[(size_t)k * kFft + n] = sinf(angle);
    }
  // Slaney filter bank (audio.rs:226-263)
  std::vector<float> bin_hz(kFreqs), edge(kBins + 2), width(kBins + 1);
  for (int f = 0; f < kFreqs; ++f) bin_hz[f] = (float)f * (16000.0f / 2.0f) / (float)(kFreqs - 1);
  const float lo = hz_to_mel(0.0f), hi = hz_to_mel(8000.0f);
  for (int i = 0; i < kBins + 2; ++i) edge[i] = mel_to_hz(lo + (hi - lo) * (float)i / (float)(kBins + 1));
  for (int i = 0; i < kBins + 1; ++i) {
    width[i] = edge[i + 1] - edge[i];
    if (width[i] == 0.0f) width[i] = 1e-6f;
  }
  filters.resize((size_t)kBins * kFreqs);
  for (int m = 0; m < kBins; ++m) {
    const float norm = 2.0f / (edge[m + 2] - edge[m]);
    for (int f = 0; f < kFreqs; ++f) {
      const float rise = (bin_hz[f] - edge[m]) / width[m];
      const float fall = (edge[m + 2] - bin_hz[f]) / width[m + 1];
      const float tri = rise < fall ? rise : fall;
      filters[(size_t)m * kFreqs + f] = (tri > 0.0f ? tri : 0.0f) * norm;
    }
  }
}

// The device copy of the tables for the current device (uploaded on first use).
int mel_tables(const MelTables **out) {
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return QASR_ERR_INVALID;
  std::lock_guard<std::mutex> lk(g_tables_mu);
  MelTables &t = g_tables[dev];
  if (!t.window) {
    std::vector<float> w, c, s, f;
    host_tables(w, c, s, f);
    const size_t n = w.size() + c.size() + s.size() + f.size();
    float *buf = nullptr;
    int rc = cuda_status(cudaMalloc(&buf, n * 4), "mel tables: cudaMalloc");
    if (rc) return rc;
    float *p = buf;
    for (auto *v : {&w, &c, &s, &f}) {
      if ((rc = cuda_status(cudaMemcpy(p, v->data(), v->size() * 4, cudaMemcpyHostToDevice), "mel tables: upload"))) {
        cudaFree(buf);
        return rc;
      }
      p += v->size();
    }
    t.window = buf;
    t.cos_t = t.window + w.size();
    t.sin_t = t.cos_t + c.size();
    t.filters = t.sin_t + s.size();
  }
  *out = &t;
  return QASR_OK;
}

// Sample g of the reflect-padded signal (audio.rs:277-287).
__device__ __forceinline__ float padded_sample(const float *__restrict__ s, int n, long g) {
  constexpr int pad = kFft / 2;
  if (g < pad) {
    const long src = pad - g;
    return src < n ? s[src] : 0.0f;
  }
  if (g < pad + n) return s[g - pad];
  const long src = (long)n - 2 - (g - pad - n);
  return src >= 0 ? s[src] : 0.0f;
}

// power[k, t] = |sum_n frame_t[n] window[n] e^{-2 pi i k n / 400}|^2, k-major.
__global__ void __launch_bounds__(256)
    mel_power_kernel(float *__restrict__ power, const float *__restrict__ samples, int n_samples, int n_frames,
                     const float *__restrict__ window, const float *__restrict__ cos_t,
                     const float *__restrict__ sin_t) {
  extern __shared__ float4 mel_smem[];
  float *frames = reinterpret_cast<float *>(mel_smem);  // [32][kFramePitch]
  const int t0 = blockIdx.x * kFramesPerBlock;
  // eight independent loads per thread before the stores
  for (int base = threadIdx.x; base < kFramesPerBlock * kFft; base += blockDim.x * 8) {
    float val[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * (int)blockDim.x;
      const int f = i / kFft, j = i - f * kFft, t = t0 + f;
      val[u] = (i < kFramesPerBlock * kFft && t < n_frames)
                   ? __fmul_rn(padded_sample(samples, n_samples, (long)t * kHop + j), window[j])
                   : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int i = base + u * (int)blockDim.x;
      if (i < kFramesPerBlock * kFft) {
        const int f = i / kFft, j = i - f * kFft;
        frames[f * kFramePitch + j] = val[u];
      }
    }
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int k0 = blockIdx.y * kBinsPerBlock + warp * kBinsPerWarp;
  if (k0 >= kFreqs) return;  // warp-uniform, no barrier follows
  const float4 *row = reinterpret_cast<const float4 *>(frames + lane * kFramePitch);
  const float4 *cr[kBinsPerWarp], *sr[kBinsPerWarp];
#pragma unroll
  for (int j = 0; j < kBinsPerWarp; ++j) {
    const int k = min(k0 + j, kFreqs - 1);  // bins past 200 repeat bin 200 and are not stored
    cr[j] = reinterpret_cast<const float4 *>(cos_t + (size_t)k * kFft);
    sr[j] = reinterpret_cast<const float4 *>(sin_t + (size_t)k * kFft);
  }
  float re[kBinsPerWarp], im[kBinsPerWarp];
#pragma unroll
  for (int j = 0; j < kBinsPerWarp; ++j) re[j] = im[j] = 0.0f;
#pragma unroll 2
  for (int q = 0; q < kFft / 4; ++q) {
    const float4 w = row[q];
#pragma unroll
    for (int j = 0; j < kBinsPerWarp; ++j) {
      const float4 c = __ldg(cr[j] + q), s = __ldg(sr[j] + q);
      re[j] = __fadd_rn(re[j], __fmul_rn(w.x, c.x));
      im[j] = __fadd_rn(im[j], __fmul_rn(w.x, s.x));
      re[j] = __fadd_rn(re[j], __fmul_rn(w.y, c.y));
      im[j] = __fadd_rn(im[j], __fmul_rn(w.y, s.y));
      re[j] = __fadd_rn(re[j], __fmul_rn(w.z, c.z));
      im[j] = __fadd_rn(im[j], __fmul_rn(w.z, s.z));
      re[j] = __fadd_rn(re[j], __fmul_rn(w.w, c.w));
      im[j] = __fadd_rn(im[j], __fmul_rn(w.w, s.w));
    }
  }
  const int t = t0 + lane;
  if (t < n_frames) {
#pragma unroll
    for (int j = 0; j < kBinsPerWarp; ++j)
      if (k0 + j < kFreqs)
        power[(size_t)(k0 + j) * n_frames + t] = __fadd_rn(__fmul_rn(re[j], re[j]), __fmul_rn(im[j], im[j]));
  }
}

__device__ __forceinline__ unsigned order_key(float v) {
  const unsigned u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float order_value(unsigned key) {
  return __uint_as_float((key & 0x80000000u) ? (key & 0x7fffffffu) : ~key);
}

// mel[m, t] = log10(max(sum_k filters[m, k] power[k, t], 1e-10)); *max_key = max over all.
__global__ void __launch_bounds__(256)
    mel_log_kernel(float *__restrict__ mel, unsigned *__restrict__ max_key, const float *__restrict__ power,
                   int n_frames, const float *__restrict__ filters) {
  __shared__ float p[kFreqs][kFramesPerBlock];
  const int t0 = blockIdx.x * kFramesPerBlock;
  for (int i = threadIdx.x; i < kFreqs * kFramesPerBlock; i += blockDim.x) {
    const int k = i / kFramesPerBlock, f = i % kFramesPerBlock;
    p[k][f] = t0 + f < n_frames ? power[(size_t)k * n_frames + t0 + f] : 0.0f;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = t0 + lane;
  float top = -1e30f;
  // blockIdx.y takes kBins / gridDim.y mel bins, two per warp; the loads of
  // the sequential sum are independent of it, so unrolling runs them ahead
  const int per = kBins / gridDim.y, m0 = blockIdx.y * per;
  for (int m = m0 + warp; m < m0 + per; m += 8) {
    const float *fr = filters + (size_t)m * kFreqs;
    float acc = 0.0f;
#pragma unroll 8
    for (int k = 0; k < kFreqs; ++k) acc = __fadd_rn(acc, __fmul_rn(__ldg(fr + k), p[k][lane]));
    if (acc < 1e-10f) acc = 1e-10f;
    const float v = (float)log10((double)acc);
    if (t < n_frames) {
      mel[(size_t)m * n_frames + t] = v;
      top = fmaxf(top, v);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) top = fmaxf(top, __shfl_xor_sync(0xffffffffu, top, o));
  if (lane == 0 && top > -1e30f) atomicMax(max_key, order_key(top));
}

__global__ void __launch_bounds__(256) mel_norm_kernel(float *__restrict__ mel, const unsigned *__restrict__ max_key,
                                                       long n) {
  const float floor_v = __fsub_rn(order_value(*max_key), 8.0f);
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
    mel[i] = __fdiv_rn(__fadd_rn(fmaxf(mel[i], floor_v), 4.0f), 4.0f);
}

}  // namespace
}  // namespace qasr

using namespace qasr;

extern "C" int qasr_mel_frames(int n_samples) { return n_samples > 0 ? n_samples / kHop : 0; }

extern "C" int qasr_mel_spectrogram(float *mel, const float *samples, int n_samples, void *stream) {
  const int n_frames = qasr_mel_frames(n_samples);
  if (!mel || !samples || n_frames <= 0) {
    set_error("qasr_mel_spectrogram: invalid arguments (%d samples; at least %d needed)", n_samples, kHop);
    return QASR_ERR_INVALID;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const MelTables *tab = nullptr;
  int rc = mel_tables(&tab);
  if (rc) return rc;
  void *pw = nullptr, *key = nullptr;
  if ((rc = dev_scratch(kScratchMelPower, (size_t)kFreqs * n_frames * 4, &pw))) return rc;
  if ((rc = dev_scratch(kScratchMelMax, 4, &key))) return rc;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int smem = kFramesPerBlock * kFramePitch * 4;
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    if ((rc = cuda_status(cudaFuncSetAttribute(mel_power_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                          "qasr_mel_spectrogram: smem attribute")))
      return rc;
    attr_set[dev] = true;
  }
  const int fb = (n_frames + kFramesPerBlock - 1) / kFramesPerBlock;
  float *power = static_cast<float *>(pw);
  unsigned *max_key = static_cast<unsigned *>(key);
  mel_power_kernel<<<dim3(fb, (kFreqs + kBinsPerBlock - 1) / kBinsPerBlock), 256, smem, st>>>(
      power, samples, n_samples, n_frames, tab->window, tab->cos_t, tab->sin_t);
  if ((rc = launch_status("qasr_mel_spectrogram: power"))) return rc;
  if ((rc = cuda_status(cudaMemsetAsync(max_key, 0, 4, st), "qasr_mel_spectrogram: reset max"))) return rc;
  mel_log_kernel<<<dim3(fb, kBins / 16), 256, 0, st>>>(mel, max_key, power, n_frames, tab->filters);
  if ((rc = launch_status("qasr_mel_spectrogram: log"))) return rc;
  const long total = (long)kBins * n_frames;
  mel_norm_kernel<<<(int)std::min((total + 255) / 256, 148l * 8), 256, 0, st>>>(mel, max_key, total);
  return launch_status("qasr_mel_spectrogram: normalise");
}
