// encoder.cu -- the audio encoder's remaining per-chunk kernels:
//  * kernels::conv2d (crates/qwen-asr/src/kernels/mod.rs:790-860), the
//    three-layer conv stem of Encoder::forward (encoder.rs:290-320): im2col
//    into a [spatial, patch] matrix, then the tensor-core f32 GEMM
//    (umma_gemm.cu) with the conv weights as the row operand, which writes
//    the reference's [c_out, spatial] layout directly, then the bias;
//  * kernels::bidirectional_attention (mod.rs:1038-1122): windowed full
//    attention.  The main kernel stages one window's K and V rows of one
//    head in shared memory; each warp then takes a query: one key per lane
//    for the scores, the window max, exp and sum, then the weighted sum of V
//    rows (lanes over dimensions).  This is the softmax in two passes rather
//    than the reference's per-key running update (same value up to f32
//    rounding, and no per-key dependency chain).  Windows longer than the
//    shared-memory budget use the per-key kernel, which keeps K/V in L2.
#include <algorithm>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"
#include "umma.cuh"

namespace qasr {

// colsT[s, p] = input[ic, oh*stride + ki - pad, ow*stride + kj - pad] (0 outside),
// s = oh*w_out + ow, p = (ic*kh + ki)*kw + kj: im2col (mod.rs:790-813), transposed.
__global__ void __launch_bounds__(256) im2col_t_kernel(float *__restrict__ colsT, const float *__restrict__ in,
                                                       int c_in, int h_in, int w_in, int kh, int kw, int stride,
                                                       int pad, int h_out, int w_out) {
  const long patch = (long)c_in * kh * kw;
  const long total = patch * h_out * w_out;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long s = i / patch, p = i % patch;
    const int oh = (int)(s / w_out), ow = (int)(s % w_out);
    const int ic = (int)(p / (kh * kw)), r = (int)(p % (kh * kw)), ki = r / kw, kj = r % kw;
    const int ih = oh * stride + ki - pad, iw = ow * stride + kj - pad;
    colsT[i] = (ih >= 0 && ih < h_in && iw >= 0 && iw < w_in) ? in[((long)ic * h_in + ih) * w_in + iw] : 0.0f;
  }
}

// out[o, s] += bias[o]
__global__ void __launch_bounds__(256) bias_rows_kernel(float *__restrict__ out, const float *__restrict__ bias,
                                                        int rows, int cols) {
  const long total = (long)rows * cols;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x)
    out[i] = __fadd_rn(out[i], bias[i / cols]);
}

template <int EPL>  // elements per lane: head_dim / 32
__global__ void __launch_bounds__(256)
bidir_attention_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ k,
                       const float *__restrict__ v, int seq, int n_heads, float scale,
                       const int32_t *__restrict__ window_starts, int n_windows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long task = (long)blockIdx.x * 8 + warp;
  if (task >= (long)seq * n_heads) return;
  const int i = (int)(task / n_heads), h = (int)(task % n_heads);
  // window of query i: the last start <= i (starts are increasing)
  int lo = 0, hi = n_windows;  // window w = [starts[w], starts[w+1])
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (window_starts[mid] <= i) lo = mid; else hi = mid;
  }
  const int ws = max(0, window_starts[lo]), we = min(seq, window_starts[lo + 1]);
  const int hd = EPL * 32;
  const long hidden = (long)n_heads * hd;
  float qv[EPL], o[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    qv[e] = q[i * hidden + (long)h * hd + lane * EPL + e];
    o[e] = 0.0f;
  }
  float max_score = -1e30f, sum_exp = 0.0f;
  for (int j = ws; j < we; ++j) {
    const float *kr = k + j * hidden + (long)h * hd + lane * EPL;
    const float *vr = v + j * hidden + (long)h * hd + lane * EPL;
    float d = 0.0f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) d = fmaf(qv[e], kr[e], d);
    const float score = __fmul_rn(warp_sum(d), scale);
    if (score > max_score) {  // mod.rs:1058-1067: rescale the running state
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
  for (int e = 0; e < EPL; ++e)
    out[i * hidden + (long)h * hd + lane * EPL + e] = sum_exp > 0.0f ? __fmul_rn(o[e], inv) : o[e];
}

// Window [starts[w], starts[w+1]) of head h, queries z*8+warp, z*8+warp+8*gridDim.z, ...
// Shared memory: K [kt][HD+4] (padded: lane-per-key float4 reads are
// conflict-free), V [kt][HD], per-warp q [HD] and scores [kt].
constexpr int kBidirPadK = 4;
template <int EPL>
__global__ void __launch_bounds__(256)
bidir_attention_staged_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ k,
                              const float *__restrict__ v, int seq, int n_heads, float scale,
                              const int32_t *__restrict__ window_starts, int kt) {
  constexpr int HD = EPL * 32;
  extern __shared__ float4 bidir_smem[];
  float *sK = reinterpret_cast<float *>(bidir_smem);
  float *sV = sK + (size_t)kt * (HD + kBidirPadK);
  float *sQ = sV + (size_t)kt * HD;
  float *sP = sQ + 8 * HD;
  const int w = blockIdx.x, h = blockIdx.y;
  const int ws = max(0, window_starts[w]), we = min(seq, window_starts[w + 1]);
  const int n = we - ws;
  if (n <= 0 || n > kt) return;  // block-uniform; the host sizes kt to the longest window
  const long hidden = (long)n_heads * HD;
  stage_kv_rows<HD, kBidirPadK>(sK, sV, k, v, ws, hidden, (long)h * HD, n);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float *qs = sQ + warp * HD, *ps = sP + (size_t)warp * kt;
  for (int qi = blockIdx.z * 8 + warp; qi < n; qi += gridDim.z * 8) {
    const long row = (long)(ws + qi) * hidden + (long)h * HD;
    for (int d = lane; d < HD; d += 32) qs[d] = q[row + d];
    __syncwarp();
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) {
      // K rows padded to HD + 4 floats: the float4 reads of 8 consecutive
      // lanes cover all 32 banks; q is a broadcast read
      const float4 *kr = reinterpret_cast<const float4 *>(sK + j * (HD + kBidirPadK));
      const float4 *q4 = reinterpret_cast<const float4 *>(qs);
      float sc = 0.0f;
#pragma unroll 4
      for (int d4 = 0; d4 < HD / 4; ++d4) {
        const float4 kk = kr[d4], qq = q4[d4];
        sc = fmaf(qq.x, kk.x, sc);
        sc = fmaf(qq.y, kk.y, sc);
        sc = fmaf(qq.z, kk.z, sc);
        sc = fmaf(qq.w, kk.w, sc);
      }
      sc = __fmul_rn(sc, scale);
      ps[j] = sc;
      mx = fmaxf(mx, sc);
    }
    mx = warp_max(mx);
    float l = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float pj = expf(__fsub_rn(ps[j], mx));
      ps[j] = pj;
      l = __fadd_rn(l, pj);
    }
    l = warp_sum(l);
    __syncwarp();
    float o[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) o[e] = 0.0f;
    for (int j = 0; j < n; ++j) {  // lane owns elements lane + 32 e: conflict-free V reads
      const float pj = ps[j];
      const float *vr = sV + j * HD + lane;
#pragma unroll
      for (int e = 0; e < EPL; ++e) o[e] = fmaf(pj, vr[32 * e], o[e]);
    }
    const float inv = __fdiv_rn(1.0f, l);  // l >= 1: the max key contributes exp(0)
#pragma unroll
    for (int e = 0; e < EPL; ++e) out[row + lane + 32 * e] = __fmul_rn(o[e], inv);
    __syncwarp();  // qs / ps are rewritten by the next query
  }
}

static int grid_for(long n) { return (int)std::max(1l, std::min((n + 255) / 256, 148l * 16)); }

}  // namespace qasr

using namespace qasr;

extern "C" int qasr_conv2d(float *out, const float *input, const float *weight, const float *bias, int c_in,
                           int c_out, int h_in, int w_in, int kh, int kw, int stride, int padding, void *stream) {
  if (!out || !input || !weight || c_in <= 0 || c_out <= 0 || h_in <= 0 || w_in <= 0 || kh <= 0 || kw <= 0 ||
      stride <= 0 || padding < 0 || h_in + 2 * padding < kh || w_in + 2 * padding < kw) {
    set_error("qasr_conv2d: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const int h_out = (h_in + 2 * padding - kh) / stride + 1, w_out = (w_in + 2 * padding - kw) / stride + 1;
  const int patch = c_in * kh * kw, spatial = h_out * w_out;
  void *cols = nullptr;
  int rc = dev_scratch(kScratchIm2col, (size_t)spatial * patch * 4, &cols);
  if (rc) return rc;
  float *colsT = static_cast<float *>(cols);
  im2col_t_kernel<<<grid_for((long)spatial * patch), 256, 0, st>>>(colsT, input, c_in, h_in, w_in, kh, kw, stride,
                                                                    padding, h_out, w_out);
  if ((rc = launch_status("qasr_conv2d: im2col"))) return rc;
  // out[o, s] = sum_p weight[o, p] * colsT[s, p]: weights are the row operand
  rc = f32_gemm(out, spatial, weight, patch, colsT, nullptr, c_out, patch, spatial, st);
  if (rc == QASR_ERR_UNSUPPORTED) rc = f32_gemm_fallback(out, weight, colsT, nullptr, c_out, patch, spatial, st);
  if (rc) return rc;
  if (bias) {
    bias_rows_kernel<<<grid_for((long)c_out * spatial), 256, 0, st>>>(out, bias, c_out, spatial);
    if ((rc = launch_status("qasr_conv2d: bias"))) return rc;
  }
  return QASR_OK;
}

namespace qasr {
constexpr int kBidirMaxSmem = 200 * 1024;

size_t bidir_smem_bytes(int head_dim, int kt) {
  return ((size_t)kt * (head_dim + kBidirPadK) + (size_t)kt * head_dim + 8 * head_dim + 8 * (size_t)kt) * 4;
}

// Windowed attention with the longest window known (max_window keys).
int bidir_attention_launch(float *out, const float *q, const float *k, const float *v, int seq, int n_heads,
                           int head_dim, float scale, const int32_t *window_starts, int n_windows, int max_window,
                           cudaStream_t st) {
  const size_t smem = bidir_smem_bytes(head_dim, max_window);
  if (max_window > 0 && smem <= (size_t)kBidirMaxSmem) {
    static bool attr_set[64][2] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    const int which = head_dim == 64 ? 0 : 1;
    if (dev >= 0 && dev < 64 && !attr_set[dev][which]) {
      cudaError_t e = head_dim == 64
                          ? cudaFuncSetAttribute(bidir_attention_staged_kernel<2>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kBidirMaxSmem)
                          : cudaFuncSetAttribute(bidir_attention_staged_kernel<4>,
                                                 cudaFuncAttributeMaxDynamicSharedMemorySize, kBidirMaxSmem);
      if (int rc = cuda_status(e, "qasr_bidirectional_attention: smem attribute")) return rc;
      attr_set[dev][which] = true;
    }
    // about two queries per warp of each (window, head)
    const int qz = std::max(1, (max_window + 15) / 16);
    const dim3 grid((unsigned)n_windows, (unsigned)n_heads, (unsigned)qz);
    if (head_dim == 64)
      bidir_attention_staged_kernel<2><<<grid, 256, smem, st>>>(out, q, k, v, seq, n_heads, scale, window_starts,
                                                                 max_window);
    else
      bidir_attention_staged_kernel<4><<<grid, 256, smem, st>>>(out, q, k, v, seq, n_heads, scale, window_starts,
                                                                 max_window);
    return launch_status("qasr_bidirectional_attention");
  }
  const long tasks = (long)seq * n_heads;
  const int grid = (int)((tasks + 7) / 8);
  if (head_dim == 64)
    bidir_attention_kernel<2><<<grid, 256, 0, st>>>(out, q, k, v, seq, n_heads, scale, window_starts, n_windows);
  else
    bidir_attention_kernel<4><<<grid, 256, 0, st>>>(out, q, k, v, seq, n_heads, scale, window_starts, n_windows);
  return launch_status("qasr_bidirectional_attention");
}
}  // namespace qasr

// The window bounds are device data: they are read back once per call to size
// the shared-memory window (the encoder engine, which knows its windows, calls
// bidir_attention_launch directly).
extern "C" int qasr_bidirectional_attention(float *out, const float *q, const float *k, const float *v, int seq,
                                            int n_heads, int head_dim, float scale, const int32_t *window_starts,
                                            int n_windows, void *stream) {
  if (!out || !q || !k || !v || !window_starts || seq < 0 || n_heads <= 0 || n_windows <= 0) {
    set_error("qasr_bidirectional_attention: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (head_dim != 64 && head_dim != 128) {
    set_error("qasr_bidirectional_attention: head_dim %d unsupported (64 or 128)", head_dim);
    return QASR_ERR_UNSUPPORTED;
  }
  if (seq == 0) return QASR_OK;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  std::vector<int32_t> starts(n_windows + 1);
  int rc = cuda_status(cudaMemcpyAsync(starts.data(), window_starts, starts.size() * 4, cudaMemcpyDefault, st),
                       "qasr_bidirectional_attention: window starts");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(st), "qasr_bidirectional_attention");
  if (rc) return rc;
  int max_window = 0;
  for (int w = 0; w < n_windows; ++w)
    max_window = std::max(max_window, std::min(seq, starts[w + 1]) - std::max(0, starts[w]));
  return bidir_attention_launch(out, q, k, v, seq, n_heads, head_dim, scale, window_starts, n_windows, max_window,
                                st);
}
