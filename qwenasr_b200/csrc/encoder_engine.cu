// encoder_engine.cu -- the audio encoder on one GPU: Encoder::forward
// (crates/qwen-asr/src/encoder.rs:243-415, f32 weights) and
// EncoderInt8::forward (encoder.rs:562-667, INT8 projection weights with f32
// scales, as a V2 .qint8 file stores them), composed from the kernel-level
// entries in the reference's order.  Each projection matrix is held either as
// f32 or as INT8 + per-row scales, whichever its setter supplied, and runs
// through qasr_linear / qasr_linear_int8 accordingly.
//
// Per mel chunk of chunk_size frames (encoder.rs:281-348): three stride-2
// 3x3 convolutions (480 channels) each followed by the tanh GELU, the
// [480, h3, w3] -> [w3, 480*h3] reshape, the conv-out projection and the
// sinusoidal position rows of the chunk.  Then per layer (encoder.rs:368-403):
// LayerNorm, q/k/v projections with bias, bidirectional attention inside
// windows of tokens_per_chunk * (n_window_infer / chunk_size) tokens, output
// projection + residual, LayerNorm, fc1 + GELU, fc2 + residual.  Finally the
// post LayerNorm and proj1 + GELU + proj2 (encoder.rs:405-415).
//
// Device layout: every weight is a device copy owned by the engine; the
// activation buffers are sized for the largest mel length seen so far.
#include <algorithm>
#include <cstring>
#include <vector>

#include "common.cuh"
#include "matvec.cuh"
#include "umma.cuh"

namespace qasr {

constexpr int kConvHidden = 480;  // CONV_HIDDEN (config.rs:23)
constexpr int kMelBins = 128;
constexpr int kStemGroup = 32;  // chunks per conv-stem pass (bounds the patch buffers on long audio)

inline int grid_of(long n) { return (int)std::max(1l, std::min((n + 255) / 256, 148l * 16)); }

// The conv stem runs on B chunks at once in channel-last layout: the
// activation of chunk b at (row h, column w), channel c is act[((b*H + h)*W +
// w)*C + c].  Each convolution is then one GEMM over all B*h_out*w_out output
// positions: colsT[(b*h_out + oh)*w_out + ow, (ic*3 + ki)*3 + kj] (3x3
// kernel, stride 2, padding 1, every chunk padded on its own as in the
// reference's per-chunk kernels::conv2d) times the [c_out, c_in*9] weights.

// conv1 (one input channel) + bias + tanh GELU straight from the mel
// [128, mel_frames]: chunk b covers frames first + b*cs .. + cw; out[r, o]
// channel-last.  The GELU is the gelu_kernel body (the 480-channel rows keep
// every element in the 8-lane body of avx::gelu_inplace).
__global__ void __launch_bounds__(256) conv1_gelu_kernel(float *__restrict__ out, const float *__restrict__ mel,
                                                         int mel_frames, int first, int cs, int cw, int B, int h_out,
                                                         int w_out, const float *__restrict__ w,
                                                         const float *__restrict__ bias) {
  // one warp per output position (b, oh, ow): its 9 inputs are read once,
  // the lanes cover the kConvHidden channels (weights in shared memory,
  // stride 9 across lanes: conflict-free), stores are coalesced rows
  __shared__ float sw[kConvHidden * 9], sb[kConvHidden];
  for (int i = threadIdx.x; i < kConvHidden * 9; i += blockDim.x) sw[i] = w[i];
  for (int i = threadIdx.x; i < kConvHidden; i += blockDim.x) sb[i] = bias[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int positions = B * h_out * w_out;  // < 2^31: B <= kStemGroup
  for (int r = blockIdx.x * 8 + warp; r < positions; r += gridDim.x * 8) {
    const int ow = r % w_out, t = r / w_out, oh = t % h_out, b = t / h_out;
    float x[9];
#pragma unroll
    for (int kk = 0; kk < 9; ++kk) {
      const int ih = oh * 2 + kk / 3 - 1, iw = ow * 2 + kk % 3 - 1;
      x[kk] = (ih >= 0 && ih < kMelBins && iw >= 0 && iw < cw)
                  ? __ldg(mel + (long)ih * mel_frames + first + (long)b * cs + iw)
                  : 0.0f;
    }
    float *row = out + (long)r * kConvHidden;
    for (int o = lane; o < kConvHidden; o += 32) {
      float acc = 0.0f;
#pragma unroll
      for (int kk = 0; kk < 9; ++kk) acc = fmaf(sw[o * 9 + kk], x[kk], acc);
      row[o] = gelu_tanh_ref(__fadd_rn(acc, sb[o]));
    }
  }
}

// Patches of a channel-last activation [B, h_in, w_in, C] in channel-fastest
// order: colsT[r, (ki*3 + kj)*C + ic] (the conv weights are permuted to match
// once, conv_weight_cl_kernel), so every (position, ki, kj) copies C
// contiguous floats: float4 loads and stores.
__global__ void __launch_bounds__(256) im2col_cl_kernel(float *__restrict__ colsT, const float *__restrict__ act,
                                                        int C, int h_in, int w_in, int B, int h_out, int w_out) {
  // 32-bit index math: B <= kStemGroup keeps every index below 2^31
  const int C4 = C / 4;
  const int per_row = 9 * C4;
  const int total = B * h_out * w_out * per_row;
  float4 *dst = reinterpret_cast<float4 *>(colsT);
  const float4 *src = reinterpret_cast<const float4 *>(act);
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int r = i / per_row;
    const int rem = i - r * per_row, kk = rem / C4, c4 = rem % C4;
    const int ow = r % w_out, t = r / w_out, oh = t % h_out, b = t / h_out;
    const int ih = oh * 2 + kk / 3 - 1, iw = ow * 2 + kk % 3 - 1;
    dst[i] = (ih >= 0 && ih < h_in && iw >= 0 && iw < w_in) ? src[(((long)b * h_in + ih) * w_in + iw) * C4 + c4]
                                                             : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// dst[o, kk*C + ic] = src[o, ic*9 + kk]: the [c_out, c_in, 3, 3] weights in
// the channel-fastest patch order of im2col_cl_kernel.
__global__ void __launch_bounds__(256) conv_weight_cl_kernel(float *__restrict__ dst, const float *__restrict__ src,
                                                             int c_out, int C) {
  const long total = (long)c_out * C * 9;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long o = i / (9l * C);
    const int rem = (int)(i - o * 9l * C), kk = rem / C, ic = rem % C;
    dst[i] = src[(o * C + ic) * 9 + kk];
  }
}

// the encoder.rs:322-331 reshape per chunk, from channel-last c3 [B, h3, w3, C]:
// reshaped[b*w3 + t, c*h3 + f] = c3[b, f, t, c]
__global__ void __launch_bounds__(256) conv_reshape_cl_kernel(float *__restrict__ out, const float *__restrict__ c3,
                                                              int C, int h3, int w3, int B) {
  const long row = (long)C * h3;
  const long total = (long)B * w3 * row;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long bt = i / row;
    const int cf = (int)(i - bt * row), c = cf / h3, f = cf % h3;
    const int t = (int)(bt % w3), b = (int)(bt / w3);
    out[i] = c3[(((long)b * h3 + f) * w3 + t) * C + c];
  }
}

// x[b*w3 + t, :] += pe[t, :] (every chunk restarts its positions, encoder.rs:339-343)
__global__ void __launch_bounds__(256) add_chunk_pe_kernel(float *__restrict__ x, const float *__restrict__ pe, int B,
                                                           int w3, int D) {
  const long total = (long)B * w3 * D;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x)
    x[i] = __fadd_rn(x[i], pe[i % ((long)w3 * D)]);
}

// One projection matrix [rows, cols]: f32, or INT8 with f32 row scales.
struct EncMat {
  int rows = 0, cols = 0;
  float *f = nullptr;
  int8_t *q = nullptr;
  float *s = nullptr;
  F32Weight pw;  // digit planes of f (when the tensor-core GEMM takes the shape)
  bool ready() const { return f || q; }
  void release() {
    f32_weight_free(&pw);
    if (f) cudaFree(f);
    if (q) cudaFree(q);
    if (s) cudaFree(s);
    f = nullptr;
    q = nullptr;
    s = nullptr;
  }
};

struct EncLayerDev {
  float *attn_norm_w, *attn_norm_b, *bq, *bk, *bv, *bo;  // bk, bv follow bq in one [3D] buffer
  float *ffn_norm_w, *ffn_norm_b, *fc1_b, *fc2_b;
  EncMat wq, wk, wv, wo, fc1, fc2;
  F32Weight qkv;  // f32 q|k|v as one [3D, D] digit-plane operand (d_model a multiple of 128)
};

}  // namespace qasr

struct qasr_encoder {
  qasr_encoder_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  qasr::ScratchArena *arena = nullptr;  // this engine's kernel-level scratch
  std::vector<qasr::EncLayerDev> layers;
  float *conv_w[3] = {nullptr, nullptr, nullptr}, *conv_b[3] = {nullptr, nullptr, nullptr};
  qasr::EncMat conv_out, proj1, proj2;
  float *ln_post_w = nullptr, *ln_post_b = nullptr, *proj1_b = nullptr, *proj2_b = nullptr;
  std::vector<void *> allocs;
  // activations, grown on demand
  int tok_cap = 0, stem_cap = 0;
  qasr::F32Weight conv_pw[3];  // conv2 / conv3 weights as digit planes (conv1 has K = 9: CUDA cores)
  void *act = nullptr;
  float *x = nullptr, *xn = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr, *proj = nullptr,
        *mid = nullptr, *out = nullptr, *pe = nullptr;
  void *conv_buf = nullptr;
  float *cols = nullptr, *act_a = nullptr, *act_b = nullptr;  // stem patches, ping-pong activations
  float *mel_dev = nullptr;  // device copy of a host mel input
  size_t mel_cap = 0;
  int32_t *win = nullptr;
  int win_cap = 0;
};

using namespace qasr;

static int enc_alloc(qasr_encoder *e, float **p, size_t n) {
  void *q = nullptr;
  int rc = cuda_status(cudaMalloc(&q, n * 4), "qasr_encoder: cudaMalloc");
  if (rc) return rc;
  e->allocs.push_back(q);
  *p = static_cast<float *>(q);
  return QASR_OK;
}

static int enc_copy(qasr_encoder *e, float *dst, const float *src, size_t n, const char *what) {
  if (!src) {
    set_error("qasr_encoder: %s is NULL", what);
    return QASR_ERR_INVALID;
  }
  return cuda_status(cudaMemcpyAsync(dst, src, n * 4, cudaMemcpyDefault, e->stream), what);
}

// f32 weights into m (replacing an INT8 copy).
static int mat_set_f32(qasr_encoder *e, EncMat &m, const float *src, const char *what) {
  if (!src) {
    set_error("qasr_encoder: %s is NULL", what);
    return QASR_ERR_INVALID;
  }
  const size_t n = (size_t)m.rows * m.cols;
  if (m.q) {
    int rc = cuda_status(cudaStreamSynchronize(e->stream), what);
    if (rc) return rc;
    m.release();
  }
  if (!m.f) {
    int rc = cuda_status(cudaMalloc(&m.f, n * 4), "qasr_encoder: cudaMalloc");
    if (rc) return rc;
  }
  int rc = cuda_status(cudaMemcpyAsync(m.f, src, n * 4, cudaMemcpyDefault, e->stream), what);
  if (rc) return rc;
  // the constant operand's digit planes, once (unsupported shapes stay on qasr_linear)
  if ((rc = cuda_status(cudaStreamSynchronize(e->stream), what))) return rc;
  f32_weight_free(&m.pw);
  rc = f32_weight_prepare(&m.pw, m.f, m.rows, m.cols, e->stream);
  return rc == QASR_ERR_UNSUPPORTED ? QASR_OK : rc;
}

// INT8 weights + row scales into m (replacing an f32 copy).
static int mat_set_i8(qasr_encoder *e, EncMat &m, const int8_t *src, const float *scales, const char *what) {
  if (!src || !scales) {
    set_error("qasr_encoder: %s (or its scales) is NULL", what);
    return QASR_ERR_INVALID;
  }
  const size_t n = (size_t)m.rows * m.cols;
  if (m.f) {
    int rc = cuda_status(cudaStreamSynchronize(e->stream), what);
    if (rc) return rc;
    m.release();
  }
  if (!m.q) {
    int rc = cuda_status(cudaMalloc(&m.q, n), "qasr_encoder: cudaMalloc");
    if (!rc) rc = cuda_status(cudaMalloc(&m.s, (size_t)m.rows * 4), "qasr_encoder: cudaMalloc");
    if (rc) return rc;
  }
  int rc = cuda_status(cudaMemcpyAsync(m.q, src, n, cudaMemcpyDefault, e->stream), what);
  if (!rc) rc = cuda_status(cudaMemcpyAsync(m.s, scales, (size_t)m.rows * 4, cudaMemcpyDefault, e->stream), what);
  return rc;
}

// y [T, rows] = x [T, cols] m^T (+ bias): kernels::linear or linear_int8.
static int mat_apply(float *y, const float *x, const EncMat &m, const float *bias, int T, cudaStream_t st) {
  if (m.q)
    return bias ? qasr_linear_int8(y, x, m.q, m.s, bias, T, m.cols, m.rows, st)
                : qasr_linear_nobias_int8(y, x, m.q, m.s, T, m.cols, m.rows, st);
  if (m.pw.planes) {
    const int rc = f32_gemm_prepared(y, m.rows, x, m.cols, m.pw, bias, T, st);
    if (rc != QASR_ERR_UNSUPPORTED) return rc;
  }
  return bias ? qasr_linear(y, x, m.f, bias, T, m.cols, m.rows, st)
              : qasr_linear_nobias(y, x, m.f, T, m.cols, m.rows, st);
}

// The f32 q|k|v weights of a layer as one [3D, D] digit-plane operand, so
// the three projections run as one GEMM with a split output; the separate
// planes are then dropped.  d_model not a multiple of 128 keeps three GEMMs.
static int prepare_qkv(qasr_encoder *e, EncLayerDev &L) {
  f32_weight_free(&L.qkv);  // callers synchronised e->stream
  const int D = e->cfg.d_model;
  if (D % 128 || !L.wq.f || !L.wk.f || !L.wv.f) return QASR_OK;
  const size_t n = (size_t)D * D;
  float *tmp = nullptr;
  int rc = cuda_status(cudaMalloc(&tmp, 3 * n * 4), "qasr_encoder: q|k|v weights");
  if (rc) return rc;
  const float *src[3] = {L.wq.f, L.wk.f, L.wv.f};
  for (int i = 0; i < 3 && !rc; ++i)
    rc = cuda_status(cudaMemcpyAsync(tmp + i * n, src[i], n * 4, cudaMemcpyDeviceToDevice, e->stream),
                     "qasr_encoder: q|k|v weights");
  if (!rc) rc = f32_weight_prepare(&L.qkv, tmp, 3 * D, D, e->stream);
  if (rc == QASR_ERR_UNSUPPORTED) rc = QASR_OK;
  const int rs = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder: q|k|v weights");
  cudaFree(tmp);
  if (!rc && !rs && L.qkv.planes)
    for (EncMat *m : {&L.wq, &L.wk, &L.wv}) f32_weight_free(&m->pw);
  return rc ? rc : rs;
}

// conv i (1 or 2) of the stem over `rows` patch rows: y [rows, 480] =
// cols [rows, 480*9] W_i^T + b_i.
static int conv_gemm(qasr_encoder *e, int i, float *y, const float *cols, int rows, cudaStream_t st) {
  const int CH = kConvHidden;
  if (e->conv_pw[i].planes) {
    const int rc = f32_gemm_prepared(y, CH, cols, (long)CH * 9, e->conv_pw[i], e->conv_b[i], rows, st);
    if (rc != QASR_ERR_UNSUPPORTED) return rc;
  }
  return f32_gemm_fallback(y, cols, e->conv_w[i], e->conv_b[i], rows, CH * 9, CH, st);
}

// conv2 / conv3 (3x3, stride 2, padding 1, CH -> CH channels) of the
// channel-last activation act [B, h_in, w_in, CH] into y [B*h_out*w_out, CH]:
// an implicit GEMM (patch digits straight from act) when the weights have
// their digit planes, else patches into e->cols and the CUDA-core GEMM.
static int conv_stage(qasr_encoder *e, int i, float *y, const float *act, int h_in, int w_in, int B, int h_out,
                      int w_out, cudaStream_t st) {
  const int CH = kConvHidden;
  const long rows = (long)B * h_out * w_out;
  if (e->conv_pw[i].planes) {
    const int rc = f32_gemm_prepared_conv(y, CH, act, CH, h_in, w_in, B, h_out, w_out, e->conv_pw[i], e->conv_b[i],
                                          st);
    if (rc != QASR_ERR_UNSUPPORTED) return rc;
  }
  im2col_cl_kernel<<<grid_of(rows * CH * 9 / 4), 256, 0, st>>>(e->cols, act, CH, h_in, w_in, B, h_out, w_out);
  if (int rc = launch_status("qasr_encoder_forward: conv patches")) return rc;
  return conv_gemm(e, i, y, e->cols, (int)rows, st);
}

// conv2 / conv3 after their weights change: the weights into the
// channel-fastest patch order, then their digit planes
static int prepare_convs(qasr_encoder *e) {
  const int CH = kConvHidden;
  float *tmp = nullptr;
  int rc = cuda_status(cudaMalloc(&tmp, (size_t)CH * CH * 9 * 4), "qasr_encoder: conv weights");
  for (int i = 1; i < 3 && !rc; ++i) {
    conv_weight_cl_kernel<<<grid_of((long)CH * CH * 9), 256, 0, e->stream>>>(tmp, e->conv_w[i], CH, CH);
    rc = launch_status("qasr_encoder: conv weight order");
    if (!rc)
      rc = cuda_status(cudaMemcpyAsync(e->conv_w[i], tmp, (size_t)CH * CH * 9 * 4, cudaMemcpyDeviceToDevice,
                                       e->stream),
                       "qasr_encoder: conv weight order");
  }
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder: conv weights");
  if (tmp) cudaFree(tmp);
  for (int i = 1; i < 3 && !rc; ++i) {
    f32_weight_free(&e->conv_pw[i]);
    rc = f32_weight_prepare(&e->conv_pw[i], e->conv_w[i], kConvHidden, kConvHidden * 9, e->stream);
    if (rc == QASR_ERR_UNSUPPORTED) rc = QASR_OK;
  }
  return rc;
}

static std::vector<EncMat *> enc_mats(qasr_encoder *e) {
  std::vector<EncMat *> v = {&e->conv_out, &e->proj1, &e->proj2};
  for (auto &L : e->layers)
    for (EncMat *m : {&L.wq, &L.wk, &L.wv, &L.wo, &L.fc1, &L.fc2}) v.push_back(m);
  return v;
}

extern "C" void qasr_encoder_free(qasr_encoder *e) {
  if (!e) return;
  cudaSetDevice(e->device);
  if (e->stream) cudaStreamSynchronize(e->stream);
  for (EncMat *m : enc_mats(e)) m->release();
  for (auto &L : e->layers) f32_weight_free(&L.qkv);
  for (auto &pw : e->conv_pw) f32_weight_free(&pw);
  for (void *p : e->allocs) cudaFree(p);
  if (e->act) cudaFree(e->act);
  if (e->conv_buf) cudaFree(e->conv_buf);
  if (e->win) cudaFree(e->win);
  if (e->mel_dev) cudaFree(e->mel_dev);
  if (e->stream) cudaStreamDestroy(e->stream);
  arena_free(e->arena);
  delete e;
}

static int chunk_tokens(int w) {  // three stride-2 3x3 convolutions with padding 1
  const int w1 = (w + 2 - 3) / 2 + 1, w2 = (w1 + 2 - 3) / 2 + 1;
  return (w2 + 2 - 3) / 2 + 1;
}

extern "C" qasr_encoder *qasr_encoder_create(const qasr_encoder_config *cfg, int device) {
  if (!cfg || cfg->d_model <= 0 || cfg->n_layers <= 0 || cfg->n_heads <= 0 || cfg->ffn_dim <= 0 ||
      cfg->output_dim <= 0 || cfg->chunk_size <= 0 || cfg->n_window_infer < cfg->chunk_size ||
      cfg->head_dim * cfg->n_heads != cfg->d_model) {
    set_error("qasr_encoder_create: invalid config");
    return nullptr;
  }
  if (cfg->head_dim != 64 && cfg->head_dim != 128) {
    set_error("qasr_encoder_create: head_dim must be 64 or 128");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error("qasr_encoder_create: cudaSetDevice(%d) failed", device);
    return nullptr;
  }
  qasr_encoder *e = new qasr_encoder();
  e->cfg = *cfg;
  e->device = device;
  int rc = cuda_status(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking), "qasr_encoder_create");
  if (!rc && !(e->arena = arena_create(device))) {
    set_error("qasr_encoder_create: scratch arena");
    rc = QASR_ERR_ALLOC;
  }
  const int D = cfg->d_model, F = cfg->ffn_dim, O = cfg->output_dim, CH = kConvHidden;
  const int h3 = chunk_tokens(kMelBins);  // frequency rows after the stem: 16
  e->layers.resize(cfg->n_layers);
  const int cin[3] = {1, CH, CH};
  for (int i = 0; i < 3 && !rc; ++i) {
    rc = enc_alloc(e, &e->conv_w[i], (size_t)CH * cin[i] * 9);
    if (!rc) rc = enc_alloc(e, &e->conv_b[i], CH);
  }
  // projection matrices: shapes now, storage when a setter supplies f32 or INT8
  e->conv_out.rows = D;
  e->conv_out.cols = CH * h3;
  e->proj1.rows = D;
  e->proj1.cols = D;
  e->proj2.rows = O;
  e->proj2.cols = D;
  for (auto &L : e->layers) {
    float **pp[] = {&L.attn_norm_w, &L.attn_norm_b, &L.bo, &L.ffn_norm_w, &L.ffn_norm_b, &L.fc2_b};
    for (float **p : pp)
      if (!rc) rc = enc_alloc(e, p, D);
    if (!rc) rc = enc_alloc(e, &L.bq, 3 * (size_t)D);
    if (!rc) {
      L.bk = L.bq + D;
      L.bv = L.bq + 2 * (size_t)D;
    }
    if (!rc) rc = enc_alloc(e, &L.fc1_b, F);
    for (EncMat *m : {&L.wq, &L.wk, &L.wv, &L.wo}) {
      m->rows = D;
      m->cols = D;
    }
    L.fc1.rows = F;
    L.fc1.cols = D;
    L.fc2.rows = D;
    L.fc2.cols = F;
  }
  if (!rc) rc = enc_alloc(e, &e->ln_post_w, D);
  if (!rc) rc = enc_alloc(e, &e->ln_post_b, D);
  if (!rc) rc = enc_alloc(e, &e->proj1_b, D);
  if (!rc) rc = enc_alloc(e, &e->proj2_b, O);
  if (rc) {
    qasr_encoder_free(e);
    return nullptr;
  }
  return e;
}

extern "C" int qasr_encoder_set_conv(qasr_encoder *e, const float *conv1_w, const float *conv1_b,
                                     const float *conv2_w, const float *conv2_b, const float *conv3_w,
                                     const float *conv3_b, const float *conv_out_w) {
  if (!e) {
    set_error("qasr_encoder_set_conv: null encoder");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const int CH = kConvHidden, h3 = chunk_tokens(kMelBins);
  const float *w[3] = {conv1_w, conv2_w, conv3_w}, *b[3] = {conv1_b, conv2_b, conv3_b};
  const int cin[3] = {1, CH, CH};
  int rc = QASR_OK;
  for (int i = 0; i < 3 && !rc; ++i) {
    rc = enc_copy(e, e->conv_w[i], w[i], (size_t)CH * cin[i] * 9, "conv weight");
    if (!rc) rc = enc_copy(e, e->conv_b[i], b[i], CH, "conv bias");
  }
  if (!rc) rc = mat_set_f32(e, e->conv_out, conv_out_w, "conv_out weight");
  if (!rc) rc = prepare_convs(e);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_conv");
  (void)h3;
  return rc;
}

// EncoderInt8 (encoder.rs:446-520): the convolutions stay f32, conv_out is INT8.
extern "C" int qasr_encoder_set_conv_int8(qasr_encoder *e, const float *conv1_w, const float *conv1_b,
                                          const float *conv2_w, const float *conv2_b, const float *conv3_w,
                                          const float *conv3_b, const int8_t *conv_out, const float *conv_out_s) {
  if (!e) {
    set_error("qasr_encoder_set_conv_int8: null encoder");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const int CH = kConvHidden;
  const float *w[3] = {conv1_w, conv2_w, conv3_w}, *b[3] = {conv1_b, conv2_b, conv3_b};
  const int cin[3] = {1, CH, CH};
  int rc = QASR_OK;
  for (int i = 0; i < 3 && !rc; ++i) {
    rc = enc_copy(e, e->conv_w[i], w[i], (size_t)CH * cin[i] * 9, "conv weight");
    if (!rc) rc = enc_copy(e, e->conv_b[i], b[i], CH, "conv bias");
  }
  if (!rc) rc = mat_set_i8(e, e->conv_out, conv_out, conv_out_s, "conv_out weight");
  if (!rc) rc = prepare_convs(e);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_conv_int8");
  return rc;
}

extern "C" int qasr_encoder_set_layer(qasr_encoder *e, int layer, const qasr_enc_layer_weights *w) {
  if (!e || !w || layer < 0 || layer >= e->cfg.n_layers) {
    set_error("qasr_encoder_set_layer: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const size_t D = e->cfg.d_model, F = e->cfg.ffn_dim;
  EncLayerDev &L = e->layers[layer];
  int rc = QASR_OK;
  struct {
    float *dst;
    const float *src;
    size_t n;
    const char *what;
  } items[] = {{L.attn_norm_w, w->attn_norm_w, D, "attn_norm_w"}, {L.attn_norm_b, w->attn_norm_b, D, "attn_norm_b"},
               {L.bq, w->bq, D, "bq"}, {L.bk, w->bk, D, "bk"}, {L.bv, w->bv, D, "bv"}, {L.bo, w->bo, D, "bo"},
               {L.ffn_norm_w, w->ffn_norm_w, D, "ffn_norm_w"}, {L.ffn_norm_b, w->ffn_norm_b, D, "ffn_norm_b"},
               {L.fc1_b, w->fc1_b, F, "fc1_b"}, {L.fc2_b, w->fc2_b, D, "fc2_b"}};
  for (auto &it : items)
    if (!rc) rc = enc_copy(e, it.dst, it.src, it.n, it.what);
  if (!rc) rc = mat_set_f32(e, L.wq, w->wq, "wq");
  if (!rc) rc = mat_set_f32(e, L.wk, w->wk, "wk");
  if (!rc) rc = mat_set_f32(e, L.wv, w->wv, "wv");
  if (!rc) rc = prepare_qkv(e, L);
  if (!rc) rc = mat_set_f32(e, L.wo, w->wo, "wo");
  if (!rc) rc = mat_set_f32(e, L.fc1, w->fc1_w, "fc1_w");
  if (!rc) rc = mat_set_f32(e, L.fc2, w->fc2_w, "fc2_w");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_layer");
  return rc;
}

// EncLayerInt8 (encoder.rs:424-444): INT8 projections, f32 biases and norms.
extern "C" int qasr_encoder_set_layer_int8(qasr_encoder *e, int layer, const qasr_enc_layer_weights_int8 *w) {
  if (!e || !w || layer < 0 || layer >= e->cfg.n_layers) {
    set_error("qasr_encoder_set_layer_int8: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const size_t D = e->cfg.d_model, F = e->cfg.ffn_dim;
  EncLayerDev &L = e->layers[layer];
  int rc = QASR_OK;
  struct {
    float *dst;
    const float *src;
    size_t n;
    const char *what;
  } items[] = {{L.attn_norm_w, w->attn_norm_w, D, "attn_norm_w"}, {L.attn_norm_b, w->attn_norm_b, D, "attn_norm_b"},
               {L.bq, w->bq, D, "bq"}, {L.bk, w->bk, D, "bk"}, {L.bv, w->bv, D, "bv"}, {L.bo, w->bo, D, "bo"},
               {L.ffn_norm_w, w->ffn_norm_w, D, "ffn_norm_w"}, {L.ffn_norm_b, w->ffn_norm_b, D, "ffn_norm_b"},
               {L.fc1_b, w->fc1_b, F, "fc1_b"}, {L.fc2_b, w->fc2_b, D, "fc2_b"}};
  if (L.qkv.planes) {  // the f32 q|k|v operand goes with the f32 weights
    rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_layer_int8");
    f32_weight_free(&L.qkv);
  }
  for (auto &it : items)
    if (!rc) rc = enc_copy(e, it.dst, it.src, it.n, it.what);
  if (!rc) rc = mat_set_i8(e, L.wq, w->wq, w->wq_s, "wq");
  if (!rc) rc = mat_set_i8(e, L.wk, w->wk, w->wk_s, "wk");
  if (!rc) rc = mat_set_i8(e, L.wv, w->wv, w->wv_s, "wv");
  if (!rc) rc = mat_set_i8(e, L.wo, w->wo, w->wo_s, "wo");
  if (!rc) rc = mat_set_i8(e, L.fc1, w->fc1, w->fc1_s, "fc1");
  if (!rc) rc = mat_set_i8(e, L.fc2, w->fc2, w->fc2_s, "fc2");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_layer_int8");
  return rc;
}

extern "C" int qasr_encoder_set_post(qasr_encoder *e, const float *ln_post_w, const float *ln_post_b,
                                     const float *proj1_w, const float *proj1_b, const float *proj2_w,
                                     const float *proj2_b) {
  if (!e) {
    set_error("qasr_encoder_set_post: null encoder");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const size_t D = e->cfg.d_model, O = e->cfg.output_dim;
  int rc = enc_copy(e, e->ln_post_w, ln_post_w, D, "ln_post_w");
  if (!rc) rc = enc_copy(e, e->ln_post_b, ln_post_b, D, "ln_post_b");
  if (!rc) rc = mat_set_f32(e, e->proj1, proj1_w, "proj1_w");
  if (!rc) rc = enc_copy(e, e->proj1_b, proj1_b, D, "proj1_b");
  if (!rc) rc = mat_set_f32(e, e->proj2, proj2_w, "proj2_w");
  if (!rc) rc = enc_copy(e, e->proj2_b, proj2_b, O, "proj2_b");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_post");
  return rc;
}

extern "C" int qasr_encoder_set_post_int8(qasr_encoder *e, const float *ln_post_w, const float *ln_post_b,
                                          const int8_t *proj1, const float *proj1_s, const float *proj1_b,
                                          const int8_t *proj2, const float *proj2_s, const float *proj2_b) {
  if (!e) {
    set_error("qasr_encoder_set_post_int8: null encoder");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  const size_t D = e->cfg.d_model, O = e->cfg.output_dim;
  int rc = enc_copy(e, e->ln_post_w, ln_post_w, D, "ln_post_w");
  if (!rc) rc = enc_copy(e, e->ln_post_b, ln_post_b, D, "ln_post_b");
  if (!rc) rc = mat_set_i8(e, e->proj1, proj1, proj1_s, "proj1");
  if (!rc) rc = enc_copy(e, e->proj1_b, proj1_b, D, "proj1_b");
  if (!rc) rc = mat_set_i8(e, e->proj2, proj2, proj2_s, "proj2");
  if (!rc) rc = enc_copy(e, e->proj2_b, proj2_b, O, "proj2_b");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(e->stream), "qasr_encoder_set_post_int8");
  return rc;
}

extern "C" const qasr_encoder_config *qasr_encoder_get_config(const qasr_encoder *e) { return e ? &e->cfg : nullptr; }
extern "C" int qasr_encoder_device(const qasr_encoder *e) { return e ? e->device : -1; }

qasr::ScratchArena *qasr::encoder_arena(qasr_encoder *e) { return e ? e->arena : nullptr; }

extern "C" int qasr_encoder_tokens(const qasr_encoder *e, int mel_frames) {
  if (!e || mel_frames <= 0) return 0;
  const int cs = e->cfg.chunk_size;
  int total = 0;
  for (int s = 0; s < mel_frames; s += cs) total += chunk_tokens(std::min(cs, mel_frames - s));
  return total;
}

// Encoder::forward over n independent segments at once: their tokens are
// concatenated (segment s at rows off_s ..), every per-token operation runs
// once over all rows, the attention windows restart at every segment and
// each segment's conv chunks are padded on their own, so segment s's rows
// equal a forward of that segment alone.
static int encoder_run(qasr_encoder *e, int n, const float *const *mels, const int *frames, float *const *outs,
                       const int *out_rows, int *n_tokens) {
  cudaSetDevice(e->device);
  qasr::ArenaScope arena_scope(e->arena);
  for (EncMat *m : enc_mats(e))
    if (!m->ready()) {
      set_error("qasr_encoder_forward: weights not set (call the qasr_encoder_set_* functions first)");
      return QASR_ERR_INVALID;
    }
  const qasr_encoder_config &c = e->cfg;
  const int D = c.d_model, F = c.ffn_dim, O = c.output_dim, CH = kConvHidden, cs = c.chunk_size;
  std::vector<int> seg_T(n), seg_off(n + 1, 0);
  int max_frames = 0, max_full = 0;
  for (int i = 0; i < n; ++i) {
    if (!mels[i] || !outs[i] || frames[i] <= 0) {
      set_error("qasr_encoder_forward: invalid arguments (segment %d)", i);
      return QASR_ERR_INVALID;
    }
    seg_T[i] = qasr_encoder_tokens(e, frames[i]);
    if (out_rows[i] < seg_T[i]) {
      set_error("qasr_encoder_forward: output %d has %d rows, %d tokens needed", i, out_rows[i], seg_T[i]);
      return QASR_ERR_INVALID;
    }
    seg_off[i + 1] = seg_off[i] + seg_T[i];
    max_frames = std::max(max_frames, frames[i]);
    max_full = std::max(max_full, frames[i] / cs);
  }
  const int T = seg_off[n];
  cudaStream_t st = e->stream;
  int rc = QASR_OK;
  // buffers: per-token activations, and the conv stem of up to kStemGroup chunks
  const int h1 = (kMelBins + 2 - 3) / 2 + 1, h2 = (h1 + 2 - 3) / 2 + 1, h3 = (h2 + 2 - 3) / 2 + 1;
  const int w1m = (cs + 2 - 3) / 2 + 1, w2m = (w1m + 2 - 3) / 2 + 1, w3m = (w2m + 2 - 3) / 2 + 1;
  const int gmax = std::max(1, std::min(max_full, kStemGroup));
  if (T > e->tok_cap) {
    if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_encoder_forward"))) return rc;
    if (e->act) cudaFree(e->act);
    e->act = nullptr;
    e->tok_cap = 0;
    const size_t per_tok = (size_t)7 * D + F + O + D;  // x xn q k v attn proj | mid | out | pe
    if ((rc = cuda_status(cudaMalloc(&e->act, per_tok * T * 4), "qasr_encoder_forward: buffers"))) return rc;
    float *f = static_cast<float *>(e->act);
    auto take = [&](size_t n) { float *r = f; f += n * T; return r; };
    e->x = take(D);
    e->xn = take(D);
    e->q = take(D);
    e->k = take(D);
    e->v = take(D);
    e->attn = take(D);
    e->proj = take(D);
    e->mid = take(F);
    e->out = take(O);
    e->pe = take(D);
    e->tok_cap = T;
  }
  if (gmax > e->stem_cap) {
    if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_encoder_forward"))) return rc;
    if (e->conv_buf) cudaFree(e->conv_buf);
    e->conv_buf = nullptr;
    e->stem_cap = 0;
    const size_t pos1 = (size_t)gmax * h1 * w1m, pos2 = (size_t)gmax * h2 * w2m, pos3 = (size_t)gmax * h3 * w3m;
    const size_t cols = std::max({pos1 * 9, pos2 * CH * 9, pos3 * CH * 9});
    if ((rc = cuda_status(cudaMalloc(&e->conv_buf, (cols + pos1 * CH + pos2 * CH) * 4),
                          "qasr_encoder_forward: conv buffers")))
      return rc;
    e->cols = static_cast<float *>(e->conv_buf);
    e->act_a = e->cols + cols;
    e->act_b = e->act_a + pos1 * CH;
    e->stem_cap = gmax;
  }
  // ---- conv stem (encoder.rs:281-348) per segment: groups of full chunks, then the tail chunk
  int tok = 0;
  for (int sg = 0; sg < n && !rc; ++sg) {
    const float *mel = mels[sg];
    const int mel_frames = frames[sg], tail = mel_frames % cs;
    // the stem kernels read the mel directly: a host mel is copied to the device first
    cudaPointerAttributes pa{};
    const bool on_dev = cudaPointerGetAttributes(&pa, mel) == cudaSuccess &&
                        (pa.type == cudaMemoryTypeDevice || pa.type == cudaMemoryTypeManaged);
    cudaGetLastError();  // an unknown pointer is not an error here
    if (!on_dev) {
      const size_t bytes = (size_t)kMelBins * max_frames * 4;
      if (bytes > e->mel_cap) {
        if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_encoder_forward"))) return rc;
        if (e->mel_dev) cudaFree(e->mel_dev);
        e->mel_dev = nullptr;
        e->mel_cap = 0;
        if ((rc = cuda_status(cudaMalloc(&e->mel_dev, bytes), "qasr_encoder_forward: mel buffer"))) return rc;
        e->mel_cap = bytes;
      }
      // the previous segment's stem must be done with the buffer
      if ((rc = cuda_status(cudaMemcpyAsync(e->mel_dev, mel, (size_t)kMelBins * mel_frames * 4, cudaMemcpyDefault, st),
                            "qasr_encoder_forward: mel")))
        return rc;
      mel = e->mel_dev;
    }
    for (int first = 0; first < mel_frames && !rc;) {
      const bool full = first + cs <= mel_frames;
      const int B = full ? std::min(kStemGroup, (mel_frames - first) / cs) : 1;
      const int cw = full ? cs : tail;
      const int w1 = (cw + 2 - 3) / 2 + 1, w2 = (w1 + 2 - 3) / 2 + 1, w3 = (w2 + 2 - 3) / 2 + 1;
      const long r1 = (long)B * h1 * w1, r2 = (long)B * h2 * w2, r3 = (long)B * h3 * w3;
      conv1_gelu_kernel<<<(int)std::min<long>((r1 + 7) / 8, 148l * 8), 256, 0, st>>>(
          e->act_a, mel, mel_frames, first, cs, cw, B, h1, w1, e->conv_w[0], e->conv_b[0]);
      rc = launch_status("qasr_encoder_forward: conv1");
      if (!rc) rc = conv_stage(e, 1, e->act_b, e->act_a, h1, w1, B, h2, w2, st);
      if (!rc) rc = qasr_gelu(e->act_b, (int64_t)r2 * CH, st);
      if (!rc) rc = conv_stage(e, 2, e->act_a, e->act_b, h2, w2, B, h3, w3, st);
      if (!rc) rc = qasr_gelu(e->act_a, (int64_t)r3 * CH, st);
      if (!rc) {
        conv_reshape_cl_kernel<<<grid_of(r3 * CH), 256, 0, st>>>(e->cols, e->act_a, CH, h3, w3, B);
        rc = launch_status("qasr_encoder_forward: reshape");
      }
      if (!rc) rc = mat_apply(e->x + (size_t)tok * D, e->cols, e->conv_out, nullptr, B * w3, st);
      if (!rc) rc = qasr_sinusoidal_pe(e->pe, w3, D, st);
      if (!rc) {
        add_chunk_pe_kernel<<<grid_of((long)B * w3 * D), 256, 0, st>>>(e->x + (size_t)tok * D, e->pe, B, w3, D);
        rc = launch_status("qasr_encoder_forward: positions");
      }
      tok += B * w3;
      first += B * cw;
    }
  }
  if (rc) return rc;
  // ---- attention windows (encoder.rs:350-357)
  const int tpc = chunk_tokens(cs);
  const int wsize = tpc * (c.n_window_infer / cs);
  std::vector<int32_t> starts;
  int max_window = 0;
  for (int i = 0; i < n; ++i)
    for (int w0 = 0; w0 < seg_T[i]; w0 += wsize) {
      starts.push_back(seg_off[i] + w0);
      max_window = std::max(max_window, std::min(wsize, seg_T[i] - w0));
    }
  const int nw = (int)starts.size();
  starts.push_back(T);
  if (nw + 1 > e->win_cap) {
    if (e->win) cudaFree(e->win);
    e->win = nullptr;
    if ((rc = cuda_status(cudaMalloc(&e->win, (nw + 1) * 4), "qasr_encoder_forward: windows"))) return rc;
    e->win_cap = nw + 1;
  }
  if ((rc = cuda_status(cudaMemcpyAsync(e->win, starts.data(), (nw + 1) * 4, cudaMemcpyHostToDevice, st), "windows")))
    return rc;
  // the host vector must outlive the copy
  if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_encoder_forward"))) return rc;
  const float scale = 1.0f / sqrtf((float)c.head_dim);
  const int64_t td = (int64_t)T * D;
  for (int l = 0; l < c.n_layers && !rc; ++l) {
    const EncLayerDev &L = e->layers[l];
    rc = qasr_layer_norm(e->xn, e->x, L.attn_norm_w, L.attn_norm_b, T, D, 1e-5f, st);
    bool fused = false;
    if (!rc && L.qkv.planes) {  // one digit pass and one launch for q, k and v
      const int r = f32_gemm_prepared_split3(e->q, D, e->k, D, D, e->v, D, 2 * D, e->xn, D, L.qkv, L.bq, T, st);
      if (r != QASR_ERR_UNSUPPORTED) {
        rc = r;
        fused = true;
      }
    }
    if (!fused) {
      if (!rc) rc = mat_apply(e->q, e->xn, L.wq, L.bq, T, st);
      if (!rc) rc = mat_apply(e->k, e->xn, L.wk, L.bk, T, st);
      if (!rc) rc = mat_apply(e->v, e->xn, L.wv, L.bv, T, st);
    }
    if (!rc)
      rc = bidir_attention_launch(e->attn, e->q, e->k, e->v, T, c.n_heads, c.head_dim, scale, e->win, nw,
                                  max_window, st);
    if (!rc) rc = mat_apply(e->proj, e->attn, L.wo, L.bo, T, st);
    if (!rc) rc = qasr_add_inplace(e->x, e->proj, td, st);
    if (!rc) rc = qasr_layer_norm(e->xn, e->x, L.ffn_norm_w, L.ffn_norm_b, T, D, 1e-5f, st);
    if (!rc) rc = mat_apply(e->mid, e->xn, L.fc1, L.fc1_b, T, st);
    if (!rc) rc = qasr_gelu(e->mid, (int64_t)T * F, st);
    if (!rc) rc = mat_apply(e->proj, e->mid, L.fc2, L.fc2_b, T, st);
    if (!rc) rc = qasr_add_inplace(e->x, e->proj, td, st);
  }
  // ---- post LayerNorm and projections (encoder.rs:405-415)
  if (!rc) rc = qasr_layer_norm(e->xn, e->x, e->ln_post_w, e->ln_post_b, T, D, 1e-5f, st);
  if (!rc) rc = mat_apply(e->q, e->xn, e->proj1, e->proj1_b, T, st);
  if (!rc) rc = qasr_gelu(e->q, td, st);
  if (!rc) rc = mat_apply(e->out, e->q, e->proj2, e->proj2_b, T, st);
  for (int i = 0; i < n && !rc; ++i)
    rc = cuda_status(cudaMemcpyAsync(outs[i], e->out + (size_t)seg_off[i] * O, (size_t)seg_T[i] * O * 4,
                                     cudaMemcpyDefault, st),
                     "encoder output");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(st), "qasr_encoder_forward");
  if (!rc && n_tokens)
    for (int i = 0; i < n; ++i) n_tokens[i] = seg_T[i];
  return rc;
}

extern "C" int qasr_encoder_forward(qasr_encoder *e, const float *mel, int mel_frames, float *out, int out_rows,
                                    int *n_tokens) {
  if (!e || !mel || !out || mel_frames <= 0) {
    set_error("qasr_encoder_forward: invalid arguments");
    return QASR_ERR_INVALID;
  }
  float *outs[1] = {out};
  int T = 0;
  const int rc = encoder_run(e, 1, &mel, &mel_frames, outs, &out_rows, &T);
  if (!rc && n_tokens) *n_tokens = T;
  return rc;
}

extern "C" int qasr_encoder_forward_batch(qasr_encoder *e, const float *const *mels, const int *mel_frames, int n,
                                          float *const *outs, const int *out_rows, int *n_tokens) {
  if (!e || !mels || !mel_frames || !outs || !out_rows || n <= 0) {
    set_error("qasr_encoder_forward_batch: invalid arguments");
    return QASR_ERR_INVALID;
  }
  return encoder_run(e, n, mels, mel_frames, outs, out_rows, n_tokens);
}
