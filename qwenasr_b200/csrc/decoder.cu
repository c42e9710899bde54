// decoder.cu -- INT8 decoder engine: DecoderInt8 + KvCache + RopeCache +
// decoder_forward_int8 (crates/qwen-asr/src/decoder.rs:130-306, 652-965) for
// a batch of independent sequences on one GPU.
//
// Device layout (all allocated once in qasr_decoder_create):
//   per layer  wqkv  int8 [q_dim + 2*kv_dim, hidden]  (q | k | v rows; one
//                    matvec launch covers the three projections, like the
//                    fused QKV range split of kernels::linear_nobias_bf16_qkv,
//                    mod.rs:708-775), sqkv f32 scales; wo/so; gate_up/sgu
//                    (interleaved rows, decoder.rs:699-719); down/sdown;
//                    q/k/input/post norms f32.
//   globals    embed (f32 or int8 + scales), final norm, lm head int8 + scales
//   KV         k_cache/v_cache f32 [max_batch][n_layers][max_seq][kv_dim]:
//              the reference's per-sequence KvCache layout, sequences stacked.
//   RoPE       cos/sin [max_seq, head_dim], the RopeCache::ensure table.
//   work       x [B, hidden]; q_out, attn [B, q_dim]; h [B, inter];
//              attention partials/counters; argmax keys.
// Every INT8 matrix keeps the reference's row-major [out, in] layout and is
// read by TMA through one tensor map (umma_weight_map) built at creation.
//
// One decode step = 2 + 5*n_layers kernels captured once per batch size in a
// CUDA graph (programmatic dependent launch between the streaming kernels)
// and replayed: embed gather; per layer RMSNorm+QKV contraction with the q/k
// per-head norm + RoPE + KV append in its epilogue, attention, o-proj
// (+residual), RMSNorm+gate/up contraction+SwiGLU, down contraction
// (+residual); final RMSNorm + lm head + argmax.  The INT8 contractions run
// on the tensor cores (umma_matvec.cu).
#include <algorithm>
#include <cstring>
#include <vector>

#include "attention.cuh"
#include "common.cuh"
#include "matvec.cuh"
#include "step.cuh"
#include "umma.cuh"

namespace qasr {

struct LayerDev {
  int8_t *wqkv = nullptr, *wo = nullptr, *gate_up = nullptr, *down = nullptr;
  CUtensorMap tm_qkv, tm_o, tm_gu, tm_down;
  float *sqkv = nullptr, *so = nullptr, *sgu = nullptr, *sdown = nullptr;
  float *q_norm = nullptr, *k_norm = nullptr, *in_norm = nullptr, *post_norm = nullptr;
};

}  // namespace qasr

struct qasr_decoder {
  qasr_decoder_config cfg;
  int device = 0;
  cudaStream_t stream = nullptr;
  qasr::ScratchArena *arena = nullptr;  // this engine's kernel-level scratch
  std::vector<qasr::LayerDev> layers;
  void *embed = nullptr;
  float *embed_s = nullptr, *norm = nullptr, *lm_s = nullptr;
  int8_t *lm = nullptr;
  bool lm_tied = false;
  bool globals_ready = false;  // set_globals succeeded (the lm head tensor map exists)
  float *k_cache = nullptr, *v_cache = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  float *x = nullptr, *q_out = nullptr, *attn = nullptr, *h = nullptr;
  float *partials = nullptr, *logits = nullptr;
  unsigned *attn_ctr = nullptr, *am_ctr = nullptr;
  CUtensorMap tm_k, tm_v, tm_lm;
  unsigned long long *am_keys = nullptr;
  int32_t *tok = nullptr, *pos = nullptr, *next = nullptr;
  int *err = nullptr;
  int32_t *h_tok = nullptr, *h_pos = nullptr, *h_next = nullptr;  // pinned staging
  int *h_err = nullptr;
  bool keep_logits = false;
  // prefill work buffers (decoder_prefill_int8's DecoderBuffers), grown on demand
  int pf_cap = 0;
  float *pf_x = nullptr, *pf_xn = nullptr, *pf_q = nullptr, *pf_k = nullptr, *pf_v = nullptr, *pf_attn = nullptr,
        *pf_proj = nullptr, *pf_gu = nullptr, *pf_h = nullptr;
  void *pf_block = nullptr;
  unsigned char *pf_meta = nullptr;  // row positions / slots and attention segments of a prefill
  size_t pf_meta_cap = 0;
  int32_t *emb_ids = nullptr;  // device ids of qasr_decoder_embed, grown on demand
  int emb_cap = 0;
  std::vector<cudaGraphExec_t> graphs;  // per M (index M), built lazily
  // the persistent decode-step kernel (decode_step.cu): tensor maps and layer
  // pointers in device memory, its zeroed scratch block and attention partials
  int step_kernel = 1;  // 0: the persistent kernel where it covers the shape; 1: per-layer kernels (default)
  CUtensorMap *step_maps = nullptr;
  qasr::StepLayerPtrs *step_layers = nullptr;
  unsigned char *step_scratch = nullptr;
  qasr::StepScratch step_layout{};
  float *step_part = nullptr;
  bool step_dirty = true;  // weights changed since the device tables were written
  unsigned long long *step_trace = nullptr;  // caller's phase-timeline buffer (qasr_decoder_trace) or null
  int64_t step_trace_n = 0;
  CUtensorMap tm_k16, tm_v16;
  std::vector<void *> allocs;
  long seq_stride() const { return (long)cfg.n_layers * cfg.max_seq * cfg.n_kv_heads * cfg.head_dim; }
};

namespace qasr {

// Embedding gather for the step's tokens (f32 or int8 table).
__global__ void step_embed_kernel(float *__restrict__ x, const void *__restrict__ table,
                                  const float *__restrict__ scales, int is_int8, const int32_t *__restrict__ ids,
                                  int dim, int vocab, int *err) {
  const int m = blockIdx.x;
  int id = ids[m];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0) atomicExch(err, 1);
    id = 0;
  }
  float4 *d = reinterpret_cast<float4 *>(x + (size_t)m * dim);
  if (is_int8) {
    const int8_t *tab = static_cast<const int8_t *>(table);
    const uint32_t *src = reinterpret_cast<const uint32_t *>(tab + (size_t)id * dim);
    const float s = scales[id];
    for (int c = threadIdx.x; c < dim / 4; c += blockDim.x) {
      float f[4];
      i8x4_to_f32(src[c], f);
      d[c] = make_float4(__fmul_rn(f[0], s), __fmul_rn(f[1], s), __fmul_rn(f[2], s), __fmul_rn(f[3], s));
    }
  } else {
    const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(table) + (size_t)id * dim);
    for (int c = threadIdx.x; c < dim / 4; c += blockDim.x) d[c] = src[c];
  }
}

}  // namespace qasr

using namespace qasr;

// kernels launched by the decode step (the rope table kernel lives in norm_rope.cu)
extern "C" int qasr_rms_norm(float *, const float *, const float *, int, int, float, void *);
extern "C" int qasr_rope_cache_table(float *, float *, int, int, float, void *);

static void *dalloc(qasr_decoder *d, size_t bytes, int *rc) {
  void *p = nullptr;
  if (*rc) return nullptr;
  cudaError_t e = cudaMalloc(&p, bytes ? bytes : 16);
  if (e != cudaSuccess) {
    *rc = cuda_status(e, "qasr_decoder: cudaMalloc");
    return nullptr;
  }
  d->allocs.push_back(p);
  return p;
}

extern "C" void qasr_decoder_free(qasr_decoder *d) {
  if (!d) return;
  cudaSetDevice(d->device);
  if (d->stream) cudaStreamSynchronize(d->stream);
  for (auto g : d->graphs)
    if (g) cudaGraphExecDestroy(g);
  for (void *p : d->allocs) cudaFree(p);
  if (d->pf_block) cudaFree(d->pf_block);
  if (d->emb_ids) cudaFree(d->emb_ids);
  if (d->h_tok) cudaFreeHost(d->h_tok);
  if (d->stream) cudaStreamDestroy(d->stream);
  arena_free(d->arena);
  delete d;
}

extern "C" qasr_decoder *qasr_decoder_create(const qasr_decoder_config *cfg, int device) {
  if (!cfg || cfg->hidden <= 0 || cfg->hidden % 128 || cfg->inter <= 0 || cfg->inter % 64 || cfg->n_layers <= 0 ||
      cfg->n_heads <= 0 || cfg->n_kv_heads <= 0 || cfg->n_heads % cfg->n_kv_heads || cfg->vocab <= 0 ||
      cfg->max_batch <= 0 || cfg->max_batch > 8 || cfg->max_seq <= 0) {
    set_error("qasr_decoder_create: invalid config");
    return nullptr;
  }
  if (cfg->head_dim != 128 || cfg->n_heads / cfg->n_kv_heads > 2) {
    set_error("qasr_decoder_create: head_dim must be 128 and GQA group <= 2");
    return nullptr;
  }
  if (cudaSetDevice(device) != cudaSuccess) {
    set_error("qasr_decoder_create: cudaSetDevice(%d) failed", device);
    return nullptr;
  }
  qasr_decoder *d = new qasr_decoder();
  d->cfg = *cfg;
  d->device = device;
  int rc = cuda_status(cudaStreamCreateWithFlags(&d->stream, cudaStreamNonBlocking), "qasr_decoder_create");
  if (!rc && !(d->arena = arena_create(device))) {
    set_error("qasr_decoder_create: scratch arena");
    rc = QASR_ERR_ALLOC;
  }
  const int H = cfg->hidden, I = cfg->inter, L = cfg->n_layers, hd = cfg->head_dim;
  const int q_dim = cfg->n_heads * hd, kv_dim = cfg->n_kv_heads * hd, qkv_rows = q_dim + 2 * kv_dim;
  const int B = cfg->max_batch;
  d->layers.resize(L);
  for (int l = 0; l < L; ++l) {
    LayerDev &ld = d->layers[l];
    ld.wqkv = (int8_t *)dalloc(d, (size_t)qkv_rows * H, &rc);
    ld.sqkv = (float *)dalloc(d, (size_t)qkv_rows * 4, &rc);
    ld.wo = (int8_t *)dalloc(d, (size_t)H * q_dim, &rc);
    ld.so = (float *)dalloc(d, (size_t)H * 4, &rc);
    ld.gate_up = (int8_t *)dalloc(d, (size_t)2 * I * H, &rc);
    ld.sgu = (float *)dalloc(d, (size_t)2 * I * 4, &rc);
    ld.down = (int8_t *)dalloc(d, (size_t)H * I, &rc);
    ld.sdown = (float *)dalloc(d, (size_t)H * 4, &rc);
    ld.q_norm = (float *)dalloc(d, (size_t)hd * 4, &rc);
    ld.k_norm = (float *)dalloc(d, (size_t)hd * 4, &rc);
    ld.in_norm = (float *)dalloc(d, (size_t)H * 4, &rc);
    ld.post_norm = (float *)dalloc(d, (size_t)H * 4, &rc);
    if (!rc) rc = umma_weight_map(&ld.tm_qkv, ld.wqkv, qkv_rows, H);
    if (!rc) rc = umma_weight_map(&ld.tm_o, ld.wo, H, q_dim);
    if (!rc) rc = umma_weight_map(&ld.tm_gu, ld.gate_up, 2 * I, H);
    if (!rc) rc = umma_weight_map(&ld.tm_down, ld.down, H, I);
  }
  d->embed = dalloc(d, (size_t)cfg->vocab * H * (cfg->embed_is_int8 ? 1 : 4), &rc);
  if (cfg->embed_is_int8) d->embed_s = (float *)dalloc(d, (size_t)cfg->vocab * 4, &rc);
  d->norm = (float *)dalloc(d, (size_t)H * 4, &rc);
  const size_t kv_elems = (size_t)B * d->seq_stride();
  d->k_cache = (float *)dalloc(d, kv_elems * 4, &rc);
  d->v_cache = (float *)dalloc(d, kv_elems * 4, &rc);
  d->rope_cos = (float *)dalloc(d, (size_t)cfg->max_seq * hd * 4, &rc);
  d->rope_sin = (float *)dalloc(d, (size_t)cfg->max_seq * hd * 4, &rc);
  d->x = (float *)dalloc(d, (size_t)B * H * 4, &rc);
  d->q_out = (float *)dalloc(d, (size_t)B * q_dim * 4, &rc);
  d->attn = (float *)dalloc(d, (size_t)B * q_dim * 4, &rc);
  d->h = (float *)dalloc(d, (size_t)B * I * 4, &rc);
  const int G = cfg->n_heads / cfg->n_kv_heads;
  d->partials =
      (float *)dalloc(d, (size_t)(attn_decode_grid() + B * cfg->n_kv_heads) * G * kAttnPartStride * 4, &rc);
  d->attn_ctr = (unsigned *)dalloc(d, (size_t)B * cfg->n_kv_heads * 4, &rc);
  d->am_keys = (unsigned long long *)dalloc(d, 8 * 8, &rc);
  d->am_ctr = (unsigned *)dalloc(d, 16, &rc);
  d->tok = (int32_t *)dalloc(d, 8 * 4, &rc);
  d->pos = (int32_t *)dalloc(d, 8 * 4, &rc);
  d->next = (int32_t *)dalloc(d, 8 * 4, &rc);
  d->err = (int *)dalloc(d, 16, &rc);
  d->step_maps = (CUtensorMap *)dalloc(d, (size_t)(3 + 4 * L) * sizeof(CUtensorMap), &rc);
  d->step_layers = (qasr::StepLayerPtrs *)dalloc(d, (size_t)L * sizeof(qasr::StepLayerPtrs), &rc);
  d->step_layout = qasr::step_scratch_layout(L, std::max({(long)qkv_rows, (long)H, 2l * I}));
  d->step_scratch = (unsigned char *)dalloc(d, d->step_layout.total, &rc);
  d->step_part = (float *)dalloc(d, (size_t)(attn_grid() + qasr::kStepMaxPairs) * 2 * 132 * 4, &rc);
  if (!rc) rc = cuda_status(cudaHostAlloc((void **)&d->h_tok, 4 * 64, cudaHostAllocDefault), "cudaHostAlloc");
  if (rc) {
    qasr_decoder_free(d);
    return nullptr;
  }
  d->h_pos = d->h_tok + 16;
  d->h_next = d->h_tok + 32;
  d->h_err = reinterpret_cast<int *>(d->h_tok + 48);
  cudaStream_t st = d->stream;
  rc = cuda_status(cudaMemsetAsync(d->k_cache, 0, kv_elems * 4, st), "memset");
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->v_cache, 0, kv_elems * 4, st), "memset");
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->attn_ctr, 0, (size_t)B * cfg->n_kv_heads * 4, st), "memset");
  if (!rc) rc = attn_make_tensor_map(&d->tm_k, d->k_cache, (long)B * L * cfg->max_seq, kv_dim);
  if (!rc) rc = attn_make_tensor_map(&d->tm_v, d->v_cache, (long)B * L * cfg->max_seq, kv_dim);
  if (!rc) rc = step_kv_map(&d->tm_k16, d->k_cache, (long)B * L * cfg->max_seq, kv_dim);
  if (!rc) rc = step_kv_map(&d->tm_v16, d->v_cache, (long)B * L * cfg->max_seq, kv_dim);
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->step_scratch, 0, d->step_layout.total, st), "memset");
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->am_keys, 0, 64, st), "memset");
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->am_ctr, 0, 16, st), "memset");
  if (!rc) rc = cuda_status(cudaMemsetAsync(d->err, 0, 16, st), "memset");
  if (!rc) rc = qasr_rope_cache_table(d->rope_cos, d->rope_sin, cfg->max_seq, hd, cfg->theta, st);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(st), "qasr_decoder_create");
  if (rc) {
    qasr_decoder_free(d);
    return nullptr;
  }
  d->graphs.assign(9, nullptr);
  return d;
}

static int copy_in(qasr_decoder *d, void *dst, const void *src, size_t bytes, const char *what) {
  if (!src) {
    set_error("qasr_decoder: %s is NULL", what);
    return QASR_ERR_INVALID;
  }
  return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, d->stream), what);
}

extern "C" int qasr_decoder_set_layer(qasr_decoder *d, int layer, const qasr_dec_layer_weights *w) {
  if (!d || !w || layer < 0 || layer >= d->cfg.n_layers) {
    set_error("qasr_decoder_set_layer: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  const qasr_decoder_config &c = d->cfg;
  const size_t H = c.hidden, I = c.inter, q_dim = (size_t)c.n_heads * c.head_dim, kv = (size_t)c.n_kv_heads * c.head_dim;
  LayerDev &ld = d->layers[layer];
  int rc = 0;
  if (!rc) rc = copy_in(d, ld.wqkv, w->wq, q_dim * H, "wq");
  if (!rc) rc = copy_in(d, ld.wqkv + q_dim * H, w->wk, kv * H, "wk");
  if (!rc) rc = copy_in(d, ld.wqkv + (q_dim + kv) * H, w->wv, kv * H, "wv");
  if (!rc) rc = copy_in(d, ld.sqkv, w->wq_s, q_dim * 4, "wq_s");
  if (!rc) rc = copy_in(d, ld.sqkv + q_dim, w->wk_s, kv * 4, "wk_s");
  if (!rc) rc = copy_in(d, ld.sqkv + q_dim + kv, w->wv_s, kv * 4, "wv_s");
  if (!rc) rc = copy_in(d, ld.wo, w->wo, H * q_dim, "wo");
  if (!rc) rc = copy_in(d, ld.so, w->wo_s, H * 4, "wo_s");
  if (w->gate_up || w->gate_up_s) {  // both NULL: qasr_decoder_set_gate_up supplies them
    if (!rc) rc = copy_in(d, ld.gate_up, w->gate_up, 2 * I * H, "gate_up");
    if (!rc) rc = copy_in(d, ld.sgu, w->gate_up_s, 2 * I * 4, "gate_up_s");
  }
  if (!rc) rc = copy_in(d, ld.down, w->down, H * I, "down");
  if (!rc) rc = copy_in(d, ld.sdown, w->down_s, H * 4, "down_s");
  if (!rc) rc = copy_in(d, ld.q_norm, w->q_norm, c.head_dim * 4, "q_norm");
  if (!rc) rc = copy_in(d, ld.k_norm, w->k_norm, c.head_dim * 4, "k_norm");
  if (!rc) rc = copy_in(d, ld.in_norm, w->input_norm, H * 4, "input_norm");
  if (!rc) rc = copy_in(d, ld.post_norm, w->post_attn_norm, H * 4, "post_attn_norm");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(d->stream), "qasr_decoder_set_layer");
  d->step_dirty = true;
  return rc;
}

namespace qasr {
// fused[2r] = gate[r], fused[2r+1] = up[r] (rows of `cols` bytes), and the scales alike.
__global__ void __launch_bounds__(256) interleave_rows_kernel(int8_t *__restrict__ fused, float *__restrict__ fused_s,
                                                              const int8_t *__restrict__ gate,
                                                              const float *__restrict__ gate_s,
                                                              const int8_t *__restrict__ up,
                                                              const float *__restrict__ up_s, int rows, int cols) {
  const int vec = cols / 16;  // uint4 per row
  const long total = (long)2 * rows * vec;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long r2 = i / vec, c = i % vec;
    const long r = r2 >> 1;
    const int8_t *src = (r2 & 1) ? up : gate;
    reinterpret_cast<uint4 *>(fused + r2 * cols)[c] = reinterpret_cast<const uint4 *>(src + r * cols)[c];
    if (c == 0) fused_s[r2] = (r2 & 1) ? up_s[r] : gate_s[r];
  }
}
}  // namespace qasr

// DecoderInt8::load's gate/up fusion (decoder.rs:699-719) on the device.
extern "C" int qasr_decoder_set_gate_up(qasr_decoder *d, int layer, const int8_t *gate, const float *gate_s,
                                        const int8_t *up, const float *up_s) {
  if (!d || layer < 0 || layer >= d->cfg.n_layers || !gate || !gate_s || !up || !up_s) {
    set_error("qasr_decoder_set_gate_up: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  const qasr_decoder_config &c = d->cfg;
  const size_t H = c.hidden, I = c.inter;
  LayerDev &ld = d->layers[layer];
  void *tmp = nullptr;
  int rc = cuda_status(cudaMalloc(&tmp, 2 * I * H + 2 * I * 4), "qasr_decoder_set_gate_up: staging");
  if (rc) return rc;
  int8_t *g = static_cast<int8_t *>(tmp), *u = g + I * H;
  float *gs = reinterpret_cast<float *>(u + I * H), *us = gs + I;
  rc = copy_in(d, g, gate, I * H, "gate");
  if (!rc) rc = copy_in(d, u, up, I * H, "up");
  if (!rc) rc = copy_in(d, gs, gate_s, I * 4, "gate_s");
  if (!rc) rc = copy_in(d, us, up_s, I * 4, "up_s");
  if (!rc) {
    const long total = (long)2 * I * (H / 16);
    interleave_rows_kernel<<<(int)std::min((total + 255) / 256, 148l * 8), 256, 0, d->stream>>>(
        ld.gate_up, ld.sgu, g, gs, u, us, (int)I, (int)H);
    rc = launch_status("qasr_decoder_set_gate_up");
  }
  const int rc2 = cuda_status(cudaStreamSynchronize(d->stream), "qasr_decoder_set_gate_up");
  cudaFree(tmp);
  d->step_dirty = true;
  return rc ? rc : rc2;
}

extern "C" int qasr_decoder_set_globals(qasr_decoder *d, const void *embed, const float *embed_scales,
                                        const float *norm, const int8_t *lm_head, const float *lm_head_s) {
  if (!d) {
    set_error("qasr_decoder_set_globals: null decoder");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  const qasr_decoder_config &c = d->cfg;
  const size_t VH = (size_t)c.vocab * c.hidden;
  int rc = QASR_OK;
  if (!lm_head && !c.embed_is_int8) {
    set_error("qasr_decoder_set_globals: a tied lm head needs the INT8 embedding table");
    return QASR_ERR_INVALID;
  }
  if (c.embed_is_int8 && !lm_head) {
    rc = copy_in(d, d->embed, embed, VH, "embed");  // tied: one copy serves the gather and the lm head
    d->lm_tied = true;
  } else {
    rc = copy_in(d, d->embed, embed, VH * (c.embed_is_int8 ? 1 : 4), "embed");
    d->lm_tied = false;
  }
  if (!rc && c.embed_is_int8) rc = copy_in(d, d->embed_s, embed_scales, (size_t)c.vocab * 4, "embed_scales");
  if (!rc) rc = copy_in(d, d->norm, norm, (size_t)c.hidden * 4, "norm");
  if (!rc && lm_head) {
    if (!d->lm) {
      int arc = 0;
      d->lm = (int8_t *)dalloc(d, VH, &arc);
      d->lm_s = (float *)dalloc(d, (size_t)c.vocab * 4, &arc);
      if (arc) return arc;
    }
    rc = copy_in(d, d->lm, lm_head, VH, "lm_head");
    if (!rc) rc = copy_in(d, d->lm_s, lm_head_s, (size_t)c.vocab * 4, "lm_head_s");
  }
  if (!rc)
    rc = umma_weight_map(&d->tm_lm, d->lm_tied ? static_cast<const int8_t *>(d->embed) : d->lm, c.vocab, c.hidden);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(d->stream), "qasr_decoder_set_globals");
  d->globals_ready = rc == QASR_OK;
  d->step_dirty = true;
  return rc;
}

extern "C" int qasr_decoder_kv(qasr_decoder *d, int slot, float **k, float **v) {
  if (!d || !k || !v || slot < 0 || slot >= d->cfg.max_batch) {
    set_error("qasr_decoder_kv: invalid arguments");
    return QASR_ERR_INVALID;
  }
  *k = d->k_cache + (size_t)slot * d->seq_stride();
  *v = d->v_cache + (size_t)slot * d->seq_stride();
  return QASR_OK;
}

extern "C" void *qasr_decoder_stream(qasr_decoder *d) { return d ? (void *)d->stream : nullptr; }

extern "C" int qasr_decoder_keep_logits(qasr_decoder *d, int enable) {
  if (!d) return QASR_ERR_INVALID;
  if (enable && !d->logits) {
    int rc = 0;
    cudaSetDevice(d->device);
    qasr::ArenaScope arena_scope(d->arena);
    d->logits = (float *)dalloc(d, (size_t)d->cfg.max_batch * d->cfg.vocab * 4, &rc);
    if (rc) return rc;
  }
  if ((bool)enable != d->keep_logits) {
    for (auto &g : d->graphs)
      if (g) {
        cudaGraphExecDestroy(g);
        g = nullptr;
      }
  }
  d->keep_logits = enable != 0;
  return QASR_OK;
}

extern "C" const float *qasr_decoder_logits(qasr_decoder *d) { return d && d->keep_logits ? d->logits : nullptr; }

static bool step_params(qasr_decoder *d, int M, StepParams *out);

extern "C" int qasr_decoder_set_step_kernel(qasr_decoder *d, int mode) {
  if (!d || mode < 0 || mode > 1) {
    set_error("qasr_decoder_set_step_kernel: invalid arguments (mode 0 or 1)");
    return QASR_ERR_INVALID;
  }
  if (mode != d->step_kernel) {
    cudaSetDevice(d->device);
    for (auto &g : d->graphs)
      if (g) {
        cudaGraphExecDestroy(g);
        g = nullptr;
      }
  }
  d->step_kernel = mode;
  return QASR_OK;
}

extern "C" int qasr_decoder_trace(qasr_decoder *d, unsigned long long *stamps, int64_t n) {
  if (!d || n < 0) {
    set_error("qasr_decoder_trace: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  for (auto &g : d->graphs)
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  d->step_trace = n ? stamps : nullptr;
  d->step_trace_n = n;
  return QASR_OK;
}

extern "C" int qasr_decoder_trace_stride(const qasr_decoder *d) {
  return d ? step_trace_stride(d->cfg.n_layers) : -1;
}

extern "C" int qasr_decoder_step_kernel(const qasr_decoder *d, int M) {
  if (!d || M < 1 || M > d->cfg.max_batch) return -1;
  StepParams q{};
  return step_params(const_cast<qasr_decoder *>(d), M, &q) ? 0 : 1;
}

// Optional per-kernel-class timing of an eager step: events recorded before
// the first and after every kernel, durations summed per class.
struct StepMarks {
  std::vector<cudaEvent_t> ev;
  std::vector<int> cls;
  cudaStream_t st;
  void mark(int c) {
    cudaEvent_t e;
    cudaEventCreate(&e);
    cudaEventRecord(e, st);
    ev.push_back(e);
    cls.push_back(c);
  }
  ~StepMarks() {
    for (auto e : ev) cudaEventDestroy(e);
  }
};
#define MARK(c) \
  if (marks) marks->mark(c)

// Write the persistent kernel's tables (tensor maps, layer pointers) to the
// device when the weights changed; never inside a stream capture.
static int step_upload(qasr_decoder *d) {
  if (!d->step_dirty) return QASR_OK;
  const qasr_decoder_config &c = d->cfg;
  std::vector<CUtensorMap> maps((size_t)3 + 4 * c.n_layers);
  std::vector<StepLayerPtrs> lp((size_t)c.n_layers);
  maps[0] = d->tm_k16;
  maps[1] = d->tm_v16;
  maps[2] = d->tm_lm;
  for (int l = 0; l < c.n_layers; ++l) {
    const LayerDev &L = d->layers[l];
    maps[3 + 4 * l] = L.tm_qkv;
    maps[4 + 4 * l] = L.tm_o;
    maps[5 + 4 * l] = L.tm_gu;
    maps[6 + 4 * l] = L.tm_down;
    lp[l] = StepLayerPtrs{L.sqkv, L.so, L.sgu, L.sdown, L.q_norm, L.k_norm, L.in_norm, L.post_norm};
  }
  int rc = cuda_status(cudaMemcpy(d->step_maps, maps.data(), maps.size() * sizeof(CUtensorMap), cudaMemcpyHostToDevice),
                       "decode step tables");
  if (!rc)
    rc = cuda_status(cudaMemcpy(d->step_layers, lp.data(), lp.size() * sizeof(StepLayerPtrs), cudaMemcpyHostToDevice),
                     "decode step tables");
  if (!rc) d->step_dirty = false;
  return rc;
}

// Parameters of the persistent kernel for a step of M sequences; false when
// the engine uses the per-layer kernels (by choice or because the kernel does
// not cover the shape).
static bool step_params(qasr_decoder *d, int M, StepParams *out) {
  if (d->step_kernel != 0) return false;
  const qasr_decoder_config &c = d->cfg;
  StepParams q{};
  q.maps = d->step_maps;
  q.layers = d->step_layers;
  q.final_norm = d->norm;
  q.lm_s = d->lm_tied ? d->embed_s : d->lm_s;
  q.x = d->x;
  q.q_out = d->q_out;
  q.attn = d->attn;
  q.h = d->h;
  q.k_cache = d->k_cache;
  q.v_cache = d->v_cache;
  q.seq_stride = d->seq_stride();
  q.rope_cos = d->rope_cos;
  q.rope_sin = d->rope_sin;
  q.pos = d->pos;
  unsigned char *b = d->step_scratch;
  const StepScratch &o = d->step_layout;
  q.sync = reinterpret_cast<unsigned *>(b + o.sync);
  q.tile_ctr = reinterpret_cast<unsigned *>(b + o.tile_ctr);
  q.pair_ctr = reinterpret_cast<unsigned *>(b + o.pair_ctr);
  q.keys = reinterpret_cast<unsigned long long *>(b + o.keys);
  q.am_ctr = reinterpret_cast<unsigned *>(b + o.am_ctr);
  q.acc = reinterpret_cast<long long *>(b + o.acc);
  q.part = d->step_part;
  q.logits = d->keep_logits ? d->logits : nullptr;
  q.next = d->next;
  q.err = d->err;
  q.trace = d->step_trace && d->step_trace_n >= (int64_t)attn_grid() * step_trace_stride(c.n_layers) ? d->step_trace
                                                                                                      : nullptr;
  q.M = M;
  q.H = c.hidden;
  q.I = c.inter;
  q.NQ = c.n_heads;
  q.NKV = c.n_kv_heads;
  q.L = c.n_layers;
  q.V = c.vocab;
  q.max_seq = c.max_seq;
  q.eps = c.eps;
  q.scale = 1.0f / sqrtf((float)c.head_dim);
  if (step_plan(q, attn_grid()) != QASR_OK) return false;
  *out = q;
  return true;
}

// Enqueue the kernels of one decode step for M sequences on d->stream.
static int enqueue_step(qasr_decoder *d, int M, StepMarks *marks = nullptr) {
  const qasr_decoder_config &c = d->cfg;
  if (!d->globals_ready) {
    set_error("qasr_decoder: qasr_decoder_set_globals must succeed before a step");
    return QASR_ERR_INVALID;
  }
  cudaStream_t st = d->stream;
  MARK(-1);
  const int H = c.hidden, I = c.inter, hd = c.head_dim;
  const int q_dim = c.n_heads * hd, kv_dim = c.n_kv_heads * hd, qkv_rows = q_dim + 2 * kv_dim;
  const int G = c.n_heads / c.n_kv_heads;
  const void *emb_tab = d->embed;
  step_embed_kernel<<<M, 256, 0, st>>>(d->x, emb_tab, d->embed_s, c.embed_is_int8, d->tok, H, c.vocab, d->err);
  MARK(QASR_K_EMBED);
  int rc = launch_status("decode step: embed");
  StepParams sp;
  if (!rc && step_params(d, M, &sp)) {
    // the whole step as one persistent kernel after its scratch is zeroed
    rc = cuda_status(cudaMemsetAsync(d->step_scratch, 0, d->step_layout.total, st), "decode step: scratch");
    if (!rc) rc = step_launch(sp, attn_grid(), st);
    MARK(QASR_K_STEP);
    return rc;
  }
  // in-step timeline of the per-layer kernels (qasr_decoder_trace): launch
  // 5*l + {0 q|k|v, 1 attention, 2 o-proj, 3 gate/up, 4 down}, 5*L the lm head
  unsigned long long *ts =
      d->step_trace && d->step_trace_n >= 2 * (5 * (int64_t)c.n_layers + 1) ? d->step_trace : nullptr;
  auto tslot = [&](int launch) { return ts ? ts + 2 * launch : nullptr; };
  auto mvp = [&](const CUtensorMap &tm, const float *x, long xs, const float *nw, const float *sc, float *y, long ys,
                 int K, int N) {
    UmmaParams p{};
    p.tmap = tm;
    p.x = x; p.x_stride = xs; p.norm_w = nw; p.eps = c.eps; p.scales = sc; p.y = y; p.y_stride = ys;
    p.M = M; p.K = K; p.N = N;
    p.keys = d->am_keys; p.counter = d->am_ctr; p.ids = d->next; p.err = d->err;
    return p;
  };
  auto mv = [&](const CUtensorMap &tm, const float *x, long xs, const float *nw, const float *sc, float *y, long ys,
                int K, int N, MvEpi e, int launch) {
    UmmaParams p = mvp(tm, x, xs, nw, sc, y, ys, K, N);
    p.tstamp = tslot(launch);
    return umma_launch(p, e, st, true);
  };
  for (int l = 0; l < c.n_layers && !rc; ++l) {
    const LayerDev &L = d->layers[l];
    // input RMSNorm fused into the q|k|v matvec; its epilogue applies the q/k
    // per-head norm + RoPE and appends K/V (one launch)
    {
      UmmaParams p = mvp(L.tm_qkv, d->x, H, L.in_norm, L.sqkv, nullptr, 0, H, qkv_rows);
      p.post.q_out = d->q_out; p.post.k_cache = d->k_cache; p.post.v_cache = d->v_cache;
      p.post.seq_stride = d->seq_stride(); p.post.layer = l; p.post.max_seq = c.max_seq;
      p.post.n_heads = c.n_heads; p.post.n_kv = c.n_kv_heads; p.post.positions = d->pos;
      p.post.q_norm = L.q_norm; p.post.k_norm = L.k_norm; p.post.cos_tab = d->rope_cos; p.post.sin_tab = d->rope_sin;
      p.tstamp = tslot(5 * l);
      if ((rc = umma_launch(p, MvEpi::QkvPost, st, true))) break;
    }
    MARK(QASR_K_QKV);
    AttnDecodeParams a{};
    a.tm_k = d->tm_k; a.tm_v = d->tm_v;
    a.q = d->q_out; a.q_stride = q_dim; a.layer = l; a.n_layers = c.n_layers; a.max_seq = c.max_seq;
    a.n_kv_heads = c.n_kv_heads; a.positions = d->pos; a.scale = 1.0f / sqrtf((float)hd); a.M = M;
    a.partials = d->partials; a.counters = d->attn_ctr; a.out = d->attn; a.out_stride = q_dim; a.err = d->err;
    a.tstamp = tslot(5 * l + 1);
    if ((rc = attn_decode_launch(a, G, st, true))) break;
    MARK(QASR_K_ATTN);
    if ((rc = mv(L.tm_o, d->attn, q_dim, nullptr, L.so, d->x, H, q_dim, H, MvEpi::Residual, 5 * l + 2))) break;
    MARK(QASR_K_OPROJ);
    // post-attention RMSNorm fused into the gate/up matvec, SwiGLU in its epilogue
    if ((rc = mv(L.tm_gu, d->x, H, L.post_norm, L.sgu, d->h, I, H, 2 * I, MvEpi::SwiGLU, 5 * l + 3))) break;
    MARK(QASR_K_GATEUP);
    if ((rc = mv(L.tm_down, d->h, I, nullptr, L.sdown, d->x, H, I, H, MvEpi::Residual, 5 * l + 4))) break;
    MARK(QASR_K_DOWN);
  }
  if (rc) return rc;
  // final RMSNorm fused into the lm head, argmax in its epilogue
  rc = mv(d->tm_lm, d->x, H, d->norm, d->lm_tied ? d->embed_s : d->lm_s, d->keep_logits ? d->logits : nullptr, c.vocab,
          H, c.vocab, MvEpi::Argmax, 5 * c.n_layers);
  MARK(QASR_K_LMHEAD);
  return rc;
}

static int run_graph(qasr_decoder *d, int M) {
  if (int rc = step_upload(d)) return rc;
  if (!d->graphs[M]) {
    cudaGraph_t graph = nullptr;
    int rc = cuda_status(cudaStreamBeginCapture(d->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
    if (rc) return rc;
    int erc = enqueue_step(d, M);
    rc = cuda_status(cudaStreamEndCapture(d->stream, &graph), "end capture");
    if (erc || rc) {
      if (graph) cudaGraphDestroy(graph);
      cudaGetLastError();  // do not leave the capture error sticky for later calls
      return erc ? erc : rc;
    }
    cudaGraphExec_t exec = nullptr;
    rc = cuda_status(cudaGraphInstantiate(&exec, graph, 0), "graph instantiate");
    cudaGraphDestroy(graph);
    if (rc) return rc;
    d->graphs[M] = exec;
  }
  return cuda_status(cudaGraphLaunch(d->graphs[M], d->stream), "graph launch");
}

extern "C" int qasr_decoder_step_device(qasr_decoder *d, const int32_t *tokens, const int32_t *positions, int M,
                                        int32_t *next_tokens) {
  if (!d || !tokens || !positions || !next_tokens || M <= 0 || M > d->cfg.max_batch) {
    set_error("qasr_decoder_step_device: invalid arguments (M=%d)", M);
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  int rc = cuda_status(cudaMemcpyAsync(d->tok, tokens, M * 4, cudaMemcpyDeviceToDevice, d->stream), "tokens");
  if (!rc) rc = cuda_status(cudaMemcpyAsync(d->pos, positions, M * 4, cudaMemcpyDeviceToDevice, d->stream), "pos");
  if (!rc) rc = run_graph(d, M);
  if (!rc) rc = cuda_status(cudaMemcpyAsync(next_tokens, d->next, M * 4, cudaMemcpyDeviceToDevice, d->stream), "next");
  return rc;
}

extern "C" int qasr_decoder_step(qasr_decoder *d, const int32_t *tokens, const int32_t *positions, int M,
                                 int32_t *next_tokens) {
  if (!d || !tokens || !positions || !next_tokens || M <= 0 || M > d->cfg.max_batch) {
    set_error("qasr_decoder_step: invalid arguments (M=%d)", M);
    return QASR_ERR_INVALID;
  }
  for (int m = 0; m < M; ++m) {
    if (tokens[m] < 0 || tokens[m] >= d->cfg.vocab) {
      set_error("qasr_decoder_step: token %d of sequence %d outside [0,%d)", tokens[m], m, d->cfg.vocab);
      return QASR_ERR_INVALID;
    }
    if (positions[m] < 0 || positions[m] >= d->cfg.max_seq) {
      set_error("qasr_decoder_step: position %d of sequence %d outside [0,%d)", positions[m], m, d->cfg.max_seq);
      return QASR_ERR_INVALID;
    }
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  std::memcpy(d->h_tok, tokens, M * 4);
  std::memcpy(d->h_pos, positions, M * 4);
  int rc = cuda_status(cudaMemcpyAsync(d->tok, d->h_tok, M * 4, cudaMemcpyHostToDevice, d->stream), "tokens H2D");
  if (!rc) rc = cuda_status(cudaMemcpyAsync(d->pos, d->h_pos, M * 4, cudaMemcpyHostToDevice, d->stream), "pos H2D");
  if (!rc) rc = run_graph(d, M);
  if (!rc) rc = cuda_status(cudaMemcpyAsync(d->h_next, d->next, M * 4, cudaMemcpyDeviceToHost, d->stream), "D2H");
  if (!rc) rc = cuda_status(cudaMemcpyAsync(d->h_err, d->err, 4, cudaMemcpyDeviceToHost, d->stream), "err D2H");
  if (!rc) rc = cuda_status(cudaStreamSynchronize(d->stream), "qasr_decoder_step");
  if (rc) return rc;
  if (*d->h_err) {
    set_error("qasr_decoder_step: device reported bad input (code %d)", *d->h_err);
    cudaMemsetAsync(d->err, 0, 4, d->stream);
    cudaStreamSynchronize(d->stream);
    return QASR_ERR_INVALID;
  }
  std::memcpy(next_tokens, d->h_next, M * 4);
  return QASR_OK;
}

extern "C" int64_t qasr_decoder_step_bytes(const qasr_decoder *d, const int32_t *positions, int M) {
  if (!d || !positions || M <= 0) return 0;
  const qasr_decoder_config &c = d->cfg;
  const int64_t H = c.hidden, I = c.inter, q_dim = (int64_t)c.n_heads * c.head_dim,
                kv = (int64_t)c.n_kv_heads * c.head_dim;
  const int64_t w_layer = (q_dim + 2 * kv) * H + H * q_dim + 2 * I * H + H * I;
  const int64_t s_layer = 4 * ((q_dim + 2 * kv) + H + 2 * I + H);
  const int64_t n_layer = 4 * (2 * c.head_dim + 2 * H);
  int64_t bytes = c.n_layers * (w_layer + s_layer + n_layer);
  bytes += (int64_t)c.vocab * H + 4 * (int64_t)c.vocab;  // lm head + scales
  for (int m = 0; m < M; ++m) bytes += (int64_t)c.n_layers * 2 * (positions[m] + 1) * kv * 4;
  return bytes;
}

extern "C" int qasr_decoder_profile_step(qasr_decoder *d, const int32_t *tokens, const int32_t *positions, int M,
                                         float *class_ms, int *class_launches, int n_classes) {
  if (!d || !tokens || !positions || !class_ms || M <= 0 || M > d->cfg.max_batch || n_classes < QASR_K_COUNT) {
    set_error("qasr_decoder_profile_step: invalid arguments");
    return QASR_ERR_INVALID;
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  std::memcpy(d->h_tok, tokens, M * 4);
  std::memcpy(d->h_pos, positions, M * 4);
  int rc = cuda_status(cudaMemcpyAsync(d->tok, d->h_tok, M * 4, cudaMemcpyHostToDevice, d->stream), "tokens H2D");
  if (!rc) rc = cuda_status(cudaMemcpyAsync(d->pos, d->h_pos, M * 4, cudaMemcpyHostToDevice, d->stream), "pos H2D");
  if (rc) return rc;
  if ((rc = step_upload(d))) return rc;
  StepMarks marks;
  marks.st = d->stream;
  rc = enqueue_step(d, M, &marks);
  if (!rc) rc = cuda_status(cudaStreamSynchronize(d->stream), "qasr_decoder_profile_step");
  if (rc) return rc;
  for (int i = 0; i < n_classes; ++i) {
    class_ms[i] = 0.0f;
    if (class_launches) class_launches[i] = 0;
  }
  for (size_t i = 1; i < marks.ev.size(); ++i) {
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, marks.ev[i - 1], marks.ev[i]);
    const int c = marks.cls[i];
    if (c >= 0 && c < n_classes) {
      class_ms[c] += ms;
      if (class_launches) class_launches[c] += 1;
    }
  }
  return QASR_OK;
}

// decoder_prefill_int8 (decoder.rs:751-842) for sequence `slot`: the prompt
// rows embeds[0..seq) (host or device, [seq, hidden] f32) at positions
// start_pos.. go through every layer; their K/V rows are written to the
// slot's cache.  The projections run as tensor-core GEMMs over all rows
// (the reference: seq_len matvecs), the norms, RoPE, attention and SwiGLU
// are the kernel-level entries, in the reference's order.
namespace qasr {
// apply_rope_neox with a position per row: x[r, head, :] rotated by the
// table row pos[r] (the arithmetic of apply_rope_kernel).
__global__ void rope_rows_kernel(float *__restrict__ x, const float *__restrict__ cos_tab,
                                 const float *__restrict__ sin_tab, const int32_t *__restrict__ pos, int rows,
                                 int n_heads, int head_dim) {
  const int half = head_dim / 2;
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (long)rows * n_heads * half) return;
  const int dd = (int)(t % half);
  const long sh = t / half;
  const int r = (int)(sh / n_heads);
  float *vec = x + sh * head_dim;
  const float *c = cos_tab + (size_t)pos[r] * head_dim, *sn = sin_tab + (size_t)pos[r] * head_dim;
  const float x1 = vec[dd], x2 = vec[half + dd];
  vec[dd] = __fadd_rn(__fmul_rn(x1, c[dd]), __fmul_rn(-x2, sn[dd]));
  vec[half + dd] = __fadd_rn(__fmul_rn(x2, c[half + dd]), __fmul_rn(x1, sn[half + dd]));
}

// KV append with a destination per row: row r of k/v goes to cache row
// (layer * max_seq + pos[r]) of sequence slot[r].
__global__ void kv_append_rows_kernel(float *__restrict__ k_cache, float *__restrict__ v_cache,
                                      const float *__restrict__ k_new, const float *__restrict__ v_new,
                                      const int32_t *__restrict__ slot, const int32_t *__restrict__ pos, int rows,
                                      int layer, int max_seq, int kv_dim, long seq_stride) {
  const long t = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const int per_row = kv_dim / 4;
  if (t >= (long)rows * per_row) return;
  const int r = (int)(t / per_row), c = (int)(t % per_row);
  const size_t dst = (size_t)slot[r] * seq_stride + ((size_t)layer * max_seq + pos[r]) * kv_dim;
  reinterpret_cast<float4 *>(k_cache + dst)[c] = reinterpret_cast<const float4 *>(k_new + (size_t)r * kv_dim)[c];
  reinterpret_cast<float4 *>(v_cache + dst)[c] = reinterpret_cast<const float4 *>(v_new + (size_t)r * kv_dim)[c];
}
}  // namespace qasr

// decoder_prefill_int8 (decoder.rs:751-842) for n sequences at once: their
// prompt rows are concatenated, every per-row operation (norms, the q|k|v,
// o, gate/up and down GEMMs with their fused epilogues, SwiGLU) runs once over
// all rows, RoPE and the KV append take each row's position and slot, and
// one causal-attention launch covers every sequence (grid z).  Sequence i's
// cache ends up exactly as a prefill of it alone would leave it.
extern "C" int qasr_decoder_prefill_batch(qasr_decoder *d, const int *slots, const float *const *embeds,
                                          const int *seqs, const int *start_pos, int n) {
  if (!d || !slots || !embeds || !seqs || !start_pos || n <= 0 || n > d->cfg.max_batch) {
    set_error("qasr_decoder_prefill: invalid arguments");
    return QASR_ERR_INVALID;
  }
  const qasr_decoder_config &c = d->cfg;
  int R = 0, max_seq_q = 0;
  for (int i = 0; i < n; ++i) {
    if (!embeds[i] || slots[i] < 0 || slots[i] >= c.max_batch || seqs[i] <= 0 || start_pos[i] < 0) {
      set_error("qasr_decoder_prefill: invalid arguments (sequence %d)", i);
      return QASR_ERR_INVALID;
    }
    if (start_pos[i] + seqs[i] > c.max_seq) {
      set_error("qasr_decoder_prefill: positions %d..%d outside the cache (max_seq %d)", start_pos[i],
                start_pos[i] + seqs[i] - 1, c.max_seq);
      return QASR_ERR_INVALID;
    }
    for (int j = 0; j < i; ++j)
      if (slots[j] == slots[i]) {
        set_error("qasr_decoder_prefill: slot %d given twice", slots[i]);
        return QASR_ERR_INVALID;
      }
    R += seqs[i];
    max_seq_q = std::max(max_seq_q, seqs[i]);
  }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  cudaStream_t st = d->stream;
  const int H = c.hidden, I = c.inter, hd = c.head_dim;
  const int q_dim = c.n_heads * hd, kv_dim = c.n_kv_heads * hd;
  int rc = QASR_OK;
  // buffers: activations for R rows, then per-row positions / slots and the segment table
  const size_t per_row = (size_t)2 * H + 2 * q_dim + 2 * kv_dim + H + 2 * I + I;
  const size_t meta_bytes = (size_t)2 * R * 4 + (size_t)n * sizeof(CaSeg) + 256;
  if (R > d->pf_cap || meta_bytes > d->pf_meta_cap) {
    const int cap = std::max(R, 64);
    void *blk = nullptr;
    if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_decoder_prefill"))) return rc;
    const size_t meta = std::max(meta_bytes, (size_t)2 * cap * 4 + (size_t)c.max_batch * sizeof(CaSeg) + 256);
    if ((rc = cuda_status(cudaMalloc(&blk, per_row * cap * 4 + meta), "qasr_decoder_prefill: buffers"))) return rc;
    if (d->pf_block) cudaFree(d->pf_block);
    d->pf_block = blk;
    float *f = static_cast<float *>(blk);
    auto take = [&](size_t k) { float *r = f; f += k * cap; return r; };
    d->pf_x = take(H);
    d->pf_xn = take(H);
    d->pf_q = take(q_dim);
    d->pf_attn = take(q_dim);
    d->pf_k = take(kv_dim);
    d->pf_v = take(kv_dim);
    d->pf_proj = take(H);
    d->pf_gu = take(2 * I);
    d->pf_h = take(I);
    d->pf_meta = reinterpret_cast<unsigned char *>(f);
    d->pf_cap = cap;
    d->pf_meta_cap = meta;
  }
  // host tables -> device: row positions and slots, then the attention segments
  std::vector<int32_t> row_pos(R), row_slot(R);
  std::vector<CaSeg> segs(n);
  const long seq_stride = d->seq_stride();
  for (int i = 0, r0 = 0; i < n; r0 += seqs[i], ++i) {
    for (int j = 0; j < seqs[i]; ++j) {
      row_pos[r0 + j] = start_pos[i] + j;
      row_slot[r0 + j] = slots[i];
    }
    segs[i] = CaSeg{r0, seqs[i], start_pos[i] + seqs[i], start_pos[i], (long)slots[i] * seq_stride};
  }
  int32_t *d_pos = reinterpret_cast<int32_t *>(d->pf_meta), *d_slot = d_pos + R;
  CaSeg *d_segs = reinterpret_cast<CaSeg *>(d->pf_meta + ((2 * (size_t)R * 4 + 15) & ~(size_t)15));
  rc = cuda_status(cudaMemcpyAsync(d_pos, row_pos.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st), "prefill meta");
  if (!rc)
    rc = cuda_status(cudaMemcpyAsync(d_slot, row_slot.data(), (size_t)R * 4, cudaMemcpyHostToDevice, st),
                     "prefill meta");
  if (!rc)
    rc = cuda_status(cudaMemcpyAsync(d_segs, segs.data(), (size_t)n * sizeof(CaSeg), cudaMemcpyHostToDevice, st),
                     "prefill meta");
  for (int i = 0, r0 = 0; i < n && !rc; r0 += seqs[i], ++i)
    rc = cuda_status(cudaMemcpyAsync(d->pf_x + (size_t)r0 * H, embeds[i], (size_t)seqs[i] * H * 4, cudaMemcpyDefault,
                                     st),
                     "prefill embeds");
  if (rc) return rc;
  const float scale = 1.0f / sqrtf((float)hd);
  const long nq = (long)R * c.n_heads * (hd / 2), nk = (long)R * c.n_kv_heads * (hd / 2);
  const long nkv = (long)R * (kv_dim / 4);
  for (int l = 0; l < c.n_layers && !rc; ++l) {
    const LayerDev &L = d->layers[l];
    const size_t kv_rows = (size_t)kv_dim * H;
    if ((rc = qasr_rms_norm(d->pf_xn, d->pf_x, L.in_norm, R, H, c.eps, st))) break;
    // q, k, v: the three row ranges of the fused q|k|v matrix, one GEMM when
    // the tensor-core path takes it (more than 8 rows), else three matvec calls
    rc = R > 8 ? int8_gemm_split3(d->pf_q, q_dim, d->pf_k, kv_dim, q_dim, d->pf_v, kv_dim, q_dim + kv_dim, d->pf_xn, H,
                                  L.wqkv, L.sqkv, R, H, q_dim + 2 * kv_dim, st)
               : QASR_ERR_UNSUPPORTED;
    if (rc == QASR_ERR_UNSUPPORTED) {
      if ((rc = qasr_linear_nobias_int8(d->pf_q, d->pf_xn, L.wqkv, L.sqkv, R, H, q_dim, st))) break;
      if ((rc = qasr_linear_nobias_int8(d->pf_k, d->pf_xn, L.wqkv + (size_t)q_dim * H, L.sqkv + q_dim, R, H, kv_dim,
                                        st)))
        break;
      if ((rc = qasr_linear_nobias_int8(d->pf_v, d->pf_xn, L.wqkv + (size_t)q_dim * H + kv_rows,
                                        L.sqkv + q_dim + kv_dim, R, H, kv_dim, st)))
        break;
    } else if (rc) {
      break;
    }
    if ((rc = qasr_rms_norm_per_head(d->pf_q, L.q_norm, R, c.n_heads, hd, c.eps, st))) break;
    if ((rc = qasr_rms_norm_per_head(d->pf_k, L.k_norm, R, c.n_kv_heads, hd, c.eps, st))) break;
    rope_rows_kernel<<<(int)((nq + 255) / 256), 256, 0, st>>>(d->pf_q, d->rope_cos, d->rope_sin, d_pos, R, c.n_heads,
                                                              hd);
    rope_rows_kernel<<<(int)((nk + 255) / 256), 256, 0, st>>>(d->pf_k, d->rope_cos, d->rope_sin, d_pos, R,
                                                              c.n_kv_heads, hd);
    kv_append_rows_kernel<<<(int)((nkv + 255) / 256), 256, 0, st>>>(d->k_cache, d->v_cache, d->pf_k, d->pf_v, d_slot,
                                                                    d_pos, R, l, c.max_seq, kv_dim, seq_stride);
    if ((rc = launch_status("qasr_decoder_prefill: rope / kv append"))) break;
    // causal attention of every sequence over its cache (layer l)
    const size_t lay = (size_t)l * c.max_seq * kv_dim;
    if ((rc = causal_attention_segments(d->pf_attn, d->pf_q, d->k_cache + lay, d->v_cache + lay, d_segs, n, max_seq_q,
                                        c.n_heads, c.n_kv_heads, hd, scale, st)))
      break;
    // o-proj + residual, gate/up + SwiGLU, down + residual: fused GEMM
    // epilogues when the tensor-core GEMM takes the shape (more than 8 rows)
    const bool fused = R > 8;
    rc = fused ? int8_gemm_epi(d->pf_x, H, d->pf_attn, q_dim, L.wo, L.so, R, q_dim, H, 1, st) : QASR_ERR_UNSUPPORTED;
    if (rc == QASR_ERR_UNSUPPORTED) {
      if ((rc = qasr_linear_nobias_int8(d->pf_proj, d->pf_attn, L.wo, L.so, R, q_dim, H, st))) break;
      if ((rc = qasr_add_inplace(d->pf_x, d->pf_proj, (int64_t)R * H, st))) break;
    } else if (rc) {
      break;
    }
    if ((rc = qasr_rms_norm(d->pf_xn, d->pf_x, L.post_norm, R, H, c.eps, st))) break;
    rc = fused ? int8_gemm_epi(d->pf_h, I, d->pf_xn, H, L.gate_up, L.sgu, R, H, 2 * I, 2, st) : QASR_ERR_UNSUPPORTED;
    if (rc == QASR_ERR_UNSUPPORTED) {
      if ((rc = qasr_linear_nobias_int8(d->pf_gu, d->pf_xn, L.gate_up, L.sgu, R, H, 2 * I, st))) break;
      if ((rc = qasr_swiglu_multiply(d->pf_h, d->pf_gu, R, I, st))) break;
    } else if (rc) {
      break;
    }
    rc = fused ? int8_gemm_epi(d->pf_x, H, d->pf_h, I, L.down, L.sdown, R, I, H, 1, st) : QASR_ERR_UNSUPPORTED;
    if (rc == QASR_ERR_UNSUPPORTED) {
      if ((rc = qasr_linear_nobias_int8(d->pf_proj, d->pf_h, L.down, L.sdown, R, I, H, st))) break;
      if ((rc = qasr_add_inplace(d->pf_x, d->pf_proj, (int64_t)R * H, st))) break;
    } else if (rc) {
      break;
    }
  }
  if (!rc) rc = cuda_status(cudaStreamSynchronize(st), "qasr_decoder_prefill");
  return rc;
}

extern "C" int qasr_decoder_prefill(qasr_decoder *d, int slot, const float *embeds, int seq, int start_pos) {
  return qasr_decoder_prefill_batch(d, &slot, &embeds, &seq, &start_pos, 1);
}

extern "C" const qasr_decoder_config *qasr_decoder_get_config(const qasr_decoder *d) { return d ? &d->cfg : nullptr; }
extern "C" int qasr_decoder_device(const qasr_decoder *d) { return d ? d->device : -1; }

qasr::ScratchArena *qasr::decoder_arena(qasr_decoder *d) { return d ? d->arena : nullptr; }

// QwenCtx::tok_embed_to_f32 (context.rs:115-124) for n host ids: rows of the
// engine's embedding table (dequantised when INT8) into out [n, hidden].
extern "C" int qasr_decoder_embed(qasr_decoder *d, const int32_t *ids, int n, float *out) {
  if (!d || !ids || !out || n <= 0) {
    set_error("qasr_decoder_embed: invalid arguments");
    return QASR_ERR_INVALID;
  }
  if (!d->globals_ready) {
    set_error("qasr_decoder_embed: qasr_decoder_set_globals has not succeeded");
    return QASR_ERR_INVALID;
  }
  const qasr_decoder_config &c = d->cfg;
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= c.vocab) {
      set_error("qasr_decoder_embed: id %d (index %d) outside [0,%d)", ids[i], i, c.vocab);
      return QASR_ERR_INVALID;
    }
  cudaSetDevice(d->device);
  qasr::ArenaScope arena_scope(d->arena);
  cudaStream_t st = d->stream;
  int rc = QASR_OK;
  if (n > d->emb_cap) {
    if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_decoder_embed"))) return rc;
    if (d->emb_ids) cudaFree(d->emb_ids);
    d->emb_ids = nullptr;
    d->emb_cap = 0;
    if ((rc = cuda_status(cudaMalloc(&d->emb_ids, (size_t)std::max(n, 64) * 4), "qasr_decoder_embed: ids"))) return rc;
    d->emb_cap = std::max(n, 64);
  }
  if ((rc = cuda_status(cudaMemcpyAsync(d->emb_ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, st), "embed ids")))
    return rc;
  step_embed_kernel<<<n, 256, 0, st>>>(out, d->embed, d->embed_s, c.embed_is_int8, d->emb_ids, c.hidden, c.vocab,
                                       d->err);
  if ((rc = launch_status("qasr_decoder_embed"))) return rc;
  return cuda_status(cudaStreamSynchronize(st), "qasr_decoder_embed");
}

// Residual stream after the last prefill (device, [seq, hidden]); NULL before one.
extern "C" const float *qasr_decoder_prefill_hidden(qasr_decoder *d) { return d ? d->pf_x : nullptr; }
