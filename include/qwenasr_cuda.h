/*
 * qwenasr_cuda.h -- C ABI of the B200 (sm_100a) kernel library for the
 * QwenASR per-layer hot path.
 *
 * Two layers of entry points:
 *
 *  1. Kernel level.  One function per function of the reference's kernel
 *     module (crates/qwen-asr/src/kernels/mod.rs), same argument order and
 *     meaning, with device pointers and an explicit CUDA stream appended
 *     (`stream` is a cudaStream_t; NULL = the legacy default stream).  The
 *     reference functions mutate slices in place where these do, and return
 *     nothing; here every function returns a status (QASR_OK or a negative
 *     QASR_ERR_*), with a message in qasr_last_error().  Fused entries
 *     (qasr_pre_attn_block, qasr_ln_pe, ...) replace a sequence of reference
 *     calls and name the sequence.
 *
 *  2. Decoder engine.  An opaque qasr_decoder owning INT8 decoder weights on
 *     one GPU, KV caches for a batch of independent sequences and the
 *     captured decode-step graph: the device counterpart of DecoderInt8 +
 *     KvCache + RopeCache + decoder_forward_int8 (crates/qwen-asr/src/
 *     decoder.rs:130-306, 652-965), driven by QwenCtx::decoder_forward_token
 *     (context.rs:311) in the reference.
 *
 * Layouts are the reference's: row-major f32 activations [rows, cols]; INT8
 * weights row-major [out, in] with f32 per-row scales [out]
 * (quantize.rs:78-84); the fused gate/up weight with rows interleaved
 * g0,u0,g1,u1,... (decoder.rs:699-719); KV cache per sequence
 * [n_layers, max_seq, kv_dim] f32 with row (layer*max_seq + pos)
 * (decoder.rs:194-202); RoPE tables [pos, head_dim] with duplicated halves
 * (decoder.rs:253-289).
 *
 * Thread safety: entry points may be called from several host threads on
 * distinct streams/engines; one qasr_decoder must not be driven from two
 * threads at once.
 */
#ifndef QWENASR_CUDA_H
#define QWENASR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden default visibility; everything declared
 * here is exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

#define QASR_OK 0
#define QASR_ERR_INVALID (-1)     /* null pointer, bad shape or out-of-range id */
#define QASR_ERR_CUDA (-2)        /* a CUDA call or kernel launch failed */
#define QASR_ERR_ALLOC (-3)       /* device allocation failed */
#define QASR_ERR_UNSUPPORTED (-4) /* shape outside what a specialised kernel handles */
#define QASR_ERR_TIMEOUT (-5)     /* a bounded device-side wait gave up */

/* Message of the last failing call on this host thread ("" if none). */
const char *qasr_last_error(void);
/* Library version string. */
const char *qasr_version(void);

/* ======================================================================
 * Kernel level (device pointers)
 * ==================================================================== */

/* kernels::rms_norm (mod.rs:897-918; x86 row kernel avx::rms_norm_row,
 * avx.rs:377-415).  out[s,:] = x[s,:] * (1/sqrt(sum(x^2)/hidden + eps)) * w.
 * Bit-exact with the reference's x86_64 path (same summation tree). */
int qasr_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps, void *stream);

/* kernels::rms_norm_per_head (mod.rs:920-935), in place.  Bit-exact
 * (sequential per-head sum, as in the reference). */
int qasr_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim, float eps, void *stream);

/* kernels::layer_norm (mod.rs:866-895; avx::layer_norm_row avx.rs:420-481).
 * Bit-exact with the x86_64 path. */
int qasr_layer_norm(float *out, const float *x, const float *w, const float *b, int seq, int hidden, float eps,
                    void *stream);

/* kernels::compute_rope_neox (mod.rs:1228-1245): cos/sin [seq, head_dim]
 * for the given positions (halves duplicated). */
int qasr_compute_rope_neox(float *cos_out, float *sin_out, const int32_t *positions, int seq, int head_dim,
                           float theta, void *stream);

/* RopeCache::ensure (decoder.rs:253-289): table rows 0..n_pos-1. */
int qasr_rope_cache_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta, void *stream);

/* kernels::apply_rope_neox (mod.rs:1247-1267), in place; cos_v/sin_v are
 * [seq, head_dim].  Bit-exact. */
int qasr_apply_rope_neox(float *x, const float *cos_v, const float *sin_v, int seq, int n_heads, int head_dim,
                         void *stream);

/* KvCache::k_at / v_at copies (decoder.rs:194-202, calls at 805-810 and
 * 894-895): rows k_new[s], v_new[s] -> cache row (layer*max_seq + start_pos + s).
 * Bit-exact (a copy).  Fails with QASR_ERR_INVALID when start_pos+seq > max_seq. */
int qasr_kv_append(float *k_cache, float *v_cache, const float *k_new, const float *v_new, int layer,
                   int max_seq, int kv_dim, int start_pos, int seq, void *stream);

/* kernels::sinusoidal_pe (mod.rs:1213-1226): pe [n_pos, d_model]. */
int qasr_sinusoidal_pe(float *pe, int n_pos, int d_model, void *stream);

/* kernels::gelu (mod.rs:948-963; avx::gelu_inplace avx.rs:536-563): the
 * tanh form with the reference's fast exp, in place.  Bit-exact on the
 * 8-aligned body; the last n%8 elements use tanhf like the reference tail. */
int qasr_gelu(float *x, int64_t n, void *stream);

/* Exact-erf GELU 0.5*x*(1+erf(x/sqrt(2))), in place: the encoder activation
 * of the reference's Metal encoder (encoder_gpu.rs:470,480). */
int qasr_gelu_erf(float *x, int64_t n, void *stream);

/* kernels::silu (mod.rs:941-946), in place. */
int qasr_silu(float *x, int64_t n, void *stream);

/* kernels::swiglu_multiply (mod.rs:965-985; avx::swiglu_interleaved
 * avx.rs:568-599): out[s,j] = silu(gu[s,2j]) * gu[s,2j+1].  Bit-exact on the
 * 8-aligned body (reference fast exp); tail uses expf. */
int qasr_swiglu_multiply(float *out, const float *gate_up, int seq, int inter, void *stream);

/* kernels::add_inplace (mod.rs:482-484). */
int qasr_add_inplace(float *a, const float *b, int64_t n, void *stream);

/* kernels::linear_nobias_int8 (mod.rs:650-661; generic::int8_matvec_fused
 * generic.rs:39-49): y[s,o] = scales[o] * sum_k w[o,k]*x[s,k].  Any seq: up
 * to 8 rows as a weight-streaming tensor-core contraction, more as one
 * tensor-core GEMM over all rows (the reference runs seq matvecs). */
int qasr_linear_nobias_int8(float *y, const float *x, const int8_t *w, const float *scales, int seq, int in_dim,
                            int out_dim, void *stream);

/* kernels::linear_int8 (mod.rs:664-673): as above plus bias[o] (may be NULL). */
int qasr_linear_int8(float *y, const float *x, const int8_t *w, const float *scales, const float *bias, int seq,
                     int in_dim, int out_dim, void *stream);

/* kernels::linear (mod.rs:531-565; cblas_sgemm in the reference):
 * y[s,o] = sum_k x[s,k]*w[o,k] + b[o] (b may be NULL), f32 weights [out, in].
 * Tensor cores for in_dim % 16 == 0, in_dim >= 128, out_dim >= 128 (each
 * operand as three exact int8 digit planes); a CUDA-core kernel otherwise. */
int qasr_linear(float *y, const float *x, const float *w, const float *b, int seq, int in_dim, int out_dim,
                void *stream);

/* kernels::linear_nobias (mod.rs:567-568). */
int qasr_linear_nobias(float *y, const float *x, const float *w, int seq, int in_dim, int out_dim, void *stream);

/* kernels::matmul_t (mod.rs:503-528): c[m,n] = sum_k a[m,k]*b[n,k]. */
int qasr_matmul_t(float *c, const float *a, const float *b, int m, int k, int n, void *stream);

/* kernels::conv2d (mod.rs:790-860): out [c_out, h_out*w_out] = weight
 * [c_out, c_in*kh*kw] x im2col(input [c_in, h_in, w_in]) + bias[c_out] (bias
 * may be NULL); h_out = (h_in + 2*padding - kh)/stride + 1, same for w.  The
 * product runs as the tensor-core f32 GEMM when c_in*kh*kw and the output
 * size allow (see qasr_linear), on CUDA cores otherwise. */
int qasr_conv2d(float *out, const float *input, const float *weight, const float *bias, int c_in, int c_out,
                int h_in, int w_in, int kh, int kw, int stride, int padding, void *stream);

/* kernels::bidirectional_attention (mod.rs:1038-1122): full attention inside
 * windows [window_starts[w], window_starts[w+1]) (device int32 array of
 * n_windows+1 increasing entries, the last = seq), q/k/v/out [seq,
 * n_heads*head_dim]; head_dim 64 or 128. */
int qasr_bidirectional_attention(float *out, const float *q, const float *k, const float *v, int seq, int n_heads,
                                 int head_dim, float scale, const int32_t *window_starts, int n_windows,
                                 void *stream);

/* audio::mel_spectrogram (audio.rs:271-385): frames for n_samples 16 kHz
 * samples (n_samples / 160; 0 = too short, where the reference returns None). */
int qasr_mel_frames(int n_samples);
/* mel [128, n_frames] (device) = normalised log-mel of samples [n_samples]
 * (device): reflect padding of 200, periodic Hann window, 400-point DFT, hop
 * 160, last frame dropped, 128 Slaney mel bins, log10 with a 1e-10 floor,
 * clamped at the global max - 8, then (v + 4) / 4.  The power spectrum and
 * the mel sums follow the reference's f32 operation order exactly; log10 is
 * correctly rounded (glibc's log10f is within one ulp of it).  The constant
 * tables are uploaded on the first call per device (do not make that call
 * under stream capture). */
int qasr_mel_spectrogram(float *mel, const float *samples, int n_samples, void *stream);

/* kernels::causal_attention (mod.rs:1124-1207): GQA causal attention of
 * seq_q queries at global positions q_offset.. over k/v [seq_k, n_kv*hd].
 * head_dim must be 64 or 128. */
int qasr_causal_attention(float *out, const float *q, const float *k, const float *v, int seq_q, int seq_k,
                          int n_heads, int n_kv_heads, int head_dim, float scale, int q_offset, void *stream);

/* quantize_f32_to_int8 (quantize.rs:633-662): symmetric per-row INT8,
 * scale = absmax/127, q = round-half-away(v*127/absmax) clamped.  Bit-exact. */
int qasr_quantize_f32_to_int8(const float *data, int64_t out_dim, int64_t in_dim, int8_t *q, float *scales,
                              void *stream);

/* Embedding gather: dst[i,:] = table[ids[i],:] (f32 table, BASELINE decode
 * config) -- bit-exact copy.  Ids outside [0,vocab) set *bad_id_flag (device
 * int, may be NULL) and produce a zero row. */
int qasr_embed_gather_f32(float *dst, const float *table, const int32_t *ids, int n, int dim, int64_t vocab,
                          int *bad_id_flag, void *stream);

/* tok_embed_int8_to_f32 (decoder.rs:639-646) for n ids: dst[i,d] =
 * f32(table[id,d]) * scales[id].  Bit-exact. */
int qasr_embed_gather_int8(float *dst, const int8_t *table, const float *scales, const int32_t *ids, int n, int dim,
                           int64_t vocab, int *bad_id_flag, void *stream);

/* ---------------------------------------------------------------- fused */

/* The decoder pre-attention block of decoder_prefill_int8
 * (decoder.rs:770-810) on given projections:
 *   x_norm = rms_norm(x, w_in)                              (mod.rs:897)
 *   q, k   = rms_norm_per_head(q|k, q_norm_w|k_norm_w)      (mod.rs:920)
 *   q, k   = apply_rope_neox(q|k, cos/sin rows start_pos..) (mod.rs:1247)
 *   cache rows start_pos.. of layer `layer` <- k, v         (decoder.rs:805-810)
 * q is rotated in place; k_out (may be NULL) receives the rotated k.
 * cos_tab/sin_tab are full RopeCache tables (row = position).  Bit-exact.
 * Shapes: head_dim 128, hidden <= 2048, n_heads + n_kv_heads <= 24 with
 * n_kv_heads <= 8 (the published models); others return
 * QASR_ERR_UNSUPPORTED. */
int qasr_pre_attn_block(float *x_norm, const float *x, const float *w_in, int seq, int hidden, float *q,
                        const float *k, const float *v, float *k_out, const float *q_norm_w, const float *k_norm_w,
                        int n_heads, int n_kv_heads, int head_dim, float eps, const float *cos_tab,
                        const float *sin_tab, int start_pos, float *k_cache, float *v_cache, int layer,
                        int max_seq, void *stream);

/* Encoder LayerNorm + sinusoidal position add: out[r,:] =
 * layer_norm(x[r,:]) + pe[r % n_pos, :]  (layer_norm mod.rs:866 bit-exact,
 * then the add of encoder.rs:341-343).  pe is [n_pos, hidden]. */
int qasr_ln_pe(float *out, const float *x, const float *w, const float *b, const float *pe, int rows, int hidden,
               int n_pos, float eps, void *stream);

/* The encoder's elementwise steps in one launch (the ln_pe_gelu entry of the
 * fused family): out = qasr_ln_pe(x) as above, and exact-erf GELU in place on
 * act [n_act] (the FFN activation; qasr_gelu_erf's arithmetic).  Replaces
 * layer_norm (mod.rs:866) + the PE add (encoder.rs:341-343) + gelu
 * (mod.rs:948) of a config-2 pass; both results are bit-identical to the
 * separate entries.  act 16-byte aligned; n_act may be 0. */
int qasr_ln_pe_gelu_erf(float *out, const float *x, const float *w, const float *b, const float *pe, int rows,
                        int hidden, int n_pos, float eps, float *act, int64_t n_act, void *stream);

/* Post-attention RMSNorm + fused gate/up INT8 matvec + SwiGLU for M tokens
 * (decoder.rs:911-921): h[m,j] = silu(g)*u with g,u the interleaved rows
 * 2j, 2j+1 of w_gate_up applied to rms_norm(x[m]).  M <= 8. */
int qasr_int8_norm_gateup_swiglu(float *h, const float *x, const float *norm_w, const int8_t *w_gate_up,
                                 const float *scales, int M, int hidden, int inter, float eps, void *stream);

/* INT8 matvec with the residual add folded in (decoder.rs:907-908 and
 * 922-924): x[m,o] += scales[o] * sum_k w[o,k]*a[m,k].  M <= 8. */
int qasr_int8_matvec_residual(float *x, const float *a, const int8_t *w, const float *scales, int M, int in_dim,
                              int out_dim, void *stream);

/* Final RMSNorm + INT8 lm-head + first-max argmax (decoder.rs:929-964) for
 * M tokens: ids_out[m] = argmax_o scales[o]*dot(w[o], rms_norm(x[m])).
 * logits_out [M, vocab] may be NULL.  M <= 8. */
int qasr_final_norm_lmhead_argmax(int32_t *ids_out, float *logits_out, const float *x, const float *norm_w,
                                  const int8_t *w, const float *scales, int M, int hidden, int vocab, float eps,
                                  void *stream);

/* Same result as qasr_final_norm_lmhead_argmax, but the call allocates no
 * device memory.  No counterpart in the reference (its CPU path has no device
 * allocations to avoid).  For hosts that may not allocate once serving has
 * started: a runtime with its own pool or a hard memory budget.  The argmax
 * scratch is a fixed 256-byte array in the library; its device address is
 * looked up on the first call on each device (make that first call before any
 * stream capture), and every call clears it with a 256-byte memset on
 * `stream` before its kernel.  Limits: M <= 8, hidden a multiple of 512 and
 * <= 3072, x / w / norm_w 16-byte aligned; larger M returns QASR_ERR_INVALID,
 * other shapes QASR_ERR_UNSUPPORTED.  If a bounded device-side wait gives
 * up, every id of the call is -1.  The scratch is shared by all calls on one
 * device, so calls that overlap in time on one device race and must be
 * serialised. */
int qasr_final_norm_lmhead_argmax_noalloc(int32_t *ids_out, float *logits_out, const float *x, const float *norm_w,
                                          const int8_t *w, const float *scales, int M, int hidden, int vocab,
                                          float eps, void *stream);

/* ======================================================================
 * Decoder engine
 * ==================================================================== */

typedef struct qasr_decoder qasr_decoder;

typedef struct {
  int hidden;     /* 1024 (0.6B) / 2048 (1.7B) */
  int inter;      /* 3072 / 6144 */
  int n_layers;   /* 28 */
  int n_heads;    /* 16 */
  int n_kv_heads; /* 8 */
  int head_dim;   /* 128 */
  int vocab;      /* 151936 */
  float eps;      /* 1e-6 */
  float theta;    /* 1e6 */
  int max_batch;  /* sequences decoded together, 1..8 */
  int max_seq;    /* KV capacity per sequence */
  int embed_is_int8; /* 1: INT8 token table + scales (qint8 V2), 0: f32 table */
} qasr_decoder_config;

/* One decoder layer's weights, host or device pointers (copied). */
typedef struct {
  const int8_t *wq; const float *wq_s;        /* [n_heads*hd, hidden] */
  const int8_t *wk; const float *wk_s;        /* [n_kv*hd, hidden] */
  const int8_t *wv; const float *wv_s;        /* [n_kv*hd, hidden] */
  const int8_t *wo; const float *wo_s;        /* [hidden, n_heads*hd] */
  const int8_t *gate_up; const float *gate_up_s; /* [2*inter, hidden], interleaved rows */
  const int8_t *down; const float *down_s;    /* [hidden, inter] */
  const float *q_norm; const float *k_norm;   /* [hd] */
  const float *input_norm; const float *post_attn_norm; /* [hidden] */
} qasr_dec_layer_weights;

/* DecoderInt8 + KvCache allocation on `device` (decoder.rs:652-747,140-150).
 * Returns NULL on failure (message in qasr_last_error()). */
qasr_decoder *qasr_decoder_create(const qasr_decoder_config *cfg, int device);
void qasr_decoder_free(qasr_decoder *dec);

/* Upload weights (host or device pointers; copied). */
int qasr_decoder_set_layer(qasr_decoder *dec, int layer, const qasr_dec_layer_weights *w);
/* DecoderInt8::load's gate/up fusion (decoder.rs:699-719) on the device:
 * gate and up [inter, hidden] INT8 (host or device) with their scales,
 * interleaved g0,u0,g1,u1,... into layer `layer`'s fused matrix.  For this,
 * qasr_decoder_set_layer may be given gate_up = gate_up_s = NULL. */
int qasr_decoder_set_gate_up(qasr_decoder *dec, int layer, const int8_t *gate, const float *gate_s, const int8_t *up,
                             const float *up_s);
/* embed: f32 [vocab, hidden] or int8 [vocab, hidden] (+ embed_scales);
 * final norm [hidden]; lm_head int8 [vocab, hidden] + scales.  When lm_head
 * is NULL the lm head is tied to the INT8 embedding table (decoder.rs:950-963). */
int qasr_decoder_set_globals(qasr_decoder *dec, const void *embed, const float *embed_scales, const float *norm,
                             const int8_t *lm_head, const float *lm_head_s);

/* Device pointers of sequence `slot`'s KV cache, [n_layers, max_seq, kv_dim]. */
int qasr_decoder_kv(qasr_decoder *dec, int slot, float **k_cache, float **v_cache);

/* One greedy decode step for sequences 0..M-1 (decoder_forward_int8,
 * decoder.rs:845-965, per sequence): token ids and positions in, next ids
 * out, all HOST buffers.  Sequence m embeds tokens[m], writes its K/V at
 * row positions[m] of its cache and attends over rows 0..positions[m]. */
int qasr_decoder_step(qasr_decoder *dec, const int32_t *tokens, const int32_t *positions, int M, int32_t *next_tokens);

/* decoder_prefill_int8 (decoder.rs:751-842) for sequence `slot`: the prompt
 * rows embeds [seq, hidden] f32 (host or device pointer) at positions
 * start_pos .. start_pos+seq-1 run through every layer and their K/V rows
 * are written to the slot's cache (KvCache with len = start_pos).  The next
 * decode step for the slot is at position start_pos + seq.  Synchronous. */
int qasr_decoder_prefill(qasr_decoder *dec, int slot, const float *embeds, int seq, int start_pos);
/* decoder_prefill_int8 for n sequences at once (distinct slots): their rows
 * go through the layers together, each with its own positions, slot and
 * causal attention; every slot's cache ends up as a prefill of it alone
 * would leave it.  embeds[i] [seqs[i], hidden] host or device.  Synchronous. */
int qasr_decoder_prefill_batch(qasr_decoder *dec, const int *slots, const float *const *embeds, const int *seqs,
                               const int *start_pos, int n);

/* Device pointer to the residual stream [seq, hidden] left by the last
 * prefill (the reference's bufs.pref_x); NULL before the first prefill. */
const float *qasr_decoder_prefill_hidden(qasr_decoder *dec);

/* Same step on DEVICE buffers, enqueued on the engine's stream without a
 * host synchronisation; next_tokens may alias tokens. */
int qasr_decoder_step_device(qasr_decoder *dec, const int32_t *tokens, const int32_t *positions, int M,
                             int32_t *next_tokens);

/* The engine's CUDA stream (cudaStream_t) and, after a step, the device
 * pointer of the last step's logits [M, vocab] (NULL unless enabled). */
void *qasr_decoder_stream(qasr_decoder *dec);
/* The configuration and device the engine was created with (NULL / -1 for NULL). */
const qasr_decoder_config *qasr_decoder_get_config(const qasr_decoder *dec);
int qasr_decoder_device(const qasr_decoder *dec);
/* QwenCtx::tok_embed_to_f32 (context.rs:115-124) for n host ids: rows of
 * the engine's embedding table (dequantised when INT8) into out [n, hidden]
 * (device).  Ids outside [0, vocab) are rejected.  Synchronous. */
int qasr_decoder_embed(qasr_decoder *dec, const int32_t *ids, int n, float *out);
int qasr_decoder_keep_logits(qasr_decoder *dec, int enable);
const float *qasr_decoder_logits(qasr_decoder *dec);

/* How the engine runs a decode step.  mode 1 (the default): per-layer
 * kernels (5 launches per layer, replayed as one CUDA graph with
 * programmatic dependent launch); mode 0: one persistent kernel for the whole
 * step (every layer, the lm head and the argmax) on every SM, wherever it
 * covers the shape (up to 8 sequences, 2 query heads per kv head, hidden <=
 * 2048), else the per-layer kernels.  Same results within the parity bars.
 * No counterpart in the reference (a CPU engine has no launches to fuse). */
int qasr_decoder_set_step_kernel(qasr_decoder *dec, int mode);
/* 0 if a step of M sequences runs as the persistent kernel, 1 if it runs as
 * per-layer kernels, -1 for bad arguments. */
int qasr_decoder_step_kernel(const qasr_decoder *dec, int M);
/* In-step timeline of the decode step (for profiling; no counterpart in the
 * reference).  While `stamps` (device memory, n values) is set, every step
 * writes %globaltimer stamps (ns):
 *  - per-layer kernels (step kernel mode 1): launch i = 5*layer + {0 q|k|v,
 *    1 attention, 2 o-proj, 3 gate/up, 4 down}, i = 5*n_layers the lm head;
 *    stamps[2i] = the earliest CTA past its dependency wait (atomic min: set
 *    it to all ones first), stamps[2i+1] = the last CTA's exit (atomic max:
 *    set it to 0 first); needs n >= 2*(5*n_layers + 1);
 *  - the persistent kernel (mode 0): CTA c writes stamps[c * stride +
 *    layer * 20 + phase * 4 + e], phase 0..4 as above, e 0..3 (entry,
 *    dependency met, input staged, results published), the lm head as layer
 *    n_layers; stride = qasr_decoder_trace_stride, n >= SMs x stride.
 * n = 0 turns it off.  Changing it re-captures the step graphs. */
int qasr_decoder_trace(qasr_decoder *dec, unsigned long long *stamps, int64_t n);
int qasr_decoder_trace_stride(const qasr_decoder *dec);

/* Kernel classes of a decode step, for qasr_decoder_profile_step. */
#define QASR_K_EMBED 0     /* token embedding gather */
#define QASR_K_NORM 1      /* input / post-attention / final RMSNorm */
#define QASR_K_QKV 2       /* RMSNorm + q|k|v INT8 matvec + q/k norm, RoPE, KV append */
#define QASR_K_QKV_POST 3  /* (fused into QASR_K_QKV; no separate launch) */
#define QASR_K_ATTN 4      /* split-K decode attention */
#define QASR_K_OPROJ 5     /* o-proj INT8 matvec + residual */
#define QASR_K_GATEUP 6    /* gate/up INT8 matvec + SwiGLU */
#define QASR_K_DOWN 7      /* down INT8 matvec + residual */
#define QASR_K_LMHEAD 8    /* lm head INT8 matvec + argmax */
#define QASR_K_STEP 9      /* the persistent kernel: all of the above but the embedding gather */
#define QASR_K_COUNT 10

/* Run one decode step eagerly (no graph) with CUDA events around every
 * kernel; class_ms[c] receives the summed device time of class c and
 * class_launches[c] (may be NULL) its launch count.  Same results as
 * qasr_decoder_step; for profiling and rooflines. */
int qasr_decoder_profile_step(qasr_decoder *dec, const int32_t *tokens, const int32_t *positions, int M,
                              float *class_ms, int *class_launches, int n_classes);

/* Bytes the decode step reads/writes per call, by the algorithmic model
 * (weights + scales + norms + lm head + K/V rows attended); for rooflines. */
int64_t qasr_decoder_step_bytes(const qasr_decoder *dec, const int32_t *positions, int M);

/* ======================================================================
 * Audio encoder engine (f32 weights)
 * ==================================================================== */

typedef struct qasr_encoder qasr_encoder;

typedef struct {
  int d_model;        /* 896 (0.6B) / 1024 (1.7B) */
  int n_layers;       /* 18 / 24 */
  int n_heads;        /* 14 / 16 */
  int head_dim;       /* 64 */
  int ffn_dim;        /* 3584 / 4096 */
  int output_dim;     /* the decoder hidden size: 1024 / 2048 */
  int chunk_size;     /* mel frames per conv chunk: 2 * n_window = 100 */
  int n_window_infer; /* 800: attention windows of chunk tokens * (n_window_infer / chunk_size) */
} qasr_encoder_config;

typedef struct {
  const float *attn_norm_w, *attn_norm_b;        /* [d_model] */
  const float *wq, *bq, *wk, *bk, *wv, *bv;      /* [d_model, d_model], [d_model] */
  const float *wo, *bo;
  const float *ffn_norm_w, *ffn_norm_b;          /* [d_model] */
  const float *fc1_w, *fc1_b;                    /* [ffn, d_model], [ffn] */
  const float *fc2_w, *fc2_b;                    /* [d_model, ffn], [d_model] */
} qasr_enc_layer_weights;

/* Encoder (encoder.rs:20-240) on `device`: weight buffers allocated, values
 * set by the calls below (host or device pointers, copied).  NULL on failure. */
qasr_encoder *qasr_encoder_create(const qasr_encoder_config *cfg, int device);
void qasr_encoder_free(qasr_encoder *enc);

/* Conv stem: conv1 [480, 1, 3, 3], conv2/conv3 [480, 480, 3, 3] with biases
 * [480], conv_out [d_model, 480*16] (no bias). */
int qasr_encoder_set_conv(qasr_encoder *enc, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                          const float *conv2_b, const float *conv3_w, const float *conv3_b, const float *conv_out_w);
int qasr_encoder_set_layer(qasr_encoder *enc, int layer, const qasr_enc_layer_weights *w);
/* ln_post [d_model], proj1 [d_model, d_model] + bias, proj2 [output_dim, d_model] + bias. */
int qasr_encoder_set_post(qasr_encoder *enc, const float *ln_post_w, const float *ln_post_b, const float *proj1_w,
                          const float *proj1_b, const float *proj2_w, const float *proj2_b);

/* EncLayerInt8 (encoder.rs:424-444): the projection matrices INT8 [out, in]
 * with f32 per-row scales (the qwen-asr-quantize format), biases and norms f32. */
typedef struct {
  const float *attn_norm_w, *attn_norm_b;
  const int8_t *wq; const float *wq_s, *bq;
  const int8_t *wk; const float *wk_s, *bk;
  const int8_t *wv; const float *wv_s, *bv;
  const int8_t *wo; const float *wo_s, *bo;
  const float *ffn_norm_w, *ffn_norm_b;
  const int8_t *fc1; const float *fc1_s, *fc1_b;
  const int8_t *fc2; const float *fc2_s, *fc2_b;
} qasr_enc_layer_weights_int8;

/* EncoderInt8 (encoder.rs:446-520, the encoder of a V2 .qint8 file): the
 * same engine with INT8 projections, run through qasr_linear_int8 /
 * qasr_linear_nobias_int8 as EncoderInt8::forward does.  Each matrix keeps
 * whichever form its latest setter supplied. */
int qasr_encoder_set_conv_int8(qasr_encoder *enc, const float *conv1_w, const float *conv1_b, const float *conv2_w,
                               const float *conv2_b, const float *conv3_w, const float *conv3_b,
                               const int8_t *conv_out, const float *conv_out_s);
int qasr_encoder_set_layer_int8(qasr_encoder *enc, int layer, const qasr_enc_layer_weights_int8 *w);
int qasr_encoder_set_post_int8(qasr_encoder *enc, const float *ln_post_w, const float *ln_post_b,
                               const int8_t *proj1, const float *proj1_s, const float *proj1_b, const int8_t *proj2,
                               const float *proj2_s, const float *proj2_b);

/* Encoder tokens produced for mel_frames frames (13 per full 100-frame chunk). */
int qasr_encoder_tokens(const qasr_encoder *enc, int mel_frames);
const qasr_encoder_config *qasr_encoder_get_config(const qasr_encoder *enc);
int qasr_encoder_device(const qasr_encoder *enc);

/* Encoder::forward (encoder.rs:243-415): mel [128, mel_frames] f32 (host or
 * device) -> out [n_tokens, output_dim] (host or device, out_rows >= n_tokens).
 * Synchronous. */
int qasr_encoder_forward(qasr_encoder *enc, const float *mel, int mel_frames, float *out, int out_rows,
                         int *n_tokens);
/* qasr_encoder_forward over n independent segments at once (their tokens
 * concatenated on the device, attention windows restarting per segment):
 * outs[i] receives segment i's rows exactly as a forward of it alone would,
 * n_tokens[i] their count.  Synchronous. */
int qasr_encoder_forward_batch(qasr_encoder *enc, const float *const *mels, const int *mel_frames, int n,
                               float *const *outs, const int *out_rows, int *n_tokens);

/* ======================================================================
 * .qint8 model files (quantize.rs) and the V2 load path (context.rs:341-420)
 * ==================================================================== */

typedef struct qasr_qint8 qasr_qint8;

/* QuantFile::open (quantize.rs:130-280): mmap a V1 or V2 .qint8 file and
 * parse its tensor table.  Truncated tables and tensors whose bytes run past
 * the end of the file are rejected.  NULL on failure.  Needs no GPU. */
qasr_qint8 *qasr_qint8_open(const char *path);
void qasr_qint8_close(qasr_qint8 *f);
int qasr_qint8_version(const qasr_qint8 *f); /* 1 or 2 */
int qasr_qint8_count(const qasr_qint8 *f);
int qasr_qint8_find(const qasr_qint8 *f, const char *name); /* index, -1 if absent */
/* Tensor i: name, dtype (0 INT8, 1 F32, 2 BF16), dims and shape (up to 8),
 * pointers into the mapping (scales NULL unless INT8; F32/BF16 data may be
 * unaligned).  Any output pointer may be NULL. */
int qasr_qint8_tensor(const qasr_qint8 *f, int i, const char **name, int *dtype, int *n_dims, int64_t *shape,
                      const void **data, const float **scales);
/* QwenConfig::detect (config.rs:110-156) from the tensor shapes; either
 * output may be NULL.  max_batch / max_seq of dec are left unchanged. */
int qasr_qint8_detect(const qasr_qint8 *f, qasr_decoder_config *dec, qasr_encoder_config *enc);
/* DecoderInt8::load (decoder.rs:680-748) / EncoderInt8::load_from_qint8
 * (encoder.rs:466-520) into engines created with the detected configs. */
int qasr_qint8_load_decoder(const qasr_qint8 *f, qasr_decoder *dec);
int qasr_qint8_load_encoder(const qasr_qint8 *f, qasr_encoder *enc);

/* ======================================================================
 * Transcription (transcribe.rs), token ids out
 * ==================================================================== */

/* Prompt rows of a segment with n_audio_tokens encoder rows: PREFIX_HEAD (3)
 * + n_prompt + PREFIX_TAIL (6) + audio + SUFFIX_BASE (6) + n_force. */
int qasr_transcribe_prompt_len(int n_audio_tokens, int n_prompt, int n_force);

/* transcribe_segment (transcribe.rs:67-244) for n_segments (<= the decoder's
 * max_batch) independent segments at once, decoded as one batch (the
 * segmented mode, transcribe.rs:354-420, without past-text conditioning):
 * samples[i] (host or device, 16 kHz f32, n_samples[i] >= 160) -> log-mel ->
 * encoder -> prompt embeddings with the reference's special tokens and the
 * optional prompt / forced-language ids -> prefill into KV slot i -> greedy
 * decode.  ids[i * ids_stride + j] (host) receives generated token j of
 * segment i, n_ids[i] how many: max_new, or when stop_at_eos is set up to and
 * including the first <|endoftext|> / <|im_end|>.  The encoder's output size
 * must equal the decoder's hidden size and both engines must be on one
 * device.  Synchronous. */
int qasr_transcribe_batch(qasr_decoder *dec, qasr_encoder *enc, const float *const *samples, const int *n_samples,
                          int n_segments, const int32_t *prompt_tokens, int n_prompt, const int32_t *force_tokens,
                          int n_force, int max_new, int stop_at_eos, int32_t *ids, int ids_stride, int *n_ids);

/* The segment loop of transcribe_audio (transcribe.rs:354-420, past-text
 * conditioning off) over n_segments independent segments, spread over
 * n_lanes engine lanes (decs[l], encs[l]: one decoder + encoder pair per
 * lane, no engine in two lanes, each pair on one device).  Segments go in
 * full batches of the smallest lane's max_batch to whichever lane is free
 * (so lanes beyond ceil(n_segments / max_batch) stay idle); lane 0
 * runs on the calling thread, the others on threads of their own, so lanes on
 * one GPU overlap their work and lanes on several GPUs run side by side.
 * Outputs as qasr_transcribe_batch, indexed by segment; the ids of a segment
 * do not depend on the lane or batch it ran in.  Synchronous; on an error the
 * first failing lane's message is reported and the other lanes stop after
 * their current batch. */
int qasr_transcribe_lanes(qasr_decoder *const *decs, qasr_encoder *const *encs, int n_lanes,
                          const float *const *samples, const int *n_samples, int n_segments,
                          const int32_t *prompt_tokens, int n_prompt, const int32_t *force_tokens, int n_force,
                          int max_new, int stop_at_eos, int32_t *ids, int ids_stride, int *n_ids);

/* ======================================================================
 * Streaming transcription (transcribe.rs:445-1495), token ids out
 * ==================================================================== */

typedef struct qasr_stream qasr_stream;

typedef struct {
  float chunk_sec;            /* stream_chunk_sec: audio per step (2.0) */
  int rollback;               /* stream_rollback: uncommitted tail tokens (5) */
  int unfixed_chunks;         /* stream_unfixed_chunks: chunks before commits start (2) */
  int max_new_tokens;         /* stream_max_new_tokens per chunk (32; <= 0 means 32) */
  int past_text_conditioning; /* feed the committed tokens back as prompt (0) */
  int incremental;            /* 1: stream_push_audio / StreamState semantics; 0: transcribe_stream */
} qasr_stream_config;

/* The QwenCtx defaults (context.rs:499-512), incremental. */
void qasr_stream_default_config(qasr_stream_config *cfg);
/* A stream over an encoder and a decoder on one device; it decodes in the
 * decoder's KV slot 0 (batch of one).  NULL on failure. */
qasr_stream *qasr_stream_create(qasr_decoder *dec, qasr_encoder *enc, const qasr_stream_config *cfg);
void qasr_stream_free(qasr_stream *s);
/* Prompt / forced-language token ids (placed as in transcribe_segment). */
int qasr_stream_set_prompt(qasr_stream *s, const int32_t *prompt, int n_prompt, const int32_t *force, int n_force);
/* Byte length of every token's text (tokenizer.decode_bytes(t).len()), used by
 * the byte-level realignment of committed tokens after a re-anchor. */
int qasr_stream_set_token_bytes(qasr_stream *s, const int32_t *bytes, int n);
/* stream_push_audio (transcribe.rs:960-1495): samples = all audio received
 * so far (16 kHz f32, host or device); processes every complete chunk after
 * the cursor (and the rest when finalize).  emitted (host, cap entries)
 * receives the token ids committed by this call.  With incremental = 0, one
 * call with the whole buffer and finalize = 1 is transcribe_stream. */
int qasr_stream_push(qasr_stream *s, const float *samples, int64_t n_samples, int finalize, int32_t *emitted, int cap,
                     int *n_emitted);
/* StreamState::reset / audio_cursor / audio_trim_request / apply_audio_trim. */
int qasr_stream_reset(qasr_stream *s);
int64_t qasr_stream_audio_cursor(const qasr_stream *s);
int64_t qasr_stream_trim_request(const qasr_stream *s);
int qasr_stream_apply_trim(qasr_stream *s, int64_t trim);
/* All committed ids so far (StreamState::text) and the decoded but not yet
 * committed ones (unfixed_text); *n = the full count, up to cap copied. */
int qasr_stream_emitted(const qasr_stream *s, int32_t *ids, int cap, int *n);
int qasr_stream_unfixed(const qasr_stream *s, int32_t *ids, int cap, int *n);

/* Host helpers of the transcription drivers (no GPU):
 * stream_tail_repeat_blocks (transcribe.rs:42-59) and find_split_point
 * (transcribe.rs:250-275). */
int qasr_stream_tail_repeat(const int32_t *tokens, int n, int max_period, int *best_reps, int *best_period);
int64_t qasr_find_split_point(const float *samples, int64_t n, int64_t target_sample, float search_sec);
/* transcribe_audio's segment plan (transcribe.rs:317-345): starts[i] = the
 * first sample of segment i, *n_segments their count (up to 127). */
int qasr_plan_segments(const float *samples, int64_t n, float segment_sec, float search_sec, int64_t *starts, int cap,
                       int *n_segments);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* QWENASR_CUDA_H */
