/*
 * oracle.h -- CPU restatement of the QwenASR reference kernel path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * CUDA kernels in qwenasr_b200/csrc and the timed CPU baseline in bench.py.
 * Nothing in the product library links it, loads it or calls it.
 *
 * What it restates: the x86_64 code path of crates/qwen-asr (Rust), i.e. the
 * AVX2/FMA row kernels of src/kernels/avx.rs, the scalar kernels of
 * src/kernels/generic.rs that mod.rs dispatches to on x86_64 (the INT8
 * matvec, mod.rs:396-402), the scalar helpers of src/kernels/mod.rs and the
 * per-layer compositions of src/decoder.rs.  AVX lanes are emulated with
 * 8-wide float arrays and fmaf(), so every rounding step happens in the same
 * order as the intrinsics; scalar Rust code is restated with the same
 * left-to-right evaluation and no FMA contraction (Rust never contracts, so
 * this file is compiled with -ffp-contract=off).  Transcendentals call glibc
 * expf/logf/powf/sinf/cosf/tanhf, which is what Rust's f32 methods lower to
 * on Linux.
 *
 * Pinning: the reference is a Rust crate and no Rust toolchain exists on the
 * build or GPU machines, so no output of the reference itself can be produced
 * here.  The reference's own kernel tests (crates/qwen-asr/tests/kernels.rs)
 * pin only properties (norm statistics, GELU signs, SiLU formula, vector op
 * identities); tests/test_oracle.py re-runs every one of them against this
 * library.  Beyond those properties, parity is UNPINNED against reference
 * output: the restatement is checked by code reading and by independent
 * float64 re-derivations in tests/test_oracle.py.
 *
 * All matrices are row-major.  INT8 weights are [out, in] with f32 per-row
 * scales [out] (src/quantize.rs:78-84).
 */
#ifndef QWENASR_ORACLE_H
#define QWENASR_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* thread pool (mod.rs:288 set_threads, MAX_THREADS = 16 at mod.rs:177) */
void orc_set_threads(int n);
int orc_get_threads(void);

/* ---- row kernels (avx.rs / mod.rs) ---- */
void orc_rms_norm(float *out, const float *x, const float *w, int seq, int hidden, float eps);
void orc_rms_norm_per_head(float *x, const float *w, int seq, int n_heads, int head_dim, float eps);
void orc_layer_norm(float *out, const float *x, const float *w, const float *b, int seq, int hidden, float eps);
void orc_compute_rope_neox(float *cos_out, float *sin_out, const int32_t *positions, int seq, int head_dim, float theta);
void orc_rope_cache_table(float *cos_out, float *sin_out, int n_pos, int head_dim, float theta);
void orc_apply_rope_neox(float *x, const float *cos_v, const float *sin_v, int seq, int n_heads, int head_dim);
void orc_sinusoidal_pe(float *pe, int n_pos, int d_model);
void orc_gelu(float *x, long n);            /* tanh GELU, avx.rs:536 */
void orc_gelu_erf(float *x, long n);        /* exact-erf GELU (Metal path semantics) */
void orc_silu(float *x, long n);            /* mod.rs:941 */
void orc_swiglu_multiply(float *out, const float *gate_up, int seq, int inter);   /* avx.rs:568 */
void orc_swiglu_decode(float *out, const float *gate_up, int inter);              /* decoder.rs:916-921 */
void orc_softmax(float *x, int rows, int cols);
float orc_fast_exp(float x);               /* one lane of fast_exp_avx, avx.rs:487 */
float orc_dot_f32(const float *a, const float *b, int n);
float orc_dot_f32_generic(const float *a, const float *b, int n);
void orc_vec_scale_inplace(float *dst, float s, int n);
void orc_vec_axpy_inplace(float *dst, const float *src, float alpha, int n);
void orc_vec_scale_add(float *dst, const float *src, float c, int n);
void orc_add_inplace(float *a, const float *b, long n);

/* ---- matvec / linear ---- */
void orc_linear_nobias_int8(float *y, const float *x, const int8_t *w, const float *scales,
                            int seq, int in_dim, int out_dim);
void orc_linear_int8(float *y, const float *x, const int8_t *w, const float *scales,
                     const float *bias, int seq, int in_dim, int out_dim);
void orc_linear(float *y, const float *x, const float *w, const float *bias,
                int seq, int in_dim, int out_dim);   /* f32 GEMM, fp64-accumulated stand-in for cblas_sgemm */
void orc_bf16_matvec_generic(float *y, const float *x, const uint16_t *w, const float *bias, int in_dim, int out_dim);
void orc_bf16_matvec(float *y, const float *x, const uint16_t *w, const float *bias, int in_dim, int out_dim);

/* ---- attention ---- */
void orc_causal_attention(float *out, const float *q, const float *k, const float *v,
                          int seq_q, int seq_k, int n_heads, int n_kv_heads, int head_dim,
                          float scale, int q_offset);
void orc_bidirectional_attention(float *out, const float *q, const float *k, const float *v,
                                 int seq, int n_heads, int head_dim, float scale,
                                 const int32_t *window_starts, int n_windows);

/* ---- quantizer / embeddings (quantize.rs:633, decoder.rs:631-646) ---- */
void orc_quantize_f32_to_int8(const float *data, int64_t out_dim, int64_t in_dim, int8_t *q, float *scales);
void orc_embed_int8(float *dst, const int8_t *table, const float *scales, int token, int dim);
void orc_embed_bf16(float *dst, const uint16_t *table, int token, int dim);
int orc_argmax_first(const float *x, int n);
void orc_interleave_gate_up(const int8_t *gate, const float *gate_s, const int8_t *up, const float *up_s,
                            int inter, int hidden, int8_t *fused, float *fused_s);

/* ---- INT8 decoder (decoder.rs:845-965 / 751-842) ---- */
typedef struct {
    const int8_t *wq; const float *wq_s;        /* [q_dim, hidden] */
    const int8_t *wk; const float *wk_s;        /* [kv_dim, hidden] */
    const int8_t *wv; const float *wv_s;        /* [kv_dim, hidden] */
    const int8_t *wo; const float *wo_s;        /* [hidden, q_dim] */
    const int8_t *gate_up; const float *gate_up_s;  /* [2*inter, hidden], rows interleaved g,u */
    const int8_t *down; const float *down_s;    /* [hidden, inter] */
    const float *q_norm; const float *k_norm;   /* [head_dim] */
    const float *input_norm; const float *post_attn_norm;  /* [hidden] */
} orc_dec_layer;

typedef struct {
    int hidden, inter, n_layers, n_heads, n_kv_heads, head_dim, vocab;
    float eps, theta;
    const orc_dec_layer *layers;
    const float *norm;                           /* [hidden] */
    const int8_t *lm_head; const float *lm_head_s;  /* [vocab, hidden] */
} orc_decoder;

/* KV cache of one sequence: k, v = [n_layers, max_seq, kv_dim] f32 (decoder.rs:130-202). */
int orc_decoder_forward_int8(const orc_decoder *dec, float *k_cache, float *v_cache, int max_seq,
                             int pos, const float *input_embed, float *logits_out, float *x_out);
void orc_decoder_prefill_int8(const orc_decoder *dec, float *k_cache, float *v_cache, int max_seq,
                              int start_pos, const float *input_embeds, int seq_len, float *x_out);

/* Config-1 block (decoder pre-attention at 0.6B shapes): rms_norm of x, per-head norm + RoPE of
 * q and k, KV append of k and v at rows start_pos.. of a [max_seq, kv_dim] layer slab. */
void orc_pre_attn_block(float *x_norm, const float *x, const float *w_in, int seq, int hidden,
                        float *q, float *k, const float *v, const float *q_norm_w, const float *k_norm_w,
                        int n_heads, int n_kv_heads, int head_dim, float eps,
                        const float *cos_tab, const float *sin_tab, int start_pos,
                        float *k_cache, float *v_cache);

/* ---- log-mel front end (audio.rs:202-385): 16 kHz, 400-point DFT, hop 160, 128 Slaney bins ---- */
#define ORC_MEL_NFFT 400
#define ORC_MEL_FREQS 201
#define ORC_MEL_HOP 160
#define ORC_MEL_BINS 128
void orc_mel_filters(float *filters);                              /* [128, 201] */
void orc_mel_tables(float *window, float *cos_t, float *sin_t);     /* [400], [201, 400] x2 */
int orc_mel_frames(int n_samples);
int orc_mel_spectrogram(float *mel, const float *samples, int n_samples);  /* mel [128, n_frames] */

#ifdef __cplusplus
}
#endif
#endif
