// qwenasr_cuda.rs -- Rust declarations of the C ABI in qwenasr_cuda.h, for a
// crate of the reference (crates/qwen-asr) that links libqwenasr_b200.so.
// No Rust toolchain exists where this library is built, so this file is not
// compiled here; tests/test_abi.py checks that it declares every function of
// the header with the same number of arguments.
#![allow(non_camel_case_types, dead_code)]
use std::os::raw::{c_char, c_int, c_void};

pub const QASR_OK: c_int = 0;
pub const QASR_ERR_INVALID: c_int = -1;
pub const QASR_ERR_CUDA: c_int = -2;
pub const QASR_ERR_ALLOC: c_int = -3;
pub const QASR_ERR_UNSUPPORTED: c_int = -4;
pub const QASR_ERR_TIMEOUT: c_int = -5;

#[repr(C)]
pub struct QasrDecoder {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrDecoderConfig {
    pub hidden: c_int,
    pub inter: c_int,
    pub n_layers: c_int,
    pub n_heads: c_int,
    pub n_kv_heads: c_int,
    pub head_dim: c_int,
    pub vocab: c_int,
    pub eps: f32,
    pub theta: f32,
    pub max_batch: c_int,
    pub max_seq: c_int,
    pub embed_is_int8: c_int,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrDecLayerWeights {
    pub wq: *const i8, pub wq_s: *const f32, pub wk: *const i8, pub wk_s: *const f32,
    pub wv: *const i8, pub wv_s: *const f32, pub wo: *const i8, pub wo_s: *const f32,
    pub gate_up: *const i8, pub gate_up_s: *const f32, pub down: *const i8, pub down_s: *const f32,
    pub q_norm: *const f32, pub k_norm: *const f32, pub input_norm: *const f32, pub post_attn_norm: *const f32,
}

#[repr(C)]
pub struct QasrEncoder {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrEncoderConfig {
    pub d_model: c_int,
    pub n_layers: c_int,
    pub n_heads: c_int,
    pub head_dim: c_int,
    pub ffn_dim: c_int,
    pub output_dim: c_int,
    pub chunk_size: c_int,
    pub n_window_infer: c_int,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrEncLayerWeights {
    pub attn_norm_w: *const f32, pub attn_norm_b: *const f32,
    pub wq: *const f32, pub bq: *const f32, pub wk: *const f32, pub bk: *const f32,
    pub wv: *const f32, pub bv: *const f32, pub wo: *const f32, pub bo: *const f32,
    pub ffn_norm_w: *const f32, pub ffn_norm_b: *const f32,
    pub fc1_w: *const f32, pub fc1_b: *const f32, pub fc2_w: *const f32, pub fc2_b: *const f32,
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrEncLayerWeightsInt8 {
    pub attn_norm_w: *const f32, pub attn_norm_b: *const f32,
    pub wq: *const i8, pub wq_s: *const f32, pub bq: *const f32,
    pub wk: *const i8, pub wk_s: *const f32, pub bk: *const f32,
    pub wv: *const i8, pub wv_s: *const f32, pub bv: *const f32,
    pub wo: *const i8, pub wo_s: *const f32, pub bo: *const f32,
    pub ffn_norm_w: *const f32, pub ffn_norm_b: *const f32,
    pub fc1: *const i8, pub fc1_s: *const f32, pub fc1_b: *const f32,
    pub fc2: *const i8, pub fc2_s: *const f32, pub fc2_b: *const f32,
}

#[repr(C)]
pub struct QasrQint8 {
    _private: [u8; 0],
}

#[repr(C)]
pub struct QasrStream {
    _private: [u8; 0],
}

#[repr(C)]
#[derive(Clone, Copy)]
pub struct QasrStreamConfig {
    pub chunk_sec: f32,
    pub rollback: c_int,
    pub unfixed_chunks: c_int,
    pub max_new_tokens: c_int,
    pub past_text_conditioning: c_int,
    pub incremental: c_int,
}

#[link(name = "qwenasr_b200")]
extern "C" {
    pub fn qasr_last_error() -> *const c_char;
    pub fn qasr_version() -> *const c_char;
    pub fn qasr_rms_norm(out: *mut f32, x: *const f32, w: *const f32, seq: c_int, hidden: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_rms_norm_per_head(x: *mut f32, w: *const f32, seq: c_int, n_heads: c_int, head_dim: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_layer_norm(out: *mut f32, x: *const f32, w: *const f32, b: *const f32, seq: c_int, hidden: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_compute_rope_neox(cos_out: *mut f32, sin_out: *mut f32, positions: *const i32, seq: c_int, head_dim: c_int, theta: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_rope_cache_table(cos_out: *mut f32, sin_out: *mut f32, n_pos: c_int, head_dim: c_int, theta: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_apply_rope_neox(x: *mut f32, cos_v: *const f32, sin_v: *const f32, seq: c_int, n_heads: c_int, head_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_kv_append(k_cache: *mut f32, v_cache: *mut f32, k_new: *const f32, v_new: *const f32, layer: c_int, max_seq: c_int, kv_dim: c_int, start_pos: c_int, seq: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_sinusoidal_pe(pe: *mut f32, n_pos: c_int, d_model: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_gelu(x: *mut f32, n: i64, stream: *mut c_void) -> c_int;
    pub fn qasr_gelu_erf(x: *mut f32, n: i64, stream: *mut c_void) -> c_int;
    pub fn qasr_silu(x: *mut f32, n: i64, stream: *mut c_void) -> c_int;
    pub fn qasr_swiglu_multiply(out: *mut f32, gate_up: *const f32, seq: c_int, inter: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_add_inplace(a: *mut f32, b: *const f32, n: i64, stream: *mut c_void) -> c_int;
    pub fn qasr_linear_nobias_int8(y: *mut f32, x: *const f32, w: *const i8, scales: *const f32, seq: c_int, in_dim: c_int, out_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_linear_int8(y: *mut f32, x: *const f32, w: *const i8, scales: *const f32, bias: *const f32, seq: c_int, in_dim: c_int, out_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_linear(y: *mut f32, x: *const f32, w: *const f32, b: *const f32, seq: c_int, in_dim: c_int, out_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_linear_nobias(y: *mut f32, x: *const f32, w: *const f32, seq: c_int, in_dim: c_int, out_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_matmul_t(c: *mut f32, a: *const f32, b: *const f32, m: c_int, k: c_int, n: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_conv2d(out: *mut f32, input: *const f32, weight: *const f32, bias: *const f32, c_in: c_int, c_out: c_int, h_in: c_int, w_in: c_int, kh: c_int, kw: c_int, stride: c_int, padding: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_bidirectional_attention(out: *mut f32, q: *const f32, k: *const f32, v: *const f32, seq: c_int, n_heads: c_int, head_dim: c_int, scale: f32, window_starts: *const i32, n_windows: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_mel_frames(n_samples: c_int) -> c_int;
    pub fn qasr_mel_spectrogram(mel: *mut f32, samples: *const f32, n_samples: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_causal_attention(out: *mut f32, q: *const f32, k: *const f32, v: *const f32, seq_q: c_int, seq_k: c_int, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int, scale: f32, q_offset: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_quantize_f32_to_int8(data: *const f32, out_dim: i64, in_dim: i64, q: *mut i8, scales: *mut f32, stream: *mut c_void) -> c_int;
    pub fn qasr_embed_gather_f32(dst: *mut f32, table: *const f32, ids: *const i32, n: c_int, dim: c_int, vocab: i64, bad_id_flag: *mut c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_embed_gather_int8(dst: *mut f32, table: *const i8, scales: *const f32, ids: *const i32, n: c_int, dim: c_int, vocab: i64, bad_id_flag: *mut c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_pre_attn_block(x_norm: *mut f32, x: *const f32, w_in: *const f32, seq: c_int, hidden: c_int, q: *mut f32, k: *const f32, v: *const f32, k_out: *mut f32, q_norm_w: *const f32, k_norm_w: *const f32, n_heads: c_int, n_kv_heads: c_int, head_dim: c_int, eps: f32, cos_tab: *const f32, sin_tab: *const f32, start_pos: c_int, k_cache: *mut f32, v_cache: *mut f32, layer: c_int, max_seq: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_ln_pe(out: *mut f32, x: *const f32, w: *const f32, b: *const f32, pe: *const f32, rows: c_int, hidden: c_int, n_pos: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_ln_pe_gelu_erf(out: *mut f32, x: *const f32, w: *const f32, b: *const f32, pe: *const f32, rows: c_int, hidden: c_int, n_pos: c_int, eps: f32, act: *mut f32, n_act: i64, stream: *mut c_void) -> c_int;
    pub fn qasr_int8_norm_gateup_swiglu(h: *mut f32, x: *const f32, norm_w: *const f32, w_gate_up: *const i8, scales: *const f32, M: c_int, hidden: c_int, inter: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_int8_matvec_residual(x: *mut f32, a: *const f32, w: *const i8, scales: *const f32, M: c_int, in_dim: c_int, out_dim: c_int, stream: *mut c_void) -> c_int;
    pub fn qasr_final_norm_lmhead_argmax(ids_out: *mut i32, logits_out: *mut f32, x: *const f32, norm_w: *const f32, w: *const i8, scales: *const f32, M: c_int, hidden: c_int, vocab: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_final_norm_lmhead_argmax_noalloc(ids_out: *mut i32, logits_out: *mut f32, x: *const f32, norm_w: *const f32, w: *const i8, scales: *const f32, M: c_int, hidden: c_int, vocab: c_int, eps: f32, stream: *mut c_void) -> c_int;
    pub fn qasr_decoder_create(cfg: *const QasrDecoderConfig, device: c_int) -> *mut QasrDecoder;
    pub fn qasr_decoder_free(dec: *mut QasrDecoder);
    pub fn qasr_decoder_set_layer(dec: *mut QasrDecoder, layer: c_int, w: *const QasrDecLayerWeights) -> c_int;
    pub fn qasr_decoder_set_gate_up(dec: *mut QasrDecoder, layer: c_int, gate: *const i8, gate_s: *const f32, up: *const i8, up_s: *const f32) -> c_int;
    pub fn qasr_decoder_set_globals(dec: *mut QasrDecoder, embed: *const c_void, embed_scales: *const f32, norm: *const f32, lm_head: *const i8, lm_head_s: *const f32) -> c_int;
    pub fn qasr_decoder_kv(dec: *mut QasrDecoder, slot: c_int, k_cache: *mut *mut f32, v_cache: *mut *mut f32) -> c_int;
    pub fn qasr_decoder_step(dec: *mut QasrDecoder, tokens: *const i32, positions: *const i32, M: c_int, next_tokens: *mut i32) -> c_int;
    pub fn qasr_decoder_prefill(dec: *mut QasrDecoder, slot: c_int, embeds: *const f32, seq: c_int, start_pos: c_int) -> c_int;
    pub fn qasr_decoder_prefill_batch(dec: *mut QasrDecoder, slots: *const c_int, embeds: *const *const f32, seqs: *const c_int, start_pos: *const c_int, n: c_int) -> c_int;
    pub fn qasr_decoder_prefill_hidden(dec: *mut QasrDecoder) -> *const f32;
    pub fn qasr_decoder_step_device(dec: *mut QasrDecoder, tokens: *const i32, positions: *const i32, M: c_int, next_tokens: *mut i32) -> c_int;
    pub fn qasr_decoder_stream(dec: *mut QasrDecoder) -> *mut c_void;
    pub fn qasr_decoder_get_config(dec: *const QasrDecoder) -> *const QasrDecoderConfig;
    pub fn qasr_decoder_device(dec: *const QasrDecoder) -> c_int;
    pub fn qasr_decoder_embed(dec: *mut QasrDecoder, ids: *const i32, n: c_int, out: *mut f32) -> c_int;
    pub fn qasr_decoder_keep_logits(dec: *mut QasrDecoder, enable: c_int) -> c_int;
    pub fn qasr_decoder_set_step_kernel(dec: *mut QasrDecoder, mode: c_int) -> c_int;
    pub fn qasr_decoder_step_kernel(dec: *const QasrDecoder, M: c_int) -> c_int;
    pub fn qasr_decoder_trace(dec: *mut QasrDecoder, stamps: *mut u64, n: i64) -> c_int;
    pub fn qasr_decoder_trace_stride(dec: *const QasrDecoder) -> c_int;
    pub fn qasr_decoder_logits(dec: *mut QasrDecoder) -> *const f32;
    pub fn qasr_decoder_profile_step(dec: *mut QasrDecoder, tokens: *const i32, positions: *const i32, M: c_int, class_ms: *mut f32, class_launches: *mut c_int, n_classes: c_int) -> c_int;
    pub fn qasr_decoder_step_bytes(dec: *const QasrDecoder, positions: *const i32, M: c_int) -> i64;
    pub fn qasr_encoder_create(cfg: *const QasrEncoderConfig, device: c_int) -> *mut QasrEncoder;
    pub fn qasr_encoder_free(enc: *mut QasrEncoder);
    pub fn qasr_encoder_set_conv(enc: *mut QasrEncoder, conv1_w: *const f32, conv1_b: *const f32, conv2_w: *const f32, conv2_b: *const f32, conv3_w: *const f32, conv3_b: *const f32, conv_out_w: *const f32) -> c_int;
    pub fn qasr_encoder_set_layer(enc: *mut QasrEncoder, layer: c_int, w: *const QasrEncLayerWeights) -> c_int;
    pub fn qasr_encoder_set_post(enc: *mut QasrEncoder, ln_post_w: *const f32, ln_post_b: *const f32, proj1_w: *const f32, proj1_b: *const f32, proj2_w: *const f32, proj2_b: *const f32) -> c_int;
    pub fn qasr_encoder_set_conv_int8(enc: *mut QasrEncoder, conv1_w: *const f32, conv1_b: *const f32, conv2_w: *const f32, conv2_b: *const f32, conv3_w: *const f32, conv3_b: *const f32, conv_out: *const i8, conv_out_s: *const f32) -> c_int;
    pub fn qasr_encoder_set_layer_int8(enc: *mut QasrEncoder, layer: c_int, w: *const QasrEncLayerWeightsInt8) -> c_int;
    pub fn qasr_encoder_set_post_int8(enc: *mut QasrEncoder, ln_post_w: *const f32, ln_post_b: *const f32, proj1: *const i8, proj1_s: *const f32, proj1_b: *const f32, proj2: *const i8, proj2_s: *const f32, proj2_b: *const f32) -> c_int;
    pub fn qasr_encoder_tokens(enc: *const QasrEncoder, mel_frames: c_int) -> c_int;
    pub fn qasr_encoder_get_config(enc: *const QasrEncoder) -> *const QasrEncoderConfig;
    pub fn qasr_encoder_device(enc: *const QasrEncoder) -> c_int;
    pub fn qasr_encoder_forward(enc: *mut QasrEncoder, mel: *const f32, mel_frames: c_int, out: *mut f32, out_rows: c_int, n_tokens: *mut c_int) -> c_int;
    pub fn qasr_encoder_forward_batch(enc: *mut QasrEncoder, mels: *const *const f32, mel_frames: *const c_int, n: c_int, outs: *const *mut f32, out_rows: *const c_int, n_tokens: *mut c_int) -> c_int;
    pub fn qasr_qint8_open(path: *const c_char) -> *mut QasrQint8;
    pub fn qasr_qint8_close(f: *mut QasrQint8);
    pub fn qasr_qint8_version(f: *const QasrQint8) -> c_int;
    pub fn qasr_qint8_count(f: *const QasrQint8) -> c_int;
    pub fn qasr_qint8_find(f: *const QasrQint8, name: *const c_char) -> c_int;
    pub fn qasr_qint8_tensor(f: *const QasrQint8, i: c_int, name: *mut *const c_char, dtype: *mut c_int, n_dims: *mut c_int, shape: *mut i64, data: *mut *const c_void, scales: *mut *const f32) -> c_int;
    pub fn qasr_qint8_detect(f: *const QasrQint8, dec: *mut QasrDecoderConfig, enc: *mut QasrEncoderConfig) -> c_int;
    pub fn qasr_qint8_load_decoder(f: *const QasrQint8, dec: *mut QasrDecoder) -> c_int;
    pub fn qasr_qint8_load_encoder(f: *const QasrQint8, enc: *mut QasrEncoder) -> c_int;
    pub fn qasr_transcribe_prompt_len(n_audio_tokens: c_int, n_prompt: c_int, n_force: c_int) -> c_int;
    pub fn qasr_transcribe_batch(dec: *mut QasrDecoder, enc: *mut QasrEncoder, samples: *const *const f32, n_samples: *const c_int, n_segments: c_int, prompt_tokens: *const i32, n_prompt: c_int, force_tokens: *const i32, n_force: c_int, max_new: c_int, stop_at_eos: c_int, ids: *mut i32, ids_stride: c_int, n_ids: *mut c_int) -> c_int;
    pub fn qasr_transcribe_lanes(decs: *const *mut QasrDecoder, encs: *const *mut QasrEncoder, n_lanes: c_int, samples: *const *const f32, n_samples: *const c_int, n_segments: c_int, prompt_tokens: *const i32, n_prompt: c_int, force_tokens: *const i32, n_force: c_int, max_new: c_int, stop_at_eos: c_int, ids: *mut i32, ids_stride: c_int, n_ids: *mut c_int) -> c_int;
    pub fn qasr_stream_default_config(cfg: *mut QasrStreamConfig);
    pub fn qasr_stream_create(dec: *mut QasrDecoder, enc: *mut QasrEncoder, cfg: *const QasrStreamConfig) -> *mut QasrStream;
    pub fn qasr_stream_free(s: *mut QasrStream);
    pub fn qasr_stream_set_prompt(s: *mut QasrStream, prompt: *const i32, n_prompt: c_int, force: *const i32, n_force: c_int) -> c_int;
    pub fn qasr_stream_set_token_bytes(s: *mut QasrStream, bytes: *const i32, n: c_int) -> c_int;
    pub fn qasr_stream_push(s: *mut QasrStream, samples: *const f32, n_samples: i64, finalize: c_int, emitted: *mut i32, cap: c_int, n_emitted: *mut c_int) -> c_int;
    pub fn qasr_stream_reset(s: *mut QasrStream) -> c_int;
    pub fn qasr_stream_audio_cursor(s: *const QasrStream) -> i64;
    pub fn qasr_stream_trim_request(s: *const QasrStream) -> i64;
    pub fn qasr_stream_apply_trim(s: *mut QasrStream, trim: i64) -> c_int;
    pub fn qasr_stream_emitted(s: *const QasrStream, ids: *mut i32, cap: c_int, n: *mut c_int) -> c_int;
    pub fn qasr_stream_unfixed(s: *const QasrStream, ids: *mut i32, cap: c_int, n: *mut c_int) -> c_int;
    pub fn qasr_stream_tail_repeat(tokens: *const i32, n: c_int, max_period: c_int, best_reps: *mut c_int, best_period: *mut c_int) -> c_int;
    pub fn qasr_find_split_point(samples: *const f32, n: i64, target_sample: i64, search_sec: f32) -> i64;
    pub fn qasr_plan_segments(samples: *const f32, n: i64, segment_sec: f32, search_sec: f32, starts: *mut i64, cap: c_int, n_segments: *mut c_int) -> c_int;
}
