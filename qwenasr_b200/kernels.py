"""Host-side mirror of the reference's kernel module on the B200.

Each function keeps the name, argument order and in-place semantics of the
function it replaces in crates/qwen-asr/src/kernels/mod.rs (cited per
function): Rust slices become contiguous torch CUDA tensors that are mutated
in place, lengths stay explicit.  Work is enqueued on torch's current CUDA
stream through the C ABI of libqwenasr_b200.so; nothing here computes on the
CPU, and every call raises QasrError (from the library's status) or
ValueError (bad tensors) instead of falling back.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib

__all__ = [
    "rms_norm", "rms_norm_per_head", "layer_norm", "compute_rope_neox", "rope_cache_table", "apply_rope_neox",
    "kv_append", "sinusoidal_pe", "gelu", "gelu_erf", "silu", "swiglu_multiply", "add_inplace",
    "linear_nobias_int8", "linear_int8", "causal_attention", "quantize_f32_to_int8", "embed_gather",
    "pre_attn_block", "ln_pe", "ln_pe_gelu_erf", "int8_norm_gateup_swiglu", "int8_matvec_residual", "final_norm_lmhead_argmax",
]


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t, dtype=None, name="tensor", numel=None):
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if numel is not None and t.numel() < numel:
        raise ValueError(f"{name} has {t.numel()} elements, needs {numel}")
    return C.c_void_p(t.data_ptr())


f32, i8, i32 = torch.float32, torch.int8, torch.int32


def rms_norm(out, x, weight, seq_len, hidden, eps):
    """kernels::rms_norm (mod.rs:897): out = x * rsqrt(mean(x^2)+eps) * weight (bit-exact)."""
    n = seq_len * hidden
    _lib.call("qasr_rms_norm", _ptr(out, f32, "out", n), _ptr(x, f32, "x", n), _ptr(weight, f32, "weight", hidden),
              seq_len, hidden, C.c_float(eps), _stream())


def rms_norm_per_head(x, weight, seq_len, n_heads, head_dim, eps):
    """kernels::rms_norm_per_head (mod.rs:920), in place (bit-exact)."""
    _lib.call("qasr_rms_norm_per_head", _ptr(x, f32, "x", seq_len * n_heads * head_dim),
              _ptr(weight, f32, "weight", head_dim), seq_len, n_heads, head_dim, C.c_float(eps), _stream())


def layer_norm(out, x, weight, bias, seq_len, hidden, eps):
    """kernels::layer_norm (mod.rs:866) (bit-exact)."""
    n = seq_len * hidden
    _lib.call("qasr_layer_norm", _ptr(out, f32, "out", n), _ptr(x, f32, "x", n), _ptr(weight, f32, "weight", hidden),
              _ptr(bias, f32, "bias", hidden), seq_len, hidden, C.c_float(eps), _stream())


def compute_rope_neox(cos_out, sin_out, positions, seq, head_dim, theta):
    """kernels::compute_rope_neox (mod.rs:1228)."""
    _lib.call("qasr_compute_rope_neox", _ptr(cos_out, f32, "cos_out", seq * head_dim),
              _ptr(sin_out, f32, "sin_out", seq * head_dim), _ptr(positions, i32, "positions", seq), seq, head_dim,
              C.c_float(theta), _stream())


def rope_cache_table(cos_out, sin_out, n_pos, head_dim, theta):
    """RopeCache::ensure (decoder.rs:253) table rows 0..n_pos."""
    _lib.call("qasr_rope_cache_table", _ptr(cos_out, f32, "cos_out", n_pos * head_dim),
              _ptr(sin_out, f32, "sin_out", n_pos * head_dim), n_pos, head_dim, C.c_float(theta), _stream())


def apply_rope_neox(x, cos_vals, sin_vals, seq, n_heads, head_dim):
    """kernels::apply_rope_neox (mod.rs:1247), in place (bit-exact)."""
    _lib.call("qasr_apply_rope_neox", _ptr(x, f32, "x", seq * n_heads * head_dim),
              _ptr(cos_vals, f32, "cos_vals", seq * head_dim), _ptr(sin_vals, f32, "sin_vals", seq * head_dim),
              seq, n_heads, head_dim, _stream())


def kv_append(k_cache, v_cache, k_new, v_new, layer, max_seq, kv_dim, start_pos, seq):
    """KvCache::k_at/v_at copies (decoder.rs:194-202, 805-810)."""
    cap = (layer + 1) * max_seq * kv_dim
    _lib.call("qasr_kv_append", _ptr(k_cache, f32, "k_cache", cap), _ptr(v_cache, f32, "v_cache", cap),
              _ptr(k_new, f32, "k_new", seq * kv_dim), _ptr(v_new, f32, "v_new", seq * kv_dim), layer, max_seq, kv_dim,
              start_pos, seq, _stream())


def sinusoidal_pe(pe, n_pos, d_model):
    """kernels::sinusoidal_pe (mod.rs:1213)."""
    _lib.call("qasr_sinusoidal_pe", _ptr(pe, f32, "pe", n_pos * d_model), n_pos, d_model, _stream())


def gelu(x, n):
    """kernels::gelu (mod.rs:948): tanh GELU with the reference's fast exp, in place."""
    _lib.call("qasr_gelu", _ptr(x, f32, "x", n), C.c_int64(n), _stream())


def gelu_erf(x, n):
    """Exact-erf GELU (encoder_gpu.rs:470 semantics), in place."""
    _lib.call("qasr_gelu_erf", _ptr(x, f32, "x", n), C.c_int64(n), _stream())


def silu(x, n):
    """kernels::silu (mod.rs:941), in place."""
    _lib.call("qasr_silu", _ptr(x, f32, "x", n), C.c_int64(n), _stream())


def swiglu_multiply(out, gate_up, seq_len, intermediate):
    """kernels::swiglu_multiply (mod.rs:965) over interleaved gate/up (bit-exact body)."""
    _lib.call("qasr_swiglu_multiply", _ptr(out, f32, "out", seq_len * intermediate),
              _ptr(gate_up, f32, "gate_up", 2 * seq_len * intermediate), seq_len, intermediate, _stream())


def add_inplace(a, b, n):
    """kernels::add_inplace (mod.rs:482)."""
    _lib.call("qasr_add_inplace", _ptr(a, f32, "a", n), _ptr(b, f32, "b", n), C.c_int64(n), _stream())


def linear_nobias_int8(y, x, w_int8, scales, seq_len, in_dim, out_dim):
    """kernels::linear_nobias_int8 (mod.rs:650)."""
    _lib.call("qasr_linear_nobias_int8", _ptr(y, f32, "y", seq_len * out_dim), _ptr(x, f32, "x", seq_len * in_dim),
              _ptr(w_int8, i8, "w_int8", out_dim * in_dim), _ptr(scales, f32, "scales", out_dim), seq_len, in_dim,
              out_dim, _stream())


def linear_int8(y, x, w_int8, scales, bias, seq_len, in_dim, out_dim):
    """kernels::linear_int8 (mod.rs:664); bias may be None."""
    _lib.call("qasr_linear_int8", _ptr(y, f32, "y", seq_len * out_dim), _ptr(x, f32, "x", seq_len * in_dim),
              _ptr(w_int8, i8, "w_int8", out_dim * in_dim), _ptr(scales, f32, "scales", out_dim),
              _ptr(bias, f32, "bias", out_dim), seq_len, in_dim, out_dim, _stream())


def linear(y, x, w, b, seq_len, in_dim, out_dim):
    """kernels::linear (mod.rs:531): y = x @ w^T + b, f32 weights; b may be None."""
    _lib.call("qasr_linear", _ptr(y, f32, "y", seq_len * out_dim), _ptr(x, f32, "x", seq_len * in_dim),
              _ptr(w, f32, "w", out_dim * in_dim), _ptr(b, f32, "b", out_dim), seq_len, in_dim, out_dim, _stream())


def linear_nobias(y, x, w, seq_len, in_dim, out_dim):
    """kernels::linear_nobias (mod.rs:567)."""
    _lib.call("qasr_linear_nobias", _ptr(y, f32, "y", seq_len * out_dim), _ptr(x, f32, "x", seq_len * in_dim),
              _ptr(w, f32, "w", out_dim * in_dim), seq_len, in_dim, out_dim, _stream())


def matmul_t(c, a, b, m, k, n):
    """kernels::matmul_t (mod.rs:503): c = a @ b^T."""
    _lib.call("qasr_matmul_t", _ptr(c, f32, "c", m * n), _ptr(a, f32, "a", m * k), _ptr(b, f32, "b", n * k), m, k, n,
              _stream())


def conv2d(out, inp, weight, bias, c_in, c_out, h_in, w_in, kh, kw, stride, padding):
    """kernels::conv2d (mod.rs:815): out [c_out, h_out*w_out]; bias may be None."""
    h_out = (h_in + 2 * padding - kh) // stride + 1
    w_out = (w_in + 2 * padding - kw) // stride + 1
    _lib.call("qasr_conv2d", _ptr(out, f32, "out", c_out * h_out * w_out), _ptr(inp, f32, "input", c_in * h_in * w_in),
              _ptr(weight, f32, "weight", c_out * c_in * kh * kw), _ptr(bias, f32, "bias", c_out), c_in, c_out, h_in,
              w_in, kh, kw, stride, padding, _stream())


def bidirectional_attention(out, q, k, v, seq, n_heads, head_dim, scale, window_starts, n_windows):
    """kernels::bidirectional_attention (mod.rs:1094); window_starts int32 [n_windows+1] on the device."""
    _lib.call("qasr_bidirectional_attention", _ptr(out, f32, "out", seq * n_heads * head_dim),
              _ptr(q, f32, "q", seq * n_heads * head_dim), _ptr(k, f32, "k", seq * n_heads * head_dim),
              _ptr(v, f32, "v", seq * n_heads * head_dim), seq, n_heads, head_dim, C.c_float(scale),
              _ptr(window_starts, i32, "window_starts", n_windows + 1), n_windows, _stream())


def mel_frames(n_samples: int) -> int:
    """Frames audio::mel_spectrogram produces for n_samples (0 = too short)."""
    return int(_lib.load().qasr_mel_frames(int(n_samples)))


def mel_spectrogram(mel, samples, n_samples):
    """audio::mel_spectrogram (audio.rs:271): mel [128, n_frames] from 16 kHz samples, both on the device."""
    n_frames = mel_frames(n_samples)
    _lib.call("qasr_mel_spectrogram", _ptr(mel, f32, "mel", 128 * max(n_frames, 1)),
              _ptr(samples, f32, "samples", n_samples), n_samples, _stream())


def causal_attention(out, q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, scale, q_offset):
    """kernels::causal_attention (mod.rs:1174)."""
    _lib.call("qasr_causal_attention", _ptr(out, f32, "out", seq_q * n_heads * head_dim),
              _ptr(q, f32, "q", seq_q * n_heads * head_dim), _ptr(k, f32, "k", seq_k * n_kv_heads * head_dim),
              _ptr(v, f32, "v", seq_k * n_kv_heads * head_dim), seq_q, seq_k, n_heads, n_kv_heads, head_dim,
              C.c_float(scale), q_offset, _stream())


def quantize_f32_to_int8(data, out_dim, in_dim, q_out, scales_out):
    """quantize_f32_to_int8 (quantize.rs:633) into preallocated q_out/scales_out (bit-exact)."""
    _lib.call("qasr_quantize_f32_to_int8", _ptr(data, f32, "data", out_dim * in_dim), C.c_int64(out_dim),
              C.c_int64(in_dim), _ptr(q_out, i8, "q_out", out_dim * in_dim), _ptr(scales_out, f32, "scales_out", out_dim),
              _stream())


def embed_gather(dst, table, ids, n, dim, vocab, scales=None, bad_id_flag=None):
    """Token embedding gather: f32 table (copy) or INT8 table + scales
    (tok_embed_int8_to_f32, decoder.rs:639)."""
    if table.dtype == i8:
        _lib.call("qasr_embed_gather_int8", _ptr(dst, f32, "dst", n * dim), _ptr(table, i8, "table", vocab * dim),
                  _ptr(scales, f32, "scales", vocab), _ptr(ids, i32, "ids", n), n, dim, C.c_int64(vocab),
                  _ptr(bad_id_flag, i32, "bad_id_flag"), _stream())
    else:
        _lib.call("qasr_embed_gather_f32", _ptr(dst, f32, "dst", n * dim), _ptr(table, f32, "table", vocab * dim),
                  _ptr(ids, i32, "ids", n), n, dim, C.c_int64(vocab), _ptr(bad_id_flag, i32, "bad_id_flag"), _stream())


def pre_attn_block(x_norm, x, w_in, seq, hidden, q, k, v, k_out, q_norm_w, k_norm_w, n_heads, n_kv_heads, head_dim,
                   eps, cos_tab, sin_tab, start_pos, k_cache, v_cache, layer, max_seq):
    """Fused decoder pre-attention block (decoder.rs:770-810): rms_norm, per-head
    q/k norm, NeoX RoPE, KV append -- one kernel, bit-exact."""
    q_dim, kv_dim = n_heads * head_dim, n_kv_heads * head_dim
    cap = (layer + 1) * max_seq * kv_dim
    tab = (start_pos + seq) * head_dim
    _lib.call("qasr_pre_attn_block", _ptr(x_norm, f32, "x_norm", seq * hidden), _ptr(x, f32, "x", seq * hidden),
              _ptr(w_in, f32, "w_in", hidden), seq, hidden, _ptr(q, f32, "q", seq * q_dim),
              _ptr(k, f32, "k", seq * kv_dim), _ptr(v, f32, "v", seq * kv_dim), _ptr(k_out, f32, "k_out", seq * kv_dim),
              _ptr(q_norm_w, f32, "q_norm_w", head_dim), _ptr(k_norm_w, f32, "k_norm_w", head_dim), n_heads,
              n_kv_heads, head_dim, C.c_float(eps), _ptr(cos_tab, f32, "cos_tab", tab), _ptr(sin_tab, f32, "sin_tab", tab),
              start_pos, _ptr(k_cache, f32, "k_cache", cap), _ptr(v_cache, f32, "v_cache", cap), layer, max_seq,
              _stream())


def ln_pe(out, x, weight, bias, pe, rows, hidden, n_pos, eps):
    """Encoder LayerNorm + sinusoidal position add (mod.rs:866 + encoder.rs:341-343)."""
    _lib.call("qasr_ln_pe", _ptr(out, f32, "out", rows * hidden), _ptr(x, f32, "x", rows * hidden),
              _ptr(weight, f32, "weight", hidden), _ptr(bias, f32, "bias", hidden), _ptr(pe, f32, "pe", n_pos * hidden),
              rows, hidden, n_pos, C.c_float(eps), _stream())


def ln_pe_gelu_erf(out, x, weight, bias, pe, rows, hidden, n_pos, eps, act, n_act):
    """LayerNorm + sinusoidal position add (mod.rs:866 + encoder.rs:341-343)
    and exact-erf GELU in place on the FFN activation, one launch."""
    _lib.call("qasr_ln_pe_gelu_erf", _ptr(out, f32, "out", rows * hidden), _ptr(x, f32, "x", rows * hidden),
              _ptr(weight, f32, "weight", hidden), _ptr(bias, f32, "bias", hidden), _ptr(pe, f32, "pe", n_pos * hidden),
              rows, hidden, n_pos, C.c_float(eps), _ptr(act, f32, "act", n_act), C.c_int64(n_act), _stream())


def int8_norm_gateup_swiglu(h, x, norm_w, w_gate_up, scales, M, hidden, inter, eps):
    """Post-attention RMSNorm + gate/up INT8 matvec + SwiGLU (decoder.rs:911-921)."""
    _lib.call("qasr_int8_norm_gateup_swiglu", _ptr(h, f32, "h", M * inter), _ptr(x, f32, "x", M * hidden),
              _ptr(norm_w, f32, "norm_w", hidden), _ptr(w_gate_up, i8, "w_gate_up", 2 * inter * hidden),
              _ptr(scales, f32, "scales", 2 * inter), M, hidden, inter, C.c_float(eps), _stream())


def int8_matvec_residual(x, a, w, scales, M, in_dim, out_dim):
    """x += INT8 matvec(a) (decoder.rs:907-908, 922-924)."""
    _lib.call("qasr_int8_matvec_residual", _ptr(x, f32, "x", M * out_dim), _ptr(a, f32, "a", M * in_dim),
              _ptr(w, i8, "w", out_dim * in_dim), _ptr(scales, f32, "scales", out_dim), M, in_dim, out_dim, _stream())


def final_norm_lmhead_argmax(ids_out, logits_out, x, norm_w, w, scales, M, hidden, vocab, eps):
    """Final RMSNorm + INT8 lm head + first-max argmax (decoder.rs:929-964)."""
    _lib.call("qasr_final_norm_lmhead_argmax", _ptr(ids_out, i32, "ids_out", M),
              _ptr(logits_out, f32, "logits_out", M * vocab), _ptr(x, f32, "x", M * hidden),
              _ptr(norm_w, f32, "norm_w", hidden), _ptr(w, i8, "w", vocab * hidden), _ptr(scales, f32, "scales", vocab),
              M, hidden, vocab, C.c_float(eps), _stream())
