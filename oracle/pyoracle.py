"""numpy front end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as
the checker, and by bench.py's CPU-baseline / reference legs.  The product
package (qwenasr_b200) never imports this module.

Every function restates the reference function named in its docstring
(paths relative to crates/qwen-asr/src of ZhaoChaoqun/QwenASR) on float32
numpy arrays, returning new arrays instead of mutating the caller's (except
where noted).
"""
from __future__ import annotations

import ctypes as C
import math
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

f32p = C.POINTER(C.c_float)
i8p = C.POINTER(C.c_int8)
i32p = C.POINTER(C.c_int32)
u16p = C.POINTER(C.c_uint16)


def build(force: bool = False) -> str:
    """Compile liboracle.so with oracle/Makefile (g++, no GPU needed)."""
    if force or not os.path.exists(_LIB_PATH) or (
        os.path.getmtime(_LIB_PATH) < max(os.path.getmtime(os.path.join(_HERE, f)) for f in ("oracle.cpp", "oracle.h"))
    ):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _lib.orc_fast_exp.restype = C.c_float
        _lib.orc_fast_exp.argtypes = [C.c_float]
        _lib.orc_dot_f32.restype = C.c_float
        _lib.orc_dot_f32_generic.restype = C.c_float
        _lib.orc_argmax_first.restype = C.c_int
        _lib.orc_decoder_forward_int8.restype = C.c_int
        for name in ("orc_rms_norm", "orc_rms_norm_per_head", "orc_layer_norm", "orc_vec_scale_inplace",
                     "orc_vec_axpy_inplace", "orc_vec_scale_add", "orc_compute_rope_neox", "orc_rope_cache_table"):
            getattr(_lib, name).restype = None
    return _lib


def _p(a, t=f32p):
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def set_threads(n: int) -> None:
    """kernels::set_threads (mod.rs:288), capped at 16 like MAX_THREADS."""
    lib().orc_set_threads(int(n))


def rms_norm(x, w, eps=1e-6):
    """kernels::rms_norm -> avx::rms_norm_row (mod.rs:897, avx.rs:377)."""
    x = _f32(x)
    seq, hidden = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    lib().orc_rms_norm(_p(out), _p(x), _p(_f32(w)), seq, hidden, C.c_float(eps))
    return out


def rms_norm_per_head(x, w, n_heads, head_dim, eps=1e-6):
    """kernels::rms_norm_per_head (mod.rs:920); returns the normalised copy."""
    out = _f32(x).copy()
    seq = out.size // (n_heads * head_dim)
    lib().orc_rms_norm_per_head(_p(out), _p(_f32(w)), seq, n_heads, head_dim, C.c_float(eps))
    return out


def layer_norm(x, w, b, eps=1e-5):
    """kernels::layer_norm -> avx::layer_norm_row (mod.rs:866, avx.rs:420)."""
    x = _f32(x)
    seq, hidden = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    lib().orc_layer_norm(_p(out), _p(x), _p(_f32(w)), _p(_f32(b)), seq, hidden, C.c_float(eps))
    return out


def compute_rope_neox(positions, head_dim, theta=1e6):
    """kernels::compute_rope_neox (mod.rs:1228) -> (cos, sin) [seq, head_dim]."""
    pos = np.ascontiguousarray(positions, dtype=np.int32)
    cos = np.empty((pos.size, head_dim), np.float32)
    sin = np.empty_like(cos)
    lib().orc_compute_rope_neox(_p(cos), _p(sin), _p(pos, i32p), pos.size, head_dim, C.c_float(theta))
    return cos, sin


def rope_cache_table(n_pos, head_dim, theta=1e6):
    """RopeCache::ensure table rows 0..n_pos (decoder.rs:253)."""
    cos = np.empty((n_pos, head_dim), np.float32)
    sin = np.empty_like(cos)
    lib().orc_rope_cache_table(_p(cos), _p(sin), n_pos, head_dim, C.c_float(theta))
    return cos, sin


def apply_rope_neox(x, cos, sin, n_heads, head_dim):
    """kernels::apply_rope_neox (mod.rs:1247); returns the rotated copy."""
    out = _f32(x).copy()
    seq = out.size // (n_heads * head_dim)
    lib().orc_apply_rope_neox(_p(out), _p(_f32(cos)), _p(_f32(sin)), seq, n_heads, head_dim)
    return out


def sinusoidal_pe(n_pos, d_model):
    """kernels::sinusoidal_pe (mod.rs:1213)."""
    pe = np.empty((n_pos, d_model), np.float32)
    lib().orc_sinusoidal_pe(_p(pe), n_pos, d_model)
    return pe


def gelu(x):
    """kernels::gelu -> avx::gelu_inplace (tanh GELU, avx.rs:536)."""
    out = _f32(x).copy()
    lib().orc_gelu(_p(out), C.c_long(out.size))
    return out


def gelu_erf(x):
    """Exact-erf GELU (encoder_gpu.rs:470 semantics)."""
    out = _f32(x).copy()
    lib().orc_gelu_erf(_p(out), C.c_long(out.size))
    return out


def silu(x):
    out = _f32(x).copy()
    lib().orc_silu(_p(out), C.c_long(out.size))
    return out


def swiglu_multiply(gate_up, seq, inter):
    """kernels::swiglu_multiply -> avx::swiglu_interleaved (mod.rs:965, avx.rs:568)."""
    gu = _f32(gate_up)
    out = np.empty((seq, inter), np.float32)
    lib().orc_swiglu_multiply(_p(out), _p(gu), seq, inter)
    return out


def swiglu_decode(gate_up, inter):
    """Scalar decode SwiGLU with libm exp (decoder.rs:916-921)."""
    gu = _f32(gate_up)
    out = np.empty((inter,), np.float32)
    lib().orc_swiglu_decode(_p(out), _p(gu), inter)
    return out


def softmax(x):
    out = _f32(x).copy()
    rows, cols = out.reshape(-1, out.shape[-1]).shape
    lib().orc_softmax(_p(out), rows, cols)
    return out


def fast_exp(v: float) -> float:
    return lib().orc_fast_exp(C.c_float(v))


def dot_f32(a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_dot_f32(_p(a), _p(b), a.size)


def dot_f32_generic(a, b):
    a, b = _f32(a), _f32(b)
    return lib().orc_dot_f32_generic(_p(a), _p(b), a.size)


def vec_scale_inplace(dst, s):
    out = _f32(dst).copy()
    lib().orc_vec_scale_inplace(_p(out), C.c_float(s), out.size)
    return out


def vec_axpy_inplace(dst, src, alpha):
    out = _f32(dst).copy()
    lib().orc_vec_axpy_inplace(_p(out), _p(_f32(src)), C.c_float(alpha), out.size)
    return out


def vec_scale_add(dst, src, c):
    out = _f32(dst).copy()
    lib().orc_vec_scale_add(_p(out), _p(_f32(src)), C.c_float(c), out.size)
    return out


def linear_nobias_int8(x, w, scales):
    """kernels::linear_nobias_int8 (mod.rs:650) -> generic::int8_matvec_fused."""
    x = _f32(x)
    w = np.ascontiguousarray(w, dtype=np.int8)
    out_dim, in_dim = w.shape
    seq = x.size // in_dim
    y = np.empty((seq, out_dim), np.float32)
    lib().orc_linear_nobias_int8(_p(y), _p(x), _p(w, i8p), _p(_f32(scales)), seq, in_dim, out_dim)
    return y


def linear_int8(x, w, scales, bias):
    x = _f32(x)
    w = np.ascontiguousarray(w, dtype=np.int8)
    out_dim, in_dim = w.shape
    seq = x.size // in_dim
    y = np.empty((seq, out_dim), np.float32)
    lib().orc_linear_int8(_p(y), _p(x), _p(w, i8p), _p(_f32(scales)), _p(_f32(bias)), seq, in_dim, out_dim)
    return y


def linear(x, w, bias=None):
    """kernels::linear (mod.rs:531); fp64-accumulated stand-in for cblas_sgemm."""
    x, w = _f32(x), _f32(w)
    out_dim, in_dim = w.shape
    seq = x.size // in_dim
    y = np.empty((seq, out_dim), np.float32)
    b = _f32(bias) if bias is not None else None
    lib().orc_linear(_p(y), _p(x), _p(w), _p(b) if b is not None else None, seq, in_dim, out_dim)
    return y


def bf16_matvec(x, w_bf16, bias=None, generic=False):
    x = _f32(x)
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    out_dim, in_dim = w.shape
    y = np.empty((out_dim,), np.float32)
    b = _f32(bias) if bias is not None else None
    fn = lib().orc_bf16_matvec_generic if generic else lib().orc_bf16_matvec
    fn(_p(y), _p(x), _p(w, u16p), _p(b) if b is not None else None, in_dim, out_dim)
    return y


def causal_attention(q, k, v, seq_q, seq_k, n_heads, n_kv_heads, head_dim, q_offset, scale=None):
    """kernels::causal_attention (mod.rs:1174)."""
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(head_dim), dtype=np.float32)
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((seq_q, n_heads * head_dim), np.float32)
    lib().orc_causal_attention(_p(out), _p(q), _p(k), _p(v), seq_q, seq_k, n_heads, n_kv_heads, head_dim,
                               C.c_float(scale), q_offset)
    return out


def bidirectional_attention(q, k, v, seq, n_heads, head_dim, window_starts, scale=None):
    """kernels::bidirectional_attention (mod.rs:1094)."""
    if scale is None:
        scale = 1.0 / np.sqrt(np.float32(head_dim), dtype=np.float32)
    ws = np.ascontiguousarray(window_starts, dtype=np.int32)
    q, k, v = _f32(q), _f32(k), _f32(v)
    out = np.empty((seq, n_heads * head_dim), np.float32)
    lib().orc_bidirectional_attention(_p(out), _p(q), _p(k), _p(v), seq, n_heads, head_dim, C.c_float(scale),
                                      _p(ws, i32p), ws.size - 1)
    return out


def quantize_f32_to_int8(data):
    """quantize_f32_to_int8 (quantize.rs:633) -> (int8 [out,in], scales [out])."""
    d = _f32(data)
    out_dim, in_dim = d.shape
    q = np.empty((out_dim, in_dim), np.int8)
    s = np.empty((out_dim,), np.float32)
    lib().orc_quantize_f32_to_int8(_p(d), C.c_int64(out_dim), C.c_int64(in_dim), _p(q, i8p), _p(s))
    return q, s


def embed_int8(table, scales, token):
    """tok_embed_int8_to_f32 (decoder.rs:639)."""
    table = np.ascontiguousarray(table, dtype=np.int8)
    dim = table.shape[1]
    out = np.empty((dim,), np.float32)
    lib().orc_embed_int8(_p(out), _p(table, i8p), _p(_f32(scales)), int(token), dim)
    return out


def argmax_first(x) -> int:
    x = _f32(x)
    return lib().orc_argmax_first(_p(x), x.size)


def interleave_gate_up(gate, gate_s, up, up_s):
    """Row interleave of DecoderInt8::load (decoder.rs:699-719)."""
    inter, hidden = gate.shape
    fused = np.empty((2 * inter, hidden), np.int8)
    fs = np.empty((2 * inter,), np.float32)
    lib().orc_interleave_gate_up(_p(np.ascontiguousarray(gate), i8p), _p(_f32(gate_s)),
                                 _p(np.ascontiguousarray(up), i8p), _p(_f32(up_s)), inter, hidden,
                                 _p(fused, i8p), _p(fs))
    return fused, fs


# ---------------------------------------------------------------- decoder --
class _Layer(C.Structure):
    _fields_ = [(n, t) for n, t in (
        ("wq", i8p), ("wq_s", f32p), ("wk", i8p), ("wk_s", f32p), ("wv", i8p), ("wv_s", f32p),
        ("wo", i8p), ("wo_s", f32p), ("gate_up", i8p), ("gate_up_s", f32p), ("down", i8p), ("down_s", f32p),
        ("q_norm", f32p), ("k_norm", f32p), ("input_norm", f32p), ("post_attn_norm", f32p))]


class _Decoder(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
                ("theta", C.c_float), ("layers", C.POINTER(_Layer)), ("norm", f32p),
                ("lm_head", i8p), ("lm_head_s", f32p)]


class OracleDecoder:
    """DecoderInt8 (decoder.rs:652-747) over numpy weights.

    `weights` is the dict produced by qwenasr_b200-independent test helpers:
    per layer keys wq, wq_s, wk, wk_s, wv, wv_s, wo, wo_s, gate_up, gate_up_s,
    down, down_s, q_norm, k_norm, input_norm, post_attn_norm; plus norm,
    lm_head, lm_head_s at top level and a config dict `cfg`.
    """

    def __init__(self, weights):
        self.w = weights
        cfg = weights["cfg"]
        self.cfg = cfg
        self._layers = (_Layer * cfg["n_layers"])()
        self._keep = []
        for i, lw in enumerate(weights["layers"]):
            L = self._layers[i]
            for name, _ in _Layer._fields_:
                arr = lw[name]
                arr = np.ascontiguousarray(arr)
                self._keep.append(arr)
                setattr(L, name, _p(arr, i8p if arr.dtype == np.int8 else f32p))
        norm = _f32(weights["norm"])
        lm = np.ascontiguousarray(weights["lm_head"], dtype=np.int8)
        lms = _f32(weights["lm_head_s"])
        self._keep += [norm, lm, lms]
        self._dec = _Decoder(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                             cfg["head_dim"], cfg["vocab"], C.c_float(cfg["eps"]), C.c_float(cfg["theta"]),
                             self._layers, _p(norm), _p(lm, i8p), _p(lms))

    def new_kv(self, max_seq):
        c = self.cfg
        shape = (c["n_layers"], max_seq, c["n_kv_heads"] * c["head_dim"])
        return np.zeros(shape, np.float32), np.zeros(shape, np.float32)

    def forward(self, k_cache, v_cache, pos, embed, want_logits=False):
        """decoder_forward_int8 (decoder.rs:845); returns (token, logits|None, final_x)."""
        c = self.cfg
        logits = np.empty((c["vocab"],), np.float32) if want_logits else None
        xo = np.empty((c["hidden"],), np.float32)
        tok = lib().orc_decoder_forward_int8(C.byref(self._dec), _p(k_cache), _p(v_cache), k_cache.shape[1],
                                             int(pos), _p(_f32(embed)), _p(logits) if logits is not None else None,
                                             _p(xo))
        return tok, logits, xo

    def prefill(self, k_cache, v_cache, start_pos, embeds):
        """decoder_prefill_int8 (decoder.rs:751); returns the residual stream."""
        e = _f32(embeds)
        seq = e.shape[0]
        xo = np.empty_like(e)
        lib().orc_decoder_prefill_int8(C.byref(self._dec), _p(k_cache), _p(v_cache), k_cache.shape[1],
                                       int(start_pos), _p(e), seq, _p(xo))
        return xo


def pre_attn_block(x, w_in, q, k, v, q_norm_w, k_norm_w, n_heads, n_kv_heads, head_dim, eps,
                   cos_tab, sin_tab, start_pos, k_cache, v_cache):
    """Config-1 pre-attention block (decoder.rs:770-810 order).  q is returned
    rotated; k_cache/v_cache ([max_seq, kv_dim]) are written in place."""
    x = _f32(x)
    seq, hidden = x.shape
    xn = np.empty_like(x)
    q = _f32(q).copy()
    k = _f32(k).copy()
    lib().orc_pre_attn_block(_p(xn), _p(x), _p(_f32(w_in)), seq, hidden, _p(q), _p(k), _p(_f32(v)),
                             _p(_f32(q_norm_w)), _p(_f32(k_norm_w)), n_heads, n_kv_heads, head_dim,
                             C.c_float(eps), _p(_f32(cos_tab)), _p(_f32(sin_tab)), start_pos,
                             _p(k_cache), _p(v_cache))
    return xn, q, k


MEL_BINS, MEL_FREQS, MEL_NFFT, MEL_HOP = 128, 201, 400, 160


def mel_filters():
    """build_mel_filters (audio.rs:226-263): Slaney filters [128, 201]."""
    f = np.empty((MEL_BINS, MEL_FREQS), np.float32)
    lib().orc_mel_filters(_p(f))
    return f


def mel_tables():
    """The periodic Hann window [400] and DFT cos/sin rows [201, 400] (audio.rs:303-325)."""
    w = np.empty(MEL_NFFT, np.float32)
    c = np.empty((MEL_FREQS, MEL_NFFT), np.float32)
    s = np.empty((MEL_FREQS, MEL_NFFT), np.float32)
    lib().orc_mel_tables(_p(w), _p(c), _p(s))
    return w, c, s


def mel_spectrogram(samples):
    """audio::mel_spectrogram (audio.rs:271-385): [128, n_frames] log-mel of
    16 kHz samples, or None when the input is too short for one frame."""
    x = _f32(samples).ravel()
    n_frames = len(x) // MEL_HOP
    if n_frames == 0:
        return None
    mel = np.empty((MEL_BINS, n_frames), np.float32)
    got = lib().orc_mel_spectrogram(_p(mel), _p(x), len(x))
    assert got == n_frames
    return mel


# ------------------------------------------------------------ encoder --
_CONV_HIDDEN = 480


def _conv3x3s2(x, w, b, c_in, c_out, h, wd):
    """kernels::conv2d (mod.rs:790-860) with a 3x3 kernel, stride 2, padding 1:
    an im2col product in float64 (cblas_sgemm's stand-in)."""
    ho, wo = (h - 1) // 2 + 1, (wd - 1) // 2 + 1
    xp = np.zeros((c_in, h + 2, wd + 2))
    xp[:, 1:1 + h, 1:1 + wd] = x.reshape(c_in, h, wd)
    cols = np.empty((c_in * 9, ho * wo))
    for ic in range(c_in):
        for ki in range(3):
            for kj in range(3):
                cols[(ic * 3 + ki) * 3 + kj] = xp[ic, ki:ki + 2 * ho:2, kj:kj + 2 * wo:2].ravel()
    return ((w.reshape(c_out, -1).astype(np.float64) @ cols) + b[:, None]).astype(np.float32), ho, wo


def _enc_proj(x, d, name, bias_key):
    """kernels::linear (f32 "<name>" or "<name>_w") or linear_int8 ("<name>" + "<name>_s")."""
    b = d[bias_key] if bias_key else None
    if name + "_s" in d:
        return linear_int8(x, d[name], d[name + "_s"], b) if b is not None else linear_nobias_int8(
            x, d[name], d[name + "_s"])
    return linear(x, d[name] if name in d else d[name + "_w"], b)


def encoder_forward(w, cfg, mel):
    """Encoder::forward (encoder.rs:243-415) composed from the restated
    kernels: per 100-frame chunk the conv stem (3 x conv + GELU), conv_out
    and the sinusoidal positions; windowed layers; post LayerNorm and the two
    projections.  mel [128, frames] -> [tokens, output_dim].  Matrices given
    with scales ("<m>", "<m>_s") run as EncoderInt8::forward does
    (encoder.rs:562-667: linear_int8 / linear_nobias_int8)."""
    D, CH, cs = cfg["d_model"], _CONV_HIDDEN, cfg["chunk_size"]
    frames = mel.shape[1]
    xs = []
    for s in range(0, frames, cs):
        chunk = mel[:, s:s + cs]
        c1, h1, w1 = _conv3x3s2(chunk, w["conv1_w"], w["conv1_b"], 1, CH, 128, chunk.shape[1])
        c1 = gelu(c1.ravel()).reshape(c1.shape)
        c2, h2, w2 = _conv3x3s2(c1, w["conv2_w"], w["conv2_b"], CH, CH, h1, w1)
        c2 = gelu(c2.ravel()).reshape(c2.shape)
        c3, h3, w3 = _conv3x3s2(c2, w["conv3_w"], w["conv3_b"], CH, CH, h2, w2)
        c3 = gelu(c3.ravel()).reshape(CH, h3, w3)
        reshaped = np.ascontiguousarray(c3.transpose(2, 0, 1).reshape(w3, CH * h3))
        xs.append(_enc_proj(reshaped, w, "conv_out", None) + sinusoidal_pe(w3, D))
    x = np.concatenate(xs).astype(np.float32)
    T = x.shape[0]
    tpc = 13
    wsize = tpc * (cfg["n_window_infer"] // cs)
    starts = np.array(list(range(0, T, wsize)) + [T], np.int32)
    scale = np.float32(1.0 / math.sqrt(cfg["head_dim"]))
    for L in w["layers"]:
        xn = layer_norm(x, L["attn_norm_w"], L["attn_norm_b"], 1e-5)
        q = _enc_proj(xn, L, "wq", "bq")
        k = _enc_proj(xn, L, "wk", "bk")
        v = _enc_proj(xn, L, "wv", "bv")
        a = bidirectional_attention(q, k, v, T, cfg["n_heads"], cfg["head_dim"], starts, scale)
        x = (x + _enc_proj(a, L, "wo", "bo")).astype(np.float32)
        xn = layer_norm(x, L["ffn_norm_w"], L["ffn_norm_b"], 1e-5)
        mid = gelu(_enc_proj(xn, L, "fc1", "fc1_b").ravel()).reshape(T, -1)
        x = (x + _enc_proj(mid, L, "fc2", "fc2_b")).astype(np.float32)
    xn = layer_norm(x, w["ln_post_w"], w["ln_post_b"], 1e-5)
    p1 = gelu(_enc_proj(xn, w, "proj1", "proj1_b").ravel()).reshape(T, -1)
    return _enc_proj(p1, w, "proj2", "proj2_b")
