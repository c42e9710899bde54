"""ctypes binding of libqwenasr_b200.so (the C ABI in include/qwenasr_cuda.h).

The shared library is built in-tree by qwenasr_b200/build.py.  Loading fails
loudly when it is missing: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqwenasr_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "qwenasr_cuda.h")

QASR_OK = 0
QASR_ERR_INVALID = -1
QASR_ERR_CUDA = -2
QASR_ERR_ALLOC = -3
QASR_ERR_UNSUPPORTED = -4
QASR_ERR_TIMEOUT = -5


class QasrError(RuntimeError):
    def __init__(self, code: int, fn: str, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


class DecoderConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("inter", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("vocab", C.c_int), ("eps", C.c_float),
                ("theta", C.c_float), ("max_batch", C.c_int), ("max_seq", C.c_int), ("embed_is_int8", C.c_int)]


class DecLayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "wq", "wq_s", "wk", "wk_s", "wv", "wv_s", "wo", "wo_s", "gate_up", "gate_up_s", "down", "down_s",
        "q_norm", "k_norm", "input_norm", "post_attn_norm")]


P = C.c_void_p
I = C.c_int
I64 = C.c_int64
F = C.c_float

# name -> (restype, argtypes); every function returning int is a status.
_SIGS = {
    "qasr_last_error": (C.c_char_p, []),
    "qasr_version": (C.c_char_p, []),
    "qasr_rms_norm": (I, [P, P, P, I, I, F, P]),
    "qasr_rms_norm_per_head": (I, [P, P, I, I, I, F, P]),
    "qasr_layer_norm": (I, [P, P, P, P, I, I, F, P]),
    "qasr_compute_rope_neox": (I, [P, P, P, I, I, F, P]),
    "qasr_rope_cache_table": (I, [P, P, I, I, F, P]),
    "qasr_apply_rope_neox": (I, [P, P, P, I, I, I, P]),
    "qasr_kv_append": (I, [P, P, P, P, I, I, I, I, I, P]),
    "qasr_sinusoidal_pe": (I, [P, I, I, P]),
    "qasr_gelu": (I, [P, I64, P]),
    "qasr_gelu_erf": (I, [P, I64, P]),
    "qasr_silu": (I, [P, I64, P]),
    "qasr_swiglu_multiply": (I, [P, P, I, I, P]),
    "qasr_add_inplace": (I, [P, P, I64, P]),
    "qasr_linear_nobias_int8": (I, [P, P, P, P, I, I, I, P]),
    "qasr_linear_int8": (I, [P, P, P, P, P, I, I, I, P]),
    "qasr_causal_attention": (I, [P, P, P, P, I, I, I, I, I, F, I, P]),
    "qasr_linear": (I, [P, P, P, P, I, I, I, P]),
    "qasr_linear_nobias": (I, [P, P, P, I, I, I, P]),
    "qasr_matmul_t": (I, [P, P, P, I, I, I, P]),
    "qasr_conv2d": (I, [P, P, P, P, I, I, I, I, I, I, I, I, P]),
    "qasr_bidirectional_attention": (I, [P, P, P, P, I, I, I, F, P, I, P]),
    "qasr_mel_frames": (I, [I]),
    "qasr_mel_spectrogram": (I, [P, P, I, P]),
    "qasr_quantize_f32_to_int8": (I, [P, I64, I64, P, P, P]),
    "qasr_embed_gather_f32": (I, [P, P, P, I, I, I64, P, P]),
    "qasr_embed_gather_int8": (I, [P, P, P, P, I, I, I64, P, P]),
    "qasr_pre_attn_block": (I, [P, P, P, I, I, P, P, P, P, P, P, I, I, I, F, P, P, I, P, P, I, I, P]),
    "qasr_ln_pe": (I, [P, P, P, P, P, I, I, I, F, P]),
    "qasr_ln_pe_gelu_erf": (I, [P, P, P, P, P, I, I, I, F, P, I64, P]),
    "qasr_int8_norm_gateup_swiglu": (I, [P, P, P, P, P, I, I, I, F, P]),
    "qasr_int8_matvec_residual": (I, [P, P, P, P, I, I, I, P]),
    "qasr_final_norm_lmhead_argmax": (I, [P, P, P, P, P, P, I, I, I, F, P]),
    "qasr_final_norm_lmhead_argmax_noalloc": (I, [P, P, P, P, P, P, I, I, I, F, P]),
    "qasr_decoder_create": (P, [C.POINTER(DecoderConfig), I]),
    "qasr_decoder_free": (None, [P]),
    "qasr_decoder_set_layer": (I, [P, I, C.POINTER(DecLayerWeights)]),
    "qasr_decoder_set_globals": (I, [P, P, P, P, P, P]),
    "qasr_decoder_kv": (I, [P, I, C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "qasr_decoder_step": (I, [P, P, P, I, P]),
    "qasr_decoder_prefill": (I, [P, I, P, I, I]),
    "qasr_decoder_prefill_batch": (I, [P, P, P, P, P, I]),
    "qasr_decoder_prefill_hidden": (P, [P]),
    "qasr_decoder_step_device": (I, [P, P, P, I, P]),
    "qasr_decoder_stream": (P, [P]),
    "qasr_decoder_set_gate_up": (I, [P, I, P, P, P, P]),
    "qasr_decoder_get_config": (P, [P]),
    "qasr_decoder_device": (I, [P]),
    "qasr_decoder_embed": (I, [P, P, I, P]),
    "qasr_decoder_keep_logits": (I, [P, I]),
    "qasr_decoder_set_step_kernel": (I, [P, I]),
    "qasr_decoder_step_kernel": (I, [P, I]),
    "qasr_decoder_trace": (I, [P, P, I64]),
    "qasr_decoder_trace_stride": (I, [P]),
    "qasr_decoder_logits": (P, [P]),
    "qasr_decoder_step_bytes": (I64, [P, P, I]),
    "qasr_decoder_profile_step": (I, [P, P, P, I, P, P, I]),
}

class EncoderConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("d_model", "n_layers", "n_heads", "head_dim", "ffn_dim", "output_dim",
                                       "chunk_size", "n_window_infer")]


class EncLayerWeights(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "attn_norm_w", "attn_norm_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ffn_norm_w", "ffn_norm_b",
        "fc1_w", "fc1_b", "fc2_w", "fc2_b")]


class StreamConfig(C.Structure):
    _fields_ = [("chunk_sec", C.c_float), ("rollback", C.c_int), ("unfixed_chunks", C.c_int),
                ("max_new_tokens", C.c_int), ("past_text_conditioning", C.c_int), ("incremental", C.c_int)]


class EncLayerWeightsInt8(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in (
        "attn_norm_w", "attn_norm_b", "wq", "wq_s", "bq", "wk", "wk_s", "bk", "wv", "wv_s", "bv", "wo", "wo_s", "bo",
        "ffn_norm_w", "ffn_norm_b", "fc1", "fc1_s", "fc1_b", "fc2", "fc2_s", "fc2_b")]


_SIGS.update({
    "qasr_encoder_create": (P, [C.POINTER(EncoderConfig), I]),
    "qasr_encoder_free": (None, [P]),
    "qasr_encoder_set_conv": (I, [P, P, P, P, P, P, P, P]),
    "qasr_encoder_set_layer": (I, [P, I, C.POINTER(EncLayerWeights)]),
    "qasr_encoder_set_post": (I, [P, P, P, P, P, P, P]),
    "qasr_encoder_tokens": (I, [P, I]),
    "qasr_encoder_forward": (I, [P, P, I, P, I, C.POINTER(C.c_int)]),
    "qasr_encoder_forward_batch": (I, [P, P, P, I, P, P, P]),
    "qasr_encoder_get_config": (P, [P]),
    "qasr_encoder_set_conv_int8": (I, [P, P, P, P, P, P, P, P, P]),
    "qasr_encoder_set_layer_int8": (I, [P, I, C.POINTER(EncLayerWeightsInt8)]),
    "qasr_encoder_set_post_int8": (I, [P, P, P, P, P, P, P, P, P]),
    "qasr_qint8_open": (P, [C.c_char_p]),
    "qasr_qint8_close": (None, [P]),
    "qasr_qint8_version": (I, [P]),
    "qasr_qint8_count": (I, [P]),
    "qasr_qint8_find": (I, [P, C.c_char_p]),
    "qasr_qint8_tensor": (I, [P, I, C.POINTER(C.c_char_p), C.POINTER(C.c_int), C.POINTER(C.c_int),
                              C.POINTER(C.c_int64), C.POINTER(C.c_void_p), C.POINTER(C.c_void_p)]),
    "qasr_qint8_detect": (I, [P, C.POINTER(DecoderConfig), C.POINTER(EncoderConfig)]),
    "qasr_qint8_load_decoder": (I, [P, P]),
    "qasr_qint8_load_encoder": (I, [P, P]),
    "qasr_stream_default_config": (None, [C.POINTER(StreamConfig)]),
    "qasr_stream_create": (P, [P, P, C.POINTER(StreamConfig)]),
    "qasr_stream_free": (None, [P]),
    "qasr_stream_set_prompt": (I, [P, P, I, P, I]),
    "qasr_stream_set_token_bytes": (I, [P, P, I]),
    "qasr_stream_push": (I, [P, P, I64, I, P, I, C.POINTER(C.c_int)]),
    "qasr_stream_reset": (I, [P]),
    "qasr_stream_audio_cursor": (I64, [P]),
    "qasr_stream_trim_request": (I64, [P]),
    "qasr_stream_apply_trim": (I, [P, I64]),
    "qasr_stream_emitted": (I, [P, P, I, C.POINTER(C.c_int)]),
    "qasr_stream_unfixed": (I, [P, P, I, C.POINTER(C.c_int)]),
    "qasr_stream_tail_repeat": (I, [P, I, I, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "qasr_find_split_point": (I64, [P, I64, I64, F]),
    "qasr_plan_segments": (I, [P, I64, F, F, P, I, C.POINTER(C.c_int)]),
    "qasr_encoder_device": (I, [P]),
    "qasr_transcribe_prompt_len": (I, [I, I, I]),
    "qasr_transcribe_batch": (I, [P, P, P, P, I, P, I, P, I, I, I, P, I, P]),
    "qasr_transcribe_lanes": (I, [P, P, I, P, P, I, P, I, P, I, I, I, P, I, P]),
})

KERNEL_CLASSES = ("embed", "norm", "qkv", "qkv_post", "attn", "oproj", "gateup", "down", "lmhead", "step")

_lib = None


def header_functions() -> list[str]:
    """Names of the functions declared in include/qwenasr_cuda.h."""
    txt = open(HEADER).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(qasr_[a-z0-9_]+)\s*\(", txt)))


def load(path: str | None = None):
    """Load the library (once).  Raises if the in-tree .so has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = path or LIB_PATH
    if not os.path.exists(path):
        raise RuntimeError(f"{path} is missing: build it with `python -m qwenasr_b200.build` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(path)
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def last_error() -> str:
    return (load().qasr_last_error() or b"").decode()


def check(code: int, fn: str) -> None:
    if code != QASR_OK:
        raise QasrError(code, fn, last_error())


def call(name: str, *args) -> None:
    """Call a status-returning entry point and raise QasrError on failure."""
    check(getattr(load(), name)(*args), name)
