"""Python face of the audio encoder engine (qasr_encoder_*): Encoder::forward
(crates/qwen-asr/src/encoder.rs:243-415) with f32 weights on one GPU."""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib


def _ptr(a, keep):
    if isinstance(a, torch.Tensor):
        a = a.detach().contiguous()
        if a.dtype != torch.int8:
            a = a.float()
        keep.append(a)
        return C.c_void_p(a.data_ptr())
    arr = np.ascontiguousarray(a, dtype=np.int8 if np.asarray(a).dtype == np.int8 else np.float32)
    keep.append(arr)
    return C.c_void_p(arr.ctypes.data)


class Encoder:
    def __init__(self, cfg: dict, device: int = 0):
        self.cfg = dict(cfg)
        self.device = device
        c = _lib.EncoderConfig(cfg["d_model"], cfg["n_layers"], cfg["n_heads"], cfg["head_dim"], cfg["ffn_dim"],
                               cfg["output_dim"], cfg["chunk_size"], cfg["n_window_infer"])
        self._h = _lib.load().qasr_encoder_create(C.byref(c), device)
        if not self._h:
            raise _lib.QasrError(_lib.QASR_ERR_INVALID, "qasr_encoder_create", _lib.last_error())

    def set_weights(self, w: dict) -> None:
        """f32 weights (encoder_weights_np keys), or the INT8 form of
        EncoderInt8 when the dict carries scales ("wq_s", "conv_out_s", ...;
        see synthetic.quantize_encoder)."""
        keep = []
        if "conv_out_s" in w:
            _lib.call("qasr_encoder_set_conv_int8", self._h, *[_ptr(w[k], keep) for k in (
                "conv1_w", "conv1_b", "conv2_w", "conv2_b", "conv3_w", "conv3_b")],
                _ptr(w["conv_out"], keep), _ptr(w["conv_out_s"], keep))
        else:
            _lib.call("qasr_encoder_set_conv", self._h, *[_ptr(w[k], keep) for k in (
                "conv1_w", "conv1_b", "conv2_w", "conv2_b", "conv3_w", "conv3_b", "conv_out_w")])
        for i, lw in enumerate(w["layers"]):
            if "wq_s" in lw:
                s = _lib.EncLayerWeightsInt8(*[_ptr(lw[n], keep) for n, _ in _lib.EncLayerWeightsInt8._fields_])
                _lib.call("qasr_encoder_set_layer_int8", self._h, i, C.byref(s))
            else:
                s = _lib.EncLayerWeights(*[_ptr(lw[n], keep) for n, _ in _lib.EncLayerWeights._fields_])
                _lib.call("qasr_encoder_set_layer", self._h, i, C.byref(s))
        if "proj1_s" in w:
            _lib.call("qasr_encoder_set_post_int8", self._h, *[_ptr(w[k], keep) for k in (
                "ln_post_w", "ln_post_b", "proj1", "proj1_s", "proj1_b", "proj2", "proj2_s", "proj2_b")])
        else:
            _lib.call("qasr_encoder_set_post", self._h, *[_ptr(w[k], keep) for k in (
                "ln_post_w", "ln_post_b", "proj1_w", "proj1_b", "proj2_w", "proj2_b")])

    def tokens(self, mel_frames: int) -> int:
        return _lib.load().qasr_encoder_tokens(self._h, int(mel_frames))

    def forward(self, mel) -> torch.Tensor:
        """mel [128, frames] (numpy or CUDA tensor) -> [tokens, output_dim] on the device."""
        keep = []
        frames = mel.shape[1]
        T = self.tokens(frames)
        out = torch.empty(T, self.cfg["output_dim"], dtype=torch.float32, device=f"cuda:{self.device}")
        n = C.c_int(0)
        _lib.call("qasr_encoder_forward", self._h, _ptr(mel, keep), int(frames), C.c_void_p(out.data_ptr()), T,
                  C.byref(n))
        return out

    def forward_batch(self, mels) -> list[torch.Tensor]:
        """Several mels [128, frames_i] in one pass -> [tokens_i, output_dim] each."""
        keep = []
        n = len(mels)
        ptrs = (C.c_void_p * n)(*[_ptr(m, keep) for m in mels])
        frames = (C.c_int * n)(*[int(m.shape[1]) for m in mels])
        outs = [torch.empty(self.tokens(f), self.cfg["output_dim"], dtype=torch.float32,
                            device=f"cuda:{self.device}") for f in frames]
        optr = (C.c_void_p * n)(*[o.data_ptr() for o in outs])
        rows = (C.c_int * n)(*[o.shape[0] for o in outs])
        got = (C.c_int * n)()
        _lib.call("qasr_encoder_forward_batch", self._h, ptrs, frames, n, optr, rows, got)
        return outs

    def close(self) -> None:
        if self._h:
            _lib.load().qasr_encoder_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
