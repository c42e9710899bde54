"""Python face of the streaming driver (qasr_stream_*): StreamState +
stream_push_audio and transcribe_stream (crates/qwen-asr/src/transcribe.rs:
445-1495) on the device engines, token ids out.

    s = Stream(dec, enc)                 # QwenCtx streaming defaults
    ids = s.push(buffer_so_far)          # newly committed ids
    ids += s.push(buffer_so_far, finalize=True)
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib


def default_config(**over) -> _lib.StreamConfig:
    cfg = _lib.StreamConfig()
    _lib.load().qasr_stream_default_config(C.byref(cfg))
    for k, v in over.items():
        setattr(cfg, k, v)
    return cfg


def _ids(a):
    a = np.ascontiguousarray(a if a is not None else [], dtype=np.int32)
    return a, (C.c_void_p(a.ctypes.data) if a.size else None)


class Stream:
    def __init__(self, dec, enc, **cfg):
        self.cfg = default_config(**cfg)
        self._h = _lib.load().qasr_stream_create(dec._h, enc._h, C.byref(self.cfg))
        if not self._h:
            raise _lib.QasrError(_lib.QASR_ERR_INVALID, "qasr_stream_create", _lib.last_error())
        self._cap = 4096

    def set_prompt(self, prompt=None, force=None) -> None:
        p, pp = _ids(prompt)
        f, fp = _ids(force)
        _lib.call("qasr_stream_set_prompt", self._h, pp, p.size, fp, f.size)

    def set_token_bytes(self, table) -> None:
        t, tp = _ids(table)
        _lib.call("qasr_stream_set_token_bytes", self._h, tp, t.size)

    def push(self, samples, finalize: bool = False) -> list[int]:
        """stream_push_audio: samples = all audio so far (numpy or CUDA tensor)."""
        if isinstance(samples, torch.Tensor):
            s = samples.detach().float().contiguous()
            torch.cuda.synchronize()  # read on the engine's stream
            ptr, n = s.data_ptr(), s.numel()
        else:
            s = np.ascontiguousarray(samples, dtype=np.float32)
            ptr, n = s.ctypes.data, s.size
        out = np.zeros(self._cap, np.int32)
        cnt = C.c_int(0)
        _lib.call("qasr_stream_push", self._h, C.c_void_p(ptr) if n else None, int(n), 1 if finalize else 0,
                  C.c_void_p(out.ctypes.data), self._cap, C.byref(cnt))
        del s
        return out[:cnt.value].tolist()

    def _list(self, fn) -> list[int]:
        cnt = C.c_int(0)
        _lib.call(fn, self._h, None, 0, C.byref(cnt))
        out = np.zeros(max(cnt.value, 1), np.int32)
        _lib.call(fn, self._h, C.c_void_p(out.ctypes.data), out.size, C.byref(cnt))
        return out[:cnt.value].tolist()

    def emitted(self) -> list[int]:
        return self._list("qasr_stream_emitted")

    def unfixed(self) -> list[int]:
        return self._list("qasr_stream_unfixed")

    def reset(self) -> None:
        _lib.call("qasr_stream_reset", self._h)

    @property
    def audio_cursor(self) -> int:
        return int(_lib.load().qasr_stream_audio_cursor(self._h))

    @property
    def trim_request(self) -> int:
        return int(_lib.load().qasr_stream_trim_request(self._h))

    def apply_trim(self, trim: int) -> None:
        _lib.call("qasr_stream_apply_trim", self._h, int(trim))

    def close(self) -> None:
        if self._h:
            _lib.load().qasr_stream_free(self._h)
            self._h = None


def transcribe_stream(dec, enc, samples, **cfg) -> list[int]:
    """transcribe_stream (transcribe.rs:445-800): the whole buffer chunk by
    chunk; the committed ids."""
    s = Stream(dec, enc, **dict(cfg, incremental=0))
    try:
        return s.push(samples, finalize=True)
    finally:
        s.close()


def tail_repeat_blocks(tokens, max_period: int) -> tuple[int, int]:
    t, tp = _ids(tokens)
    reps, period = C.c_int(0), C.c_int(0)
    _lib.call("qasr_stream_tail_repeat", tp, t.size, int(max_period), C.byref(reps), C.byref(period))
    return reps.value, period.value


def find_split_point(samples, target_sample: int, search_sec: float) -> int:
    s = np.ascontiguousarray(samples, dtype=np.float32)
    return int(_lib.load().qasr_find_split_point(C.c_void_p(s.ctypes.data), s.size, int(target_sample),
                                                 C.c_float(search_sec)))
