"""Python face of qasr_transcribe_batch / qasr_transcribe_lanes:
transcribe_segment (crates/qwen-asr/src/transcribe.rs:67-244) and the
segmented transcribe_audio (transcribe.rs:294-420), token ids out.

Audio -> log-mel -> encoder -> prompt embeddings (the reference's special
tokens, transcribe.rs:11-13) -> prefill -> greedy decode, for up to
`dec.max_batch` independent segments decoded together; any number of
segments over one or more engine lanes.  Text decoding stays with the
caller's tokenizer, as in the reference's host.
"""
from __future__ import annotations

import ctypes as C
from typing import Sequence

import numpy as np
import torch

from . import _lib

PREFIX_HEAD = (151644, 8948, 198)
PREFIX_TAIL = (151645, 198, 151644, 872, 198, 151669)
SUFFIX_BASE = (151670, 151645, 198, 151644, 77091, 198)
TOKEN_ENDOFTEXT, TOKEN_IM_END = 151643, 151645


def prompt_len(n_audio_tokens: int, n_prompt: int = 0, n_force: int = 0) -> int:
    return int(_lib.load().qasr_transcribe_prompt_len(int(n_audio_tokens), int(n_prompt), int(n_force)))


def _ids_arg(ids):
    if ids is None or len(ids) == 0:
        return None, 0, None
    a = np.ascontiguousarray(ids, dtype=np.int32)
    return C.c_void_p(a.ctypes.data), len(a), a


def _segment_args(segments):
    """ctypes arrays of the segments' sample pointers and lengths, and the
    arrays that keep them alive."""
    n = len(segments)
    keep = []
    ptrs = (C.c_void_p * n)()
    lens = (C.c_int * n)()
    for i, s in enumerate(segments):
        if isinstance(s, torch.Tensor):
            s = s.detach().float().contiguous()
            ptrs[i] = s.data_ptr()
            lens[i] = s.numel()
        else:
            s = np.ascontiguousarray(s, dtype=np.float32)
            ptrs[i] = s.ctypes.data
            lens[i] = s.size
        keep.append(s)
    if any(isinstance(s, torch.Tensor) for s in keep):
        torch.cuda.synchronize()  # the engines read them on their own streams
    return ptrs, lens, keep


def transcribe_ids(dec, enc, segments: Sequence, max_new: int, stop_at_eos: bool = False, prompt_tokens=None,
                   force_tokens=None) -> list[list[int]]:
    """Greedy token ids of each segment (16 kHz f32 samples: numpy arrays or
    CUDA tensors).  With stop_at_eos the ids end at the first end-of-text /
    im_end token (included), as the reference's decode loop stops there."""
    n = len(segments)
    if n == 0:
        return []
    ptrs, lens, keep = _segment_args(segments)
    pp, npr, pa = _ids_arg(prompt_tokens)
    fp, nfr, fa = _ids_arg(force_tokens)
    ids = np.zeros((n, max_new), np.int32)
    counts = (C.c_int * n)()
    _lib.call("qasr_transcribe_batch", dec._h, enc._h, ptrs, lens, n, pp, npr, fp, nfr, int(max_new), 1 if stop_at_eos else 0,
              C.c_void_p(ids.ctypes.data), int(max_new), counts)
    del pa, fa, keep
    return [ids[i, :counts[i]].tolist() for i in range(n)]


def transcribe_lanes(lanes: Sequence, segments: Sequence, max_new: int, stop_at_eos: bool = False,
                     prompt_tokens=None, force_tokens=None) -> list[list[int]]:
    """transcribe_ids over any number of independent segments, spread over
    engine lanes: lanes = [(dec, enc), ...], one decoder + encoder pair each
    (qasr_transcribe_lanes).  Lanes on one GPU overlap one another's work;
    the ids of a segment do not depend on the lane that ran it."""
    n = len(segments)
    if n == 0:
        return []
    L = len(lanes)
    decs = (C.c_void_p * L)(*[d._h for d, _ in lanes])
    encs = (C.c_void_p * L)(*[e._h for _, e in lanes])
    ptrs, lens, keep = _segment_args(segments)
    pp, npr, pa = _ids_arg(prompt_tokens)
    fp, nfr, fa = _ids_arg(force_tokens)
    ids = np.zeros((n, max_new), np.int32)
    counts = (C.c_int * n)()
    _lib.call("qasr_transcribe_lanes", decs, encs, L, ptrs, lens, n, pp, npr, fp, nfr, int(max_new),
              1 if stop_at_eos else 0, C.c_void_p(ids.ctypes.data), int(max_new), counts)
    del pa, fa, keep
    return [ids[i, :counts[i]].tolist() for i in range(n)]


def plan_segments(samples, segment_sec: float, search_sec: float = 3.0) -> list[tuple[int, int]]:
    """transcribe_audio's split of long audio (transcribe.rs:317-345):
    [(start, end)] per segment, cut at the quietest 100 ms near every
    segment_sec (no split when segment_sec <= 0)."""
    s = np.ascontiguousarray(samples, dtype=np.float32)
    starts = np.zeros(128, np.int64)
    n = C.c_int(0)
    _lib.call("qasr_plan_segments", C.c_void_p(s.ctypes.data) if s.size else None, s.size, C.c_float(segment_sec),
              C.c_float(search_sec), C.c_void_p(starts.ctypes.data), starts.size, C.byref(n))
    st = starts[:n.value].tolist()
    return [(a, b) for a, b in zip(st, st[1:] + [s.size])]


def transcribe_audio(dec, enc, samples, max_new: int, segment_sec: float = 0.0, search_sec: float = 3.0,
                     stop_at_eos: bool = True, prompt_tokens=None, force_tokens=None, lanes=None) -> list[list[int]]:
    """transcribe_audio (transcribe.rs:294-420) without past-text
    conditioning: the planned segments (each shorter than 0.5 s zero-padded
    to 0.5 s, as the reference does) transcribed independently, up to
    dec.max_batch at a time, or over `lanes` ([(dec, enc), ...], dec and enc
    then unused) when given; the ids of every segment in order."""
    s = np.ascontiguousarray(samples, dtype=np.float32)
    segs = []
    for a, b in plan_segments(s, segment_sec, search_sec):
        seg = s[a:b]
        if seg.size < 8000:
            seg = np.concatenate([seg, np.zeros(8000 - seg.size, np.float32)])
        segs.append(seg)
    return transcribe_lanes(lanes or [(dec, enc)], segs, max_new, stop_at_eos, prompt_tokens, force_tokens)
