"""INT8 decoder engine on one B200: the host face of qasr_decoder.

Mirrors DecoderInt8 + KvCache + decoder_forward_int8 of the reference
(crates/qwen-asr/src/decoder.rs:130-228, 652-965) for a batch of up to 8
independent sequences: weights are uploaded once, each sequence owns a KV
cache slot, and one call advances every sequence by one greedy token.  All
math runs in libqwenasr_b200.so; this module only owns handles and buffers.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib

LAYER_KEYS = ("wq", "wq_s", "wk", "wk_s", "wv", "wv_s", "wo", "wo_s", "gate_up", "gate_up_s", "down", "down_s",
              "q_norm", "k_norm", "input_norm", "post_attn_norm")


class _DevArray:
    """__cuda_array_interface__ view of engine-owned device memory."""

    def __init__(self, ptr, shape, typestr="<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def _host_or_dev_ptr(a, keep):
    if isinstance(a, torch.Tensor):
        if not a.is_contiguous():
            a = a.contiguous()
        keep.append(a)
        return C.c_void_p(a.data_ptr())
    arr = np.ascontiguousarray(a)
    keep.append(arr)
    return C.c_void_p(arr.ctypes.data)


class Decoder:
    """One qasr_decoder: config dict keys hidden, inter, n_layers, n_heads,
    n_kv_heads, head_dim, vocab, eps, theta."""

    def __init__(self, cfg: dict, device: int = 0, max_batch: int = 8, max_seq: int = 2048,
                 embed_is_int8: bool = False):
        self.cfg = dict(cfg)
        self.device = device
        self.max_batch = max_batch
        self.max_seq = max_seq
        c = _lib.DecoderConfig(cfg["hidden"], cfg["inter"], cfg["n_layers"], cfg["n_heads"], cfg["n_kv_heads"],
                               cfg["head_dim"], cfg["vocab"], cfg["eps"], cfg["theta"], max_batch, max_seq,
                               1 if embed_is_int8 else 0)
        lib = _lib.load()
        self._h = lib.qasr_decoder_create(C.byref(c), device)
        if not self._h:
            raise _lib.QasrError(_lib.QASR_ERR_INVALID, "qasr_decoder_create", _lib.last_error())
        self.kv_dim = cfg["n_kv_heads"] * cfg["head_dim"]

    # ---------------------------------------------------------------- weights
    def set_layer(self, i: int, w: dict) -> None:
        keep = []
        s = _lib.DecLayerWeights(*[_host_or_dev_ptr(w[k], keep) for k in LAYER_KEYS])
        _lib.call("qasr_decoder_set_layer", self._h, i, C.byref(s))

    def set_globals(self, embed, norm, lm_head=None, lm_head_s=None, embed_scales=None) -> None:
        keep = []
        _lib.call("qasr_decoder_set_globals", self._h, _host_or_dev_ptr(embed, keep),
                  _host_or_dev_ptr(embed_scales, keep) if embed_scales is not None else None,
                  _host_or_dev_ptr(norm, keep), _host_or_dev_ptr(lm_head, keep) if lm_head is not None else None,
                  _host_or_dev_ptr(lm_head_s, keep) if lm_head_s is not None else None)

    # --------------------------------------------------------------- caches
    def kv(self, slot: int):
        """(k, v) torch views of sequence `slot`'s cache [n_layers, max_seq, kv_dim]."""
        k = C.c_void_p()
        v = C.c_void_p()
        _lib.call("qasr_decoder_kv", self._h, slot, C.byref(k), C.byref(v))
        shape = (self.cfg["n_layers"], self.max_seq, self.kv_dim)
        with torch.cuda.device(self.device):
            return (torch.as_tensor(_DevArray(k.value, shape), device=f"cuda:{self.device}"),
                    torch.as_tensor(_DevArray(v.value, shape), device=f"cuda:{self.device}"))

    @property
    def stream(self) -> torch.cuda.ExternalStream:
        return torch.cuda.ExternalStream(_lib.load().qasr_decoder_stream(self._h), device=f"cuda:{self.device}")

    def set_step_kernel(self, mode: int) -> None:
        """0: the whole step as one persistent kernel where it covers the shape;
        1: per-layer kernels (the default)."""
        _lib.call("qasr_decoder_set_step_kernel", self._h, int(mode))

    def step_kernel(self, M: int) -> int:
        """0 if a step of M sequences runs as the persistent kernel, 1 if per layer."""
        return int(_lib.load().qasr_decoder_step_kernel(self._h, int(M)))

    def trace_step(self, tokens, positions) -> np.ndarray:
        """One step with the in-step timeline on (qasr_decoder_trace).  Per-layer
        kernels: uint64 [5*n_layers + 1, 2] (first CTA past its dependency
        wait, last CTA exit) per launch.  Persistent kernel: int64 %globaltimer
        stamps [CTAs, n_layers + 1, 5 phases, 4 events] (0 where a CTA had no
        part in a phase)."""
        lib = _lib.load()
        L = self.cfg["n_layers"]
        if self.step_kernel(len(tokens)) != 0:
            n = 2 * (5 * L + 1)
            buf = torch.zeros(n, dtype=torch.int64, device=f"cuda:{self.device}")
            buf[0::2] = -1  # all ones: atomic-min slots
            _lib.call("qasr_decoder_trace", self._h, C.c_void_p(buf.data_ptr()), C.c_int64(n))
            try:
                self.step(tokens, positions)
            finally:
                _lib.call("qasr_decoder_trace", self._h, None, C.c_int64(0))
            return buf.cpu().numpy().view(np.uint64).reshape(5 * L + 1, 2)
        stride = int(lib.qasr_decoder_trace_stride(self._h))
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count
        buf = torch.zeros(sms * stride, dtype=torch.int64, device=f"cuda:{self.device}")
        _lib.call("qasr_decoder_trace", self._h, C.c_void_p(buf.data_ptr()), C.c_int64(buf.numel()))
        try:
            self.step(tokens, positions)
        finally:
            _lib.call("qasr_decoder_trace", self._h, None, C.c_int64(0))
        t = buf.cpu().numpy().reshape(sms, stride)
        out = np.zeros((sms, L + 1, 5, 4), np.int64)
        out[:, :L] = t[:, :L * 20].reshape(sms, L, 5, 4)
        out[:, L, 0] = t[:, L * 20:L * 20 + 4]
        return out

    def keep_logits(self, enable: bool = True) -> None:
        _lib.call("qasr_decoder_keep_logits", self._h, 1 if enable else 0)

    def logits(self, M: int):
        p = _lib.load().qasr_decoder_logits(self._h)
        if not p:
            return None
        return torch.as_tensor(_DevArray(p, (M, self.cfg["vocab"])), device=f"cuda:{self.device}")

    # ----------------------------------------------------------------- step
    def step(self, tokens, positions) -> np.ndarray:
        """decoder_forward_int8 for len(tokens) sequences (host buffers in/out)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        out = np.empty_like(t)
        _lib.call("qasr_decoder_step", self._h, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p), t.size,
                  out.ctypes.data_as(C.c_void_p))
        return out

    def prefill(self, slot: int, embeds, start_pos: int = 0) -> None:
        """decoder_prefill_int8 for one sequence: embeds [seq, hidden] f32
        (numpy or a CUDA tensor) at positions start_pos..; fills its K/V rows."""
        if isinstance(embeds, torch.Tensor):
            e = embeds.detach().float().contiguous()
            ptr, seq = e.data_ptr(), e.shape[0]
        else:
            e = np.ascontiguousarray(embeds, dtype=np.float32)
            ptr, seq = e.ctypes.data, e.shape[0]
        _lib.call("qasr_decoder_prefill", self._h, int(slot), C.c_void_p(ptr), int(seq), int(start_pos))

    def prefill_batch(self, slots, embeds, start_pos=None) -> None:
        """decoder_prefill_int8 of several sequences at once (distinct slots)."""
        keep = []
        n = len(slots)
        sl = (C.c_int * n)(*[int(x) for x in slots])
        embeds = [e.float() if isinstance(e, torch.Tensor) else np.asarray(e, np.float32) for e in embeds]
        ptrs = (C.c_void_p * n)(*[_host_or_dev_ptr(e, keep) for e in embeds])
        lens = (C.c_int * n)(*[int(e.shape[0]) for e in embeds])
        st = (C.c_int * n)(*([int(x) for x in start_pos] if start_pos is not None else [0] * n))
        _lib.call("qasr_decoder_prefill_batch", self._h, sl, ptrs, lens, st, n)

    def prefill_hidden(self, seq: int) -> torch.Tensor:
        """Residual stream [seq, hidden] left by the last prefill (a copy)."""
        ptr = _lib.load().qasr_decoder_prefill_hidden(self._h)
        if not ptr:
            raise RuntimeError("no prefill has run")
        with torch.cuda.device(self.device):
            view = torch.as_tensor(_DevArray(ptr, (seq, self.cfg["hidden"])), device=f"cuda:{self.device}")
            return view.clone()

    def embed(self, ids) -> torch.Tensor:
        """QwenCtx::tok_embed_to_f32 for host ids: [n, hidden] rows on the device."""
        a = np.ascontiguousarray(ids, dtype=np.int32)
        out = torch.empty(a.size, self.cfg["hidden"], dtype=torch.float32, device=f"cuda:{self.device}")
        _lib.call("qasr_decoder_embed", self._h, a.ctypes.data_as(C.c_void_p), a.size, C.c_void_p(out.data_ptr()))
        return out

    def step_device(self, tokens: torch.Tensor, positions: torch.Tensor, out: torch.Tensor) -> None:
        """Same step on device int32 tensors, enqueued on the engine stream."""
        _lib.call("qasr_decoder_step_device", self._h, C.c_void_p(tokens.data_ptr()),
                  C.c_void_p(positions.data_ptr()), tokens.numel(), C.c_void_p(out.data_ptr()))

    def profile_step(self, tokens, positions) -> dict:
        """One eager step with CUDA events around each kernel: {class: (ms, launches)}."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        p = np.ascontiguousarray(positions, dtype=np.int32)
        n = len(_lib.KERNEL_CLASSES)
        ms = (C.c_float * n)()
        cnt = (C.c_int * n)()
        _lib.call("qasr_decoder_profile_step", self._h, t.ctypes.data_as(C.c_void_p), p.ctypes.data_as(C.c_void_p),
                  t.size, ms, cnt, n)
        return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(_lib.KERNEL_CLASSES)}

    def step_bytes(self, positions) -> int:
        p = np.ascontiguousarray(positions, dtype=np.int32)
        return int(_lib.load().qasr_decoder_step_bytes(self._h, p.ctypes.data_as(C.c_void_p), p.size))

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.load().qasr_decoder_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
