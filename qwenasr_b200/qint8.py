"""Python face of the .qint8 reader (qasr_qint8_*): QuantFile
(crates/qwen-asr/src/quantize.rs:130-346), QwenConfig::detect
(config.rs:110-156) and the V2 load path of QwenCtx::load (context.rs:341-420).

    f = QInt8File(path)
    dec_cfg, enc_cfg = f.detect()
    dec = Decoder(dec_cfg, max_batch=8, max_seq=2048, embed_is_int8=dec_cfg["embed_is_int8"])
    f.load_decoder(dec); enc = Encoder(enc_cfg); f.load_encoder(enc)

Opening, listing and detection run on the host only (no GPU needed).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib

DTYPES = {0: np.int8, 1: np.float32, 2: np.uint16}  # BF16 as raw 16-bit words


class QInt8File:
    def __init__(self, path: str):
        self._h = _lib.load().qasr_qint8_open(path.encode())
        if not self._h:
            raise _lib.QasrError(_lib.QASR_ERR_INVALID, "qasr_qint8_open", _lib.last_error())
        self.path = path

    @property
    def version(self) -> int:
        return int(_lib.load().qasr_qint8_version(self._h))

    def __len__(self) -> int:
        return int(_lib.load().qasr_qint8_count(self._h))

    def find(self, name: str) -> int:
        return int(_lib.load().qasr_qint8_find(self._h, name.encode()))

    def tensor(self, i: int) -> dict:
        """{name, dtype, shape, data (numpy copy), scales (numpy copy or None)}."""
        name, dt, nd = C.c_char_p(), C.c_int(), C.c_int()
        shape = (C.c_int64 * 8)()
        data, scales = C.c_void_p(), C.c_void_p()
        _lib.call("qasr_qint8_tensor", self._h, int(i), C.byref(name), C.byref(dt), C.byref(nd), shape,
                  C.byref(data), C.byref(scales))
        shp = tuple(int(shape[d]) for d in range(nd.value))
        n = int(np.prod(shp)) if shp else 0
        np_dt = DTYPES[dt.value]
        raw = C.string_at(data.value, n * np.dtype(np_dt).itemsize) if n else b""
        arr = np.frombuffer(raw, dtype=np_dt).reshape(shp) if n else np.zeros(shp, np_dt)
        sc = None
        if dt.value == 0 and shp:
            sc = np.frombuffer(C.string_at(scales.value, shp[0] * 4), dtype=np.float32).copy()
        return {"name": name.value.decode(), "dtype": dt.value, "shape": shp, "data": arr.copy(), "scales": sc}

    def names(self) -> list[str]:
        return [self.tensor(i)["name"] for i in range(len(self))]

    def detect(self) -> tuple[dict, dict | None]:
        """(decoder config dict incl. embed_is_int8, encoder config dict or None)."""
        d = _lib.DecoderConfig()
        e = _lib.EncoderConfig()
        _lib.call("qasr_qint8_detect", self._h, C.byref(d), None)
        dec = {k: getattr(d, k) for k in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "head_dim",
                                          "vocab", "eps", "theta", "embed_is_int8")}
        enc = None
        if _lib.load().qasr_qint8_detect(self._h, None, C.byref(e)) == _lib.QASR_OK:
            enc = {k: getattr(e, k) for k, _ in _lib.EncoderConfig._fields_}
        return dec, enc

    def load_decoder(self, dec) -> None:
        _lib.call("qasr_qint8_load_decoder", self._h, dec._h)

    def load_encoder(self, enc) -> None:
        _lib.call("qasr_qint8_load_encoder", self._h, enc._h)

    def close(self) -> None:
        if self._h:
            _lib.load().qasr_qint8_close(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()
