"""The .qint8 reader on the host (QuantFile::open, quantize.rs:130-346;
QwenConfig::detect, config.rs:110-156): no GPU involved.

The first tests build files byte by byte from the format description in
quantize.rs:1-35, so the parser is pinned to the format itself, not to the
test-side writer; the writer is then checked against the same parser.
"""
import struct

import numpy as np
import pytest

from qwenasr_b200 import synthetic
from qwenasr_b200._lib import QasrError
from qwenasr_b200.qint8 import QInt8File
from qint8_fixture import BF16, F32, INT8, bf16_bits, model_entries, write_qint8


def _entry(name, dt, shape, off, soff, v2=True):
    b = struct.pack("<H", len(name)) + name.encode()
    if v2:
        b += bytes([dt])
    b += bytes([len(shape)]) + b"".join(struct.pack("<I", d) for d in shape) + struct.pack("<QQ", off, soff)
    return b


def test_v2_literal_bytes(tmp_path):
    q = np.array([[1, -2, 3], [-128, 127, 0]], np.int8)
    s = np.array([0.5, 0.25], np.float32)
    f = np.array([1.5, -2.0], np.float32)
    h = bf16_bits([1.0, -3.0, 0.5])
    data = q.tobytes() + b"\0\0" + s.tobytes() + f.tobytes() + h.tobytes()  # INT8 at 0, scales at 8, F32 at 16
    table = (_entry("a.w", 0, (2, 3), 0, 8) + _entry("b", 1, (2,), 16, 0) + _entry("c", 2, (3,), 24, 0))
    p = tmp_path / "m.qint8"
    p.write_bytes(b"QINT8\x02\x00\x00" + struct.pack("<II", 3, 0) + table + data)
    with QInt8File(str(p)) as qf:
        assert qf.version == 2 and len(qf) == 3
        assert qf.find("b") == 1 and qf.find("zz") == -1
        a, b, c = (qf.tensor(i) for i in range(3))
        assert a["name"] == "a.w" and a["dtype"] == INT8 and a["shape"] == (2, 3)
        assert np.array_equal(a["data"], q) and np.array_equal(a["scales"], s)
        assert b["dtype"] == F32 and np.array_equal(b["data"], f) and b["scales"] is None
        assert c["dtype"] == BF16 and np.array_equal(c["data"], h)


def test_v1_dtype_from_scale_offset(tmp_path):
    q = np.arange(4, dtype=np.int8).reshape(2, 2)
    s = np.array([1.0, 2.0], np.float32)
    f = np.array([7.0], np.float32)
    data = q.tobytes() + s.tobytes() + f.tobytes()
    table = _entry("w", 0, (2, 2), 0, 4, v2=False) + _entry("n", 0, (1,), 12, 0, v2=False)
    p = tmp_path / "v1.qint8"
    p.write_bytes(b"QINT8\x01\x00\x00" + struct.pack("<II", 2, 0) + table + data)
    with QInt8File(str(p)) as qf:
        assert qf.version == 1
        w, n = qf.tensor(0), qf.tensor(1)
        assert w["dtype"] == INT8 and np.array_equal(w["scales"], s)
        assert n["dtype"] == F32 and n["data"].tolist() == [7.0]


@pytest.mark.parametrize("mutate", ["magic", "truncated_table", "data_past_end", "scales_past_end", "short"])
def test_corrupt_files_rejected(tmp_path, mutate):
    q = np.zeros((2, 4), np.int8)
    body = q.tobytes() + np.ones(2, np.float32).tobytes()
    table = _entry("w", 0, (2, 4), 0, 8)
    raw = b"QINT8\x02\x00\x00" + struct.pack("<II", 1, 0) + table + body
    if mutate == "magic":
        raw = b"QINT9" + raw[5:]
    elif mutate == "truncated_table":
        raw = raw[:16 + 5]
    elif mutate == "data_past_end":
        raw = raw[:16] + _entry("w", 0, (2, 400), 0, 8) + body
    elif mutate == "scales_past_end":
        raw = raw[:16] + _entry("w", 0, (2, 4), 0, 12) + body
    else:
        raw = raw[:10]
    p = tmp_path / "bad.qint8"
    p.write_bytes(raw)
    with pytest.raises(QasrError):
        QInt8File(str(p))
    with pytest.raises(QasrError):
        QInt8File(str(tmp_path / "missing.qint8"))


DEC = dict(synthetic.DEC_0_6B, n_layers=2, vocab=512)
ENC = dict(d_model=128, n_layers=3, n_heads=2, head_dim=64, ffn_dim=256, output_dim=1024, chunk_size=100,
           n_window_infer=800)


def test_writer_round_trip_and_detect(tmp_path):
    wd = synthetic.decoder_weights_np(DEC, seed=3)
    we = synthetic.quantize_encoder(synthetic.encoder_weights_np(ENC, seed=4))
    emb_q, emb_s = synthetic.quantize_np(wd["embed"])
    p = tmp_path / "model_int8.qint8"
    entries = model_entries(wd, we, int8_embed=(emb_q, emb_s), with_lm_head=False)
    write_qint8(str(p), entries)
    with QInt8File(str(p)) as qf:
        assert len(qf) == len(entries)
        for i, (name, dt, arr, sc) in enumerate(entries):
            t = qf.tensor(qf.find(name))
            assert t["dtype"] == dt and t["shape"] == np.asarray(arr).shape
            assert np.array_equal(t["data"], np.asarray(arr).astype(t["data"].dtype))
            if dt == INT8:
                assert np.array_equal(t["scales"], sc)
        dec, enc = qf.detect()
        assert {k: dec[k] for k in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "head_dim", "vocab")} == \
            {k: DEC[k] for k in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "head_dim", "vocab")}
        assert dec["embed_is_int8"] == 1
        assert enc == ENC


def test_detect_published_shapes(tmp_path):
    """The two published checkpoints' shapes give QwenConfig::detect's configs
    (config.rs:110-156): only shape metadata matters, so tensors are 1-row stubs
    except where the shape is read."""
    for dec_h, inter, enc_d, enc_l, ffn in ((1024, 3072, 896, 18, 3584), (2048, 6144, 1024, 24, 4096)):
        e = [("thinker.model.embed_tokens.weight", INT8, np.zeros((151936, dec_h), np.int8), np.ones(151936, np.float32)),
             ("thinker.audio_tower.proj2.weight", INT8, np.zeros((dec_h, 1), np.int8), np.ones(dec_h, np.float32))]
        for i in range(28):
            lp = f"thinker.model.layers.{i}."
            e.append((lp + "self_attn.q_proj.weight", INT8, np.zeros((2048, 1), np.int8), np.ones(2048, np.float32)))
        e.append(("thinker.model.layers.0.self_attn.k_proj.weight", INT8, np.zeros((1024, 1), np.int8),
                  np.ones(1024, np.float32)))
        e.append(("thinker.model.layers.0.self_attn.q_norm.weight", F32, np.ones(128, np.float32), None))
        e.append(("thinker.model.layers.0.mlp.gate_proj.weight", INT8, np.zeros((inter, 1), np.int8),
                  np.ones(inter, np.float32)))
        for i in range(enc_l):
            e.append((f"thinker.audio_tower.layers.{i}.self_attn.q_proj.weight", INT8,
                      np.zeros((enc_d, 1), np.int8), np.ones(enc_d, np.float32)))
        e.append(("thinker.audio_tower.layers.0.fc1.weight", INT8, np.zeros((ffn, 1), np.int8),
                  np.ones(ffn, np.float32)))
        p = tmp_path / f"d{dec_h}.qint8"
        write_qint8(str(p), e)
        with QInt8File(str(p)) as qf:
            dec, enc = qf.detect()
        want = synthetic.DEC_0_6B if dec_h == 1024 else synthetic.DEC_1_7B
        assert {k: dec[k] for k in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "head_dim", "vocab")} == \
            {k: want[k] for k in ("hidden", "inter", "n_layers", "n_heads", "n_kv_heads", "head_dim", "vocab")}
        assert enc == (synthetic.ENC_0_6B if dec_h == 1024 else synthetic.ENC_1_7B)


def test_decoder_only_file_has_no_encoder(tmp_path):
    wd = synthetic.decoder_weights_np(DEC, seed=5)
    p = tmp_path / "dec.qint8"
    write_qint8(str(p), model_entries(wd))
    with QInt8File(str(p)) as qf:
        dec, enc = qf.detect()
        assert enc is None and dec["embed_is_int8"] == 0
