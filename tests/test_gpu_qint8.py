"""Loading a V2 .qint8 file into the device engines (DecoderInt8::load,
decoder.rs:680-748; EncoderInt8::load_from_qint8, encoder.rs:466-520).

An engine loaded from the file must equal an engine given the same weights
through the setters bit for bit (same kernels, same bytes: this pins the
loader, including the on-device gate/up interleave), and both must match the
oracle: greedy ids identical, logits and encoder rows within 2e-3 relative.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qwenasr_b200 import synthetic  # noqa: E402
from qwenasr_b200.decoder import Decoder  # noqa: E402
from qwenasr_b200.encoder import Encoder  # noqa: E402
from qwenasr_b200.qint8 import QInt8File  # noqa: E402
from qwenasr_b200.transcribe import transcribe_ids  # noqa: E402
from oracle.pyoracle import encoder_forward  # noqa: E402
from qint8_fixture import model_entries, write_qint8  # noqa: E402

ENC = dict(d_model=128, n_layers=2, n_heads=2, head_dim=64, ffn_dim=256, output_dim=1024, chunk_size=100,
           n_window_infer=800)


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.abs(ref) + math.sqrt(float(np.mean(ref * ref)) + 1e-30)
    return float(np.max(np.abs(got - ref) / scale))


def _direct_decoder(cfg, wd, emb_q, emb_s, tied, max_seq, max_batch=2):
    dec = Decoder(cfg, device=0, max_batch=max_batch, max_seq=max_seq, embed_is_int8=True)
    for i, lw in enumerate(wd["layers"]):
        dec.set_layer(i, lw)
    if tied:
        dec.set_globals(emb_q, wd["norm"], embed_scales=emb_s)
    else:
        dec.set_globals(emb_q, wd["norm"], wd["lm_head"], wd["lm_head_s"], embed_scales=emb_s)
    return dec


@pytest.mark.parametrize("tied", [False, True])
def test_decoder_from_file(orc, tmp_path, tied):
    orc.set_threads(8)
    cfg = dict(synthetic.DEC_0_6B, n_layers=2, vocab=4096)
    wd = synthetic.decoder_weights_np(cfg, seed=40 + tied)
    emb_q, emb_s = synthetic.quantize_np(wd["embed"])
    path = str(tmp_path / "model_int8.qint8")
    write_qint8(path, model_entries(wd, int8_embed=(emb_q, emb_s), with_lm_head=not tied))
    with QInt8File(path) as qf:
        dcfg, _ = qf.detect()
        assert dcfg["embed_is_int8"] == 1 and dcfg["n_layers"] == 2
        a = Decoder(dcfg, device=0, max_batch=2, max_seq=64, embed_is_int8=True)
        qf.load_decoder(a)
    b = _direct_decoder(cfg, wd, emb_q, emb_s, tied, 64)
    wo = dict(wd, lm_head=emb_q if tied else wd["lm_head"], lm_head_s=emb_s if tied else wd["lm_head_s"])
    od = orc.OracleDecoder(wo)
    rng = np.random.default_rng(tied)
    ids = rng.integers(0, cfg["vocab"], 12).astype(np.int32)
    rows = np.stack([orc.embed_int8(emb_q, emb_s, int(t)) for t in ids[:11]])
    kh, vh = od.new_kv(64)
    od.prefill(kh, vh, 0, rows)
    for dec in (a, b):
        dec.prefill(0, rows, 0)
        dec.keep_logits(True)
    tok = np.array([ids[11]], np.int32)
    for pos in range(11, 15):
        na = a.step(tok, [pos])
        la = a.logits(1).cpu().numpy()
        nb = b.step(tok, [pos])
        lb = b.logits(1).cpu().numpy()
        assert np.array_equal(la, lb) and int(na[0]) == int(nb[0])
        ref_tok, ref_logits, _ = od.forward(kh, vh, pos, orc.embed_int8(emb_q, emb_s, int(tok[0])), want_logits=True)
        assert int(na[0]) == ref_tok
        assert rel_err(la[0], ref_logits) < 2e-3
        tok = na.astype(np.int32)
    ka, _ = a.kv(0)
    kb, _ = b.kv(0)
    assert torch.equal(ka, kb)
    a.close()
    b.close()


def test_int8_encoder_and_file(orc, tmp_path):
    """EncoderInt8::forward against the oracle composition with linear_int8;
    the file-loaded encoder equals the directly set one."""
    orc.set_threads(8)
    we = synthetic.quantize_encoder(synthetic.encoder_weights_np(ENC, seed=50))
    wd = synthetic.decoder_weights_np(dict(synthetic.DEC_0_6B, n_layers=1, vocab=256), seed=51)
    mel = np.random.default_rng(50).standard_normal((128, 230)).astype(np.float32)
    direct = Encoder(ENC, device=0)
    direct.set_weights(we)
    out = direct.forward(mel).cpu().numpy()
    ref = encoder_forward(we, ENC, mel)
    assert out.shape == ref.shape
    rms = math.sqrt(float(np.mean(ref.astype(np.float64) ** 2)))
    assert float(np.max(np.abs(out - ref) / (np.abs(ref) + rms))) < 2e-3
    path = str(tmp_path / "enc.qint8")
    write_qint8(path, model_entries(wd, we))
    with QInt8File(path) as qf:
        _, ecfg = qf.detect()
        assert ecfg == ENC
        loaded = Encoder(ecfg, device=0)
        qf.load_encoder(loaded)
    assert np.array_equal(loaded.forward(mel).cpu().numpy(), out)
    direct.close()
    loaded.close()


def test_transcribe_from_v2_file(tmp_path):
    """A self-contained V2 file (INT8 decoder with the tied INT8 embedding
    table and INT8 encoder) transcribes exactly like engines set directly."""
    cfg = dict(synthetic.DEC_0_6B, n_layers=2)  # full vocabulary: the prompt's special ids
    wd = synthetic.decoder_weights_np(cfg, seed=60)
    emb_q, emb_s = synthetic.quantize_np(wd["embed"])
    we = synthetic.quantize_encoder(synthetic.encoder_weights_np(ENC, seed=61))
    path = str(tmp_path / "model_int8.qint8")
    write_qint8(path, model_entries(wd, we, int8_embed=(emb_q, emb_s), with_lm_head=False))
    audio = [synthetic.synthetic_audio(s, seed=62 + i) for i, s in enumerate((1.2, 0.8))]
    with QInt8File(path) as qf:
        dcfg, ecfg = qf.detect()
        dec = Decoder(dcfg, device=0, max_batch=2, max_seq=96, embed_is_int8=True)
        enc = Encoder(ecfg, device=0)
        qf.load_decoder(dec)
        qf.load_encoder(enc)
    got = transcribe_ids(dec, enc, audio, 10)
    dec2 = _direct_decoder(cfg, wd, emb_q, emb_s, True, 96)
    enc2 = Encoder(ENC, device=0)
    enc2.set_weights(we)
    assert transcribe_ids(dec2, enc2, audio, 10) == got
    for e in (dec, dec2, enc, enc2):
        e.close()


def test_load_rejects_mismatched_engine(tmp_path):
    from qwenasr_b200._lib import QasrError
    cfg = dict(synthetic.DEC_0_6B, n_layers=2, vocab=4096)
    wd = synthetic.decoder_weights_np(cfg, seed=70)
    path = str(tmp_path / "m.qint8")
    write_qint8(path, model_entries(wd))  # f32 embedding table
    with QInt8File(path) as qf:
        bad = Decoder(dict(cfg, n_layers=3), device=0, max_batch=1, max_seq=32)
        with pytest.raises(QasrError, match="layers"):
            qf.load_decoder(bad)
        bad.close()
        wrong_kind = Decoder(cfg, device=0, max_batch=1, max_seq=32, embed_is_int8=True)
        with pytest.raises(QasrError, match="embed_is_int8"):
            qf.load_decoder(wrong_kind)
        wrong_kind.close()
        with pytest.raises(QasrError):
            qf.load_encoder(Encoder(ENC, device=0))  # the file has no encoder
