"""GPU parity of streaming transcription (transcribe_stream and
StreamState/stream_push_audio, transcribe.rs:445-1495) through qasr_stream_*
against the restatement in stream_oracle.py over the CPU oracle decoder.

Both sides get the same encoder rows (the device encoder's), so the check is
exact: every push emits the same token ids, and the committed / pending
tokens and the trim request agree.  20 s of audio at 2 s chunks crosses the
8 s encoder windows, the 200-row re-anchor and, on a random-weight model,
the degeneracy reset; past-text conditioning exercises the rollback prefix
and the device-side longest-common-prefix reuse of the KV cache.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qwenasr_b200 import kernels as K  # noqa: E402
from qwenasr_b200 import synthetic  # noqa: E402
from qwenasr_b200.decoder import Decoder  # noqa: E402
from qwenasr_b200.encoder import Encoder  # noqa: E402
from qwenasr_b200.stream import Stream, transcribe_stream  # noqa: E402
from stream_oracle import OracleStream  # noqa: E402

DEC = dict(synthetic.DEC_0_6B, n_layers=2)  # full vocabulary: the prompt's special ids
ENC = dict(d_model=128, n_layers=2, n_heads=2, head_dim=64, ffn_dim=256, output_dim=1024, chunk_size=100,
           n_window_infer=800)
MAX_SEQ = 2048
TOK_BYTES = (np.arange(DEC["vocab"]) % 4 + 1).astype(np.int32)


@pytest.fixture(scope="module")
def engines(orc):
    orc.set_threads(8)
    wd = synthetic.decoder_weights_np(DEC, seed=81)
    we = synthetic.encoder_weights_np(ENC, seed=82)
    dec = Decoder(DEC, device=0, max_batch=1, max_seq=MAX_SEQ)
    for i, lw in enumerate(wd["layers"]):
        dec.set_layer(i, lw)
    dec.set_globals(wd["embed"], wd["norm"], wd["lm_head"], wd["lm_head_s"])
    enc = Encoder(ENC, device=0)
    enc.set_weights(we)
    yield wd, orc.OracleDecoder(wd), dec, enc
    dec.close()
    enc.close()


def _encoder(enc):
    def encode(samples):
        s = torch.from_numpy(np.ascontiguousarray(samples, np.float32)).cuda()
        mel = torch.empty(128, K.mel_frames(len(samples)), device="cuda")
        K.mel_spectrogram(mel, s, len(samples))
        torch.cuda.synchronize()
        return enc.forward(mel).cpu().numpy()
    return encode


def _oracle(engines, **kw):
    wd, od, dec, enc = engines
    return OracleStream(od, lambda ids: wd["embed"][list(ids)], _encoder(enc), MAX_SEQ, tok_bytes=TOK_BYTES, **kw)


@pytest.mark.parametrize("past", [False, True])
def test_push_audio_matches_oracle(engines, past):
    wd, od, dec, enc = engines
    audio = synthetic.synthetic_audio(20.0, seed=90 + past)
    s = Stream(dec, enc, past_text_conditioning=int(past))
    s.set_token_bytes(TOK_BYTES)
    o = _oracle(engines, past_text_conditioning=past)
    for end, fin in ((1.5, False), (3.0, False), (7.7, False), (12.0, False), (20.0, True)):
        buf = audio[:int(end * 16000)]
        got = s.push(buf, finalize=fin)
        assert got == o.push(buf, finalize=fin), end
        assert s.audio_cursor == o.cursor and s.trim_request == o.trim_request
        assert s.emitted() == o.emitted
        text_start = o.raw.index(151704) + 1 if 151704 in o.raw else 0
        assert s.unfixed() == o.raw[text_start:][len(o.stable):]
    # the paths this case is meant to cover were taken
    assert o.chunk_idx >= 9 and o.resets > 0 and o.max_reused > 0
    assert o.max_prefix > 0 if past else len(s.emitted()) > 0
    s.close()


@pytest.mark.parametrize("past", [False, True])
def test_transcribe_stream_matches_oracle(engines, past):
    audio = synthetic.synthetic_audio(17.0, seed=95 + past)
    got = transcribe_stream(engines[2], engines[3], audio, past_text_conditioning=int(past))
    o = _oracle(engines, past_text_conditioning=past, incremental=False)
    assert got == o.push(audio, finalize=True)


def test_stream_prompt_reset_and_device_buffer(engines):
    """Prompt / forced ids in the prompt rows; reset starts over; a device
    sample buffer gives the host result."""
    wd, od, dec, enc = engines
    audio = synthetic.synthetic_audio(6.0, seed=99)
    s = Stream(dec, enc)
    s.set_prompt([1000, 2000], [3000])
    o = _oracle(engines, prompt=(1000, 2000), force=(3000,))
    assert s.push(audio, finalize=True) == o.push(audio, finalize=True)
    first = s.emitted()
    s.reset()
    assert s.audio_cursor == 0 and s.emitted() == []
    assert s.push(torch.from_numpy(audio).cuda(), finalize=True) == first
    s.close()
