"""GPU parity of the audio encoder engine (Encoder::forward, encoder.rs:243-415)
against a host composition of the oracle's kernels::* restatements (conv2d
as an fp64 im2col GEMM, cblas_sgemm's stand-in)."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qwenasr_b200 import synthetic  # noqa: E402
from qwenasr_b200.encoder import Encoder  # noqa: E402
from oracle.pyoracle import encoder_forward as encoder_forward_ref  # noqa: E402

SMALL = dict(d_model=128, n_layers=2, n_heads=2, head_dim=64, ffn_dim=256, output_dim=256, chunk_size=100,
             n_window_infer=800)


@pytest.mark.parametrize("frames", [250, 100, 37])
def test_encoder_forward_matches_oracle(orc, frames):
    orc.set_threads(8)
    w = synthetic.encoder_weights_np(SMALL, seed=frames)
    rng = np.random.default_rng(frames)
    mel = rng.standard_normal((128, frames)).astype(np.float32)
    enc = Encoder(SMALL, device=0)
    enc.set_weights(w)
    out = enc.forward(mel).cpu().numpy()
    ref = encoder_forward_ref(w, SMALL, mel)
    assert out.shape == ref.shape
    rms = math.sqrt(float(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(out - ref) / (np.abs(ref) + rms)))
    assert err < 2e-3, err
    # a device mel gives the same rows
    out2 = enc.forward(torch.from_numpy(mel).cuda()).cpu().numpy()
    assert np.array_equal(out, out2)
    enc.close()


def test_encoder_forward_batch_equals_single(orc):
    """qasr_encoder_forward_batch: ragged segments (a tail chunk, a sub-chunk
    one, several windows) in one pass give each segment's single-forward rows
    bit for bit; host and device mels mixed."""
    w = synthetic.encoder_weights_np(SMALL, seed=7)
    rng = np.random.default_rng(7)
    mels = [rng.standard_normal((128, f)).astype(np.float32) for f in (250, 37, 1000, 100)]
    enc = Encoder(SMALL, device=0)
    enc.set_weights(w)
    single = [enc.forward(m).cpu().numpy() for m in mels]
    batch = enc.forward_batch([mels[0], torch.from_numpy(mels[1]).cuda(), mels[2], torch.from_numpy(mels[3]).cuda()])
    for a, b in zip(single, batch):
        assert np.array_equal(a, b.cpu().numpy())
    enc.close()
