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

SMALL = dict(d_model=128, n_layers=2, n_heads=2, head_dim=64, ffn_dim=256, output_dim=256, chunk_size=100,
             n_window_infer=800)


def _conv(x, w, b, c_in, c_out, h, wd):
    ho, wo = (h - 1) // 2 + 1, (wd - 1) // 2 + 1
    xp = np.zeros((c_in, h + 2, wd + 2))
    xp[:, 1:1 + h, 1:1 + wd] = x.reshape(c_in, h, wd)
    cols = np.empty((c_in * 9, ho * wo))
    for ic in range(c_in):
        for ki in range(3):
            for kj in range(3):
                cols[(ic * 3 + ki) * 3 + kj] = xp[ic, ki:ki + 2 * ho:2, kj:kj + 2 * wo:2].ravel()
    return ((w.reshape(c_out, -1).astype(np.float64) @ cols) + b[:, None]).astype(np.float32), ho, wo


def encoder_forward_ref(orc, w, cfg, mel):
    D, CH, cs = cfg["d_model"], synthetic.CONV_HIDDEN, cfg["chunk_size"]
    frames = mel.shape[1]
    xs = []
    for s in range(0, frames, cs):
        chunk = mel[:, s:s + cs]
        c1, h1, w1 = _conv(chunk, w["conv1_w"], w["conv1_b"], 1, CH, 128, chunk.shape[1])
        c1 = orc.gelu(c1.ravel()).reshape(c1.shape)
        c2, h2, w2 = _conv(c1, w["conv2_w"], w["conv2_b"], CH, CH, h1, w1)
        c2 = orc.gelu(c2.ravel()).reshape(c2.shape)
        c3, h3, w3 = _conv(c2, w["conv3_w"], w["conv3_b"], CH, CH, h2, w2)
        c3 = orc.gelu(c3.ravel()).reshape(CH, h3, w3)
        reshaped = np.ascontiguousarray(c3.transpose(2, 0, 1).reshape(w3, CH * h3))
        xs.append(orc.linear(reshaped, w["conv_out_w"]) + orc.sinusoidal_pe(w3, D))
    x = np.concatenate(xs).astype(np.float32)
    T = x.shape[0]
    tpc = 13
    wsize = tpc * (cfg["n_window_infer"] // cs)
    starts = np.array(list(range(0, T, wsize)) + [T], np.int32)
    scale = np.float32(1.0 / math.sqrt(cfg["head_dim"]))
    for L in w["layers"]:
        xn = orc.layer_norm(x, L["attn_norm_w"], L["attn_norm_b"], 1e-5)
        q = orc.linear(xn, L["wq"], L["bq"])
        k = orc.linear(xn, L["wk"], L["bk"])
        v = orc.linear(xn, L["wv"], L["bv"])
        a = orc.bidirectional_attention(q, k, v, T, cfg["n_heads"], cfg["head_dim"], starts, scale)
        x = (x + orc.linear(a, L["wo"], L["bo"])).astype(np.float32)
        xn = orc.layer_norm(x, L["ffn_norm_w"], L["ffn_norm_b"], 1e-5)
        mid = orc.gelu(orc.linear(xn, L["fc1_w"], L["fc1_b"]).ravel()).reshape(T, -1)
        x = (x + orc.linear(mid, L["fc2_w"], L["fc2_b"])).astype(np.float32)
    xn = orc.layer_norm(x, w["ln_post_w"], w["ln_post_b"], 1e-5)
    p1 = orc.gelu(orc.linear(xn, w["proj1_w"], w["proj1_b"]).ravel()).reshape(T, -1)
    return orc.linear(p1, w["proj2_w"], w["proj2_b"])


@pytest.mark.parametrize("frames", [250, 100, 37])
def test_encoder_forward_matches_oracle(orc, frames):
    orc.set_threads(8)
    w = synthetic.encoder_weights_np(SMALL, seed=frames)
    rng = np.random.default_rng(frames)
    mel = rng.standard_normal((128, frames)).astype(np.float32)
    enc = Encoder(SMALL, device=0)
    enc.set_weights(w)
    out = enc.forward(mel).cpu().numpy()
    ref = encoder_forward_ref(orc, w, SMALL, mel)
    assert out.shape == ref.shape
    rms = math.sqrt(float(np.mean(ref.astype(np.float64) ** 2)))
    err = float(np.max(np.abs(out - ref) / (np.abs(ref) + rms)))
    assert err < 2e-3, err
    # a device mel gives the same rows
    out2 = enc.forward(torch.from_numpy(mel).cuda()).cpu().numpy()
    assert np.array_equal(out, out2)
    enc.close()
