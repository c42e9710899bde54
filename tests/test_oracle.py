"""Pins the CPU oracle (oracle/) before it is trusted as the parity checker.

Part 1 re-runs every test of the reference's crates/qwen-asr/tests/kernels.rs
that touches this path, with the same inputs and tolerances.  Part 2 checks
the restatement against independent float64 derivations of each formula and
against hand-derived known answers.  No reference-produced vectors exist (the
reference is Rust and no Rust toolchain is available), so this is the whole
pinning evidence.
"""
import math

import numpy as np
import pytest


# ---------------------------------------------------------------- part 1 --
# crates/qwen-asr/tests/kernels.rs, test by test.

def _bf16_trunc(v):
    return (np.asarray(v, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def test_ref_bf16_matvec_vs_generic(orc):  # kernels.rs:19-44
    in_dim, out_dim = 128, 16
    x = (np.arange(in_dim, dtype=np.float32) * np.float32(0.01) - np.float32(0.64)).astype(np.float32)
    v = (np.arange(out_dim * in_dim, dtype=np.float32) * np.float32(0.001) - np.float32(0.5)).astype(np.float32)
    w = _bf16_trunc(v).reshape(out_dim, in_dim)
    bias = np.arange(out_dim, dtype=np.float32) * np.float32(0.1)
    y_gen = orc.bf16_matvec(x, w, bias, generic=True)
    y_disp = orc.bf16_matvec(x, w, None) + bias
    assert np.max(np.abs(y_gen - y_disp)) < 0.01


def test_ref_dot_f32_vs_generic(orc):  # kernels.rs:46-58
    n = 1024
    a = np.arange(n, dtype=np.float32) * np.float32(0.01) - np.float32(5.0)
    b = np.arange(n, dtype=np.float32) * 7 + 3
    b = b.astype(np.float32) * np.float32(0.002) - np.float32(1.0)
    g, d = orc.dot_f32_generic(a, b), orc.dot_f32(a, b)
    assert abs(g - d) < 0.01 * max(abs(g), 1.0)


def test_ref_rms_norm(orc):  # kernels.rs:60-72
    dim = 128
    x = np.arange(dim, dtype=np.float32) * np.float32(0.02) - np.float32(1.28)
    out = orc.rms_norm(x[None], np.ones(dim, np.float32), 1e-6)[0]
    rms = math.sqrt(float(np.sum(out * out)) / dim)
    assert abs(rms - 1.0) < 0.01


def test_ref_layer_norm(orc):  # kernels.rs:74-89
    dim = 128
    x = np.arange(dim, dtype=np.float32) * np.float32(0.05) - np.float32(3.2)
    out = orc.layer_norm(x[None], np.ones(dim, np.float32), np.zeros(dim, np.float32), 1e-5)[0]
    mean = float(out.mean())
    var = float(((out - mean) ** 2).mean())
    assert abs(mean) < 0.01 and abs(var - 1.0) < 0.02


def test_ref_softmax(orc):  # kernels.rs:91-103
    x = orc.softmax(np.arange(1, 11, dtype=np.float32)[None])[0]
    assert abs(float(x.sum()) - 1.0) < 1e-5
    assert np.all(np.diff(x) >= 0) and x[0] > 0 and x[9] > 0


def test_ref_gelu(orc):  # kernels.rs:105-113
    x = orc.gelu(np.array([0.0, 1.0, -1.0, 2.0, -0.5], np.float32))
    assert abs(x[0]) < 1e-5 and x[1] > 0.5 and x[2] < 0.0


def test_ref_silu(orc):  # kernels.rs:115-124
    orig = np.array([0.0, 1.0, -1.0, 5.0], np.float32)
    exp = orig / (1.0 + np.exp(-orig))
    assert np.max(np.abs(orc.silu(orig) - exp)) < 1e-5


def test_ref_vec_ops(orc):  # kernels.rs:126-152
    n = 256
    a = np.arange(n, dtype=np.float32) * np.float32(0.1)
    b = (n - np.arange(n)).astype(np.float32) * np.float32(0.1)
    assert np.all(np.abs(orc.vec_scale_inplace(a, 2.0) - a * 2) < 1e-5)
    assert np.all(np.abs(orc.vec_axpy_inplace(a, b, 0.5) - (a + 0.5 * b)) < 1e-5)
    assert np.max(np.abs(orc.vec_scale_add(a, b, 0.9) - (a * np.float32(0.9) + b))) < 1e-4


# ---------------------------------------------------------------- part 2 --
# Independent float64 derivations and known answers.

def test_rms_norm_matches_float64(orc):
    rng = np.random.default_rng(1)
    for hidden in (1024, 896, 8, 23, 2048):
        x = rng.standard_normal((5, hidden)).astype(np.float32)
        w = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
        ref = x.astype(np.float64) / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6) * w
        got = orc.rms_norm(x, w, 1e-6)
        assert np.max(np.abs(got - ref) / (np.abs(ref) + 1e-3)) < 2e-6


def test_layer_norm_matches_float64(orc):
    rng = np.random.default_rng(2)
    for hidden in (896, 1024, 13, 40):
        x = rng.standard_normal((4, hidden)).astype(np.float32)
        w = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
        b = (0.02 * rng.standard_normal(hidden)).astype(np.float32)
        xd = x.astype(np.float64)
        mu = xd.mean(-1, keepdims=True)
        ref = (xd - mu) / np.sqrt(((xd - mu) ** 2).mean(-1, keepdims=True) + 1e-5) * w + b
        got = orc.layer_norm(x, w, b, 1e-5)
        assert np.max(np.abs(got - ref)) < 5e-6


def test_rope_identity_at_pos0_and_rotation(orc):
    cos, sin = orc.rope_cache_table(16, 128, 1e6)
    assert np.all(cos[0] == 1.0) and np.all(sin[0] == 0.0)
    # halves duplicated (decoder.rs:276-281)
    assert np.array_equal(cos[:, :64], cos[:, 64:]) and np.array_equal(sin[:, :64], sin[:, 64:])
    inv = 1.0 / (1e6 ** (np.arange(64) * 2 / 128.0))
    ang = np.arange(16)[:, None] * inv[None]
    assert np.max(np.abs(cos[:, :64] - np.cos(ang))) < 1e-6
    # compute_rope_neox with the same positions gives the same table
    c2, s2 = orc.compute_rope_neox(np.arange(16), 128, 1e6)
    assert np.array_equal(c2, cos) and np.array_equal(s2, sin)
    rng = np.random.default_rng(3)
    x = rng.standard_normal((16, 2 * 128)).astype(np.float32)
    y = orc.apply_rope_neox(x, cos, sin, 2, 128)
    assert np.array_equal(y[0], x[0])
    # rotation preserves the norm of each (d, d+64) pair
    xr = x.reshape(16, 2, 2, 64)
    yr = y.reshape(16, 2, 2, 64)
    assert np.allclose((xr ** 2).sum(2), (yr ** 2).sum(2), rtol=1e-5, atol=1e-6)


def test_fast_exp_accuracy(orc):
    # avx.rs:485 states ~1e-4 relative error for |x| < 88
    for v in np.linspace(-80, 80, 321):
        got = orc.fast_exp(float(v))
        assert abs(got - math.exp(float(np.float32(v)))) <= 2e-4 * math.exp(float(np.float32(v)))
    assert orc.fast_exp(0.0) == 1.0


def test_gelu_variants(orc):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(1003).astype(np.float32) * 3
    xd = x.astype(np.float64)
    tanh_ref = 0.5 * xd * (1 + np.tanh(0.7978845608028654 * (xd + 0.044715 * xd ** 3)))
    assert np.max(np.abs(orc.gelu(x) - tanh_ref)) < 1e-3
    erf_ref = 0.5 * xd * (1 + np.vectorize(math.erf)(xd / math.sqrt(2)))
    assert np.max(np.abs(orc.gelu_erf(x) - erf_ref)) < 2e-6


def test_swiglu_forms(orc):
    rng = np.random.default_rng(5)
    inter = 3072 + 5
    gu = rng.standard_normal(2 * inter).astype(np.float32)
    g, u = gu[0::2].astype(np.float64), gu[1::2].astype(np.float64)
    ref = g / (1 + np.exp(-g)) * u
    dec = orc.swiglu_decode(gu, inter)
    pre = orc.swiglu_multiply(gu[None], 1, inter)[0]
    assert np.max(np.abs(dec - ref)) < 1e-6
    assert np.max(np.abs(pre - ref)) < 1e-3
    # scalar tail of the AVX path uses libm exp, identical to the decode form
    assert np.array_equal(pre[-5:], dec[-5:])


def test_sinusoidal_pe_known_answers(orc):
    pe = orc.sinusoidal_pe(4, 896)
    assert np.all(pe[0, :448] == 0.0) and np.all(pe[0, 448:] == 1.0)
    ts = math.log(10000.0) / 447
    ref = np.array([[p * math.exp(-d * ts) for d in range(448)] for p in range(4)])
    assert np.max(np.abs(pe[:, :448] - np.sin(ref))) < 2e-6
    assert np.max(np.abs(pe[:, 448:] - np.cos(ref))) < 2e-6


def test_quantizer_rule(orc):
    # quantize.rs:633-662: scale = absmax/127, q = round(v*127/absmax), half away from zero
    d = np.array([[127.0, -63.5, 0.5, -0.5, 1.5, 0.0],
                  [0.0, 0.0, 0.0, 0.0, 0.0, 0.0],
                  [-254.0, 1.0, 2.0, 3.0, -1.0, 127.0]], np.float32)
    q, s = orc.quantize_f32_to_int8(d)
    assert s.tolist() == [1.0, 0.0, 2.0]
    assert q[0].tolist() == [127, -64, 1, -1, 2, 0]
    assert q[1].tolist() == [0] * 6
    assert q[2].tolist() == [-127, 1, 1, 2, -1, 64]


def test_int8_matvec_matches_float64(orc):
    rng = np.random.default_rng(6)
    w = rng.integers(-128, 128, size=(300, 1024), dtype=np.int8)
    s = rng.random(300).astype(np.float32) * 0.01
    x = rng.standard_normal((3, 1024)).astype(np.float32)
    ref = (x.astype(np.float64) @ w.astype(np.float64).T) * s
    got = orc.linear_nobias_int8(x, w, s)
    scale = np.sqrt((ref ** 2).mean())
    assert np.max(np.abs(got - ref)) < 1e-4 * scale


def test_threading_does_not_change_results(orc):
    rng = np.random.default_rng(7)
    w = rng.integers(-128, 128, size=(517, 256), dtype=np.int8)
    s = rng.random(517).astype(np.float32)
    x = rng.standard_normal((2, 256)).astype(np.float32)
    orc.set_threads(1)
    a = orc.linear_nobias_int8(x, w, s)
    orc.set_threads(7)
    b = orc.linear_nobias_int8(x, w, s)
    orc.set_threads(1)
    assert np.array_equal(a, b)


def test_causal_attention_matches_float64(orc):
    rng = np.random.default_rng(8)
    nh, nkv, hd, sk = 4, 2, 128, 37
    q = rng.standard_normal((3, nh * hd)).astype(np.float32)
    k = rng.standard_normal((sk, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((sk, nkv * hd)).astype(np.float32)
    off = sk - 3
    got = orc.causal_attention(q, k, v, 3, sk, nh, nkv, hd, off)
    ref = np.zeros_like(got, dtype=np.float64)
    for h in range(nh):
        kv = h // (nh // nkv)
        for i in range(3):
            n = off + i + 1
            sc = k[:n, kv * hd:(kv + 1) * hd].astype(np.float64) @ q[i, h * hd:(h + 1) * hd] / math.sqrt(hd)
            p = np.exp(sc - sc.max())
            p /= p.sum()
            ref[i, h * hd:(h + 1) * hd] = p @ v[:n, kv * hd:(kv + 1) * hd]
    assert np.max(np.abs(got - ref)) < 2e-5


def test_argmax_first_max_tie(orc):
    x = np.array([1.0, 3.0, 2.0, 3.0, -1.0], np.float32)
    assert orc.argmax_first(x) == 1


def test_embed_and_interleave(orc):
    rng = np.random.default_rng(9)
    t = rng.integers(-128, 128, size=(10, 16), dtype=np.int8)
    s = rng.random(10).astype(np.float32)
    e = orc.embed_int8(t, s, 7)
    assert np.array_equal(e, t[7].astype(np.float32) * s[7])
    g = rng.integers(-128, 128, size=(3, 4), dtype=np.int8)
    u = rng.integers(-128, 128, size=(3, 4), dtype=np.int8)
    f, fs = orc.interleave_gate_up(g, np.arange(3, dtype=np.float32), u, np.arange(3, 6, dtype=np.float32))
    assert np.array_equal(f[0::2], g) and np.array_equal(f[1::2], u)
    assert fs.tolist() == [0, 3, 1, 4, 2, 5]


# ------------------------------------------------------- log-mel front end --
# crates/qwen-asr/tests/audio.rs, then float64 and loop-level cross-checks.

def test_ref_mel_spectrogram_short_audio(orc):  # audio.rs tests:47-60
    n = 8000
    i = np.arange(n, dtype=np.float32)
    s = (np.sin(np.float32(2.0) * np.float32(np.pi) * np.float32(440.0) * i / np.float32(16000.0)) *
         np.float32(0.5)).astype(np.float32)
    mel = orc.mel_spectrogram(s)
    assert mel is not None
    assert 20 < mel.shape[1] < 80 and mel.shape == (128, 50)
    # 440 Hz is 6.6 on the Slaney scale: filter 17 or 18 (centres 0.35 mel apart) peaks
    assert int(np.argmax(mel[:, 25])) in (17, 18)


def test_ref_mel_spectrogram_shape_and_range(orc):  # audio.rs tests:22-45 (11 s of synthetic audio for jfk.wav)
    from qwenasr_b200.synthetic import synthetic_audio
    s = synthetic_audio(11.0, seed=3)
    mel = orc.mel_spectrogram(s)
    assert mel.shape == (128, 1100)
    assert mel.min() >= -1.0 and mel.max() <= 2.0
    # the clamp: nothing below max - 8 in log10 units, i.e. 2 in normalised units
    assert mel.max() - mel.min() <= 2.0 + 1e-6


def test_mel_frame_count_and_too_short(orc):
    assert orc.mel_spectrogram(np.zeros(159, np.float32)) is None
    assert orc.mel_spectrogram(np.zeros(0, np.float32)) is None
    for n in (160, 170, 399, 401, 5287):
        assert orc.mel_spectrogram(np.ones(n, np.float32)).shape == (128, n // 160)


def test_mel_filters_slaney(orc):
    f = orc.mel_filters().astype(np.float64)
    assert f.shape == (128, 201) and (f >= 0).all()
    # each filter is a triangle over its two neighbours' centres, height 2/(width in Hz)
    hz = np.arange(201) * 8000.0 / 200.0

    def to_mel(h):
        return np.where(h >= 1000, 15 + np.log(np.maximum(h, 1e-9) / 1000) * 27 / np.log(6.4), 3 * h / 200)

    def to_hz(m):
        return np.where(m >= 15, 1000 * np.exp(np.log(6.4) / 27 * (m - 15)), 200 * m / 3)

    edges = to_hz(np.linspace(0, to_mel(np.array(8000.0)), 130))
    for m in (0, 40, 90, 127):
        lo, c, hi = edges[m], edges[m + 1], edges[m + 2]
        tri = np.maximum(np.minimum((hz - lo) / (c - lo), (hi - hz) / (hi - c)), 0) * 2 / (hi - lo)
        # f32 edges: near the triangle's feet the rise/fall terms cancel, hence the atol
        np.testing.assert_allclose(f[m], tri, rtol=2e-5, atol=1e-4 * tri.max())


def _mel_loop(orc, s):
    """Pure-Python loop restatement of audio.rs:271-385 on the oracle's tables
    (f32 scalar arithmetic, sequential sums), for a couple of frames."""
    win, ct, st = orc.mel_tables()
    filt = orc.mel_filters()
    n = len(s)
    frames = n // 160
    padded = np.zeros(n + 400, np.float32)
    for i in range(200):
        padded[i] = s[200 - i] if 200 - i < n else 0.0
        src = n - 2 - i
        padded[200 + n + i] = s[src] if src >= 0 else 0.0
    padded[200:200 + n] = s
    out = np.empty((frames, 128), np.float32)
    for t in range(frames):
        w = [padded[t * 160 + i] * win[i] for i in range(400)]
        power = []
        for k in range(201):
            re = np.float32(0)
            im = np.float32(0)
            for i in range(400):
                re = np.float32(re + w[i] * ct[k, i])
                im = np.float32(im + w[i] * st[k, i])
            power.append(np.float32(re * re + im * im))
        for m in range(128):
            acc = np.float32(0)
            for k in range(201):
                acc = np.float32(acc + filt[m, k] * power[k])
            out[t, m] = np.float32(math.log10(max(float(acc), float(np.float32(1e-10)))))
    top = out.max()
    return ((np.maximum(out, np.float32(top - np.float32(8))) + np.float32(4)) / np.float32(4)).T


@pytest.mark.parametrize("n", [170, 330])
def test_mel_matches_loop_restatement(orc, n):
    """Short inputs whose reflect padding runs off the signal (zeros)."""
    s = np.random.default_rng(n).standard_normal(n).astype(np.float32) * 0.1
    got = orc.mel_spectrogram(s)
    ref = _mel_loop(orc, s)
    # log10 in the loop is correctly rounded; the oracle calls glibc log10f (<= 1 ulp apart)
    assert np.max(np.abs(got - ref)) <= 2.5e-7


def test_mel_matches_float64(orc):
    """Whole pipeline against a float64 numpy derivation (numpy's reflect pad,
    rfft, the same filter bank): f32 DFT rounding only."""
    from qwenasr_b200.synthetic import synthetic_audio
    s = synthetic_audio(2.0, seed=11)
    got = orc.mel_spectrogram(s)
    n = len(s)
    x = np.pad(s.astype(np.float64), 200, mode="reflect")
    win = 0.5 * (1 - np.cos(2 * np.pi * np.arange(400) / 400))
    fr = np.stack([x[t * 160:t * 160 + 400] * win for t in range(n // 160)])
    p = np.abs(np.fft.rfft(fr, axis=1)) ** 2
    lm = np.log10(np.maximum(p @ orc.mel_filters().astype(np.float64).T, 1e-10))
    ref = ((np.maximum(lm, lm.max() - 8) + 4) / 4).T
    assert np.max(np.abs(got - ref)) < 2e-4


def test_encoder_composition_runs(orc):
    """The oracle's Encoder::forward composition (the encoder parity checker
    and CPU baseline): 13 tokens per full 100-frame chunk, the tail chunk's
    three stride-2 convs, finite rows of output_dim."""
    from qwenasr_b200 import synthetic
    cfg = dict(d_model=128, n_layers=1, n_heads=2, head_dim=64, ffn_dim=256, output_dim=96, chunk_size=100,
               n_window_infer=800)
    w = synthetic.encoder_weights_np(cfg, seed=5)
    mel = np.random.default_rng(5).standard_normal((128, 137)).astype(np.float32)
    out = orc.encoder_forward(w, cfg, mel)
    assert out.shape == (13 + 5, 96) and np.isfinite(out).all()
