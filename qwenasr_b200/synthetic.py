"""Seeded synthetic inputs and random-init weights of the benchmark configs.

No model checkpoints exist on the build or GPU machines, so weights are
random with the architecture's shapes (config.rs:56-82 defaults, 0.6B/1.7B
shapes of config.rs:110-156):  matrices ~ N(0, 0.02) quantised per output
channel to INT8 by the qwen-asr-quantize rule (quantize.rs:633-662), norm
weights ~ N(1, 0.02), embedding table ~ N(0, 0.02).  The gate/up matrices
are stored with rows interleaved g0,u0,g1,u1,... as DecoderInt8::load does
(decoder.rs:699-719).

Two generators with the same distributions:
  * layer_weights_np: numpy on the host (parity tests, CPU baseline);
  * layer_weights_gpu: torch on the GPU, quantised by the library's own
    qasr_quantize_f32_to_int8 kernel (benchmarks at full size).
"""
from __future__ import annotations

import numpy as np

DEC_0_6B = dict(hidden=1024, inter=3072, n_layers=28, n_heads=16, n_kv_heads=8, head_dim=128, vocab=151936,
                eps=1e-6, theta=1e6)
DEC_1_7B = dict(DEC_0_6B, hidden=2048, inter=6144)


def quantize_np(w: np.ndarray):
    """quantize_f32_to_int8 (quantize.rs:633-662) in numpy: absmax/127 scales,
    round half away from zero, clamp to [-128, 127]."""
    w = np.asarray(w, np.float32)
    absmax = np.abs(w).max(axis=1)
    scales = (absmax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax > 0, np.float32(127.0) / absmax, np.float32(0.0)).astype(np.float32)
    v = (w * inv[:, None]).astype(np.float32)
    a = np.abs(v)
    r = np.floor(a)
    q = np.copysign(r + (a - r >= np.float32(0.5)), v)  # a - r is exact: half away from zero
    return np.clip(q, -128, 127).astype(np.int8), scales


def interleave_rows(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    out = np.empty((a.shape[0] * 2,) + a.shape[1:], a.dtype)
    out[0::2] = a
    out[1::2] = b
    return out


def layer_weights_np(cfg: dict, rng: np.random.Generator, quantize=quantize_np) -> dict:
    """One decoder layer (DecLayerInt8, decoder.rs:652-663) as numpy arrays."""
    H, I, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    q_dim, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd
    out = {}
    for name, shape in (("wq", (q_dim, H)), ("wk", (kv, H)), ("wv", (kv, H)), ("wo", (H, q_dim)),
                        ("down", (H, I))):
        out[name], out[name + "_s"] = quantize((rng.standard_normal(shape, np.float32) * np.float32(0.02)))
    g, gs = quantize(rng.standard_normal((I, H), np.float32) * np.float32(0.02))
    u, us = quantize(rng.standard_normal((I, H), np.float32) * np.float32(0.02))
    out["gate_up"] = interleave_rows(g, u)
    out["gate_up_s"] = interleave_rows(gs, us)
    for name, n in (("q_norm", hd), ("k_norm", hd), ("input_norm", H), ("post_attn_norm", H)):
        out[name] = (1.0 + 0.02 * rng.standard_normal(n)).astype(np.float32)
    return out


def decoder_weights_np(cfg: dict, seed: int, quantize=quantize_np) -> dict:
    """Full random decoder: layers, f32 embedding table, final norm, INT8 lm head
    (quantised from the embedding table, i.e. tied weights in INT8 form)."""
    rng = np.random.default_rng(seed)
    layers = [layer_weights_np(cfg, rng, quantize) for _ in range(cfg["n_layers"])]
    emb = rng.standard_normal((cfg["vocab"], cfg["hidden"]), np.float32) * np.float32(0.02)
    lm, lms = quantize(emb)
    norm = (1.0 + 0.02 * rng.standard_normal(cfg["hidden"])).astype(np.float32)
    return dict(cfg=dict(cfg), layers=layers, embed=emb, norm=norm, lm_head=lm, lm_head_s=lms)


def layer_weights_gpu(cfg: dict, gen, device, quantize_gpu) -> dict:
    """Same distributions on the GPU (torch.Generator `gen`); quantize_gpu(w)
    -> (int8, scales) is the library's quantiser."""
    import torch
    H, I, hd = cfg["hidden"], cfg["inter"], cfg["head_dim"]
    q_dim, kv = cfg["n_heads"] * hd, cfg["n_kv_heads"] * hd

    def rn(*shape):
        return torch.randn(*shape, generator=gen, device=device, dtype=torch.float32) * 0.02

    out = {}
    for name, shape in (("wq", (q_dim, H)), ("wk", (kv, H)), ("wv", (kv, H)), ("wo", (H, q_dim)),
                        ("down", (H, I))):
        out[name], out[name + "_s"] = quantize_gpu(rn(*shape))
    g, gs = quantize_gpu(rn(I, H))
    u, us = quantize_gpu(rn(I, H))
    out["gate_up"] = torch.stack([g, u], 1).reshape(2 * I, H).contiguous()
    out["gate_up_s"] = torch.stack([gs, us], 1).reshape(2 * I).contiguous()
    for name, n in (("q_norm", hd), ("k_norm", hd), ("input_norm", H), ("post_attn_norm", H)):
        out[name] = 1.0 + 0.02 * torch.randn(n, generator=gen, device=device, dtype=torch.float32)
    return out


# Audio encoder (encoder.rs; 0.6B config: d_model 896, 18 layers, 14 x 64
# heads, ffn 3584, output = decoder hidden 1024, chunk 100 frames, window 800).
ENC_0_6B = dict(d_model=896, n_layers=18, n_heads=14, head_dim=64, ffn_dim=3584, output_dim=1024, chunk_size=100,
                n_window_infer=800)
CONV_HIDDEN = 480


def encoder_weights_np(cfg: dict, seed: int) -> dict:
    """f32 encoder weights: matrices ~ N(0, 0.02) (conv kernels N(0, 0.05)),
    LayerNorm weights ~ N(1, 0.02), biases ~ N(0, 0.02)."""
    rng = np.random.default_rng(seed)
    D, F, O, CH = cfg["d_model"], cfg["ffn_dim"], cfg["output_dim"], CONV_HIDDEN

    def mat(*shape, s=0.02):
        return (rng.standard_normal(shape) * s).astype(np.float32)

    def ones(n):
        return (1 + 0.02 * rng.standard_normal(n)).astype(np.float32)

    w = {"conv1_w": mat(CH, 1, 3, 3, s=0.05), "conv1_b": mat(CH), "conv2_w": mat(CH, CH, 3, 3, s=0.05),
         "conv2_b": mat(CH), "conv3_w": mat(CH, CH, 3, 3, s=0.05), "conv3_b": mat(CH), "conv_out_w": mat(D, CH * 16),
         "ln_post_w": ones(D), "ln_post_b": mat(D), "proj1_w": mat(D, D), "proj1_b": mat(D), "proj2_w": mat(O, D),
         "proj2_b": mat(O), "layers": []}
    for _ in range(cfg["n_layers"]):
        w["layers"].append({"attn_norm_w": ones(D), "attn_norm_b": mat(D), "wq": mat(D, D), "bq": mat(D),
                            "wk": mat(D, D), "bk": mat(D), "wv": mat(D, D), "bv": mat(D), "wo": mat(D, D),
                            "bo": mat(D), "ffn_norm_w": ones(D), "ffn_norm_b": mat(D), "fc1_w": mat(F, D),
                            "fc1_b": mat(F), "fc2_w": mat(D, F), "fc2_b": mat(D)})
    return w


ENC_1_7B = dict(ENC_0_6B, d_model=1024, n_layers=24, n_heads=16, ffn_dim=4096, output_dim=2048)

SAMPLE_RATE = 16000


def synthetic_audio(seconds: float, seed: int) -> np.ndarray:
    """16 kHz mono test signal: pink noise at -20 dBFS RMS plus three
    sinusoids of random frequency in [200, 3000] Hz (amplitude 0.05 each,
    random phase), float32 in [-1, 1].  Stands in for speech recordings,
    which do not exist on these machines."""
    rng = np.random.default_rng(seed)
    n = int(round(seconds * SAMPLE_RATE))
    if n == 0:
        return np.zeros(0, np.float32)
    spec = np.fft.rfft(rng.standard_normal(n))
    f = np.arange(len(spec), dtype=np.float64)
    f[0] = 1.0
    pink = np.fft.irfft(spec / np.sqrt(f), n)
    pink *= 0.1 / max(np.sqrt(np.mean(pink * pink)), 1e-12)
    t = np.arange(n, dtype=np.float64) / SAMPLE_RATE
    for hz, ph in zip(rng.uniform(200.0, 3000.0, 3), rng.uniform(0.0, 2 * np.pi, 3)):
        pink += 0.05 * np.sin(2 * np.pi * hz * t + ph)
    return np.clip(pink, -1.0, 1.0).astype(np.float32)


def encoder_weights_gpu(cfg: dict, gen, device) -> dict:
    """encoder_weights_np's distributions drawn on the GPU with torch (for
    benchmarks at full size; the values differ from the numpy draw)."""
    import torch
    D, F, O, CH = cfg["d_model"], cfg["ffn_dim"], cfg["output_dim"], CONV_HIDDEN

    def mat(*shape, s=0.02):
        return torch.randn(*shape, generator=gen, device=device) * s

    def ones(n):
        return 1.0 + 0.02 * torch.randn(n, generator=gen, device=device)

    w = {"conv1_w": mat(CH, 1, 3, 3, s=0.05), "conv1_b": mat(CH), "conv2_w": mat(CH, CH, 3, 3, s=0.05),
         "conv2_b": mat(CH), "conv3_w": mat(CH, CH, 3, 3, s=0.05), "conv3_b": mat(CH), "conv_out_w": mat(D, CH * 16),
         "ln_post_w": ones(D), "ln_post_b": mat(D), "proj1_w": mat(D, D), "proj1_b": mat(D), "proj2_w": mat(O, D),
         "proj2_b": mat(O), "layers": []}
    for _ in range(cfg["n_layers"]):
        w["layers"].append({"attn_norm_w": ones(D), "attn_norm_b": mat(D), "wq": mat(D, D), "bq": mat(D),
                            "wk": mat(D, D), "bk": mat(D), "wv": mat(D, D), "bv": mat(D), "wo": mat(D, D),
                            "bo": mat(D), "ffn_norm_w": ones(D), "ffn_norm_b": mat(D), "fc1_w": mat(F, D),
                            "fc1_b": mat(F), "fc2_w": mat(D, F), "fc2_b": mat(D)})
    return w


def quantize_encoder(w: dict, quantize=quantize_np) -> dict:
    """The EncoderInt8 form of f32 encoder weights (what qwen-asr-quantize
    writes to a V2 file): conv_out, q/k/v/o, fc1, fc2, proj1, proj2 as INT8
    with per-row scales (keys "<m>" + "<m>_s"); convolutions, biases and norms
    stay f32."""
    out = {k: w[k] for k in ("conv1_w", "conv1_b", "conv2_w", "conv2_b", "conv3_w", "conv3_b", "ln_post_w",
                             "ln_post_b", "proj1_b", "proj2_b")}
    for dst, src in (("conv_out", "conv_out_w"), ("proj1", "proj1_w"), ("proj2", "proj2_w")):
        out[dst], out[dst + "_s"] = quantize(np.asarray(w[src], np.float32))
    out["layers"] = []
    for L in w["layers"]:
        q = {k: L[k] for k in ("attn_norm_w", "attn_norm_b", "bq", "bk", "bv", "bo", "ffn_norm_w", "ffn_norm_b",
                               "fc1_b", "fc2_b")}
        for dst, src in (("wq", "wq"), ("wk", "wk"), ("wv", "wv"), ("wo", "wo"), ("fc1", "fc1_w"), ("fc2", "fc2_w")):
            q[dst], q[dst + "_s"] = quantize(np.asarray(L[src], np.float32))
        out["layers"].append(q)
    return out
