"""GPU parity of every kernel-level entry point against the CPU oracle.

Bars: bit-exact for copies, gathers, KV indexing,
quantisation and the row kernels whose reference summation order is
reproduced (rms_norm, rms_norm_per_head, layer_norm, apply_rope_neox, the
reference fast-exp GELU/SwiGLU bodies); 1e-5 relative for f32 norms/RoPE
tables computed with transcendentals; 2e-3 relative for INT8 matvecs.
"""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qwenasr_b200 import kernels as K  # noqa: E402

DEV = "cuda:0"


def T(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def H(t):
    torch.cuda.synchronize()
    return t.detach().cpu().numpy()


def rel_close(got, ref, rtol):
    """|got-ref| <= rtol * (|ref| + rms(ref)): relative, with the row's RMS as
    the floor so cancellation near zero does not dominate."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.abs(ref) + math.sqrt(float(np.mean(ref * ref)) + 1e-30)
    err = np.max(np.abs(got - ref) / scale)
    return err <= rtol, err


@pytest.fixture(scope="module", autouse=True)
def _lib():
    from qwenasr_b200 import build
    build.build()
    assert torch.cuda.is_available()


# ------------------------------------------------------------------ norms --
@pytest.mark.parametrize("seq,hidden", [(512, 1024), (3, 896), (5, 23), (2, 2048), (1, 8), (4, 40)])
def test_rms_norm_bitexact(orc, seq, hidden):
    rng = np.random.default_rng(seq * 1000 + hidden)
    x = rng.standard_normal((seq, hidden)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
    out = torch.empty(seq, hidden, device=DEV)
    K.rms_norm(out, T(x), T(w), seq, hidden, 1e-6)
    assert np.array_equal(H(out), orc.rms_norm(x, w, 1e-6))


@pytest.mark.parametrize("seq,nh,hd", [(512, 16, 128), (512, 8, 128), (3, 8, 64), (2, 3, 100)])
def test_rms_norm_per_head_bitexact(orc, seq, nh, hd):
    rng = np.random.default_rng(seq + nh + hd)
    x = rng.standard_normal((seq, nh * hd)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    t = T(x)
    K.rms_norm_per_head(t, T(w), seq, nh, hd, 1e-6)
    assert np.array_equal(H(t), orc.rms_norm_per_head(x, w, nh, hd, 1e-6))


@pytest.mark.parametrize("seq,hidden", [(3000, 896), (7, 40), (3, 13), (2, 1024)])
def test_layer_norm_bitexact(orc, seq, hidden):
    rng = np.random.default_rng(seq + hidden)
    x = rng.standard_normal((seq, hidden)).astype(np.float32)
    w = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
    b = (0.02 * rng.standard_normal(hidden)).astype(np.float32)
    out = torch.empty(seq, hidden, device=DEV)
    K.layer_norm(out, T(x), T(w), T(b), seq, hidden, 1e-5)
    assert np.array_equal(H(out), orc.layer_norm(x, w, b, 1e-5))


# ------------------------------------------------------------------- RoPE --
def test_rope_table_and_compute(orc):
    n, hd = 4096, 128
    cos = torch.empty(n, hd, device=DEV)
    sin = torch.empty(n, hd, device=DEV)
    K.rope_cache_table(cos, sin, n, hd, 1e6)
    rc, rs = orc.rope_cache_table(n, hd, 1e6)
    gc, gs = H(cos), H(sin)
    # inv_freq is computed exactly as RopeCache does (host f32 powf); cos/sin of
    # the f32 angle are correctly rounded here, glibc's cosf/sinf are within
    # ~0.56 ulp, so about 1% of entries differ by one ulp (values in [-1, 1]).
    assert np.max(np.abs(gc - rc)) <= 2.5e-7 and np.max(np.abs(gs - rs)) <= 2.5e-7
    exact = np.mean(gc == rc) * 0.5 + np.mean(gs == rs) * 0.5
    assert exact > 0.98, exact
    pos = np.array([0, 1, 7, 1023, 4095, 20000], np.int32)
    c2 = torch.empty(pos.size, hd, device=DEV)
    s2 = torch.empty(pos.size, hd, device=DEV)
    K.compute_rope_neox(c2, s2, T(pos), pos.size, hd, 1e6)
    oc, os_ = orc.compute_rope_neox(pos, hd, 1e6)
    assert np.max(np.abs(H(c2) - oc)) <= 2.5e-7 and np.max(np.abs(H(s2) - os_)) <= 2.5e-7


@pytest.mark.parametrize("seq,nh,hd", [(512, 16, 128), (9, 8, 64), (3, 2, 6)])
def test_apply_rope_bitexact(orc, seq, nh, hd):
    rng = np.random.default_rng(nh * hd)
    x = rng.standard_normal((seq, nh * hd)).astype(np.float32)
    c, s = orc.rope_cache_table(seq + 5, hd, 1e6)
    c, s = c[5:], s[5:]
    t = T(x)
    K.apply_rope_neox(t, T(c), T(s), seq, nh, hd)
    assert np.array_equal(H(t), orc.apply_rope_neox(x, c, s, nh, hd))


def test_kv_append_bitexact_and_bounds():
    rng = np.random.default_rng(3)
    L, S, D = 4, 64, 1024
    kc = torch.zeros(L, S, D, device=DEV)
    vc = torch.zeros(L, S, D, device=DEV)
    kn = rng.standard_normal((5, D)).astype(np.float32)
    vn = rng.standard_normal((5, D)).astype(np.float32)
    K.kv_append(kc, vc, T(kn), T(vn), 2, S, D, 40, 5)
    k, v = H(kc), H(vc)
    assert np.array_equal(k[2, 40:45], kn) and np.array_equal(v[2, 40:45], vn)
    k[2, 40:45] = 0
    v[2, 40:45] = 0
    assert not k.any() and not v.any()
    from qwenasr_b200 import QasrError
    with pytest.raises(QasrError):
        K.kv_append(kc, vc, T(kn), T(vn), 2, S, D, 60, 5)


# ---------------------------------------------- config 1: pre-attn block --
@pytest.mark.parametrize("start_pos,layer", [(0, 0), (100, 3)])
def test_pre_attn_block_bitexact(orc, start_pos, layer):
    """x [512,1024], Q [512,16x128], K/V [512,8x128] ~ N(0,1),
    norm weights ~ N(1,0.02), eps 1e-6, RoPE theta 1e6, KV capacity 4096."""
    rng = np.random.default_rng(2024 + start_pos)
    S, Hd, nh, nkv, hd, cap, nl = 512, 1024, 16, 8, 128, 4096, 4
    x = rng.standard_normal((S, Hd)).astype(np.float32)
    w_in = (1 + 0.02 * rng.standard_normal(Hd)).astype(np.float32)
    q = rng.standard_normal((S, nh * hd)).astype(np.float32)
    k = rng.standard_normal((S, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((S, nkv * hd)).astype(np.float32)
    qw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    kw = (1 + 0.02 * rng.standard_normal(hd)).astype(np.float32)
    cos, sin = orc.rope_cache_table(cap, hd, 1e6)
    kc_ref = np.zeros((cap, nkv * hd), np.float32)
    vc_ref = np.zeros_like(kc_ref)
    xn_ref, q_ref, k_ref = orc.pre_attn_block(x, w_in, q, k, v, qw, kw, nh, nkv, hd, 1e-6, cos, sin, start_pos,
                                              kc_ref, vc_ref)
    xn = torch.empty(S, Hd, device=DEV)
    qt = T(q)
    kout = torch.empty(S, nkv * hd, device=DEV)
    kc = torch.zeros(nl, cap, nkv * hd, device=DEV)
    vc = torch.zeros(nl, cap, nkv * hd, device=DEV)
    K.pre_attn_block(xn, T(x), T(w_in), S, Hd, qt, T(k), T(v), kout, T(qw), T(kw), nh, nkv, hd, 1e-6, T(cos), T(sin),
                     start_pos, kc, vc, layer, cap)
    assert np.array_equal(H(xn), xn_ref)
    assert np.array_equal(H(qt), q_ref)
    assert np.array_equal(H(kout), k_ref)
    kg, vg = H(kc), H(vc)
    assert np.array_equal(kg[layer], kc_ref) and np.array_equal(vg[layer], vc_ref)
    kg[layer] = 0
    vg[layer] = 0
    assert not kg.any() and not vg.any()


# ---------------------------------------------------- config 2: encoder ----
def test_sinusoidal_pe(orc):
    pe = torch.empty(375, 896, device=DEV)
    K.sinusoidal_pe(pe, 375, 896)
    ref = orc.sinusoidal_pe(375, 896)
    g = H(pe)
    # one-ulp differences from glibc's expf/sinf/cosf rounding (see the RoPE test)
    assert np.max(np.abs(g - ref)) <= 2.5e-7
    assert np.mean(g == ref) > 0.98


def test_ln_pe_config2(orc):
    """BASELINE config 2 LN + PE: x [8x375, 896] ~ N(0,1), gamma ~ N(1,.02),
    beta ~ N(0,.02), eps 1e-5, PE per 375-frame item."""
    rng = np.random.default_rng(77)
    rows, d, npos = 3000, 896, 375
    x = rng.standard_normal((rows, d)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    pe = orc.sinusoidal_pe(npos, d)
    ref = orc.layer_norm(x, g, b, 1e-5) + np.tile(pe, (rows // npos, 1))
    out = torch.empty(rows, d, device=DEV)
    K.ln_pe(out, T(x), T(g), T(b), T(pe), rows, d, npos, 1e-5)
    assert np.array_equal(H(out), ref)


@pytest.mark.parametrize("rows,n_act", [(3000, 3000 * 3584), (37, 1001), (0, 4099), (13, 0)])
def test_ln_pe_gelu_erf_config2(orc, rows, n_act):
    """The one-launch config-2 pass: LN + PE bit-exact with the oracle, the
    GELU part bit-identical to qasr_gelu_erf and within 1e-5 of the oracle."""
    rng = np.random.default_rng(78 + rows)
    d, npos = 896, 375
    x = rng.standard_normal((max(rows, 1), d)).astype(np.float32)
    g = (1 + 0.02 * rng.standard_normal(d)).astype(np.float32)
    b = (0.02 * rng.standard_normal(d)).astype(np.float32)
    pe = orc.sinusoidal_pe(npos, d)
    a = (rng.standard_normal(max(n_act, 1)) * 3).astype(np.float32)
    out = torch.zeros(max(rows, 1), d, device=DEV)
    act = T(a)
    act_sep = T(a)
    K.ln_pe_gelu_erf(out, T(x), T(g), T(b), T(pe), rows, d, npos, 1e-5, act, n_act)
    if n_act:
        K.gelu_erf(act_sep, n_act)
        assert np.array_equal(H(act)[:n_act], H(act_sep)[:n_act])
        ok, err = rel_close(H(act)[:n_act], orc.gelu_erf(a[:n_act]), 1e-5)
        assert ok, err
    if rows:
        pe_rows = pe[np.arange(rows) % npos]
        assert np.array_equal(H(out)[:rows], orc.layer_norm(x[:rows], g, b, 1e-5) + pe_rows)


@pytest.mark.parametrize("n", [3000 * 3584, 1003, 8])
def test_gelu_tanh_reference_form(orc, n):
    rng = np.random.default_rng(n)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    t = T(x)
    K.gelu(t, n)
    g, ref = H(t), orc.gelu(x)
    body = n - n % 8
    assert np.array_equal(g[:body], ref[:body])
    assert np.allclose(g[body:], ref[body:], rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("n", [3000 * 3584, 1001])
def test_gelu_erf(orc, n):
    rng = np.random.default_rng(n + 1)
    x = (rng.standard_normal(n) * 3).astype(np.float32)
    t = T(x)
    K.gelu_erf(t, n)
    ok, err = rel_close(H(t), orc.gelu_erf(x), 1e-5)
    assert ok, err


def test_silu(orc):
    x = np.random.default_rng(5).standard_normal(4099).astype(np.float32) * 4
    t = T(x)
    K.silu(t, x.size)
    assert np.allclose(H(t), orc.silu(x), rtol=1e-6, atol=1e-7)


@pytest.mark.parametrize("seq,inter", [(512, 3072), (3, 3077)])
def test_swiglu_multiply(orc, seq, inter):
    gu = np.random.default_rng(inter).standard_normal((seq, 2 * inter)).astype(np.float32) * 3
    out = torch.empty(seq, inter, device=DEV)
    K.swiglu_multiply(out, T(gu), seq, inter)
    g, ref = H(out), orc.swiglu_multiply(gu, seq, inter)
    body = inter - inter % 8
    assert np.array_equal(g[:, :body], ref[:, :body])
    assert np.allclose(g[:, body:], ref[:, body:], rtol=1e-6, atol=1e-7)


def test_add_inplace():
    rng = np.random.default_rng(9)
    a, b = rng.standard_normal(1027).astype(np.float32), rng.standard_normal(1027).astype(np.float32)
    ta = T(a)
    K.add_inplace(ta, T(b), a.size)
    assert np.array_equal(H(ta), a + b)


# ----------------------------------------------- quantiser / gathers -------
def test_quantize_bitexact(orc):
    rng = np.random.default_rng(12)
    w = (rng.standard_normal((1000, 1024)) * 0.02).astype(np.float32)
    w[1] = 0
    w[2, :3] = [127.0, 63.5, -0.5]
    w[2, 3:] = 0
    q = torch.empty(1000, 1024, dtype=torch.int8, device=DEV)
    s = torch.empty(1000, device=DEV)
    K.quantize_f32_to_int8(T(w), 1000, 1024, q, s)
    qr, sr = orc.quantize_f32_to_int8(w)
    assert np.array_equal(H(q), qr) and np.array_equal(H(s), sr)


def test_embed_gather(orc):
    rng = np.random.default_rng(13)
    V, D = 151936, 1024
    table = (rng.standard_normal((V, D)) * 0.02).astype(np.float32)
    ids = rng.integers(0, V, 8).astype(np.int32)
    out = torch.empty(8, D, device=DEV)
    K.embed_gather(out, T(table), T(ids), 8, D, V)
    assert np.array_equal(H(out), table[ids])
    qt, qs = orc.quantize_f32_to_int8(table[:5000])
    ids2 = rng.integers(0, 5000, 5).astype(np.int32)
    out2 = torch.empty(5, D, device=DEV)
    K.embed_gather(out2, T(qt), T(ids2), 5, D, 5000, scales=T(qs))
    ref = np.stack([orc.embed_int8(qt, qs, int(i)) for i in ids2])
    assert np.array_equal(H(out2), ref)
    flag = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.embed_gather(out, T(table), T(np.array([0, V, -1, 5, 0, 0, 0, 0], np.int32)), 8, D, V, bad_id_flag=flag)
    assert int(H(flag)[0]) == 1


# --------------------------------------------------------- INT8 matvecs ----
@pytest.mark.parametrize("seq", [1, 3, 4, 8, 11])
@pytest.mark.parametrize("out_dim,in_dim", [(4096, 1024), (1024, 3072), (300, 896), (6144, 1024)])
def test_linear_nobias_int8(orc, seq, out_dim, in_dim):
    rng = np.random.default_rng(seq * 7 + out_dim + in_dim)
    w, s = orc.quantize_f32_to_int8((rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float32))
    x = rng.standard_normal((seq, in_dim)).astype(np.float32)
    y = torch.empty(seq, out_dim, device=DEV)
    K.linear_nobias_int8(y, T(x), T(w), T(s), seq, in_dim, out_dim)
    ok, err = rel_close(H(y), orc.linear_nobias_int8(x, w, s), 2e-3)
    assert ok and err < 5e-5, err


def test_linear_int8_bias(orc):
    rng = np.random.default_rng(21)
    w, s = orc.quantize_f32_to_int8((rng.standard_normal((896, 896)) * 0.02).astype(np.float32))
    b = (rng.standard_normal(896) * 0.1).astype(np.float32)
    x = rng.standard_normal((13, 896)).astype(np.float32)
    y = torch.empty(13, 896, device=DEV)
    K.linear_int8(y, T(x), T(w), T(s), T(b), 13, 896, 896)
    ok, err = rel_close(H(y), orc.linear_int8(x, w, s, b), 2e-3)
    assert ok and err < 5e-5, err


@pytest.mark.parametrize("seq,out_dim,in_dim,bias", [
    (33, 1024, 1024, False),    # just past one 32-token block
    (200, 4096, 1024, False),   # decoder prefill q|k|v rows
    (390, 896, 896, True),      # encoder projection, one 30 s window of tokens
    (100, 1000, 3072, True),    # rows not a multiple of the 128-row tile
    (1000, 4096, 1024, False),  # 64-token blocks (N = 192 MMAs), ragged last block
    (3000, 1000, 1024, True),   # 64-token blocks with a partial last weight tile
])
def test_int8_gemm_prefill_shapes(orc, seq, out_dim, in_dim, bias):
    """seq_len > 8 runs as one tensor-core GEMM (the reference: seq_len matvecs,
    mod.rs:650-673); same 2e-3 bar as the matvecs."""
    rng = np.random.default_rng(seq + out_dim)
    w, s = orc.quantize_f32_to_int8((rng.standard_normal((out_dim, in_dim)) * 0.02).astype(np.float32))
    x = (rng.standard_normal((seq, in_dim)) * rng.uniform(0.01, 10.0, (seq, 1))).astype(np.float32)
    y = torch.empty(seq, out_dim, device=DEV)
    if bias:
        b = (rng.standard_normal(out_dim) * 0.1).astype(np.float32)
        K.linear_int8(y, T(x), T(w), T(s), T(b), seq, in_dim, out_dim)
        ref = orc.linear_int8(x, w, s, b)
    else:
        K.linear_nobias_int8(y, T(x), T(w), T(s), seq, in_dim, out_dim)
        ref = orc.linear_nobias_int8(x, w, s)
    ok, err = rel_close(H(y), ref, 2e-3)
    assert ok and err < 5e-5, err
    # a second call with fewer rows reuses the digit scratch: stale rows must not leak
    y2 = torch.full((seq // 2, out_dim), float("nan"), device=DEV)
    K.linear_nobias_int8(y2, T(x[: seq // 2]), T(w), T(s), seq // 2, in_dim, out_dim)
    ok, err = rel_close(H(y2), orc.linear_nobias_int8(x[: seq // 2], w, s), 2e-3)
    assert ok and err < 5e-5, err


@pytest.mark.parametrize("seq,out_dim,in_dim,bias", [
    (1, 896, 896, True),        # one row
    (390, 3584, 896, True),     # encoder fc1 over a window of tokens
    (390, 896, 3584, True),     # encoder fc2
    (13, 896, 7680, False),     # conv_out-like K
    (70, 200, 1008, True),      # K not a multiple of 128 (tail tile zero-filled), N < 256
    (5, 50, 100, True),         # K % 16 != 0: CUDA-core fallback
    (3, 64, 64, False),         # below one tile: CUDA-core fallback
])
def test_linear_f32(orc, seq, out_dim, in_dim, bias):
    """kernels::linear (mod.rs:531, cblas_sgemm in the reference) against an
    fp64-accumulated oracle; both operands become exact int8 digit planes."""
    rng = np.random.default_rng(seq * 3 + out_dim + in_dim)
    w = (rng.standard_normal((out_dim, in_dim)) * rng.uniform(0.001, 0.2, (out_dim, 1))).astype(np.float32)
    x = (rng.standard_normal((seq, in_dim)) * rng.uniform(0.01, 5.0, (seq, 1))).astype(np.float32)
    b = (rng.standard_normal(out_dim) * 0.1).astype(np.float32) if bias else None
    y = torch.empty(seq, out_dim, device=DEV)
    if bias:
        K.linear(y, T(x), T(w), T(b), seq, in_dim, out_dim)
    else:
        K.linear_nobias(y, T(x), T(w), seq, in_dim, out_dim)
    ok, err = rel_close(H(y), orc.linear(x, w, b), 1e-5)
    assert ok, err


def test_matmul_t(orc):
    rng = np.random.default_rng(3)
    a = rng.standard_normal((17, 256)).astype(np.float32)
    b = rng.standard_normal((130, 256)).astype(np.float32)
    c = torch.empty(17, 130, device=DEV)
    K.matmul_t(c, T(a), T(b), 17, 256, 130)
    ok, err = rel_close(H(c), a.astype(np.float64) @ b.astype(np.float64).T, 1e-5)
    assert ok, err


@pytest.mark.parametrize("M", [1, 5, 8])
def test_matvec_residual_and_gateup_swiglu(orc, M):
    rng = np.random.default_rng(M)
    Hd, I = 1024, 3072
    wd, sd = orc.quantize_f32_to_int8((rng.standard_normal((Hd, I)) * 0.02).astype(np.float32))
    a = rng.standard_normal((M, I)).astype(np.float32)
    x = rng.standard_normal((M, Hd)).astype(np.float32)
    xt = T(x)
    K.int8_matvec_residual(xt, T(a), T(wd), T(sd), M, I, Hd)
    ok, err = rel_close(H(xt), x + orc.linear_nobias_int8(a, wd, sd), 2e-3)
    assert ok and err < 5e-5, err
    g, gs = orc.quantize_f32_to_int8((rng.standard_normal((I, Hd)) * 0.02).astype(np.float32))
    u, us = orc.quantize_f32_to_int8((rng.standard_normal((I, Hd)) * 0.02).astype(np.float32))
    gu, gus = orc.interleave_gate_up(g, gs, u, us)
    nw = (1 + 0.02 * rng.standard_normal(Hd)).astype(np.float32)
    h = torch.empty(M, I, device=DEV)
    K.int8_norm_gateup_swiglu(h, T(x), T(nw), T(gu), T(gus), M, Hd, I, 1e-6)
    xn = orc.rms_norm(x, nw, 1e-6)
    ref = np.stack([orc.swiglu_decode(orc.linear_nobias_int8(xn[m:m + 1], gu, gus)[0], I) for m in range(M)])
    ok, err = rel_close(H(h), ref, 2e-3)
    assert ok and err < 5e-5, err


@pytest.mark.parametrize("M", [1, 3, 8])
def test_final_norm_lmhead_argmax(orc, M):
    rng = np.random.default_rng(100 + M)
    V, Hd = 151936, 1024
    emb = (rng.standard_normal((V, Hd)) * 0.02).astype(np.float32)
    w, s = orc.quantize_f32_to_int8(emb)
    nw = (1 + 0.02 * rng.standard_normal(Hd)).astype(np.float32)
    x = rng.standard_normal((M, Hd)).astype(np.float32)
    ids = torch.empty(M, dtype=torch.int32, device=DEV)
    logits = torch.empty(M, V, device=DEV)
    K.final_norm_lmhead_argmax(ids, logits, T(x), T(nw), T(w), T(s), M, Hd, V, 1e-6)
    xn = orc.rms_norm(x, nw, 1e-6)
    ref_logits = orc.linear_nobias_int8(xn, w, s)
    ok, err = rel_close(H(logits), ref_logits, 2e-3)
    assert ok and err < 5e-5, err
    assert H(ids).tolist() == [orc.argmax_first(ref_logits[m]) for m in range(M)]
    # repeated calls re-arm the device-side keys/counter
    ids2 = torch.empty(M, dtype=torch.int32, device=DEV)
    K.final_norm_lmhead_argmax(ids2, None, T(x), T(nw), T(w), T(s), M, Hd, V, 1e-6)
    assert H(ids2).tolist() == H(ids).tolist()


def test_argmax_first_max_tie_rule():
    """Equal maxima: the lowest index wins (strict '>' scan, decoder.rs:942-947)."""
    V, Hd = 4096, 128
    w = np.zeros((V, Hd), np.int8)
    for r in (77, 1500, 4000):
        w[r, :] = 100
    s = np.ones(V, np.float32)
    x = np.ones((1, Hd), np.float32)
    nw = np.ones(Hd, np.float32)
    ids = torch.empty(1, dtype=torch.int32, device=DEV)
    K.final_norm_lmhead_argmax(ids, None, T(x), T(nw), T(w), T(s), 1, Hd, V, 1e-6)
    assert int(H(ids)[0]) == 77


# ------------------------------------------------------------ attention ----
@pytest.mark.parametrize("seq_q,seq_k,off,nh,nkv,hd", [
    (37, 37, 0, 16, 8, 128), (1, 1024, 1023, 16, 8, 128), (4, 200, 196, 16, 8, 128), (404, 404, 0, 16, 8, 128),
    (33, 100, 67, 16, 8, 128), (50, 50, 0, 8, 8, 64), (29, 70, 41, 6, 2, 64), (9, 40, 31, 16, 1, 128)])
def test_causal_attention(orc, seq_q, seq_k, off, nh, nkv, hd):
    """Prefill shapes, key tiles crossed at offsets, GQA groups of 1, 2, 3, 16."""
    rng = np.random.default_rng(seq_q + seq_k)
    q = rng.standard_normal((seq_q, nh * hd)).astype(np.float32)
    k = rng.standard_normal((seq_k, nkv * hd)).astype(np.float32)
    v = rng.standard_normal((seq_k, nkv * hd)).astype(np.float32)
    out = torch.empty(seq_q, nh * hd, device=DEV)
    scale = 1.0 / math.sqrt(hd)
    K.causal_attention(out, T(q), T(k), T(v), seq_q, seq_k, nh, nkv, hd, scale, off)
    ref = orc.causal_attention(q, k, v, seq_q, seq_k, nh, nkv, hd, off, np.float32(scale))
    assert np.max(np.abs(H(out) - ref)) < 2e-5


# -------------------------------------------------------- encoder kernels --
def _conv2d_ref(x, w, b, c_in, c_out, h, wd, kh, kw, stride, pad):
    """fp64 im2col + GEMM (conv2d, mod.rs:790-860, cblas_sgemm in the reference)."""
    ho, wo = (h + 2 * pad - kh) // stride + 1, (wd + 2 * pad - kw) // stride + 1
    xp = np.zeros((c_in, h + 2 * pad, wd + 2 * pad))
    xp[:, pad:pad + h, pad:pad + wd] = x.reshape(c_in, h, wd)
    cols = np.empty((c_in * kh * kw, ho * wo))
    for ic in range(c_in):
        for ki in range(kh):
            for kj in range(kw):
                cols[(ic * kh + ki) * kw + kj] = xp[ic, ki:ki + stride * ho:stride, kj:kj + stride * wo:stride].ravel()
    out = w.reshape(c_out, -1).astype(np.float64) @ cols
    return out + (b[:, None] if b is not None else 0.0)


@pytest.mark.parametrize("c_in,c_out,h,w,bias", [
    (1, 480, 128, 100, True),    # encoder conv1: [1,128,chunk] -> [480,64,50] (patch 9: CUDA cores)
    (480, 480, 64, 50, True),    # conv2 -> [480,32,25] (patch 4320: tensor cores)
    (480, 480, 32, 25, False),   # conv3 -> [480,16,13]
])
def test_conv2d_encoder_stem(c_in, c_out, h, w, bias):
    rng = np.random.default_rng(c_in + h)
    x = rng.standard_normal((c_in, h, w)).astype(np.float32)
    wt = (rng.standard_normal((c_out, c_in, 3, 3)) * 0.05).astype(np.float32)
    b = (rng.standard_normal(c_out) * 0.1).astype(np.float32) if bias else None
    ho, wo = (h - 1) // 2 + 1, (w - 1) // 2 + 1
    out = torch.empty(c_out, ho * wo, device=DEV)
    K.conv2d(out, T(x), T(wt), T(b) if bias else None, c_in, c_out, h, w, 3, 3, 2, 1)
    ok, err = rel_close(H(out), _conv2d_ref(x, wt, b, c_in, c_out, h, w, 3, 3, 2, 1), 1e-5)
    assert ok, err


@pytest.mark.parametrize("seq,n_heads,hd,win", [(390, 14, 64, 104), (37, 2, 128, 37), (50, 3, 64, 7),
                                                (1000, 2, 128, 1000), (300, 2, 64, "ragged")])
def test_bidirectional_attention(orc, seq, n_heads, hd, win):
    """Windows held in shared memory, a window too long for it (1000 keys of
    128 dims: the L2 kernel), and ragged windows including one-key ones."""
    rng = np.random.default_rng(seq + (win if win != "ragged" else 1))
    q, k, v = (rng.standard_normal((seq, n_heads * hd)).astype(np.float32) for _ in range(3))
    if win == "ragged":
        starts = np.array([0, 1, 2, 40, 41, 170, 299, seq], np.int32)
    else:
        starts = np.array(list(range(0, seq, win)) + [seq], np.int32)
    scale = 1.0 / math.sqrt(hd)
    out = torch.empty(seq, n_heads * hd, device=DEV)
    K.bidirectional_attention(out, T(q), T(k), T(v), seq, n_heads, hd, scale, T(starts), len(starts) - 1)
    ref = orc.bidirectional_attention(q, k, v, seq, n_heads, hd, starts, np.float32(scale))
    assert np.max(np.abs(H(out) - ref)) < 2e-5
