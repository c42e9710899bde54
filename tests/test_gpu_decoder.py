"""GPU parity of the INT8 decoder engine (one greedy decode step per call)
against the oracle's decoder_forward_int8 (decoder.rs:845-965), sequence by
sequence: identical greedy token ids, logits within 2e-3 relative, and the
K/V rows written to each sequence's cache within 2e-3 relative."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

from qwenasr_b200 import synthetic  # noqa: E402
from qwenasr_b200.decoder import Decoder  # noqa: E402

DEV = "cuda:0"


def rel_err(got, ref):
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    scale = np.abs(ref) + math.sqrt(float(np.mean(ref * ref)) + 1e-30)
    return float(np.max(np.abs(got - ref) / scale))


def build_pair(orc, cfg, seed, max_seq, max_batch=8):
    w = synthetic.decoder_weights_np(cfg, seed)
    od = orc.OracleDecoder(w)
    dec = Decoder(cfg, device=0, max_batch=max_batch, max_seq=max_seq)
    for i, lw in enumerate(w["layers"]):
        dec.set_layer(i, lw)
    dec.set_globals(w["embed"], w["norm"], w["lm_head"], w["lm_head_s"])
    return w, od, dec


def prefill_random_kv(dec, od, slot, upto, rng):
    """Random K/V history rows 0..upto-1 in both engines (stand-in for a prefill)."""
    k, v = dec.kv(slot)
    kh, vh = od.new_kv(dec.max_seq)
    kh[:, :upto] = rng.standard_normal((kh.shape[0], upto, kh.shape[2])).astype(np.float32)
    vh[:, :upto] = rng.standard_normal((vh.shape[0], upto, vh.shape[2])).astype(np.float32)
    k.copy_(torch.from_numpy(kh))
    v.copy_(torch.from_numpy(vh))
    torch.cuda.synchronize()
    return kh, vh


SMALL = dict(synthetic.DEC_0_6B, n_layers=2, vocab=4096)


@pytest.mark.parametrize("M", [1, 3, 8])
def test_decode_step_small(orc, M):
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=100 + M, max_seq=1100)
    rng = np.random.default_rng(M)
    positions = np.array([0, 17, 1023, 5, 300, 999, 64, 1][:M], np.int32)
    tokens = rng.integers(0, SMALL["vocab"], M).astype(np.int32)
    hist = [prefill_random_kv(dec, od, m, int(positions[m]), rng) for m in range(M)]
    dec.keep_logits(True)
    nxt = dec.step(tokens, positions)
    logits = dec.logits(M).cpu().numpy()
    for m in range(M):
        kh, vh = hist[m]
        tok, ref_logits, _ = od.forward(kh, vh, int(positions[m]), w["embed"][tokens[m]], want_logits=True)
        assert int(nxt[m]) == tok, (m, int(nxt[m]), tok)
        assert rel_err(logits[m], ref_logits) < 2e-3
        kg, vg = dec.kv(m)
        p = int(positions[m])
        assert rel_err(kg[:, p].cpu().numpy(), kh[:, p]) < 2e-3
        assert rel_err(vg[:, p].cpu().numpy(), vh[:, p]) < 2e-3
        # history rows untouched, rows after p untouched
        assert np.array_equal(kg[:, :p].cpu().numpy(), kh[:, :p])
        assert not kg[:, p + 1:].cpu().numpy().any()
    dec.close()


@pytest.mark.parametrize("M,positions", [(1, [0]), (2, [0, 1]), (5, [3, 64, 200, 1023, 65]), (8, [1023] * 8)])
def test_persistent_and_per_layer_steps_agree(orc, M, positions):
    """The persistent step kernel and the per-layer kernels (the default) give
    the oracle's ids and logits within 2e-3, at histories from empty to full."""
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=300 + M, max_seq=1100, max_batch=8)
    assert dec.step_kernel(M) == 1  # the default path is the per-layer kernels
    rng = np.random.default_rng(40 + M)
    pos = np.array(positions, np.int32)
    tokens = rng.integers(0, SMALL["vocab"], M).astype(np.int32)
    hist = [prefill_random_kv(dec, od, m, int(pos[m]), rng) for m in range(M)]
    dec.keep_logits(True)
    results = {}
    for mode in (0, 1):
        dec.set_step_kernel(mode)
        assert dec.step_kernel(M) == mode
        nxt = dec.step(tokens, pos)
        results[mode] = (nxt.copy(), dec.logits(M).cpu().numpy().copy())
    for m in range(M):
        kh, vh = hist[m]
        tok, ref_logits, _ = od.forward(kh, vh, int(pos[m]), w["embed"][tokens[m]], want_logits=True)
        for mode in (0, 1):
            ids, logits = results[mode]
            assert int(ids[m]) == tok, (mode, m, int(ids[m]), tok)
            assert rel_err(logits[m], ref_logits) < 2e-3, mode
    dec.close()


def test_step_timeline_in_both_modes(orc):
    """qasr_decoder_trace: a traced step gives the untraced step's ids, every
    per-layer launch stamps a start before its end in launch order, and the
    persistent kernel stamps every phase of every layer on some CTA."""
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=77, max_seq=300, max_batch=4)
    rng = np.random.default_rng(77)
    pos = np.array([5, 120, 250], np.int32)
    tokens = rng.integers(0, SMALL["vocab"], 3).astype(np.int32)
    for m in range(3):
        prefill_random_kv(dec, od, m, int(pos[m]), rng)
    L = SMALL["n_layers"]
    ref = dec.step(tokens, pos).copy()
    t = dec.trace_step(tokens, pos)
    assert t.shape == (5 * L + 1, 2)
    start, end = t[:, 0].astype(np.int64), t[:, 1].astype(np.int64)
    assert (t[:, 0] != np.uint64(2**64 - 1)).all() and (end > start).all()
    assert (np.diff(start) > 0).all()  # PDL lets a launch start early, never before its predecessor
    assert (dec.step(tokens, pos) == ref).all()
    dec.set_step_kernel(0)
    if dec.step_kernel(3) == 0:
        p = dec.trace_step(tokens, pos)
        assert p.shape[1:] == (L + 1, 5, 4)
        assert (p[:, :L, :, 0].max(axis=0) > 0).all()  # every phase entered by some CTA
        assert (p[:, L, 0, 0] > 0).any()  # the lm head
        assert (dec.step(tokens, pos) == ref).all()
    dec.close()


def test_greedy_loop_matches_oracle(orc):
    """Five greedy steps fed back through both engines give the same ids."""
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=7, max_seq=64, max_batch=2)
    rng = np.random.default_rng(1)
    toks = rng.integers(0, SMALL["vocab"], 2).astype(np.int32)
    caches = [od.new_kv(64) for _ in range(2)]
    gpu_ids, ref_ids = [], []
    t_gpu, t_ref = toks.copy(), toks.copy()
    for step in range(5):
        pos = np.array([step, step], np.int32)
        t_gpu = dec.step(t_gpu, pos)
        nxt = []
        for m in range(2):
            tok, _, _ = od.forward(caches[m][0], caches[m][1], step, w["embed"][t_ref[m]])
            nxt.append(tok)
        t_ref = np.array(nxt, np.int32)
        gpu_ids.append(t_gpu.tolist())
        ref_ids.append(t_ref.tolist())
    assert gpu_ids == ref_ids
    dec.close()


def test_step_input_validation(orc):
    w, od, dec = build_pair(orc, dict(SMALL, n_layers=1), seed=3, max_seq=32, max_batch=2)
    from qwenasr_b200 import QasrError
    with pytest.raises(QasrError, match="outside"):
        dec.step([SMALL["vocab"]], [0])
    with pytest.raises(QasrError, match="outside"):
        dec.step([1], [32])
    with pytest.raises(QasrError):
        dec.step([1, 2, 3], [0, 0, 0])  # M > max_batch
    # device path: a bad id is flagged on the device and reported by the next host step
    assert dec.step([1], [0]).shape == (1,)
    dec.close()


def test_device_step_matches_host_step(orc):
    w, od, dec = build_pair(orc, SMALL, seed=9, max_seq=128, max_batch=4)
    toks = np.array([5, 6, 7, 8], np.int32)
    pos = np.array([3, 3, 3, 3], np.int32)
    host = dec.step(toks, pos)
    t = torch.from_numpy(toks).to(DEV)
    p = torch.from_numpy(pos).to(DEV)
    out = torch.empty(4, dtype=torch.int32, device=DEV)
    dec.step_device(t, p, out)
    dec.stream.synchronize()
    assert out.cpu().numpy().tolist() == host.tolist()
    dec.close()


FULL_CASES = {
    # the benchmarked configuration (0.6B, 28 layers, full vocab, KV 1024) at
    # the batch sizes whose kernel choices differ (attention CTA width from
    # M = 4, cluster sizes per M), and the 1.7B decode shape of the
    # segmented workload (KV around 480)
    "0.6b_m2": ("DEC_0_6B", 1024, [1023, 600]),
    "0.6b_m4": ("DEC_0_6B", 1024, [1023, 17, 1023, 700]),
    "0.6b_m8": ("DEC_0_6B", 1024, [1023, 1023, 600, 1023, 17, 900, 1023, 512]),
    "1.7b_m8": ("DEC_1_7B", 480, [479, 479, 300, 479, 100, 479, 479, 5]),
}


@pytest.mark.slow
@pytest.mark.parametrize("case,mode", [(c, 1) for c in FULL_CASES] + [("0.6b_m8", 0), ("1.7b_m8", 0)])
def test_decode_step_full_depth(orc, case, mode):
    """All 28 layers and the 151936-row lm head, sequences at mixed positions:
    ids identical to the oracle's, logits and the new K/V rows within 2e-3
    (mode 1: the per-layer kernels, mode 0: the persistent step kernel)."""
    orc.set_threads(16)
    name, max_seq, pos = FULL_CASES[case]
    cfg = getattr(synthetic, name)
    M = len(pos)
    w, od, dec = build_pair(orc, cfg, seed=2026 + M, max_seq=max_seq, max_batch=M)
    dec.set_step_kernel(mode)
    assert dec.step_kernel(M) == mode
    rng = np.random.default_rng(5 + M)
    positions = np.array(pos, np.int32)
    tokens = rng.integers(0, cfg["vocab"], M).astype(np.int32)
    dec.keep_logits(True)
    hist = []
    for m in range(M):
        hist.append(prefill_random_kv(dec, od, m, int(positions[m]), rng))
    nxt = dec.step(tokens, positions)
    logits = dec.logits(M).cpu().numpy()
    for m in range(M):
        kh, vh = hist[m]
        p = int(positions[m])
        tok, ref_logits, _ = od.forward(kh, vh, p, w["embed"][tokens[m]], want_logits=True)
        assert int(nxt[m]) == tok, (m, int(nxt[m]), tok)
        assert rel_err(logits[m], ref_logits) < 2e-3
        kg, vg = dec.kv(m)
        assert rel_err(kg[:, p].cpu().numpy(), kh[:, p]) < 2e-3
        assert rel_err(vg[:, p].cpu().numpy(), vh[:, p]) < 2e-3
        hist[m] = None
    dec.close()


@pytest.mark.parametrize("P", [1, 37, 129])
def test_prefill_then_decode_matches_oracle(orc, P):
    """decoder_prefill_int8 (decoder.rs:751-842) in two chunks, then one decode
    step at position P: K/V rows, residual stream, logits and the greedy id
    against the oracle's prefill + forward."""
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=50 + P, max_seq=256, max_batch=1)
    rng = np.random.default_rng(P)
    ids = rng.integers(0, SMALL["vocab"], P + 1).astype(np.int32)
    emb = w["embed"][ids[:P]]
    kh, vh = od.new_kv(256)
    ref_x = od.prefill(kh, vh, 0, emb)
    cut = P // 2
    if cut:
        dec.prefill(0, emb[:cut], 0)
    dec.prefill(0, torch.from_numpy(emb[cut:]).to(DEV), cut)  # host and device prompt rows
    kg, vg = dec.kv(0)
    assert rel_err(kg[:, :P].cpu().numpy(), kh[:, :P]) < 2e-3
    assert rel_err(vg[:, :P].cpu().numpy(), vh[:, :P]) < 2e-3
    assert not kg[:, P:].cpu().numpy().any()
    assert rel_err(dec.prefill_hidden(P - cut).cpu().numpy(), ref_x[cut:]) < 2e-3
    dec.keep_logits(True)
    nxt = dec.step(ids[P:P + 1], [P])
    tok, ref_logits, _ = od.forward(kh, vh, P, w["embed"][ids[P]], want_logits=True)
    assert int(nxt[0]) == tok
    assert rel_err(dec.logits(1).cpu().numpy()[0], ref_logits) < 2e-3
    with pytest.raises(Exception, match="outside"):
        dec.prefill(0, emb[:1], 256)
    dec.close()


def test_segment_batch_greedy_matches_oracle(orc):
    """segments.decode_batch (the per-rank work of the batched-segment mode):
    prompts of different lengths prefilled into their own slots, then greedy
    steps at per-sequence positions; ids equal the oracle's prefill + forward."""
    from qwenasr_b200 import segments
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL, seed=9, max_seq=96, max_batch=3)
    rng = np.random.default_rng(5)
    lens = [5, 0, 23]
    prompts = [w["embed"][rng.integers(0, SMALL["vocab"], n)] for n in lens]
    first = rng.integers(0, SMALL["vocab"], 3).astype(np.int32)
    got = segments.decode_batch(dec, prompts, first, 4)
    for i, n in enumerate(lens):
        kh, vh = od.new_kv(96)
        if n:
            od.prefill(kh, vh, 0, prompts[i])
        tok, ids = int(first[i]), []
        for k in range(4):
            tok, _, _ = od.forward(kh, vh, n + k, w["embed"][tok])
            ids.append(tok)
        assert got[i] == ids, (i, got[i], ids)
    dec.close()


SMALL_1P7B = dict(synthetic.DEC_1_7B, n_layers=2, vocab=4096)


@pytest.mark.parametrize("M", [1, 8])
def test_decode_step_1p7b_shapes(orc, M):
    """The 1.7B decoder shapes (hidden 2048, intermediate 6144): every
    contraction has K = 2048 or 6144 and the planner's cluster / stage
    choices differ from 0.6B.  Prefill a prompt per slot, then two greedy
    steps: ids, logits and K/V rows against the oracle."""
    orc.set_threads(8)
    w, od, dec = build_pair(orc, SMALL_1P7B, seed=70 + M, max_seq=128, max_batch=M)
    rng = np.random.default_rng(70 + M)
    P = [int(p) for p in rng.integers(1, 60, M)]
    caches, toks = [], rng.integers(0, SMALL_1P7B["vocab"], M).astype(np.int32)
    for m in range(M):
        kh, vh = od.new_kv(128)
        emb = w["embed"][rng.integers(0, SMALL_1P7B["vocab"], P[m])]
        od.prefill(kh, vh, 0, emb)
        dec.prefill(m, emb, 0)
        caches.append((kh, vh))
    dec.keep_logits(True)
    pos = np.array(P, np.int32)
    for _ in range(2):
        nxt = dec.step(toks, pos)
        logits = dec.logits(M).cpu().numpy()
        for m in range(M):
            kh, vh = caches[m]
            tok, ref_logits, _ = od.forward(kh, vh, int(pos[m]), w["embed"][toks[m]], want_logits=True)
            assert int(nxt[m]) == tok
            assert rel_err(logits[m], ref_logits) < 2e-3
            kg, _ = dec.kv(m)
            assert rel_err(kg[:, :pos[m] + 1].cpu().numpy(), kh[:, :pos[m] + 1]) < 2e-3
        toks = nxt.astype(np.int32)
        pos = pos + 1
    dec.close()


def test_long_prefill_matches_oracle(orc):
    """A 1000-row prompt in one prefill: every projection (split q|k|v,
    o-proj + residual, gate/up + SwiGLU, down + residual) runs with 64-token
    blocks; K/V rows and the residual stream against the oracle's prefill."""
    orc.set_threads(16)
    P = 1000
    w, od, dec = build_pair(orc, SMALL, seed=77, max_seq=1024, max_batch=1)
    rng = np.random.default_rng(77)
    emb = w["embed"][rng.integers(0, SMALL["vocab"], P)]
    kh, vh = od.new_kv(1024)
    ref_x = od.prefill(kh, vh, 0, emb)
    dec.prefill(0, emb, 0)
    kg, vg = dec.kv(0)
    assert rel_err(kg[:, :P].cpu().numpy(), kh[:, :P]) < 2e-3
    assert rel_err(vg[:, :P].cpu().numpy(), vh[:, :P]) < 2e-3
    assert rel_err(dec.prefill_hidden(P).cpu().numpy(), ref_x) < 2e-3
    dec.close()


def test_prefill_batch_equals_single(orc):
    """qasr_decoder_prefill_batch: ragged prompts (one of a single row, one
    after 10 history rows) prefilled together leave each slot's K/V exactly as
    one prefill per slot does, and the next greedy step agrees with the oracle."""
    orc.set_threads(8)
    w, od, a = build_pair(orc, SMALL, seed=33, max_seq=256, max_batch=4)
    b = Decoder(SMALL, device=0, max_batch=4, max_seq=256)
    for i, lw in enumerate(w["layers"]):
        b.set_layer(i, lw)
    b.set_globals(w["embed"], w["norm"], w["lm_head"], w["lm_head_s"])
    rng = np.random.default_rng(33)
    lens, starts, slots = [37, 1, 120, 12], [0, 0, 10, 0], [2, 0, 3, 1]
    rows = [w["embed"][rng.integers(0, SMALL["vocab"], n)] for n in lens]
    hist = w["embed"][rng.integers(0, SMALL["vocab"], 10)]
    for dec in (a, b):
        dec.prefill(3, hist, 0)  # slot 3's first 10 rows
    a.prefill_batch(slots, rows, starts)
    for s, r, p0 in zip(slots, rows, starts):
        b.prefill(s, r, p0)
    for s in slots:
        ka, va = a.kv(s)
        kb, vb = b.kv(s)
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    toks = rng.integers(0, SMALL["vocab"], 4).astype(np.int32)
    pos = np.array([lens[slots.index(s)] + starts[slots.index(s)] for s in range(4)], np.int32)
    assert np.array_equal(a.step(toks, pos), b.step(toks, pos))
    # slot 3 (10 history rows + 120) against the oracle: row 3 of a fresh 4-row step
    kh, vh = od.new_kv(256)
    od.prefill(kh, vh, 0, np.concatenate([hist, rows[2]]))
    tok, _, _ = od.forward(kh, vh, 130, w["embed"][toks[3]])
    c = Decoder(SMALL, device=0, max_batch=4, max_seq=256)
    for i, lw in enumerate(w["layers"]):
        c.set_layer(i, lw)
    c.set_globals(w["embed"], w["norm"], w["lm_head"], w["lm_head_s"])
    c.prefill(3, hist, 0)
    c.prefill_batch(slots, rows, starts)
    assert int(c.step(toks, pos)[3]) == tok
    c.close()
    a.close()
    b.close()
