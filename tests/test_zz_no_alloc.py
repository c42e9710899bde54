"""qasr_final_norm_lmhead_argmax_noalloc: the allocation-free variant of the
final norm + lm head + argmax entry, for hosts that may not allocate device
memory once serving has started (a runtime handing out device memory from
its own pool, or one under a hard memory budget).  It is called through the C
ABI and checked against the CPU oracle's RMSNorm + INT8 matvec + first-max
argmax, the same bars as the allocating entry's test: logits within 2e-3
relative, ids identical except where the oracle's top two logits are closer
than the kernel's error could separate.

The file is named to be collected last so that the variant is exercised
both in a fresh process (run alone) and after every other GPU test.
"""
import ctypes as C
import math

import numpy as np
import pytest
import torch

from qwenasr_b200 import _lib

pytestmark = pytest.mark.gpu


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _call(ids, logits, x, nw, w, s, M, hidden, vocab, dev):
    lib = _lib.load()
    with torch.cuda.device(dev):
        stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
        rc = lib.qasr_final_norm_lmhead_argmax_noalloc(_p(ids), _p(logits), _p(x), _p(nw), _p(w), _p(s), M, hidden,
                                                       vocab, C.c_float(1e-6), stream)
    assert rc == _lib.QASR_OK, (rc, _lib.last_error())


def _inputs(orc, rng, M, hidden, vocab):
    emb = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float32)
    w, s = orc.quantize_f32_to_int8(emb)
    nw = (1 + 0.02 * rng.standard_normal(hidden)).astype(np.float32)
    return w, s, nw


def _check(orc, x, nw, w, s, ids, logits):
    """Logits within 2e-3 of the oracle's; ids equal to the oracle's first-max
    argmax unless its top-2 margin is below the measured logit error."""
    xn = orc.rms_norm(x, nw, 1e-6)
    ref = orc.linear_nobias_int8(xn, w, s).astype(np.float64)
    got = np.asarray(logits, np.float64)
    scale = np.abs(ref) + math.sqrt(float(np.mean(ref * ref)))
    err = float(np.max(np.abs(got - ref) / scale))
    assert err <= 2e-3, err
    for m in range(x.shape[0]):
        want = orc.argmax_first(ref[m].astype(np.float32))
        if int(ids[m]) != want:
            top2 = np.sort(ref[m])[-2:]
            margin = float(top2[1] - top2[0])
            assert margin <= 2 * err * scale[m].max(), (m, int(ids[m]), want, margin)
            print(f"near-tie: row {m} id {int(ids[m])} vs oracle {want}, top-2 margin {margin:.3e}")
        assert got[m, int(ids[m])] == got[m].max()


@pytest.mark.parametrize("M,hidden,vocab", [(8, 1024, 151936), (3, 2048, 151936), (1, 1024, 4096)])
def test_noalloc_matches_oracle(orc, M, hidden, vocab):
    rng = np.random.default_rng(7 * M + hidden)
    w, s, nw = _inputs(orc, rng, M, hidden, vocab)
    dw, ds, dnw = (torch.from_numpy(a).to("cuda:0") for a in (w, s, nw))
    for call in range(2):  # two calls in a row: the fixed scratch is shared by both
        x = rng.standard_normal((M, hidden)).astype(np.float32)
        ids = torch.full((M,), -2, dtype=torch.int32, device="cuda:0")
        logits = torch.empty(M, vocab, device="cuda:0")
        _call(ids, logits, torch.from_numpy(x).to("cuda:0"), dnw, dw, ds, M, hidden, vocab, 0)
        torch.cuda.synchronize()
        _check(orc, x, nw, w, s, ids.cpu().numpy(), logits.cpu().numpy())


def test_noalloc_without_logits(orc):
    rng = np.random.default_rng(11)
    M, hidden, vocab = 4, 1024, 32768
    w, s, nw = _inputs(orc, rng, M, hidden, vocab)
    x = rng.standard_normal((M, hidden)).astype(np.float32)
    ref = orc.linear_nobias_int8(orc.rms_norm(x, nw, 1e-6), w, s)
    want = [orc.argmax_first(ref[m]) for m in range(M)]
    args = [torch.from_numpy(a).to("cuda:0") for a in (x, nw, w, s)]
    for _ in range(2):
        ids = torch.full((M,), -2, dtype=torch.int32, device="cuda:0")
        _call(ids, None, *args, M, hidden, vocab, 0)
        torch.cuda.synchronize()
        assert ids.tolist() == want


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two visible GPUs")
def test_noalloc_second_device(orc):
    """A call on device 1 after device 0 in the same process: the scratch
    address and the kernel's shared-memory opt-in are per device."""
    rng = np.random.default_rng(13)
    M, hidden, vocab = 8, 1024, 8192
    w, s, nw = _inputs(orc, rng, M, hidden, vocab)
    x = rng.standard_normal((M, hidden)).astype(np.float32)
    for dev in (0, 1, 0, 1):
        d = f"cuda:{dev}"
        ids = torch.full((M,), -2, dtype=torch.int32, device=d)
        logits = torch.empty(M, vocab, device=d)
        args = [torch.from_numpy(a).to(d) for a in (x, nw, w, s)]
        _call(ids, logits, *args, M, hidden, vocab, dev)
        torch.cuda.synchronize(dev)
        _check(orc, x, nw, w, s, ids.cpu().numpy(), logits.cpu().numpy())


def test_noalloc_rejects_sizes_beyond_its_scratch():
    lib = _lib.load()
    p = C.c_void_p(256)  # never dereferenced: validation fails first
    rc = lib.qasr_final_norm_lmhead_argmax_noalloc(p, None, p, p, p, p, 9, 1024, 151936, C.c_float(1e-6), None)
    assert rc == _lib.QASR_ERR_INVALID
    assert "at most 8" in _lib.last_error()
    rc = lib.qasr_final_norm_lmhead_argmax_noalloc(p, None, p, p, p, p, 1, 4096, 151936, C.c_float(1e-6), None)
    assert rc == _lib.QASR_ERR_UNSUPPORTED
    assert "3072" in _lib.last_error()
