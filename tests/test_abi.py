"""C-ABI checks that need no GPU: the library loads, exports exactly what
include/qwenasr_cuda.h declares, and rejects bad arguments with a status code
and message before touching the device (the reference returns NULL / -1 from
its C API on bad input, c_api.rs:25-31)."""
import ctypes as C
import os

import pytest

from qwenasr_b200 import _lib


@pytest.fixture(scope="module")
def lib():
    from qwenasr_b200 import build
    build.build()
    return _lib.load()


def test_every_header_function_is_exported(lib):
    names = _lib.header_functions()
    assert len(names) >= 35
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes signature table covers all of them
    assert sorted(_lib._SIGS) == names


def test_version(lib):
    assert b"sm_100a" in lib.qasr_version()


@pytest.mark.parametrize("name,args", [
    ("qasr_rms_norm", (None, None, None, 4, 1024, C.c_float(1e-6), None)),
    ("qasr_rms_norm_per_head", (None, None, 4, 16, 128, C.c_float(1e-6), None)),
    ("qasr_layer_norm", (None, None, None, None, 4, 896, C.c_float(1e-5), None)),
    ("qasr_apply_rope_neox", (None, None, None, 1, 16, 128, None)),
    ("qasr_kv_append", (None, None, None, None, 0, 16, 1024, 0, 1, None)),
    ("qasr_gelu", (None, C.c_int64(8), None)),
    ("qasr_linear_nobias_int8", (None, None, None, None, 1, 1024, 1024, None)),
    ("qasr_causal_attention", (None, None, None, None, 1, 1, 16, 8, 128, C.c_float(0.1), 0, None)),
    ("qasr_quantize_f32_to_int8", (None, C.c_int64(4), C.c_int64(4), None, None, None)),
    ("qasr_pre_attn_block", (None,) * 3 + (1, 1024) + (None,) * 6 + (16, 8, 128, C.c_float(1e-6), None, None, 0,
                                                                      None, None, 0, 16, None)),
    ("qasr_final_norm_lmhead_argmax", (None,) * 6 + (1, 1024, 151936, C.c_float(1e-6), None)),
    ("qasr_transcribe_lanes", (None, None, 1, None, None, 1, None, 0, None, 0, 8, 0, None, 8, None)),
    ("qasr_transcribe_batch", (None, None, None, None, 1, None, 0, None, 0, 8, 0, None, 8, None)),
])
def test_null_pointers_rejected(lib, name, args):
    rc = getattr(lib, name)(*args)
    assert rc == _lib.QASR_ERR_INVALID
    assert name in _lib.last_error()


def test_shape_errors(lib):
    # kv append past the cache capacity (KvCache must grow first, decoder.rs:152)
    p = C.c_void_p(16)  # never dereferenced: validation fails first
    assert lib.qasr_kv_append(p, p, p, p, 0, 16, 1024, 10, 7, None) == _lib.QASR_ERR_INVALID
    assert "max_seq" in _lib.last_error()
    # specialised kernels refuse shapes they do not cover
    assert lib.qasr_pre_attn_block(p, p, p, 1, 1024, p, p, p, None, p, p, 16, 8, 64, C.c_float(1e-6), p, p, 0, p, p,
                                   0, 16, None) == _lib.QASR_ERR_UNSUPPORTED
    assert lib.qasr_linear_nobias_int8(p, p, p, p, 1, 100, 8, None) == _lib.QASR_ERR_UNSUPPORTED
    assert lib.qasr_causal_attention(p, p, p, p, 1, 1, 16, 8, 96, C.c_float(0.1), 0, None) == \
        _lib.QASR_ERR_UNSUPPORTED


def test_transcribe_lanes_validates_lanes(lib):
    """Lane arrays are checked before any engine is touched: no lanes, more
    than 64, or a lane without engines."""
    ids = (C.c_int * 8)()
    n = (C.c_int * 1)()
    nulls = (C.c_void_p * 2)()
    for lanes in (0, 65):
        assert lib.qasr_transcribe_lanes(nulls, nulls, lanes, None, None, 0, None, 0, None, 0, 8, 0, ids, 8,
                                         n) == _lib.QASR_ERR_INVALID
    assert lib.qasr_transcribe_lanes(nulls, nulls, 2, None, None, 0, None, 0, None, 0, 8, 0, ids, 8,
                                     n) == _lib.QASR_ERR_INVALID
    assert "lane 0" in _lib.last_error()


def test_decoder_create_rejects_bad_config(lib):
    bad = _lib.DecoderConfig(1024, 3072, 28, 16, 8, 64, 151936, 1e-6, 1e6, 8, 2048, 0)  # head_dim 64
    assert not lib.qasr_decoder_create(C.byref(bad), 0)
    assert "head_dim" in _lib.last_error()
    bad = _lib.DecoderConfig(1024, 3072, 28, 16, 8, 128, 151936, 1e-6, 1e6, 9, 2048, 0)  # batch > 8
    assert not lib.qasr_decoder_create(C.byref(bad), 0)
    assert lib.qasr_decoder_step(None, None, None, 1, None) == _lib.QASR_ERR_INVALID


def test_missing_library_fails_loudly(tmp_path):
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        saved = _lib._lib
        _lib._lib = None
        try:
            _lib.load(str(tmp_path / "nope.so"))
        finally:
            _lib._lib = saved


def _header_arg_counts():
    import re
    txt = re.sub(r"/\*.*?\*/", "", open(_lib.HEADER).read(), flags=re.S)
    out = {}
    for name, args in re.findall(r"\b(qasr_\w+)\s*\(([^;]*?)\);", txt, flags=re.S):
        a = [x for x in " ".join(args.split()).split(",") if x.strip() and x.strip() != "void"]
        out[name] = len(a)
    return out


def test_rust_binding_matches_header():
    """include/qwenasr_cuda.rs (the untested Rust extern block for the
    reference crate) declares every header function with the same arity."""
    import os
    import re
    rs = open(os.path.join(os.path.dirname(_lib.HEADER), "qwenasr_cuda.rs")).read()
    decl = {n: len([x for x in a.split(",") if x.strip()]) for n, a in re.findall(r"pub fn (qasr_\w+)\((.*?)\)", rs)}
    assert decl == _header_arg_counts()

