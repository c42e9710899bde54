"""qwenasr_b200 -- B200 (sm_100a) kernels for the QwenASR per-layer hot path.

    from qwenasr_b200 import kernels      # mirror of crates/qwen-asr/src/kernels
    from qwenasr_b200.decoder import Decoder   # INT8 decoder engine (decode step)

The compute lives in libqwenasr_b200.so (C ABI: include/qwenasr_cuda.h),
built in-tree by `python -m qwenasr_b200.build`.
"""
from ._lib import QasrError, load  # noqa: F401

__version__ = "0.1.0"
