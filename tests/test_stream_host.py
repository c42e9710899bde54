"""Host-side pieces of the transcription drivers, no GPU: the tail-repeat
detector of the streaming degeneracy check (transcribe.rs:42-59) and the
low-energy split-point search of the segmented mode (transcribe.rs:250-275),
library against the test restatement."""
import numpy as np
import pytest

from qwenasr_b200 import stream as S
from stream_oracle import find_split_point, tail_repeat_blocks


@pytest.mark.parametrize("tokens,max_period", [
    ([], 6), ([5], 6), ([1, 1], 6), ([1, 2, 1, 2, 1, 2, 1, 2], 6), ([9, 1, 2, 3, 1, 2, 3, 1, 2, 3], 6),
    ([7] * 10, 6), ([1, 2, 3, 4, 5, 6, 7] * 3, 6), ([1, 2, 3, 4, 5, 6, 7] * 3, 0), ([4, 4, 5, 4, 4, 5], 2)])
def test_tail_repeat_blocks(tokens, max_period):
    assert S.tail_repeat_blocks(tokens, max_period) == tail_repeat_blocks(tokens, max_period)


def test_tail_repeat_random():
    rng = np.random.default_rng(0)
    for _ in range(200):
        n = int(rng.integers(0, 40))
        t = rng.integers(0, 3, n).tolist()
        for mp in (0, 1, 6):
            assert S.tail_repeat_blocks(t, mp) == tail_repeat_blocks(t, mp)


@pytest.mark.parametrize("target,search", [(16000, 0.5), (800, 0.5), (31000, 0.3), (20000, 0.0)])
def test_find_split_point(target, search):
    rng = np.random.default_rng(target)
    x = (rng.standard_normal(32000) * 0.1).astype(np.float32)
    x[14000:15600] *= np.float32(0.01)  # a quiet 100 ms span
    assert S.find_split_point(x, target, search) == find_split_point(x, target, search)


def _plan_ref(x, segment_sec, search_sec):
    """transcribe.rs:317-345 restated over the test's find_split_point."""
    target = int(np.float32(segment_sec) * np.float32(16000.0))
    search = min(np.float32(search_sec), np.float32(segment_sec) / np.float32(2.0))
    margin = int(np.float32(search) * np.float32(16000.0))
    if segment_sec <= 0 or len(x) <= target + margin:
        return [(0, len(x))]
    splits, pos = [0], 0
    while pos + target + margin < len(x):
        sp = find_split_point(x, pos + target, float(search))
        splits.append(sp)
        pos = sp
        if len(splits) >= 127:
            break
    return list(zip(splits, splits[1:] + [len(x)]))


@pytest.mark.parametrize("seconds,segment_sec,search_sec", [(9.0, 2.0, 0.5), (3.0, 5.0, 1.0), (6.0, 0.0, 3.0),
                                                            (7.3, 1.5, 3.0)])
def test_plan_segments(seconds, segment_sec, search_sec):
    from qwenasr_b200.synthetic import synthetic_audio
    from qwenasr_b200.transcribe import plan_segments
    x = synthetic_audio(seconds, seed=int(seconds * 10))
    got = plan_segments(x, segment_sec, search_sec)
    assert got == _plan_ref(x, segment_sec, search_sec)
    assert got[0][0] == 0 and got[-1][1] == len(x) and all(a < b for a, b in got)
