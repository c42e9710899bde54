"""The numpy generator of synthetic weights quantises exactly like the
reference rule (as restated by the oracle), so parity tests and the CPU
baseline consume genuine .qint8-style weights."""
import numpy as np

from qwenasr_b200 import synthetic


def test_quantize_np_matches_oracle_bitwise(orc):
    rng = np.random.default_rng(11)
    w = rng.standard_normal((257, 1024)).astype(np.float32) * np.float32(0.02)
    # rows with exact .5 products and a zero row
    w[3, :4] = [127.0, 63.5, -0.5, 1.5]
    w[3, 4:] = 0
    w[7] = 0
    q1, s1 = synthetic.quantize_np(w)
    q2, s2 = orc.quantize_f32_to_int8(w)
    assert np.array_equal(q1, q2) and np.array_equal(s1, s2)


def test_layer_shapes_and_interleave():
    cfg = dict(synthetic.DEC_0_6B, n_layers=1)
    lw = synthetic.layer_weights_np(cfg, np.random.default_rng(0))
    assert lw["wq"].shape == (2048, 1024) and lw["wk"].shape == (1024, 1024)
    assert lw["wo"].shape == (1024, 2048) and lw["down"].shape == (1024, 3072)
    assert lw["gate_up"].shape == (6144, 1024) and lw["gate_up_s"].shape == (6144,)
    assert lw["wq"].dtype == np.int8 and lw["wq_s"].dtype == np.float32
    assert abs(float(lw["input_norm"].mean()) - 1.0) < 0.01
