"""The oracle's 4-bit weight restatement on its own (CPU): the packed layout
holds every code where b2_quantize_int4_rows puts it, codes stay in [-7, 7],
each group's largest magnitude maps to +-7, and the round trip is within
half a scale step of the weight."""
import numpy as np

import oracle as O


def test_packed_layout():
    # one row of two groups, codes chosen per position: weight j of each
    # 8-weight word must sit at bit 16*(j & 1) + 4*(j >> 1)
    w = np.zeros((1, 256), np.float32)
    pattern = np.array([7, -7, 1, -1, 3, -3, 0, 5], np.float32)
    w[0, :8] = pattern
    w[0, 128:136] = pattern * 2.0
    packed, scale = O.quantize_int4_rows(w)
    assert packed.shape == (1, 128) and scale.shape == (1, 2)
    assert np.array_equal(scale[0], np.array([1.0, 2.0], np.float32))
    word = int(packed[0, :4].view("<u4")[0])
    for j, q in enumerate(pattern.astype(int)):
        assert (word >> (16 * (j & 1) + 4 * (j >> 1))) & 0xF == q + 8
    assert np.array_equal(O.int4_codes(packed)[0, :8], pattern.astype(np.int32))


def test_round_trip_bounds():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((33, 512)) * 0.02).astype(np.float32)
    w[0] = 0.0                          # all-zero row: scale 0, codes 0
    w[1, 3] = 5.0                       # one dominant weight
    packed, scale = O.quantize_int4_rows(w)
    q = O.int4_codes(packed)
    assert q.min() >= -7 and q.max() <= 7
    assert np.all(scale[0] == 0) and np.all(q[0] == 0)
    g = w.reshape(33, 4, 128)
    qm = q.reshape(33, 4, 128)
    live = scale > 0
    assert np.all(np.max(np.abs(qm), axis=2)[live] == 7)
    back = O.dequantize_int4_rows(packed, scale).reshape(33, 4, 128)
    assert np.all(np.abs(back - g) <= scale[..., None] * 0.5 * (1 + 1e-6) + 1e-12)
