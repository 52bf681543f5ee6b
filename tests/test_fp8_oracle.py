"""The oracle's E4M3 restatement on its own (CPU): every finite code decodes
and re-encodes to itself, midpoints round to the even code, magnitudes
beyond 448 saturate, and the per-row scales follow max|w| / 448."""
import numpy as np

import oracle as O


def test_every_code_round_trips():
    codes = np.array([c for c in range(256) if (c & 0x7F) != 0x7F], np.uint8)  # 0x7f / 0xff are NaN
    vals = O.e4m3_decode(codes)
    back = O.e4m3_encode(vals)
    assert np.array_equal(back, codes)


def test_ties_to_even_and_saturation():
    v = O.e4m3_decode(np.arange(0, 126, dtype=np.uint8)).astype(np.float64)
    mids = ((v[:-1] + v[1:]) / 2).astype(np.float32)  # exact in float32
    got = O.e4m3_encode(mids)
    lower = np.arange(0, 125)
    want = np.where(lower % 2 == 0, lower, lower + 1)
    assert np.array_equal(got, want.astype(np.uint8))
    assert O.e4m3_encode(np.float32([449.0, 1e6, -1e30])).tolist() == [0x7E, 0x7E, 0xFE]
    assert O.e4m3_decode(np.uint8([0x7E, 0x08, 0x01])).tolist() == [448.0, 2.0 ** -6, 2.0 ** -9]


def test_row_scales():
    w = np.float32([[0, 0, 0, 0], [1, -2, 0.5, 0], [448, 1, 2, 3]])
    q, sc = O.quantize_e4m3_rows(w)
    assert sc.tolist() == [1.0, np.float32(2.0) / np.float32(448.0), 1.0]
    assert q[0].tolist() == [0, 0, 0, 0]
    assert q[2, 0] == 0x7E and O.e4m3_decode(q[1])[1] == -448.0
