"""Replay of the reference tests' random streams: std::mt19937 seeded with an
integer plus libstdc++'s uniform_real_distribution<float> (one 32-bit draw per
float: r = float(x) / 2^32, value = (b - a) * r + a in float).  numpy's legacy
RandomState(seed) seeds MT19937 exactly like std::mt19937(seed), so the cases
drawn here are the reference's own (tests/test_cuda_ops.cpp, test_attention.cpp,
test_kv_cache.cpp)."""
import numpy as np


class MT19937:
    def __init__(self, seed: int):
        self._rs = np.random.RandomState(seed)

    def __call__(self) -> int:
        return int(self._rs.randint(0, 2**32, dtype=np.uint64))

    def raw(self, n: int) -> np.ndarray:
        return self._rs.randint(0, 2**32, size=n, dtype=np.uint64)

    def uniform(self, a: float, b: float, n: int) -> np.ndarray:
        x = self.raw(n).astype(np.float32)
        r = (x / np.float32(4294967296.0)).astype(np.float32)
        r = np.where(r >= np.float32(1.0), np.nextafter(np.float32(1), np.float32(0)), r).astype(np.float32)
        return (np.float32(np.float32(b) - np.float32(a)) * r + np.float32(a)).astype(np.float32)
