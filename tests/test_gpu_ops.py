"""CUDA operators vs the CPU oracle on the reference's own seeded cases.

Each test replays the random stream of the matching TEST_CASE in the
reference's tests/test_cuda_ops.cpp (same seed, same draw order, same
tolerance) and calls the operator through the C-ABI (b2engine -> libb2engine.so).
"""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
from refrng import MT19937

pytestmark = pytest.mark.gpu


def dev(a, dtype=None):
    import torch
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a)
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


_KEEP = []


def keep(a, dtype=None):
    """Device copy of `a` that stays alive until the next test starts (a
    temporary whose data_ptr() is passed inline would be freed at once and its
    block handed to the next allocation)."""
    t = dev(a, dtype)
    _KEEP.append(t)
    return t


@pytest.fixture(autouse=True)
def _release_kept():
    yield
    _KEEP.clear()


def h16(a):
    return np.asarray(a, np.float32).astype(np.float16)


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.float().cpu().numpy()


def empty16(*shape):
    import torch
    return torch.empty(*shape, dtype=torch.float16, device="cuda")


def maxdiff(a, b):
    a = np.asarray(a, np.float32).reshape(-1)
    b = np.asarray(b, np.float32).reshape(-1)
    return float(np.max(np.abs(a - b))) if a.size else 0.0


def test_embedding_lookup(cuda):  # test_cuda_ops.cpp:41-85, tolerance 0
    import torch
    rng = MT19937(42)
    for t in range(25):
        S = 1 if t == 0 else 1 + rng() % 73
        V = 50 + rng() % 200
        H = 7 + rng() % 129
        ids = np.array([rng() % V for _ in range(S)], np.int64)
        table = h16(rng.uniform(-1, 1, V * H)).reshape(V, H)
        ref = O.embedding_lookup(ids, table.astype(np.float32))
        out = empty16(S, H)
        b2.call("b2_embedding_lookup", keep(ids).data_ptr(), keep(table).data_ptr(), out.data_ptr(), S, H,
                b2.stream_ptr())
        assert maxdiff(host(out), ref) == 0.0


def test_rmsnorm(cuda):  # test_cuda_ops.cpp:87-130, tolerance 2e-3
    rng = MT19937(43)
    for t in range(25):
        rows = 1 if t == 0 else 1 + rng() % 50
        dim = 17 + rng() % 300
        x = h16(rng.uniform(-1, 1, rows * dim)).reshape(rows, dim)
        w = h16(rng.uniform(-1, 1, dim))
        ref = O.rmsnorm(x.astype(np.float32), w.astype(np.float32), 1e-6)
        out = empty16(rows, dim)
        b2.call("b2_rmsnorm", keep(x).data_ptr(), keep(w).data_ptr(), out.data_ptr(), rows, dim, 1e-6, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 2e-3, (rows, dim)


def test_rope(cuda):  # test_cuda_ops.cpp:132-181, theta 1e6, tolerance 2e-3
    rng = MT19937(44)
    for t in range(25):
        S = 1 if t == 0 else 1 + rng() % 35
        nq = 1 + rng() % 16
        nkv = 1 + rng() % 4
        D = (1 + rng() % 32) * 2
        p0 = rng() % 100
        q = h16(rng.uniform(-1, 1, S * nq * D))
        k = h16(rng.uniform(-1, 1, S * nkv * D))
        rq, rk = O.apply_rope(q.astype(np.float32), k.astype(np.float32), S, nq, nkv, D, p0, 1e6)
        dq, dk = keep(q), keep(k)
        b2.call("b2_apply_rope", dq.data_ptr(), dk.data_ptr(), S, nq, nkv, D, p0, 1e6, b2.stream_ptr())
        assert maxdiff(host(dq), rq) <= 2e-3, (S, nq, nkv, D, p0)
        assert maxdiff(host(dk), rk) <= 2e-3


def test_causal_gqa(cuda):  # test_cuda_ops.cpp:183-235, tolerance 3e-3
    rng = MT19937(45)
    for t in range(25):
        S = 1 if t == 0 else 1 + rng() % 25
        nkv = 1 + rng() % 3
        g = 1 + rng() % 5
        nq = nkv * g
        D = 16 * (1 + rng() % 4)
        q = h16(rng.uniform(-1, 1, S * nq * D))
        k = h16(rng.uniform(-1, 1, S * nkv * D))
        v = h16(rng.uniform(-1, 1, S * nkv * D))
        ref = O.causal_gqa(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), S, nq, nkv, D)
        out = empty16(S * nq * D)
        b2.call("b2_causal_gqa", keep(q).data_ptr(), keep(k).data_ptr(), keep(v).data_ptr(), out.data_ptr(), S, nq, nkv,
                D, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 3e-3, (S, nq, nkv, D)


def test_softmax(cuda):  # test_cuda_ops.cpp:237-285, tolerance 2e-3
    rng = MT19937(46)
    for t in range(25):
        rows = 1 if t == 0 else 1 + rng() % 30
        cols = 1 + rng() % 500
        x = h16(rng.uniform(-3, 3, rows * cols)).reshape(rows, cols)
        ref = O.softmax(x.astype(np.float32))
        out = empty16(rows, cols)
        b2.call("b2_softmax", keep(x).data_ptr(), out.data_ptr(), rows, cols, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 2e-3


def test_swiglu(cuda):  # test_cuda_ops.cpp:287-329, tolerance 2e-3
    rng = MT19937(47)
    for t in range(25):
        n = 1 if t == 0 else 1 + rng() % 10000
        g = h16(rng.uniform(-2, 2, n))
        u = h16(rng.uniform(-2, 2, n))
        ref = O.swiglu(g.astype(np.float32), u.astype(np.float32))
        out = empty16(n)
        b2.call("b2_swiglu", keep(g).data_ptr(), keep(u).data_ptr(), out.data_ptr(), n, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 2e-3


def test_residual_add(cuda):  # test_cuda_ops.cpp:331-376, exact
    rng = MT19937(48)
    for t in range(25):
        n = 1 if t == 0 else 1 + rng() % 10000
        a = h16(rng.uniform(-5, 5, n))
        bb = h16(rng.uniform(-5, 5, n))
        ref = (a.astype(np.float32) + bb.astype(np.float32)).astype(np.float16)
        out = empty16(n)
        b2.call("b2_residual_add", keep(a).data_ptr(), keep(bb).data_ptr(), out.data_ptr(), n, b2.stream_ptr())
        assert maxdiff(host(out), ref) == 0.0


def test_bias_add(cuda):  # test_cuda_ops.cpp:378-426, exact
    rng = MT19937(49)
    for t in range(25):
        M = 1 if t == 0 else 1 + rng() % 50
        N = 1 if t == 0 else 1 + rng() % 200
        x = h16(rng.uniform(-5, 5, M * N)).reshape(M, N)
        bias = h16(rng.uniform(-5, 5, N))
        ref = (x.astype(np.float32) + bias.astype(np.float32)[None, :]).astype(np.float16)
        out = empty16(M, N)
        b2.call("b2_bias_add", keep(x).data_ptr(), keep(bias).data_ptr(), out.data_ptr(), M, N, b2.stream_ptr())
        assert maxdiff(host(out), ref) == 0.0


def test_matmul_transB(cuda):  # test_cuda_ops.cpp:428-478, fp16 out, tolerance 2e-3
    rng = MT19937(50)
    for t in range(25):
        M = 1 if t == 0 else 1 + rng() % 33
        K = 1 + rng() % 65
        N = 1 + rng() % 49
        A = h16(rng.uniform(-1, 1, M * K)).reshape(M, K)
        Bm = h16(rng.uniform(-1, 1, N * K)).reshape(N, K)
        ref = O.matmul_transB(A.astype(np.float32), Bm.astype(np.float32), naive=True).astype(np.float16)
        out = empty16(M, N)
        b2.call("b2_matmul_transB", keep(A).data_ptr(), keep(Bm).data_ptr(), out.data_ptr(), M, K, N, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 2e-3, (M, K, N)


def test_matmul_transB_f32(cuda):  # test_cuda_ops.cpp:675-722, fp32 out, tolerance 2e-4
    import torch
    rng = MT19937(51)
    for t in range(25):
        M = 1 if t == 0 else 1 + rng() % 33
        K = 1 + rng() % 65
        N = 1 + rng() % 49
        A = h16(rng.uniform(-1, 1, M * K)).reshape(M, K)
        Bm = h16(rng.uniform(-1, 1, N * K)).reshape(N, K)
        ref = O.matmul_transB(A.astype(np.float32), Bm.astype(np.float32), naive=True)
        out = torch.empty(M, N, dtype=torch.float32, device="cuda")
        b2.call("b2_matmul_transB_f32", keep(A).data_ptr(), keep(Bm).data_ptr(), out.data_ptr(), M, K, N,
                b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 2e-4, (M, K, N)


GEMV_SHAPES = [(1, 1), (7, 13), (33, 37), (64, 128), (128, 64), (896, 896), (128, 896), (4864, 896), (896, 4864),
               (1, 896), (896, 1), (3, 5), (17, 31), (63, 65), (129, 127), (256, 256), (512, 512), (4864, 32),
               (32, 4864), (896, 7), (7, 896), (128, 128), (64, 64), (31, 31), (13, 17)]

# Llama-3-8B / TinyLlama decode GEMV shapes (N, K) on top of the reference list
LLAMA_SHAPES = [(6144, 4096), (4096, 14336), (2560, 2048), (2048, 5632)]


@pytest.mark.parametrize("epi,seed", [(None, 1001), ("bias", 2002), ("residual", 3003)])
def test_gemv(cuda, epi, seed):  # test_cuda_ops.cpp:491-671, tol max(1e-2*max|ref|, 1e-3)
    rng = MT19937(seed)
    for N, K in GEMV_SHAPES + LLAMA_SHAPES:
        W = h16(rng.uniform(-1, 1, N * K)).reshape(N, K)
        x = h16(rng.uniform(-1, 1, K))
        extra = h16(rng.uniform(-1, 1, N)) if epi else None
        ref = W.astype(np.float64) @ x.astype(np.float64)
        if epi:
            ref = ref + extra.astype(np.float64)
        y = empty16(N)
        b2.gemv(keep(W), keep(x), y, epi=epi, extra=keep(extra) if epi else None)
        tol = max(1e-2 * max(float(np.max(np.abs(ref))), 1e-6), 1e-3)
        assert maxdiff(host(y), ref) <= tol, (N, K)


@pytest.mark.parametrize("B", [1, 2, 3, 4, 5, 8, 13])
def test_gemv_batched(cuda, B):
    import torch
    rng = np.random.default_rng(B)
    for N, K in [(33, 40), (512, 4096), (1000, 14336), (4096, 512)]:
        W = h16(rng.uniform(-1, 1, (N, K)))
        x = h16(rng.uniform(-1, 1, (B, K)))
        r = h16(rng.uniform(-1, 1, (B, N)))
        ref = x.astype(np.float64) @ W.astype(np.float64).T
        y = torch.empty(B, N, dtype=torch.float32, device="cuda")
        b2.gemv_batched(keep(W), keep(x), y, out_f32=True)
        tol = 1e-4 * max(float(np.max(np.abs(ref))), 1.0) + 1e-3
        assert maxdiff(host(y), ref) <= tol, (B, N, K)
        y16 = empty16(B, N)
        b2.gemv_batched(keep(W), keep(x), y16, epilogue=2, extra=keep(r))
        ref2 = ref + r.astype(np.float64)
        assert maxdiff(host(y16), ref2) <= max(1e-2 * float(np.max(np.abs(ref2))), 1e-3)


def test_gemv_rejects_bad_args(cuda):
    with pytest.raises(b2.B2Error) as e:
        b2.call("b2_gemv", None, None, None, 4, 4, None)
    assert e.value.status == -1
