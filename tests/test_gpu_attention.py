"""Decode / prefill attention and KV append vs the CPU oracle.

The first four tests replay the reference's seeded cases
(tests/test_attention.cpp:34-291, tests/test_kv_cache.cpp:43-196) with their
tolerances; the last ones cover BASELINE's split-KV microbench shapes
(Hq=32, Hkv=8, D=128, token-major [B, ctx, 8, 128] cache) at full size,
checked against a float64 numpy evaluation on sampled (sequence, head) pairs.
"""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
from refrng import MT19937
from test_gpu_ops import _release_kept, dev, empty16, h16, host, keep, maxdiff  # noqa: F401

pytestmark = pytest.mark.gpu


def kvview(t, sb, sh, ss):
    return b2.KVView(t.data_ptr(), sb, sh, ss, 1)


def test_decode_gqa_split_reference_cases(cuda):  # test_attention.cpp:34-175, tol 3.5e-3
    import torch
    rng = MT19937(701)
    for t in range(25):
        B = 1 if t % 4 == 0 else 1 + rng() % 3
        nkv = 2
        g = 7 if t % 3 == 0 else 1 + rng() % 7
        nq = nkv * g
        D = 64
        lens = []
        for b in range(B):
            lens.append(1 if t == 0 else 17 if t == 1 else 513 if t == 2 else 1 + rng() % 600)
        S = max(lens)
        q = h16(rng.uniform(-1, 1, B * nq * D))
        k = h16(rng.uniform(-1, 1, B * nkv * S * D))
        v = h16(rng.uniform(-1, 1, B * nkv * S * D))
        strides = (nkv * S * D, S * D, D)
        ref = O.decode_attention(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), strides,
                                 np.array(lens, np.int32), B, nq, nkv, D)
        dq, dk, dv = keep(q), keep(k), keep(v)
        dl = keep(np.array(lens, np.int32))
        split = torch.empty(8 * B * nq * (D + 2), dtype=torch.float32, device="cuda")
        out = empty16(B * nq * D)
        b2.decode_gqa_split(dq, kvview(dk, *strides), kvview(dv, *strides), dl, out, B, nq, nkv, D, S, split)
        assert maxdiff(host(out), ref) < 3.5e-3, (t, B, nq, lens)
        # no scratch: one split per (sequence, kv head) gives the same answer
        out1 = empty16(B * nq * D)
        b2.decode_gqa_split(dq, kvview(dk, *strides), kvview(dv, *strides), dl, out1, B, nq, nkv, D, S, None)
        assert maxdiff(host(out1), ref) < 3.5e-3


def test_flash_prefill_reference_cases(cuda):  # test_attention.cpp:180-291, tol 3.5e-3
    rng = MT19937(702)
    for t in range(25):
        nkv = 2
        g = 7 if t % 3 == 0 else 1 + rng() % 7
        nq = nkv * g
        D = 64
        S = [1, 15, 17, 65][t] if t < 4 else 1 + rng() % 120
        q = h16(rng.uniform(-1, 1, S * nq * D))
        k = h16(rng.uniform(-1, 1, S * nkv * D))
        v = h16(rng.uniform(-1, 1, S * nkv * D))
        ref = O.causal_gqa(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), S, nq, nkv, D)
        out = empty16(S * nq * D)
        b2.call("b2_flash_prefill_gqa", keep(q).data_ptr(), keep(k).data_ptr(), keep(v).data_ptr(), out.data_ptr(), S,
                nq, nkv, D, 1, b2.stream_ptr())
        assert maxdiff(host(out), ref) < 3.5e-3, (t, S, nq)


def test_append_kv_cache_reference_cases(cuda):  # test_kv_cache.cpp:43-96, exact
    import torch
    rng = MT19937(101)
    for t in range(25):
        T = 1 if t == 0 else 1 + rng() % 37
        p0 = 0 if t == 0 else rng() % 50
        nkv = 1 + rng() % 4
        max_seq = p0 + T + (rng() % 30)
        D = 16 * (1 + rng() % 4)
        ks = h16(rng.uniform(-2, 2, T * nkv * D))
        vs = h16(rng.uniform(-2, 2, T * nkv * D))
        dk = torch.zeros(nkv * max_seq * D, dtype=torch.float16, device="cuda")
        dv = torch.zeros_like(dk)
        b2.call("b2_append_kv_cache", keep(ks).data_ptr(), keep(vs).data_ptr(), dk.data_ptr(), dv.data_ptr(), T, p0,
                nkv, max_seq, D, b2.stream_ptr())
        exp_k = np.zeros((nkv, max_seq, D), np.float16)
        exp_v = np.zeros((nkv, max_seq, D), np.float16)
        exp_k[:, p0:p0 + T, :] = ks.reshape(T, nkv, D).transpose(1, 0, 2)
        exp_v[:, p0:p0 + T, :] = vs.reshape(T, nkv, D).transpose(1, 0, 2)
        torch.cuda.synchronize()
        assert np.array_equal(dk.cpu().numpy().view(np.uint16), exp_k.reshape(-1).view(np.uint16))
        assert np.array_equal(dv.cpu().numpy().view(np.uint16), exp_v.reshape(-1).view(np.uint16))


def test_decode_gqa_reference_cases(cuda):  # test_kv_cache.cpp:98-196, tol 3e-3
    rng = MT19937(102)
    for t in range(25):
        L = 1 if t == 0 else 1 + rng() % 64
        max_seq = L + rng() % 32
        nkv = 1 + rng() % 3
        g = 1 + rng() % 5
        nq = nkv * g
        D = 16 * (1 + rng() % 4)
        q = h16(rng.uniform(-1, 1, nq * D))
        kc = h16(rng.uniform(-1, 1, nkv * max_seq * D))
        vc = h16(rng.uniform(-1, 1, nkv * max_seq * D))
        ref = O.decode_attention(q.astype(np.float32), kc.astype(np.float32), vc.astype(np.float32),
                                 (0, max_seq * D, D), np.array([L], np.int32), 1, nq, nkv, D)
        out = empty16(nq * D)
        b2.call("b2_decode_gqa", keep(q).data_ptr(), keep(kc).data_ptr(), keep(vc).data_ptr(), out.data_ptr(), L, nq,
                nkv, max_seq, D, b2.stream_ptr())
        assert maxdiff(host(out), ref) <= 3e-3, (t, L, nq, nkv, D)


def _np_attention(q, k, v, L, scale):
    """float64 single-query attention; q [D], k/v [L, D]."""
    s = (k[:L].astype(np.float64) @ q.astype(np.float64)) * scale
    p = np.exp(s - s.max())
    return (p / p.sum()) @ v[:L].astype(np.float64)


@pytest.mark.parametrize("B,ctx", [(1, 512), (1, 4096), (1, 32768), (8, 512), (8, 4096), (8, 32768), (32, 512),
                                   (32, 4096), (32, 32768)])
def test_split_kv_baseline_shapes(cuda, B, ctx):
    """BASELINE split-KV microbench: q [B,32,128], cache [B,ctx,8,128] ~N(0,1)."""
    import torch
    nq, nkv, D = 32, 8, 128
    gen = torch.Generator(device="cuda").manual_seed(1000 + B * 7 + ctx)
    q = torch.randn(B, nq, D, generator=gen, device="cuda").half()
    k = torch.randn(B, ctx, nkv, D, generator=gen, device="cuda").half()
    v = torch.randn(B, ctx, nkv, D, generator=gen, device="cuda").half()
    lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    # ragged lengths on a second pass: shorter sequences read only their prefix
    ragged = torch.tensor([max(1, ctx - 37 * b) for b in range(B)], dtype=torch.int32, device="cuda")
    split = torch.empty(64 * B * nq * (D + 2), dtype=torch.float32, device="cuda")
    sb, sh, ss = ctx * nkv * D, D, nkv * D
    scale = 1.0 / np.sqrt(D)
    for L_t in (lens, ragged):
        out = torch.empty(B, nq, D, dtype=torch.float16, device="cuda")
        b2.decode_gqa_split(q, kvview(k, sb, sh, ss), kvview(v, sb, sh, ss), L_t, out, B, nq, nkv, D, ctx, split)
        torch.cuda.synchronize()
        Ls = L_t.cpu().numpy()
        outh = out.float().cpu().numpy()
        rs = np.random.default_rng(B + ctx)
        for b in sorted(set([0, B - 1] + list(rs.integers(0, B, 2)))):
            kb = k[b].float().cpu().numpy()
            vb = v[b].float().cpu().numpy()
            qb = q[b].float().cpu().numpy()
            for h in sorted(set([0, nq - 1] + list(rs.integers(0, nq, 3)))):
                ref = _np_attention(qb[h], kb[:, h // 4, :], vb[:, h // 4, :], int(Ls[b]), scale)
                assert maxdiff(outh[b, h], ref) < 3.5e-3, (b, h)
