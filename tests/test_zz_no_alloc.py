"""The allocation-free split-KV attention entry point (b2_decode_gqa_split_noalloc).

It serves callers that may not allocate device memory (allocator callbacks,
plugin hosts that own all device memory, allocator-free hot paths).  Shapes
the cluster-merged kernels take need no scratch; the others take their split
partials from a fixed 4 MiB array in the library, with the split count
lowered until the partials fit.  Each case runs two calls in a row (the
second call reuses the array the first one left behind) and checks the
output against the scratch-buffer entry point b2_decode_gqa_split and against
a float64 evaluation on sampled (sequence, head) pairs, within the attention
tolerance of the reference's tests (3.5e-3).  This file is collected last so
that a stop-at-first-failure run has run every other test before it.
"""
import numpy as np
import pytest

import b2engine as b2

pytestmark = pytest.mark.gpu

TOL = 3.5e-3
ARRAY_FLOATS = (4 << 20) // 4  # the library's fixed array


def _case(B, ctx, nq, nkv, D, seed, ragged):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, nq, D, generator=g, device="cuda").half()
    k = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
    v = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
    lens = [max(1, ctx - 131 * b) if ragged else ctx for b in range(B)]
    L = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, k, v, L


def _f64_attention(q, k, v, L, scale):
    """float64 single-query attention; q [D], k/v [L, D]."""
    s = (k[:L].astype(np.float64) @ q.astype(np.float64)) * scale
    p = np.exp(s - s.max())
    return (p / p.sum()) @ v[:L].astype(np.float64)


def _run_both(B, ctx, nq, nkv, D, seed, ragged):
    import torch
    q, k, v, L = _case(B, ctx, nq, nkv, D, seed, ragged)
    sb, sh, ss = ctx * nkv * D, D, nkv * D
    kv = b2.KVView(k.data_ptr(), sb, sh, ss, 1)
    vv = b2.KVView(v.data_ptr(), sb, sh, ss, 1)
    stream = b2.stream_ptr()
    out_na = torch.empty(B, nq, D, dtype=torch.float16, device="cuda")
    b2.call("b2_decode_gqa_split_noalloc", q.data_ptr(), kv, vv, L.data_ptr(), out_na.data_ptr(), B, nq, nkv, D,
            ctx, stream)
    split = torch.empty(B * nq * 16 * (D + 2) + 4096, dtype=torch.float32, device="cuda")
    out_sc = torch.empty_like(out_na)
    b2.call("b2_decode_gqa_split", q.data_ptr(), kv, vv, L.data_ptr(), out_sc.data_ptr(), B, nq, nkv, D, ctx,
            split.data_ptr(), split.numel(), stream)
    torch.cuda.synchronize()
    got = out_na.float().cpu().numpy()
    rs = np.random.default_rng(seed)
    Ls = L.cpu().numpy()
    for b in sorted({0, B - 1, int(rs.integers(0, B))}):
        kb, vb, qb = k[b].float().cpu().numpy(), v[b].float().cpu().numpy(), q[b].float().cpu().numpy()
        for h in sorted({0, nq - 1, int(rs.integers(0, nq))}):
            g = h // (nq // nkv)
            ref = _f64_attention(qb[h], kb[:, g, :], vb[:, g, :], int(Ls[b]), 1.0 / np.sqrt(D))
            assert float(np.max(np.abs(got[b, h] - ref))) <= TOL, ("float64", b, h)
    return got, out_sc.float().cpu().numpy()


@pytest.mark.parametrize("B,ctx,nq,nkv,D", [
    (1, 4096, 32, 8, 128),   # BASELINE microbench width, tensor-core kernel
    (3, 700, 14, 2, 64),     # Qwen2-0.5B heads, cluster kernel
    (8, 2048, 32, 8, 128),
    (64, 1024, 64, 8, 128),  # Llama-3-70B heads at batch 64
    (3, 700, 12, 2, 96),     # head_dim 96: global-merge kernel, several splits in the array
    (64, 256, 64, 8, 256),   # global merge whose preferred split partials exceed the array
])
def test_noalloc_matches_scratch_entry_point_twice(cuda, B, ctx, nq, nkv, D):
    for call, (seed, ragged) in enumerate([(11, False), (12, True)]):
        got, want = _run_both(B, ctx, nq, nkv, D, seed + B, ragged)
        assert np.isfinite(got).all()
        assert float(np.max(np.abs(got - want))) <= TOL, (call, B, ctx)


def test_noalloc_large_problem_runs_within_its_array(cuda):
    """A global-merge shape whose preferred two splits need more than the
    array (64 x 64 heads x 2 splits x (256 + 2) floats = 2.1 M) runs with the
    split count lowered to fit and returns B2_OK."""
    B, nq, nkv, D = 64, 64, 8, 256
    assert B * nq * 2 * (D + 2) > ARRAY_FLOATS
    got, want = _run_both(B, 256, nq, nkv, D, 5, False)
    assert float(np.max(np.abs(got - want))) <= TOL
