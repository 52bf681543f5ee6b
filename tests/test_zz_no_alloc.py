"""The allocation-free split-KV attention entry point (b2_decode_gqa_split_noalloc).

It serves callers that may not allocate device memory (allocator callbacks,
plugin hosts that own all device memory, allocator-free hot paths) by taking
its scratch from a fixed array in the library.  Its results must match the
scratch-buffer entry point b2_decode_gqa_split within the attention tolerance
of the reference's tests (3.5e-3), on two calls in a row (the second call
reuses the array the first one left behind).  This file is collected last so
that a stop-at-first-failure run has run every other test before it.
"""
import numpy as np
import pytest

import b2engine as b2

pytestmark = pytest.mark.gpu

TOL = 3.5e-3


def _case(B, ctx, nq, nkv, D, seed, ragged):
    import torch
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, nq, D, generator=g, device="cuda").half()
    k = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
    v = torch.randn(B, ctx, nkv, D, generator=g, device="cuda").half()
    lens = [max(1, ctx - 131 * b) if ragged else ctx for b in range(B)]
    L = torch.tensor(lens, dtype=torch.int32, device="cuda")
    return q, k, v, L


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
    split = torch.empty(1 << 22, dtype=torch.float32, device="cuda")  # ample: same split count
    out_ref = torch.empty_like(out_na)
    b2.call("b2_decode_gqa_split", q.data_ptr(), kv, vv, L.data_ptr(), out_ref.data_ptr(), B, nq, nkv, D, ctx,
            split.data_ptr(), split.numel(), stream)
    torch.cuda.synchronize()
    return out_na.float().cpu().numpy(), out_ref.float().cpu().numpy()


@pytest.mark.parametrize("B,ctx,nq,nkv,D", [(1, 4096, 32, 8, 128), (3, 700, 14, 2, 64), (8, 2048, 32, 8, 128)])
def test_noalloc_matches_scratch_entry_point_twice(cuda, B, ctx, nq, nkv, D):
    for call, (seed, ragged) in enumerate([(11, False), (12, True)]):
        got, want = _run_both(B, ctx, nq, nkv, D, seed + B, ragged)
        assert np.isfinite(got).all()
        assert float(np.max(np.abs(got - want))) <= TOL, (call, B, ctx)


def test_noalloc_refuses_problems_beyond_its_array(cuda):
    import torch
    B, ctx, nq, nkv, D = 1, 32768, 64, 8, 256
    q = torch.zeros(B, nq, D, dtype=torch.float16, device="cuda")
    kvbuf = torch.zeros(16, dtype=torch.float16, device="cuda")
    L = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
    view = b2.KVView(kvbuf.data_ptr(), ctx * nkv * D, D, nkv * D, 1)
    out = torch.empty_like(q)
    rc = b2.lib().b2_decode_gqa_split_noalloc(q.data_ptr(), view, view, L.data_ptr(), out.data_ptr(), B, nq, nkv, D,
                                              ctx, b2.stream_ptr())
    assert rc == -3 and b2.status_string(rc) == "workspace too small"
