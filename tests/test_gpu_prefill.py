"""tcgen05 flash prefill (b2_flash_prefill_gqa / _ex) vs the CPU oracle.

The oracle is the reference's causal GQA arithmetic (src/cpu/ops.cpp
causal_gqa, restated in oracle/b2oracle.c) on the same rounded inputs.
Tolerances: fp16, the reference's flash-prefill tolerance 3.5e-3
(tests/test_attention.cpp:180-291) on its U(-1, 1) inputs; bf16 (BASELINE's
causal-prefill config: N(0, 1) inputs, RoPE theta 5e5 applied in-kernel),
max-abs 2e-2 and mean-abs 2e-3 (bf16 keeps 8 mantissa bits: the output's own
rounding is up to 2^-9 relative).  Every call is followed by
b2_device_status, so a bounded pipeline wait that gave up fails the test.
"""
import os

import numpy as np
import pytest

import b2engine as b2
import oracle as O

pytestmark = pytest.mark.gpu

FP16_CASES = [  # (S, nq, nkv, D, batch)
    (1, 4, 2, 64, 1),
    (127, 8, 2, 64, 1),
    (128, 32, 8, 128, 1),
    (129, 32, 8, 128, 1),
    (300, 14, 2, 64, 2),
    (700, 32, 8, 128, 1),
]


def _oracle_attention(q, k, v, S, nq, nkv, D):
    O.set_threads(os.cpu_count() or 1)
    return O.causal_gqa(q.astype(np.float32), k.astype(np.float32), v.astype(np.float32), S, nq, nkv, D)


@pytest.mark.parametrize("S,nq,nkv,D,B", FP16_CASES)
def test_flash_prefill_fp16(cuda, S, nq, nkv, D, B):
    import torch
    rng = np.random.default_rng(S * 131 + nq)
    q = rng.uniform(-1, 1, (B, S, nq, D)).astype(np.float16)
    k = rng.uniform(-1, 1, (B, S, nkv, D)).astype(np.float16)
    v = rng.uniform(-1, 1, (B, S, nkv, D)).astype(np.float16)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    out = torch.empty(B, S, nq, D, dtype=torch.float16, device="cuda")
    b2.call("b2_flash_prefill_gqa", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), S, nq, nkv, D, B,
            b2.stream_ptr())
    assert b2.device_status() == 0
    got = out.float().cpu().numpy()
    for bb in range(B):
        ref = _oracle_attention(q[bb].reshape(S, -1), k[bb].reshape(S, -1), v[bb].reshape(S, -1), S, nq, nkv, D)
        assert float(np.max(np.abs(got[bb].reshape(S, -1) - ref))) < 3.5e-3, (S, nq, D, bb)


def _bf16(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(torch.bfloat16)


@pytest.mark.parametrize("S,rope", [(2048, 500000.0), (640, 0.0)])
def test_flash_prefill_bf16_rope(cuda, S, rope):
    """BASELINE's causal-prefill shape: bf16 Q [1,S,32,128], K/V [1,S,8,128]
    ~N(0,1), RoPE theta 5e5 inside the call (rope = 0: no rotation)."""
    import torch
    nq, nkv, D = 32, 8, 128
    rng = np.random.default_rng(S)
    q = _bf16(rng.standard_normal((S, nq * D)))
    k = _bf16(rng.standard_normal((S, nkv * D)))
    v = _bf16(rng.standard_normal((S, nkv * D)))
    out = torch.empty(S, nq * D, dtype=torch.bfloat16, device="cuda")
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    b2.call("b2_flash_prefill_gqa_ex", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), S, nq, nkv, D, 1,
            1, rope, 0, b2.stream_ptr())
    assert b2.device_status() == 0
    qf, kf, vf = q.float().numpy(), k.float().numpy(), v.float().numpy()
    if rope > 0:
        qf, kf = O.apply_rope(qf, kf, S, nq, nkv, D, 0, rope)
        qf, kf = _bf16(qf).float().numpy(), _bf16(kf).float().numpy()  # the kernel keeps rotated rows in bf16
    ref = _oracle_attention(qf, kf, vf, S, nq, nkv, D)
    err = np.abs(out.float().cpu().numpy() - ref)
    assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3, (float(err.max()), float(err.mean()))


@pytest.mark.slow
def test_flash_prefill_bf16_rope_s8192_sampled(cuda):
    """BASELINE's longest causal prefill, S = 8192 (bf16, RoPE theta 5e5 in
    the kernel), against the oracle on two kv head groups (q heads 0-3 and
    28-31) for the first 192 query rows (the first tiles, short causal
    windows) and the last 256 (64 key tiles each)."""
    import torch
    S, nq, nkv, D, theta = 8192, 32, 8, 128, 500000.0
    rng = np.random.default_rng(8192)
    q = _bf16(rng.standard_normal((S, nq * D)))
    k = _bf16(rng.standard_normal((S, nkv * D)))
    v = _bf16(rng.standard_normal((S, nkv * D)))
    out = torch.empty(S, nq * D, dtype=torch.bfloat16, device="cuda")
    dq, dk, dv = q.cuda(), k.cuda(), v.cuda()
    b2.call("b2_flash_prefill_gqa_ex", dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), out.data_ptr(), S, nq, nkv, D, 1,
            1, theta, 0, b2.stream_ptr())
    assert b2.device_status() == 0
    got = out.float().cpu().numpy().reshape(S, nq, D)
    O.set_threads(os.cpu_count() or 1)
    qf = q.float().numpy().reshape(S, nq, D)
    kf = k.float().numpy().reshape(S, nkv, D)
    vf = v.float().numpy().reshape(S, nkv, D)
    head, tail = 192, 256
    for g in (0, nkv - 1):
        hs = slice(4 * g, 4 * g + 4)
        qg = np.ascontiguousarray(qf[:, hs, :]).reshape(S, 4 * D)
        kg = np.ascontiguousarray(kf[:, g, :])
        vg = np.ascontiguousarray(vf[:, g, :])
        qg, kg = O.apply_rope(qg, kg, S, 4, 1, D, 0, theta)
        qg, kg = _bf16(qg).float().numpy(), _bf16(kg).float().numpy()  # rotated rows are kept in bf16
        ref_head = O.causal_gqa(qg[:head], kg[:head], vg[:head], head, 4, 1, D)
        ref_tail = O.causal_gqa_rows(qg, kg, vg, S, 4, 1, D, S - tail)
        for rows, ref in ((slice(0, head), ref_head), (slice(S - tail, S), ref_tail)):
            err = np.abs(got[rows, hs, :].reshape(ref.shape) - ref)
            assert float(err.max()) < 2e-2 and float(err.mean()) < 2e-3, (g, rows, float(err.max()))


def test_flash_prefill_fp16_rope_matches_separate_rope(cuda):
    """In-kernel RoPE (fp16) equals b2_apply_rope followed by the plain kernel."""
    import torch
    S, nq, nkv, D = 300, 8, 2, 64
    g = torch.Generator(device="cuda").manual_seed(5)
    q = torch.randn(S, nq, D, generator=g, device="cuda").half()
    k = torch.randn(S, nkv, D, generator=g, device="cuda").half()
    v = torch.randn(S, nkv, D, generator=g, device="cuda").half()
    out_a = torch.empty_like(q)
    b2.call("b2_flash_prefill_gqa_ex", q.data_ptr(), k.data_ptr(), v.data_ptr(), out_a.data_ptr(), S, nq, nkv, D, 1,
            0, 10000.0, 7, b2.stream_ptr())
    q2, k2 = q.clone(), k.clone()
    b2.call("b2_apply_rope", q2.data_ptr(), k2.data_ptr(), S, nq, nkv, D, 7, 10000.0, b2.stream_ptr())
    out_b = torch.empty_like(q)
    b2.call("b2_flash_prefill_gqa", q2.data_ptr(), k2.data_ptr(), v.data_ptr(), out_b.data_ptr(), S, nq, nkv, D, 1,
            b2.stream_ptr())
    assert b2.device_status() == 0
    assert float((out_a.float() - out_b.float()).abs().max()) < 4e-3


def test_flash_prefill_workspace_form(cuda):
    """b2_flash_prefill_gqa_ws takes the rotated q and k copies from a caller's
    b2_workspace (no allocation): same bytes as b2_flash_prefill_gqa_ex, and
    B2_ERR_WORKSPACE when the workspace is one byte short."""
    import ctypes
    import torch
    S, nq, nkv, D = 700, 32, 8, 128
    g = torch.Generator(device="cuda").manual_seed(9)
    q = torch.randn(S, nq * D, generator=g, device="cuda").bfloat16()
    k = torch.randn(S, nkv * D, generator=g, device="cuda").bfloat16()
    v = torch.randn(S, nkv * D, generator=g, device="cuda").bfloat16()
    out_a, out_b = torch.empty_like(q), torch.empty_like(q)
    st = b2.stream_ptr()
    b2.call("b2_flash_prefill_gqa_ex", q.data_ptr(), k.data_ptr(), v.data_ptr(), out_a.data_ptr(), S, nq, nkv, D, 1,
            1, 500000.0, 3, st)
    need = b2.lib().b2_flash_prefill_workspace_bytes(S, nq, nkv, D, 1)
    assert need == S * (nq + nkv) * D * 2  # rotated q and k copies
    for nbytes, want in ((need, 0), (need - 16, -3)):
        ws = ctypes.c_void_p()
        b2.call("b2_workspace_create", nbytes, ctypes.byref(ws))
        assert b2.lib().b2_workspace_bytes(ws) == nbytes
        rc = b2.lib().b2_flash_prefill_gqa_ws(q.data_ptr(), k.data_ptr(), v.data_ptr(), out_b.data_ptr(), S, nq, nkv,
                                              D, 1, 1, 500000.0, 3, ws, st)
        assert rc == want
        torch.cuda.synchronize()
        b2.call("b2_workspace_destroy", ws)
    assert b2.device_status() == 0
    assert torch.equal(out_a.view(torch.int16), out_b.view(torch.int16))
