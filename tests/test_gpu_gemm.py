"""tcgen05 GEMM (b2_matmul_transB / _f32 main path) at prefill projection shapes.

C[M,N] = A[M,K] * B[N,K]^T with half inputs and fp32 accumulation, checked
against a float64 host product of the same half-rounded inputs.  Tolerances:
fp16 output, 1e-3 * max|C| + 1e-3 (one fp16 rounding of the result is
4.9e-4 relative); fp32 output, 1e-4 * max|C| + 1e-4 (fp32 accumulation of K
products).  Ragged M/N/K exercise the TMA zero fill of partial tiles; every
call is followed by b2_device_status, so a bounded pipeline wait that gave up
fails the test instead of passing silently.
"""
import numpy as np
import pytest

import b2engine as b2

pytestmark = pytest.mark.gpu

SHAPES = [
    (128, 64, 128),      # one tile, one k block
    (200, 520, 300),     # ragged in every dimension
    (17, 4096, 1000),    # few rows (a prompt shorter than a tile)
    (512, 4096, 6144),   # Llama-3-8B q|k|v projection of a 512-token prompt
    (384, 14336, 512),   # long K (down projection width), column slice
    (1024, 2048, 5632),  # TinyLlama gate width, 256-wide tiles
]


def _run(M, K, N, f32, seed):
    import torch
    g = torch.Generator().manual_seed(seed)
    A = (torch.rand(M, K, generator=g) * 2 - 1).half()
    B = (torch.rand(N, K, generator=g) * 2 - 1).half()
    ref = (A.double() @ B.double().T).numpy()
    dA, dB = A.cuda(), B.cuda()
    out = torch.empty(M, N, dtype=torch.float32 if f32 else torch.float16, device="cuda")
    name = "b2_matmul_transB_f32" if f32 else "b2_matmul_transB"
    b2.call(name, dA.data_ptr(), dB.data_ptr(), out.data_ptr(), M, K, N, b2.stream_ptr())
    assert b2.device_status() == 0, "a tcgen05 pipeline wait gave up"
    return out.double().cpu().numpy(), ref


@pytest.mark.parametrize("M,K,N", SHAPES)
def test_tc_gemm_half_out(cuda, M, K, N):
    got, ref = _run(M, K, N, False, 1000 + M)
    tol = 1e-3 * float(np.max(np.abs(ref))) + 1e-3
    assert float(np.max(np.abs(got - ref))) <= tol, (M, K, N)


@pytest.mark.parametrize("M,K,N", SHAPES[:4])
def test_tc_gemm_f32_out(cuda, M, K, N):
    got, ref = _run(M, K, N, True, 2000 + M)
    tol = 1e-4 * float(np.max(np.abs(ref))) + 1e-4
    assert float(np.max(np.abs(got - ref))) <= tol, (M, K, N)


def test_tc_gemm_deterministic(cuda):
    a, _ = _run(256, 1024, 512, False, 7)
    b, _ = _run(256, 1024, 512, False, 7)
    assert np.array_equal(a, b)
