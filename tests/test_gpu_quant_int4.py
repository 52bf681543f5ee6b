"""4-bit weights for the batch-1/2 decode GEMVs.

Format (include/b2engine.h, b2_quantize_int4_rows): per group of 128
weights of a row, scale = max|w| / 7 and q = rint(w / scale) in [-7, 7],
packed two codes per byte.  The reference has no quantised path (its
RESULTS.md:39-40 plans INT4 weights).  Checked here:
  * b2_quantize_int4_rows: packed codes and scales bit-exact against the
    oracle's restatement (zero rows and groups, large and tiny values, one
    dominant weight);
  * b2_gemv_int4 against float64 over the dequantised weights (B = 1, 2, 3,
    half and fp32 outputs, ragged N, K = 4096 and 14336);
  * a 4-bit model's decode (b2_model_quantize_weights) teacher-forced
    against the oracle on the dequantised weights -- logits within max-abs
    2e-2 and cosine 0.9999, greedy ids under the near-tie rule -- on a small
    model and at Llama-3-8B projection widths; switching back to fp16
    restores the fp16 logits bit for bit.
"""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
from test_gpu_model import TIE_MARGIN, check_logits

pytestmark = pytest.mark.gpu


def _rows(rng, rows, K):
    w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    w[0] = 0.0                                          # all-zero row
    w[1] *= 1e4                                         # large values (fp16 range)
    w[2] *= 1e-3                                        # tiny values
    w[3, :128] = 0.0                                    # one all-zero group
    w[4, 5] = -60000.0                                  # one dominant weight: the rest of its group round to 0
    return O.f16(w)


@pytest.mark.parametrize("rows,K", [(37, 4096), (5, 128), (300, 14336)])
def test_quantize_int4_bit_exact(cuda, rows, K):
    import torch
    rng = np.random.default_rng(rows * 11 + K)
    w = _rows(rng, rows, K)
    wd = torch.from_numpy(w).half().cuda()
    q = torch.empty(rows, K // 2, dtype=torch.uint8, device="cuda")
    sc = torch.empty(rows, K // 128, dtype=torch.float32, device="cuda")
    b2.call("b2_quantize_int4_rows", wd.data_ptr(), rows, K, q.data_ptr(), sc.data_ptr(), b2.stream_ptr())
    torch.cuda.synchronize()
    q_ref, sc_ref = O.quantize_int4_rows(w)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), sc_ref.view(np.uint32))
    got = q.cpu().numpy()
    bad = np.argwhere(got != q_ref)
    assert bad.size == 0, f"{len(bad)} bytes differ, first at {bad[0]}"


@pytest.mark.parametrize("B,N,K,out_f32", [(1, 4096, 4096, 0), (2, 1000, 14336, 1), (3, 333, 2048, 0)])
def test_gemv_int4_matches_float64(cuda, B, N, K, out_f32):
    import torch
    rng = np.random.default_rng(B * 1000 + N + 7)
    w = O.f16(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    x = O.f16(rng.standard_normal((B, K)).astype(np.float32))
    q_ref, sc_ref = O.quantize_int4_rows(w)
    q = torch.from_numpy(q_ref).cuda()
    sc = torch.from_numpy(sc_ref).cuda()
    xd = torch.from_numpy(x).half().cuda()
    y = torch.empty(B, N, dtype=torch.float32 if out_f32 else torch.float16, device="cuda")
    b2.call("b2_gemv_int4", q.data_ptr(), sc.data_ptr(), xd.data_ptr(), y.data_ptr(), B, N, K, out_f32,
            b2.stream_ptr())
    torch.cuda.synchronize()
    ref = x.astype(np.float64) @ O.dequantize_int4_rows(q_ref, sc_ref).astype(np.float64).T
    got = y.float().cpu().numpy().astype(np.float64)
    tol = 1e-4 * np.sqrt(K) + (0.0 if out_f32 else 2e-3 * np.max(np.abs(ref)))
    assert float(np.max(np.abs(got - ref))) <= tol


def _int4_decode_check(cfg, seed, prompt_len, n_greedy, B=1):
    """Token-by-token decode of B prompts and their greedy continuations on
    the 4-bit model (every position through the 4-bit GEMVs), against the
    oracle on the dequantised weights."""
    m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                 theta=cfg.theta, max_batch=B, max_seq=max(256, prompt_len + n_greedy + 8))
    m.init_random(seed, 0.02)
    rng = np.random.default_rng(seed)
    ids = [list(rng.integers(0, cfg.vocab, prompt_len)) for _ in range(B)]
    m.quantize_weights("int4")
    m.reset()
    logits = []
    for pos in range(prompt_len + n_greedy):
        lg, nx = m.decode_step([s[pos] for s in ids], [pos] * B, want_logits=True, want_next=True)
        logits.append(lg.copy())
        if pos + 1 >= prompt_len:
            for b in range(B):
                ids[b].append(int(nx[b]))
    W4 = O.int4_weights(O.seeded_weights(cfg, seed))
    for b in range(B):
        ref = O.forward(cfg, W4, np.asarray(ids[b][:prompt_len + n_greedy], np.int64))
        for pos in range(prompt_len + n_greedy):
            check_logits(logits[pos][b], ref[pos], f"sequence {b} position {pos}")
        for i in range(n_greedy):
            pos = prompt_len - 1 + i
            row = ref[pos]
            if ids[b][pos + 1] != int(np.argmax(row)):
                srt = np.sort(row)[::-1]
                assert srt[0] - srt[1] < TIE_MARGIN, (b, pos, ids[b][pos + 1], int(np.argmax(row)))
    return m, ids


def test_int4_model_decode_matches_oracle(cuda):
    cfg = O.Config(vocab=1000, hidden=256, inter=768, layers=2, nq=8, nkv=2, head_dim=32, theta=10000.0)
    m, ids = _int4_decode_check(cfg, 921, 12, 20)
    # back to fp16: the fp16 path's logits again, bit for bit
    m.reset()
    m.quantize_weights("fp16")
    a = [m.decode_step([t], [p])[0].copy() for p, t in enumerate(ids[0][:6])]
    m2 = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                  theta=cfg.theta, max_batch=1, max_seq=256)
    m2.init_random(921, 0.02)
    b = [m2.decode_step([t], [p])[0].copy() for p, t in enumerate(ids[0][:6])]
    for x, y in zip(a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    m.close()
    m2.close()


def test_int4_model_decode_batch2(cuda):
    cfg = O.Config(vocab=1000, hidden=256, inter=768, layers=2, nq=8, nkv=2, head_dim=32, theta=10000.0)
    m, _ = _int4_decode_check(cfg, 923, 6, 10, B=2)
    m.close()


def test_int4_model_decode_llama8b_width(cuda):
    cfg = O.Config(vocab=4096, hidden=4096, inter=14336, layers=2, nq=32, nkv=8, head_dim=128, theta=5e5)
    m, _ = _int4_decode_check(cfg, 922, 8, 24)
    m.close()


def test_int4_rejects_unaligned_width(cuda):
    cfg = O.Config(vocab=1000, hidden=256, inter=704, layers=1, nq=8, nkv=2, head_dim=32, theta=10000.0)
    m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, max_batch=1,
                 max_seq=64)
    with pytest.raises(b2.B2Error) as e:
        m.quantize_weights("int4")
    assert e.value.status == -2
    m.close()
