"""FP8 (E4M3) weights for the decode steps.

Format: per output row, scale = max|w| / 448 and q = E4M3(w / scale) with
round-to-nearest-even and saturation (the oracle restates the OCP E4M3
encoding; the reference has no quantised path, RESULTS.md:39-40 plans one).
Checked here:
  * b2_quantize_fp8_rows: codes and scales bit-exact against the restatement
    (zero rows, subnormal-range and saturating values included);
  * b2_gemv_fp8 against float64 over the dequantised weights (B = 1, 2, 4,
    half and fp32 outputs, ragged N);
  * a quantised model's decode (b2_model_quantize_weights) teacher-forced
    against the oracle run on the dequantised weights -- logits within
    max-abs 2e-2 and cosine 0.9999, greedy ids under the near-tie rule -- on
    a small model and at Llama-3-8B projection widths (2 layers); switching
    back to fp16 restores the fp16 logits bit for bit;
  * the batched tensor-core step on the FP8 copies (E4M3 tiles by TMA,
    decoded into TMEM, A operand from TMEM) at batch 8 and 12 and at
    Llama-3-8B projection widths, against the same oracle.
"""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
from test_gpu_model import TIE_MARGIN, check_logits

pytestmark = pytest.mark.gpu


def _rows(rng, rows, K):
    w = (rng.standard_normal((rows, K)) * 0.02).astype(np.float32)
    w[0] = 0.0                                          # all-zero row: scale 1, codes 0
    w[1] *= 1e4                                         # large values (fp16 range)
    w[2] *= 1e-3                                        # tiny values
    w[3, ::7] = 0.0                                     # zeros inside a row
    w[4, 5] = -60000.0                                  # one dominant element: the rest round to subnormals / zero
    return O.f16(w)


@pytest.mark.parametrize("rows,K", [(37, 4096), (5, 112), (300, 14336)])
def test_quantize_rows_bit_exact(cuda, rows, K):
    import torch
    rng = np.random.default_rng(rows * 7 + K)
    w = _rows(rng, rows, K)
    wd = torch.from_numpy(w).half().cuda()
    q = torch.empty(rows, K, dtype=torch.uint8, device="cuda")
    sc = torch.empty(rows, dtype=torch.float32, device="cuda")
    b2.call("b2_quantize_fp8_rows", wd.data_ptr(), rows, K, q.data_ptr(), sc.data_ptr(), b2.stream_ptr())
    torch.cuda.synchronize()
    q_ref, sc_ref = O.quantize_e4m3_rows(w)
    assert np.array_equal(sc.cpu().numpy().view(np.uint32), sc_ref.view(np.uint32))
    got = q.cpu().numpy()
    bad = np.argwhere(got != q_ref)
    assert bad.size == 0, f"{len(bad)} codes differ, first at {bad[0]}: {got[tuple(bad[0])]:#x} vs {q_ref[tuple(bad[0])]:#x}"


@pytest.mark.parametrize("B,N,K,out_f32", [(1, 4096, 4096, 0), (2, 1000, 14336, 1), (4, 333, 2048, 0)])
def test_gemv_fp8_matches_float64(cuda, B, N, K, out_f32):
    import torch
    rng = np.random.default_rng(B * 1000 + N)
    w = O.f16(rng.standard_normal((N, K)).astype(np.float32) * 0.02)
    x = O.f16(rng.standard_normal((B, K)).astype(np.float32))
    q_ref, sc_ref = O.quantize_e4m3_rows(w)
    q = torch.from_numpy(q_ref).cuda()
    sc = torch.from_numpy(sc_ref).cuda()
    xd = torch.from_numpy(x).half().cuda()
    y = torch.empty(B, N, dtype=torch.float32 if out_f32 else torch.float16, device="cuda")
    b2.call("b2_gemv_fp8", q.data_ptr(), sc.data_ptr(), xd.data_ptr(), y.data_ptr(), B, N, K, out_f32,
            b2.stream_ptr())
    torch.cuda.synchronize()
    ref = x.astype(np.float64) @ O.dequantize_e4m3_rows(q_ref, sc_ref).astype(np.float64).T
    got = y.float().cpu().numpy().astype(np.float64)
    tol = 1e-4 * np.sqrt(K) + (0.0 if out_f32 else 2e-3 * np.max(np.abs(ref)))
    assert float(np.max(np.abs(got - ref))) <= tol


def _fp8_decode_check(cfg, seed, prompt_len, n_greedy):
    """Token-by-token decode of a prompt and its greedy continuation on the
    quantised model (every position through the FP8 GEMVs), against the
    oracle on the dequantised weights."""
    m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                 theta=cfg.theta, max_batch=1, max_seq=max(256, prompt_len + n_greedy + 8))
    m.init_random(seed, 0.02)
    rng = np.random.default_rng(seed)
    ids = list(rng.integers(0, cfg.vocab, prompt_len))
    m.quantize_weights("fp8")
    m.reset()
    logits = []
    for pos in range(prompt_len + n_greedy):
        lg, nx = m.decode_step([ids[pos]], [pos], want_logits=True, want_next=True)
        logits.append(lg[0].copy())
        if pos + 1 >= prompt_len:
            ids.append(int(nx[0]))
    W8 = O.fp8_weights(O.seeded_weights(cfg, seed))
    ref = O.forward(cfg, W8, np.asarray(ids[:prompt_len + n_greedy], np.int64))
    for pos in range(prompt_len + n_greedy):
        check_logits(logits[pos], ref[pos], f"position {pos}")
    for i in range(n_greedy):
        pos = prompt_len - 1 + i
        row = ref[pos]
        if ids[pos + 1] != int(np.argmax(row)):
            srt = np.sort(row)[::-1]
            assert srt[0] - srt[1] < TIE_MARGIN, (pos, ids[pos + 1], int(np.argmax(row)))
    return m, ids


def test_fp8_model_decode_matches_oracle(cuda):
    cfg = O.Config(vocab=1000, hidden=256, inter=704, layers=2, nq=8, nkv=2, head_dim=32, theta=10000.0)
    m, ids = _fp8_decode_check(cfg, 901, 12, 20)
    # back to fp16: the fp16 path's logits again, bit for bit
    m.reset()
    m.quantize_weights("fp16")
    a = [m.decode_step([t], [p])[0].copy() for p, t in enumerate(ids[:6])]
    m2 = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                  theta=cfg.theta, max_batch=1, max_seq=256)
    m2.init_random(901, 0.02)
    b = [m2.decode_step([t], [p])[0].copy() for p, t in enumerate(ids[:6])]
    for x, y in zip(a, b):
        assert np.array_equal(x.view(np.uint32), y.view(np.uint32))
    m.close()
    m2.close()


def test_fp8_model_decode_llama8b_width(cuda):
    # Llama-3-8B projection widths; a 4096-entry vocabulary keeps the host-side
    # quantisation of the oracle's lm_head small (its width is the same)
    cfg = O.Config(vocab=4096, hidden=4096, inter=14336, layers=2, nq=32, nkv=8, head_dim=128, theta=5e5)
    m, _ = _fp8_decode_check(cfg, 902, 8, 24)
    m.close()


def _fp8_batched_check(cfg, seed, B, prompt_len, n_dec):
    """B sequences decoded together on the quantised model's batched step,
    every position teacher-forced against the oracle on the dequantised
    weights."""
    m = b2.Model(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim, eps=cfg.eps,
                 theta=cfg.theta, max_batch=B, max_seq=256)
    m.init_random(seed, 0.02)
    m.quantize_weights("fp8")
    m.reset()
    rng = np.random.default_rng(seed)
    seqs = rng.integers(0, cfg.vocab, (B, prompt_len + n_dec))
    logits = []
    for pos in range(prompt_len + n_dec):
        lg, _ = m.decode_step(seqs[:, pos], [pos] * B, want_logits=True, want_next=True)
        logits.append(lg.copy())
    W8 = O.fp8_weights(O.seeded_weights(cfg, seed))
    for b in range(B):
        ref = O.forward(cfg, W8, seqs[b])
        for pos in range(prompt_len + n_dec):
            check_logits(logits[pos][b], ref[pos], f"sequence {b} position {pos}")
    m.close()


@pytest.mark.parametrize("B", [8, 12])
def test_fp8_batched_tensor_core_step(cuda, B):
    cfg = O.Config(vocab=1000, hidden=512, inter=1024, layers=2, nq=4, nkv=2, head_dim=128, theta=5e5)
    _fp8_batched_check(cfg, 903 + B, B, 6, 4)


def test_fp8_batched_llama8b_width(cuda):
    cfg = O.Config(vocab=4096, hidden=4096, inter=14336, layers=2, nq=32, nkv=8, head_dim=128, theta=5e5)
    _fp8_batched_check(cfg, 911, 8, 3, 3)
