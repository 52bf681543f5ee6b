"""Generates tests/golden/ref_cpu_golden.npz from the reference's own CPU path
(src/cpu/ops.cpp + src/model/forward_cpu.cpp compiled unmodified into
oracle/_ref/libref_cpu.so by `make -C oracle`).  Run in a container that has
the reference sources:  python tests/golden/make_golden.py
Inputs are fp16-rounded seeded values; outputs are the reference's fp32
results, which the oracle restatement must reproduce bit for bit."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as O  # noqa: E402


def f16(rng, *shape, lo=-1.0, hi=1.0):
    return rng.uniform(lo, hi, shape).astype(np.float16).astype(np.float32)


def main():
    assert O.ref_lib() is not None, "build oracle/_ref first (make -C oracle)"
    rng = np.random.default_rng(20261201)
    g = {}
    x, w = f16(rng, 7, 300), f16(rng, 300)
    g["rms_x"], g["rms_w"], g["rms_out"] = x, w, O.rmsnorm(x, w, 1e-5, ref=True)
    A, B = f16(rng, 9, 200), f16(rng, 70, 200)
    g["mm_A"], g["mm_B"], g["mm_out"] = A, B, O.matmul_transB(A, B, ref=True)
    q, k = f16(rng, 5, 4, 64), f16(rng, 5, 2, 64)
    rq, rk = O.apply_rope(q, k, 5, 4, 2, 64, 37, 500000.0, ref=True)
    g["rope_q"], g["rope_k"], g["rope_q_out"], g["rope_k_out"] = q, k, rq, rk
    q, k, v = f16(rng, 11, 6, 32), f16(rng, 11, 2, 32), f16(rng, 11, 2, 32)
    g["attn_q"], g["attn_k"], g["attn_v"] = q, k, v
    g["attn_out"] = O.causal_gqa(q, k, v, 11, 6, 2, 32, ref=True)
    gg, uu = f16(rng, 500, lo=-4, hi=4), f16(rng, 500, lo=-4, hi=4)
    g["swiglu_g"], g["swiglu_u"], g["swiglu_out"] = gg, uu, O.swiglu(gg, uu, ref=True)
    for name, bias in (("llama", False), ("qwen", True)):
        cfg = O.Config(vocab=256, hidden=64, inter=160, layers=2, nq=4, nkv=2, head_dim=16, theta=10000.0,
                       tied=True, has_bias=bias, eps=1e-6)
        W = O.seeded_weights(cfg, 555 if bias else 444)
        ids = rng.integers(0, cfg.vocab, 9)
        g[f"fwd_{name}_ids"] = ids
        g[f"fwd_{name}_logits"] = O.ref_forward(cfg, W, ids)
    np.savez_compressed(os.path.join(HERE, "ref_cpu_golden.npz"), **g)
    print("wrote", os.path.join(HERE, "ref_cpu_golden.npz"))


if __name__ == "__main__":
    main()
