"""Checkpoint loading and the full-recompute forward.

b2_model_set_tensor_bf16 takes bf16 tensors as a checkpoint stores them and
converts them to fp16 on the device by the reference loader's bit rule
(src/loader/safetensors.cpp:307-328); b2_model_forward_logits runs the whole
sequence through the batched prefill and an all-positions lm_head (the
reference's forward_gpu, src/model/forward_gpu.h:76-84)."""
import numpy as np
import pytest

import b2engine as b2
import oracle as O
import synthetic_checkpoint as SC

pytestmark = pytest.mark.gpu


def bf16_to_f16_rule(bits: np.ndarray) -> np.ndarray:
    """The loader's conversion on the host: exponent rebased, below the fp16
    normal range -> signed zero, above it -> signed infinity."""
    u = bits.astype(np.uint32)
    sign = (u & 0x8000).astype(np.uint32)
    e = ((u >> 7) & 0xFF).astype(np.int32) - 127 + 15
    mant = (u & 0x7F) << 3
    out = np.where(e <= 0, sign, np.where(e >= 31, sign | 0x7C00, sign | (np.clip(e, 0, 31).astype(np.uint32) << 10) | mant))
    return out.astype(np.uint16)


def test_bf16_conversion_bit_exact(cuda):
    """Embedding rows of crafted bf16 values (normal, below the fp16 normal
    range, signed zeros) reach the residual stream unchanged when the layers
    add nothing (W_o = W_down = 0): the step's fp32 hidden state must equal
    the loader rule's fp16 values bit for bit (zeros up to their sign).  A value above the fp16 range
    in the (untied) lm_head becomes infinity: its logit is infinite."""
    V, H, I, L, nq, nkv, D = 16, 64, 64, 1, 2, 2, 32
    m = b2.Model(V, H, I, L, nq, nkv, D, tied=False, max_batch=1, max_seq=8)
    m.init_random(3, 0.02)
    rng = np.random.default_rng(5)
    vals = rng.standard_normal((V, H)).astype(np.float32) * 0.5
    vals[0, :8] = [1e-6, -1e-6, 3e-5, -7e-5, 6.2e-5, -0.0, 0.0, 2.5]
    bits = SC.to_bf16_bits(vals)
    m.set_tensor_bf16("embed", bits)
    m.set_tensor("0.wo", np.zeros((H, nq * D), np.float16))
    m.set_tensor("0.wd", np.zeros((H, I), np.float16))
    head = rng.standard_normal((V, H)).astype(np.float32) * 0.02
    head[3, :] = 0.0
    head[3, 9] = 1e5  # beyond fp16: infinity (column 9 of every embedding row above is non-zero)
    m.set_tensor_bf16("lm_head", SC.to_bf16_bits(head))
    want = bf16_to_f16_rule(bits).view(np.float16).astype(np.float32)
    assert want[0, 0] == 0.0 and want[0, 4] != 0.0
    for tok in (0, 1, 7):
        lg = m.prefill(np.array([[tok]]))[0]
        h = m.read("hidden", np.float32, H)
        # bit for bit, except that adding the layers' zero outputs turns -0 into +0
        nz = want[tok] != 0
        assert np.array_equal(h[nz].view(np.uint32), want[tok][nz].view(np.uint32)), tok
        assert not np.any(h[~nz]), tok
        assert np.isinf(lg[3]) and np.isfinite(np.delete(lg, 3)).all(), tok
        m.reset()
    m.close()


def test_forward_logits_from_bf16_checkpoint_matches_oracle(cuda, tmp_path):
    """A Qwen2-layout checkpoint (tied head, q/k/v biases) uploaded as bf16:
    logits of every position of a 40-token sequence within max-abs 2e-2 and
    cosine >= 0.9999 of the oracle on the same weights, and the last row
    equal to b2_model_prefill's."""
    info = SC.make(str(tmp_path), vocab=700, hidden=256, inter=512, layers=2, heads=4, kv_heads=2, seed=77)
    c, t = info["config"], info["tensors"]
    H, I, V = c["hidden_size"], c["intermediate_size"], c["vocab_size"]
    nq, nkv = c["num_attention_heads"], c["num_key_value_heads"]
    D = H // nq
    m = b2.Model(V, H, I, c["num_hidden_layers"], nq, nkv, D, eps=c["rms_norm_eps"], theta=c["rope_theta"],
                 tied=True, bias=True, max_batch=1, max_seq=64)
    names = {"input_layernorm.weight": "ln1", "post_attention_layernorm.weight": "ln2",
             "self_attn.q_proj.weight": "wq", "self_attn.q_proj.bias": "bq", "self_attn.k_proj.weight": "wk",
             "self_attn.k_proj.bias": "bk", "self_attn.v_proj.weight": "wv", "self_attn.v_proj.bias": "bv",
             "self_attn.o_proj.weight": "wo", "mlp.gate_proj.weight": "wg", "mlp.up_proj.weight": "wu",
             "mlp.down_proj.weight": "wd"}
    m.set_tensor_bf16("embed", t["model.embed_tokens.weight"])
    m.set_tensor_bf16("final_norm", t["model.norm.weight"])
    for l in range(c["num_hidden_layers"]):
        for k, n in names.items():
            m.set_tensor_bf16(f"{l}.{n}", t[f"model.layers.{l}.{k}"])
    from test_gpu_reference_apps import _oracle_model
    cfg, w = _oracle_model(info)
    ids = np.random.default_rng(9).integers(0, V, 40)
    got = m.forward_logits(ids)
    ref = O.forward(cfg, w, ids, logit_row0=0)
    for i in range(len(ids)):
        a, b = got[i].astype(np.float64), ref[i].astype(np.float64)
        assert float(np.max(np.abs(a - b))) <= 2e-2, i
        assert float(a @ b / (np.linalg.norm(a) * np.linalg.norm(b))) >= 0.9999, i
    m.reset()
    last = m.prefill(ids[None, :])[0]
    assert float(np.max(np.abs(last - got[-1]))) <= 2e-3
    # longer sequences grow the workspaces: every call gives the prefix's rows
    for S in (41, 57):
        ids2 = np.random.default_rng(S).integers(0, V, S)
        assert float(np.max(np.abs(m.forward_logits(ids2)[-1] - m.prefill(ids2[None, :])[0]))) <= 2e-3
    m.close()
