"""A seeded, synthetic checkpoint directory in the layout the reference's
model loader reads (test infrastructure): config.json (Qwen2-style fields,
src/model/config.cpp:12-35), model.safetensors (bf16 tensors under the names
ModelWeights::load_and_validate expects, src/model/config.cpp:63-118, q/k/v
biases included) and tokenizer.json (the Qwen2 form: NFC, the Qwen2 split,
byte-level; a vocabulary of the 256 byte symbols, no merges, no special
tokens: every byte of a prompt is one token).
Weights ~N(0, std) rounded to bf16, norm weights 1.0.  No real model,
vocabulary or text is involved."""
from __future__ import annotations

import json
import os
import struct

import numpy as np


# the Qwen2 pre-tokenizer split (src/tokenizer/bpe.cpp:170)
QWEN2_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|"
               r"\s*[\r\n]+|\s+(?!\S)|\s+")


def byte_symbols() -> list[str]:
    """The printable-symbol stand-in of each byte used by byte-level BPE
    vocabularies: printable Latin-1 bytes stand for themselves, the others are
    shifted to code points from 256 upward, in byte order."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    sym, extra = {}, 0
    for b in range(256):
        if b in keep:
            sym[b] = chr(b)
        else:
            sym[b] = chr(256 + extra)
            extra += 1
    return [sym[b] for b in range(256)]


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, round to nearest even."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def make(path: str, *, vocab=512, hidden=256, inter=512, layers=2, heads=4, kv_heads=2, theta=1e6, eps=1e-6,
         std=0.02, seed=2024, tied=True) -> dict:
    """Write the directory; returns {tensor name: bf16 bits} and the config."""
    os.makedirs(path, exist_ok=True)
    cfg = {"model_type": "qwen2", "vocab_size": vocab, "hidden_size": hidden, "intermediate_size": inter,
           "num_hidden_layers": layers, "num_attention_heads": heads, "num_key_value_heads": kv_heads,
           "max_position_embeddings": 4096, "rms_norm_eps": eps, "rope_theta": theta, "tie_word_embeddings": tied,
           "torch_dtype": "bfloat16"}
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg, f)
    rng = np.random.default_rng(seed)
    D = hidden // heads
    kvd = kv_heads * D

    def w(*shape):
        return to_bf16_bits(rng.standard_normal(shape, dtype=np.float32) * std)

    def ones(n):
        return to_bf16_bits(np.ones(n, np.float32))

    t = {"model.embed_tokens.weight": w(vocab, hidden), "model.norm.weight": ones(hidden)}
    if not tied:
        t["lm_head.weight"] = w(vocab, hidden)
    for i in range(layers):
        p = f"model.layers.{i}."
        t[p + "input_layernorm.weight"] = ones(hidden)
        t[p + "post_attention_layernorm.weight"] = ones(hidden)
        t[p + "self_attn.q_proj.weight"] = w(hidden, hidden)
        t[p + "self_attn.q_proj.bias"] = w(hidden)
        t[p + "self_attn.k_proj.weight"] = w(kvd, hidden)
        t[p + "self_attn.k_proj.bias"] = w(kvd)
        t[p + "self_attn.v_proj.weight"] = w(kvd, hidden)
        t[p + "self_attn.v_proj.bias"] = w(kvd)
        t[p + "self_attn.o_proj.weight"] = w(hidden, hidden)
        t[p + "mlp.gate_proj.weight"] = w(inter, hidden)
        t[p + "mlp.up_proj.weight"] = w(inter, hidden)
        t[p + "mlp.down_proj.weight"] = w(hidden, inter)
    header, off = {}, 0
    for name, a in t.items():
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(os.path.join(path, "model.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        for a in t.values():
            f.write(np.ascontiguousarray(a).tobytes())
    tok = {"normalizer": {"type": "NFC"},
           "pre_tokenizer": {"type": "Sequence", "pretokenizers": [
               {"type": "Split", "pattern": {"Regex": QWEN2_SPLIT}, "behavior": "Isolated", "invert": False},
               {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": False, "use_regex": False}]},
           "decoder": {"type": "ByteLevel", "add_prefix_space": True, "trim_offsets": True, "use_regex": True},
           "model": {"type": "BPE", "vocab": {s: i for i, s in enumerate(byte_symbols())}, "merges": []},
           "added_tokens": []}
    with open(os.path.join(path, "tokenizer.json"), "w", encoding="utf-8") as f:
        json.dump(tok, f, ensure_ascii=False)
    return {"tensors": t, "config": cfg}
