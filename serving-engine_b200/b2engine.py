"""ctypes binding of the b2engine C-ABI (include/b2engine.h).

Python here is plumbing for tests and the benchmark: device memory comes from
torch tensors, every computation is a call into lib/libb2engine.so.  There is
no fallback: if the library is missing or a call fails, an exception is raised.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libb2engine.so")
_LIB = None

vp = C.c_void_p
i32 = C.c_int
i64 = C.c_int64
f32 = C.c_float
u64 = C.c_uint64


class B2Error(RuntimeError):
    def __init__(self, fn: str, status: int):
        self.status = status
        detail = lib().b2_last_error().decode()
        super().__init__(f"{fn} failed: status {status} ({status_string(status)})" + (f": {detail}" if detail else ""))


class KVView(C.Structure):
    _fields_ = [("data", vp), ("stride_b", i64), ("stride_h", i64), ("stride_s", i64), ("stride_d", i64)]


class TokenizerInfo(C.Structure):
    _fields_ = [("vocab_size", i64), ("n_ids", i64), ("n_merges", i64), ("pre_tokenizer", i32), ("nfc", i32),
                ("ignore_merges", i32), ("chat_format", i32), ("bos_id", i32), ("eos_id", i32), ("n_stop", i32),
                ("stop_ids", i32 * 4), ("n_added", i32)]


class SamplerConfig(C.Structure):
    _fields_ = [("temperature", f32), ("top_k", i32), ("top_p", f32), ("repetition_penalty", f32), ("seed", u64)]


class ModelConfig(C.Structure):
    _fields_ = [("vocab_size", i32), ("hidden_size", i32), ("intermediate_size", i32), ("num_layers", i32),
                ("num_q_heads", i32), ("num_kv_heads", i32), ("head_dim", i32), ("rms_norm_eps", f32),
                ("rope_theta", f32), ("tie_word_embeddings", i32), ("has_qkv_bias", i32), ("max_batch", i32),
                ("max_seq", i32)]


# name -> (restype, argtypes)
_SIGS = {
    "b2_version": (C.c_char_p, []),
    "b2_status_string": (C.c_char_p, [i32]),
    "b2_device_status": (i32, [i32]),
    "b2_last_error": (C.c_char_p, []),
    "b2_embedding_lookup": (i32, [vp, vp, vp, i64, i64, vp]),
    "b2_rmsnorm": (i32, [vp, vp, vp, i64, i64, f32, vp]),
    "b2_bias_add": (i32, [vp, vp, vp, i64, i64, vp]),
    "b2_residual_add": (i32, [vp, vp, vp, i64, vp]),
    "b2_apply_rope": (i32, [vp, vp, i64, i64, i64, i64, i64, f32, vp]),
    "b2_causal_gqa": (i32, [vp, vp, vp, vp, i64, i64, i64, i64, vp]),
    "b2_softmax": (i32, [vp, vp, i64, i64, vp]),
    "b2_decode_gqa": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "b2_decode_gqa_split": (i32, [vp, KVView, KVView, vp, vp, i32, i32, i32, i32, i32, vp, C.c_size_t, vp]),
    "b2_decode_gqa_split_noalloc": (i32, [vp, KVView, KVView, vp, vp, i32, i32, i32, i32, i32, vp]),
    "b2_flash_prefill_gqa": (i32, [vp, vp, vp, vp, i64, i32, i32, i32, i32, vp]),
    "b2_flash_prefill_gqa_ex": (i32, [vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, f32, i64, vp]),
    "b2_workspace_create": (i32, [C.c_size_t, C.POINTER(vp)]),
    "b2_workspace_destroy": (i32, [vp]),
    "b2_workspace_bytes": (C.c_size_t, [vp]),
    "b2_flash_prefill_workspace_bytes": (C.c_size_t, [i64, i32, i32, i32, i32]),
    "b2_flash_prefill_gqa_ws": (i32, [vp, vp, vp, vp, i64, i32, i32, i32, i32, i32, f32, i64, vp, vp]),
    "b2_swiglu": (i32, [vp, vp, vp, i64, vp]),
    "b2_matmul_transB": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "b2_matmul_transB_f32": (i32, [vp, vp, vp, i32, i32, i32, vp]),
    "b2_gemv": (i32, [vp, vp, vp, i32, i32, vp]),
    "b2_gemv_bias": (i32, [vp, vp, vp, vp, i32, i32, vp]),
    "b2_gemv_residual": (i32, [vp, vp, vp, vp, i32, i32, vp]),
    "b2_gemv_batched": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "b2_quantize_fp8_rows": (i32, [vp, i64, i32, vp, vp, vp]),
    "b2_gemv_fp8": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "b2_quantize_int4_rows": (i32, [vp, i64, i32, vp, vp, vp]),
    "b2_gemv_int4": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "b2_append_kv_cache": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, vp]),
    "b2_sampler_create": (i32, [i32, i32, C.POINTER(vp)]),
    "b2_sampler_destroy": (i32, [vp]),
    "b2_sampler_sample": (i32, [vp, vp, vp, i32, C.POINTER(SamplerConfig), vp, C.POINTER(i32)]),
    "b2_sampler_sample_async": (i32, [vp, vp, vp, i32, C.POINTER(SamplerConfig), vp, vp]),
    "b2_sampler_rng_state": (u64, [vp]),
    "b2_sampler_set_rng_state": (i32, [vp, u64]),
    "b2_nccl_unique_id": (i32, [vp]),
    "b2_model_create": (i32, [C.POINTER(ModelConfig), i32, i32, vp, C.POINTER(vp)]),
    "b2_model_create_paged": (i32, [C.POINTER(ModelConfig), i32, i32, i32, i32, vp, C.POINTER(vp)]),
    "b2_model_prefill_paged": (i32, [vp, vp, i32, vp, i32, i32, vp, vp]),
    "b2_model_decode_step_paged": (i32, [vp, vp, vp, vp, i32, i32, vp, vp]),
    "b2_model_destroy": (i32, [vp]),
    "b2_model_init_random": (i32, [vp, u64, f32]),
    "b2_model_p2p_handle": (i32, [vp, vp]),
    "b2_model_p2p_open": (i32, [vp, vp]),
    "b2_model_trace_step": (i32, [vp, i32, vp, i32, C.POINTER(i32)]),
    "b2_model_set_tensor": (i32, [vp, C.c_char_p, vp, i64, i64]),
    "b2_model_set_tensor_bf16": (i32, [vp, C.c_char_p, vp, i64, i64]),
    "b2_model_forward_logits": (i32, [vp, vp, i32, vp]),
    "b2_model_reset": (i32, [vp]),
    "b2_model_set_sampling": (i32, [vp, C.POINTER(SamplerConfig)]),
    "b2_model_quantize_weights": (i32, [vp, i32]),
    "b2_model_prefill": (i32, [vp, vp, i32, i32, vp]),
    "b2_model_decode_step": (i32, [vp, vp, vp, i32, vp, vp]),
    "b2_model_decode_enqueue": (i32, [vp, vp, vp, i32, vp]),
    "b2_model_generate_greedy": (i32, [vp, i32, vp]),
    "b2_model_sync": (i32, [vp]),
    "b2_model_stream": (vp, [vp]),
    "b2_model_buffer": (vp, [vp, C.c_char_p]),
    "b2_model_read": (i32, [vp, C.c_char_p, vp, C.c_size_t, C.c_size_t]),
    "b2_model_kv_layout": (i32, [vp, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(i64)]),
    "b2_model_step_bytes": (C.c_double, [vp, i32, i32]),
    "b2_model_step_launches": (i32, [vp, i32]),
    "b2_model_time_kernel": (i32, [vp, i32, i32, i32, C.POINTER(f32)]),
    "b2_model_kernel_bytes": (C.c_double, [vp, i32, i32, i32]),
}


_SIGS.update({
    "b2_tokenizer_load": (i32, [C.c_char_p, C.POINTER(vp)]),
    "b2_tokenizer_load_json": (i32, [C.c_char_p, C.c_size_t, C.POINTER(vp)]),
    "b2_tokenizer_destroy": (None, [vp]),
    "b2_tokenizer_encode": (i32, [vp, C.c_char_p, C.c_size_t, i32, vp, C.c_size_t, C.POINTER(C.c_size_t)]),
    "b2_tokenizer_decode": (i32, [vp, vp, C.c_size_t, i32, vp, C.c_size_t, C.POINTER(C.c_size_t)]),
    "b2_tokenizer_apply_chat_template": (i32, [vp, vp, vp, C.c_size_t, i32, vp, C.c_size_t,
                                               C.POINTER(C.c_size_t)]),
    "b2_tokenizer_token_to_id": (i32, [vp, C.c_char_p, C.c_size_t, C.POINTER(i32)]),
    "b2_tokenizer_get_info": (i32, [vp, C.POINTER(TokenizerInfo)]),
})


def exported_symbols():
    return list(_SIGS)


def lib():
    """Load the library (raises if it was not built)."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `make -C serving-engine_b200` (or __graft_entry__.build())")
        if "B2_NCCL_LIB" not in os.environ:
            # prefer the NCCL that torch ships, so both bind the same libnccl.so.2
            try:
                import importlib.util
                spec = importlib.util.find_spec("nvidia.nccl")
                for base in (spec.submodule_search_locations or []) if spec else []:
                    cand = os.path.join(base, "lib", "libnccl.so.2")
                    if os.path.exists(cand):
                        os.environ["B2_NCCL_LIB"] = cand
                        break
            except Exception:
                pass
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = L
    return _LIB


def status_string(s: int) -> str:
    return lib().b2_status_string(s).decode()


def device_status(clear: bool = True) -> int:
    """Synchronise the device; 0, or B2_ERR_TIMEOUT (-6) if a bounded wait of a
    tensor-core kernel gave up since the last clear."""
    return lib().b2_device_status(1 if clear else 0)


def call(name: str, *args) -> None:
    rc = getattr(lib(), name)(*args)
    if rc != 0:
        raise B2Error(name, rc)


def ptr(t) -> int | None:
    """Device pointer of a torch tensor (or None)."""
    return None if t is None else t.data_ptr()


def stream_ptr(stream=None) -> int | None:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream


# ---------------------------------------------------------------------------
# operator API (torch tensors in, torch tensors out; all compute in the library)
# ---------------------------------------------------------------------------

def gemv(W, x, y, epi=None, extra=None, stream=None):
    N, K = W.shape
    if epi is None:
        call("b2_gemv", ptr(W), ptr(x), ptr(y), N, K, stream_ptr(stream))
    elif epi == "bias":
        call("b2_gemv_bias", ptr(W), ptr(x), ptr(extra), ptr(y), N, K, stream_ptr(stream))
    elif epi == "residual":
        call("b2_gemv_residual", ptr(W), ptr(x), ptr(extra), ptr(y), N, K, stream_ptr(stream))
    else:
        raise ValueError(epi)


def gemv_batched(W, x, y, epilogue=0, extra=None, out_f32=False, stream=None):
    N, K = W.shape
    B = x.shape[0]
    call("b2_gemv_batched", ptr(W), ptr(x), ptr(extra), ptr(y), B, N, K, epilogue, int(out_f32), stream_ptr(stream))


def decode_gqa_split(q, kview: KVView, vview: KVView, seq_lens, out, B, nq, nkv, D, max_seq_len,
                     split_buffer=None, stream=None):
    cap = 0 if split_buffer is None else split_buffer.numel()
    call("b2_decode_gqa_split", ptr(q), kview, vview, ptr(seq_lens), ptr(out), B, nq, nkv, D, max_seq_len,
         ptr(split_buffer), cap, stream_ptr(stream))


class Sampler:
    """engine::SamplerGPU through the C-ABI."""

    def __init__(self, vocab: int, max_top_k: int = 1024):
        h = vp()
        call("b2_sampler_create", vocab, max_top_k, C.byref(h))
        self.h = h

    def sample(self, d_logits, history=(), temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0, seed=42,
               stream=None) -> int:
        import numpy as np
        hist = np.ascontiguousarray(np.asarray(history, dtype=np.int64))
        cfg = SamplerConfig(temperature, top_k, top_p, repetition_penalty, seed)
        tok = i32()
        call("b2_sampler_sample", self.h, ptr(d_logits), hist.ctypes.data if hist.size else None, hist.size,
             C.byref(cfg), stream_ptr(stream), C.byref(tok))
        return tok.value

    def sample_async(self, d_logits, d_history, history_len, d_token, temperature=0.0, top_k=0, top_p=1.0,
                     repetition_penalty=1.0, seed=42, stream=None) -> None:
        """Enqueue a draw: device history (int64), chosen id into d_token
        (device int32); no host round trip."""
        cfg = SamplerConfig(temperature, top_k, top_p, repetition_penalty, seed)
        call("b2_sampler_sample_async", self.h, ptr(d_logits), ptr(d_history) if history_len else None, history_len,
             C.byref(cfg), stream_ptr(stream), ptr(d_token))

    @property
    def rng_state(self) -> int:
        return int(lib().b2_sampler_rng_state(self.h))

    def close(self):
        if self.h:
            lib().b2_sampler_destroy(self.h)
            self.h = None

    __del__ = close


class Tokenizer:
    """engine::BPETokenizer through the C-ABI (b2_tokenizer_*): a byte-level
    BPE tokenizer read from a HF tokenizer.json (Qwen2, Llama-3 or GPT-2
    vocabularies)."""

    SPLIT_SPECIAL = 1
    ADD_SPECIAL = 2

    def __init__(self, path: str | None = None, json_text: str | bytes | None = None):
        h = vp()
        if path is not None:
            call("b2_tokenizer_load", os.fsencode(path), C.byref(h))
        else:
            data = json_text.encode() if isinstance(json_text, str) else json_text
            call("b2_tokenizer_load_json", data, len(data), C.byref(h))
        self.h = h
        info = TokenizerInfo()
        call("b2_tokenizer_get_info", self.h, C.byref(info))
        self.info = info
        self.stop_ids = [info.stop_ids[i] for i in range(info.n_stop)]

    def encode(self, text: str | bytes, split_special: bool = True, add_special: bool = False) -> list:
        """ids of `text`.  split_special: special added tokens written in the
        text become their ids (otherwise they are read as text);
        add_special: apply the file's post-processor (Llama-3's BOS)."""
        import numpy as np
        data = text.encode("utf-8") if isinstance(text, str) else bytes(text)
        flags = (self.SPLIT_SPECIAL if split_special else 0) | (self.ADD_SPECIAL if add_special else 0)
        n = C.c_size_t(0)
        buf = np.empty(len(data) + 8, np.int32)
        rc = lib().b2_tokenizer_encode(self.h, data, len(data), flags, buf.ctypes.data, buf.size, C.byref(n))
        if rc == -3:
            buf = np.empty(n.value, np.int32)
            rc = lib().b2_tokenizer_encode(self.h, data, len(data), flags, buf.ctypes.data, buf.size, C.byref(n))
        if rc != 0:
            raise B2Error("b2_tokenizer_encode", rc)
        return buf[: n.value].tolist()

    def decode_bytes(self, ids, skip_special: bool = False) -> bytes:
        import numpy as np
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int32).reshape(-1))
        n = C.c_size_t(0)
        out = C.create_string_buffer(max(16, 8 * a.size))
        rc = lib().b2_tokenizer_decode(self.h, a.ctypes.data, a.size, int(skip_special), out, len(out), C.byref(n))
        if rc == -3:
            out = C.create_string_buffer(n.value)
            rc = lib().b2_tokenizer_decode(self.h, a.ctypes.data, a.size, int(skip_special), out, len(out),
                                           C.byref(n))
        if rc != 0:
            raise B2Error("b2_tokenizer_decode", rc)
        return out.raw[: n.value]

    def decode(self, ids, skip_special: bool = False) -> str:
        """Text of `ids`; bytes that do not form UTF-8 become U+FFFD (as the
        HF library's decode does)."""
        return self.decode_bytes(ids, skip_special).decode("utf-8", errors="replace")

    def apply_chat_template(self, messages, add_generation_prompt: bool = True) -> str:
        """messages: (role, content) pairs or {"role", "content"} dicts."""
        pairs = [(m["role"], m["content"]) if isinstance(m, dict) else tuple(m) for m in messages]
        roles = (C.c_char_p * max(1, len(pairs)))(*[r.encode() for r, _ in pairs])
        contents = (C.c_char_p * max(1, len(pairs)))(*[c.encode() for _, c in pairs])
        n = C.c_size_t(0)
        cap = 256 + sum(len(r.encode()) + len(c.encode()) + 64 for r, c in pairs)
        out = C.create_string_buffer(cap)
        call("b2_tokenizer_apply_chat_template", self.h, C.cast(roles, vp), C.cast(contents, vp), len(pairs),
             int(add_generation_prompt), out, len(out), C.byref(n))
        return out.raw[: n.value].decode("utf-8", errors="replace")

    def token_to_id(self, token: str) -> int | None:
        b = token.encode()
        v = i32(-1)
        return v.value if lib().b2_tokenizer_token_to_id(self.h, b, len(b), C.byref(v)) == 0 else None

    def close(self):
        if getattr(self, "h", None):
            lib().b2_tokenizer_destroy(self.h)
            self.h = None

    __del__ = close


def nccl_unique_id() -> bytes:
    buf = (C.c_char * 128)()
    call("b2_nccl_unique_id", C.cast(buf, vp))
    return bytes(buf)


class Model:
    """A decode-path model shard (b2_model_*)."""

    def __init__(self, vocab, hidden, inter, layers, nq, nkv, head_dim, eps=1e-5, theta=10000.0, tied=False,
                 bias=False, max_batch=1, max_seq=4096, tp_rank=0, tp_size=1, nccl_id: bytes | None = None,
                 kv_blocks: int = 0, block_size: int = 16):
        """kv_blocks > 0 makes the KV cache a paged pool of kv_blocks blocks
        of block_size positions (b2_model_create_paged)."""
        self.cfg = ModelConfig(vocab, hidden, inter, layers, nq, nkv, head_dim, eps, theta, int(tied), int(bias),
                               max_batch, max_seq)
        h = vp()
        idbuf = None
        if nccl_id is not None:
            idbuf = (C.c_char * 128).from_buffer_copy(nccl_id)
        nid = C.cast(idbuf, vp) if idbuf else None
        if kv_blocks > 0:
            call("b2_model_create_paged", C.byref(self.cfg), kv_blocks, block_size, tp_rank, tp_size, nid, C.byref(h))
        else:
            call("b2_model_create", C.byref(self.cfg), tp_rank, tp_size, nid, C.byref(h))
        self.h = h
        self.block_size = block_size if kv_blocks > 0 else 0
        self.vocab = vocab
        self._B = max_batch

    def init_random(self, seed: int, std: float = 0.02):
        call("b2_model_init_random", self.h, seed, std)

    def trace_step(self, batch: int):
        """One decode step with per-launch device timestamps: an array of
        (start_ns, end_ns) rows in launch order, relative to the first start."""
        import numpy as np
        n = self.step_launches(batch)
        buf = np.zeros(2 * n, np.uint64)
        got = i32(0)
        call("b2_model_trace_step", self.h, batch, buf.ctypes.data, n, C.byref(got))
        t = buf[: 2 * got.value].astype(np.int64).reshape(-1, 2)
        return t - t[0, 0]

    def p2p_handle(self) -> bytes:
        """64-byte CUDA IPC handle of this rank's tensor-parallel exchange buffer."""
        buf = C.create_string_buffer(64)
        call("b2_model_p2p_handle", self.h, buf)
        return buf.raw

    def p2p_open(self, handles) -> None:
        """Map every rank's exchange buffer (handles in rank order); the decode
        step then exchanges partial sums over NVLink instead of NCCL."""
        blob = C.create_string_buffer(b"".join(handles), 64 * len(handles))
        call("b2_model_p2p_open", self.h, blob)

    def set_tensor(self, name: str, arr16):
        import numpy as np
        a = np.ascontiguousarray(arr16, dtype=np.float16)
        rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (1, a.size)
        call("b2_model_set_tensor", self.h, name.encode(), a.ctypes.data, rows, cols)

    def set_tensor_bf16(self, name: str, bits):
        """Upload a bf16 tensor given as its raw 16-bit patterns (uint16);
        the library converts it to fp16 on the device."""
        import numpy as np
        a = np.ascontiguousarray(bits, dtype=np.uint16)
        rows, cols = (a.shape[0], a.shape[1]) if a.ndim == 2 else (1, a.size)
        call("b2_model_set_tensor_bf16", self.h, name.encode(), a.ctypes.data, rows, cols)

    def forward_logits(self, ids):
        """fp32 logits of every position of one sequence [S, vocab] (full
        forward through the batched prefill and an all-rows lm_head)."""
        import numpy as np
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1))
        out = np.empty((a.size, self.vocab), np.float32)
        call("b2_model_forward_logits", self.h, a.ctypes.data, a.size, out.ctypes.data)
        self._B = 1
        return out

    def reset(self):
        call("b2_model_reset", self.h)

    def set_sampling(self, temperature=0.0, top_k=0, top_p=1.0, seed=42):
        """Token choice of prefill, decode steps and the device loop
        (temperature 0: greedy); resets every sequence's LCG state."""
        cfg = SamplerConfig(temperature, top_k, top_p, 1.0, seed)
        call("b2_model_set_sampling", self.h, C.byref(cfg))

    WEIGHTS = {"fp16": 0, "fp8": 1, "int4": 2}

    def quantize_weights(self, fmt="fp8"):
        """Decode GEMVs on per-row FP8 (E4M3) copies of the weights ("fp8"),
        on 4-bit copies with a scale per 128 weights ("int4", batch 1-2), or
        back on the fp16 weights ("fp16")."""
        call("b2_model_quantize_weights", self.h, self.WEIGHTS[fmt])

    def prefill(self, ids, want_logits=True):
        import numpy as np
        a = np.ascontiguousarray(np.atleast_2d(np.asarray(ids, dtype=np.int64)))
        B, S = a.shape
        self._B = B
        out = np.empty((B, self.vocab), np.float32) if want_logits else None
        call("b2_model_prefill", self.h, a.ctypes.data, B, S, out.ctypes.data if out is not None else None)
        return out

    def decode_step(self, tokens, positions, want_logits=True, want_next=False, logits_out=None):
        """One decode step through b2_model_decode_step.  logits_out: an
        optional reusable host buffer for the fp32 logits [B, vocab] (a numpy
        array, or a CPU torch tensor; page-locked memory, e.g. a torch tensor
        made with pin_memory=True, is written by the copy engine directly)."""
        import numpy as np
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).reshape(-1))
        p = np.ascontiguousarray(np.asarray(positions, dtype=np.int32).reshape(-1))
        B = t.size
        self._B = B
        lg_ptr = None
        lg = None
        if logits_out is not None:
            if hasattr(logits_out, "data_ptr"):
                import torch
                if logits_out.dtype != torch.float32 or logits_out.device.type != "cpu":
                    raise ValueError("logits_out must be a float32 tensor in host memory")
                if not logits_out.is_contiguous() or logits_out.numel() < B * self.vocab:
                    raise ValueError(f"logits_out must be contiguous with at least {B * self.vocab} elements")
                lg_ptr = logits_out.data_ptr()
            else:
                if logits_out.dtype != np.float32 or not logits_out.flags["C_CONTIGUOUS"]:
                    raise ValueError("logits_out must be a C-contiguous float32 array")
                if logits_out.size < B * self.vocab:
                    raise ValueError(f"logits_out must hold at least {B * self.vocab} elements")
                lg_ptr = logits_out.ctypes.data
            lg = logits_out
        elif want_logits:
            lg = np.empty((B, self.vocab), np.float32)
            lg_ptr = lg.ctypes.data
        nx = np.empty(B, np.int64) if want_next else None
        call("b2_model_decode_step", self.h, t.ctypes.data, p.ctypes.data, B, lg_ptr,
             nx.ctypes.data if nx is not None else None)
        return lg, nx

    def prefill_paged(self, ids, block_table, skip_blocks=0, want_logits=False):
        """One sequence's prompt into its blocks; returns (first token, logits or None)."""
        import numpy as np
        a = np.ascontiguousarray(np.asarray(ids, dtype=np.int64).reshape(-1))
        bt = np.ascontiguousarray(np.asarray(block_table, dtype=np.int32).reshape(-1))
        lg = np.empty(self.vocab, np.float32) if want_logits else None
        nx = np.empty(1, np.int64)
        call("b2_model_prefill_paged", self.h, a.ctypes.data, a.size, bt.ctypes.data, bt.size, skip_blocks,
             lg.ctypes.data if lg is not None else None, nx.ctypes.data)
        self._B = 1
        return int(nx[0]), lg

    def decode_step_paged(self, tokens, seq_lens, block_tables, want_logits=False):
        """One step of len(tokens) sequences over the pool; block_tables is
        [batch, max_blocks] int32.  Returns (next ids, logits [batch, vocab] or None)."""
        import numpy as np
        t = np.ascontiguousarray(np.asarray(tokens, dtype=np.int64).reshape(-1))
        L = np.ascontiguousarray(np.asarray(seq_lens, dtype=np.int32).reshape(-1))
        bt = np.ascontiguousarray(np.atleast_2d(np.asarray(block_tables, dtype=np.int32)))
        B = t.size
        lg = np.empty((B, self.vocab), np.float32) if want_logits else None
        nx = np.empty(B, np.int64)
        call("b2_model_decode_step_paged", self.h, t.ctypes.data, L.ctypes.data, bt.ctypes.data, bt.shape[1], B,
             lg.ctypes.data if lg is not None else None, nx.ctypes.data)
        self._B = B
        return nx, lg

    def generate_greedy(self, steps: int, fetch=True):
        """Device-resident greedy loop continuing from the last prefill / step.
        fetch=True returns the ids [steps, batch] (synchronises); fetch=False
        only enqueues the steps on the model's stream."""
        import numpy as np
        if fetch:
            out = np.empty((steps, self._B), np.int64)
            call("b2_model_generate_greedy", self.h, steps, out.ctypes.data)
            return out
        call("b2_model_generate_greedy", self.h, steps, None)
        return None

    def generate_text(self, tokenizer: "Tokenizer", prompt: str | None = None, messages=None,
                      max_new_tokens: int = 32, chunk: int = 16):
        """Text in, text out for one sequence (the reference's generate path,
        apps/generate.cpp:858-940, for any vocabulary the tokenizer reads):
        the prompt -- or the chat messages through the vocabulary's chat
        template -- is encoded (with the file's post-processor, e.g. Llama-3's
        BOS, for a plain prompt), prefilled, and decoded on the device
        `chunk` steps at a time (greedy, or the draw set_sampling configured)
        until a stop id of the tokenizer appears or max_new_tokens are
        generated.  Returns (text, prompt_ids,
        new_ids): new_ids end with the stop id when one was produced; text is
        their decode without special tokens.  Needs max_batch >= 1 and
        len(prompt_ids) + max_new_tokens <= max_seq."""
        import numpy as np
        if messages is not None:
            ids = tokenizer.encode(tokenizer.apply_chat_template(messages, add_generation_prompt=True))
        else:
            ids = tokenizer.encode(prompt, add_special=True)
        self.prefill(np.asarray(ids, np.int64)[None, :], want_logits=False)
        stop = set(tokenizer.stop_ids)
        new = []
        while len(new) < max_new_tokens:
            got = self.generate_greedy(min(chunk, max_new_tokens - len(new)))[:, 0].tolist()
            hit = next((k for k, t in enumerate(got) if t in stop), None)
            new += got if hit is None else got[: hit + 1]
            if hit is not None:
                break
        return tokenizer.decode(new, skip_special=True), ids, new

    def sync(self):
        call("b2_model_sync", self.h)

    @property
    def stream(self) -> int:
        return lib().b2_model_stream(self.h)

    def buffer(self, name: str) -> int:
        return lib().b2_model_buffer(self.h, name.encode())

    def read(self, name: str, dtype, count: int, offset_elems: int = 0):
        import numpy as np
        out = np.empty(count, dtype)
        call("b2_model_read", self.h, name.encode(), out.ctypes.data, offset_elems * out.itemsize, out.nbytes)
        return out

    def kv_layout(self):
        v = [i64() for _ in range(5)]
        call("b2_model_kv_layout", self.h, *[C.byref(x) for x in v])
        return tuple(x.value for x in v)

    def step_bytes(self, batch: int, ctx: int) -> float:
        return float(lib().b2_model_step_bytes(self.h, batch, ctx))

    KERNELS = ("qkv", "attention", "o_proj", "gate_up", "down", "lm_head")

    def time_kernel(self, kind: str, batch: int, reps: int = 3) -> float:
        ms = f32()
        call("b2_model_time_kernel", self.h, self.KERNELS.index(kind), batch, reps, C.byref(ms))
        return float(ms.value)

    def kernel_bytes(self, kind: str, batch: int, ctx: int) -> float:
        return float(lib().b2_model_kernel_bytes(self.h, self.KERNELS.index(kind), batch, ctx))

    def step_launches(self, batch: int) -> int:
        return int(lib().b2_model_step_launches(self.h, batch))

    def close(self):
        if getattr(self, "h", None):
            lib().b2_model_destroy(self.h)
            self.h = None

    __del__ = close


# ---------------------------------------------------------------------------
# paged-KV model runner
# ---------------------------------------------------------------------------

class PagedRunner:
    """Model runner over a paged KV pool, with the contract of the reference
    engine's runner (docs/runner_interface.md:18-84): the scheduler owns
    block allocation and sequence bookkeeping; the runner never allocates or
    frees blocks and only

      prefill(seq)        runs the prompt, writes its K/V into the blocks of
                          seq.block_table.physical_block_ids (skipping the
                          first seq.num_cached_tokens // block_size blocks,
                          which are shared), returns the first token id;
      decode_step(seqs)   bumps seq.block_table.num_tokens by one for each
                          sequence (the new K/V row goes to position
                          num_tokens - 1), runs one step of the batch on
                          seq.last_token_id, returns the next ids;
      step(batch)         PREFILL (one sequence) or DECODE by batch.batch_type.

    Sequences are duck-typed: .prompt_ids, .block_table (.physical_block_ids,
    .num_tokens), .last_token_id, optional .num_cached_tokens; the runner
    sets .last_logits and .last_logit_margin (top-1 minus top-2).  The
    scheduler must have allocated a sequence's next block before a step that
    crosses into it, and never hand a block shared with another sequence to a
    decode write (both as in the contract)."""

    PREFILL, DECODE = "prefill", "decode"

    def __init__(self, model: Model):
        if not model.block_size:
            raise ValueError("PagedRunner needs a model created with kv_blocks > 0")
        self.m = model
        self.bs = model.block_size

    @staticmethod
    def _diag(seq, logits):
        import numpy as np
        seq.last_logits = logits
        top = np.partition(logits, -2)[-2:]
        seq.last_logit_margin = float(top[1] - top[0])

    def prefill(self, seq, allocator=None) -> int:
        bt = seq.block_table
        skip = getattr(seq, "num_cached_tokens", 0) // self.bs
        tok, lg = self.m.prefill_paged(seq.prompt_ids, bt.physical_block_ids, skip_blocks=skip, want_logits=True)
        self._diag(seq, lg)
        return tok

    def decode_step(self, seqs, allocator=None) -> list:
        import numpy as np
        for s in seqs:
            s.block_table.num_tokens += 1
        width = max(len(s.block_table.physical_block_ids) for s in seqs)
        tables = np.zeros((len(seqs), width), np.int32)
        for i, s in enumerate(seqs):
            ids = s.block_table.physical_block_ids
            tables[i, :len(ids)] = ids
        nx, lg = self.m.decode_step_paged([s.last_token_id for s in seqs],
                                          [s.block_table.num_tokens for s in seqs], tables, want_logits=True)
        for i, s in enumerate(seqs):
            self._diag(s, lg[i])
        return [int(x) for x in nx]

    def step(self, batch) -> list:
        if batch.batch_type == self.PREFILL:
            return [self.prefill(batch.sequences[0])]
        return self.decode_step(batch.sequences)
