"""numpy front end for the CPU checker (TEST INFRASTRUCTURE ONLY).

Loads ``oracle/liboracle.so`` (the C restatement of the reference engine's CPU
path, ``oracle/b2oracle.c``) and, when it was built, ``oracle/_ref/libref_cpu.so``
(the reference's own ``src/cpu`` + ``src/model/forward_cpu.cpp`` compiled from
its sources).  Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs
import this module; the product path never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from dataclasses import dataclass

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")
i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
I64 = C.c_int64


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        L = C.CDLL(path)
        L.ora_set_threads.argtypes = [C.c_int]
        L.ora_init_scale.argtypes = [C.c_double]
        L.ora_init_scale.restype = C.c_float
        L.ora_init_tensor.argtypes = [C.c_uint64, C.c_uint64, I64, I64, I64, I64, I64, C.c_float, u16p]
        L.ora_rmsnorm.argtypes = [f32p, f32p, f32p, I64, I64, C.c_float]
        L.ora_matmul_transB_blocked.argtypes = [f32p, f32p, f32p, I64, I64, I64]
        L.ora_matmul_transB_naive.argtypes = [f32p, f32p, f32p, I64, I64, I64]
        L.ora_apply_rope.argtypes = [f32p, f32p, I64, I64, I64, I64, I64, C.c_float]
        L.ora_rope_table.argtypes = [I64, I64, I64, C.c_float, f32p, f32p]
        L.ora_causal_gqa.argtypes = [f32p, f32p, f32p, f32p, I64, I64, I64, I64]
        L.ora_causal_gqa_rows.argtypes = [f32p, f32p, f32p, f32p, I64, I64, I64, I64, I64]
        L.ora_swiglu.argtypes = [f32p, f32p, f32p, I64]
        L.ora_softmax.argtypes = [f32p, f32p, I64, I64]
        L.ora_embedding_lookup.argtypes = [i64p, f32p, f32p, I64, I64]
        L.ora_decode_attention.argtypes = [f32p, f32p, f32p, I64, I64, I64, i32p, f32p, I64, I64, I64, I64]
        L.ora_forward.argtypes = [C.c_void_p, C.c_void_p, i64p, I64, I64, C.c_void_p, C.c_void_p]
        L.ora_forward.restype = C.c_int
        L.ora_argmax.argtypes = [f32p, I64]
        L.ora_argmax.restype = I64
        L.ora_repetition_penalty.argtypes = [f32p, I64, i64p, I64, C.c_float]
        L.ora_lcg_next.argtypes = [C.POINTER(C.c_uint64)]
        L.ora_lcg_next.restype = C.c_float
        L.ora_lcg_reseed.argtypes = [C.POINTER(C.c_uint64), C.c_uint64]
        L.ora_sample_topk_topp.argtypes = [f32p, I64, C.c_int, C.c_int, C.c_float, C.c_float, C.c_float]
        L.ora_sample_topk_topp.restype = I64
        L.ora_f16_to_f32_par.argtypes = [u16p, f32p, I64]
        L.ora_set_threads(os.cpu_count() or 1)
        _LIB = L
    return _LIB


def ref_lib():
    """The reference's own CPU path, or None when it was not built here."""
    global _REF
    if _REF is None:
        path = os.path.join(HERE, "_ref", "libref_cpu.so")
        if not os.path.exists(path):
            return None
        R = C.CDLL(path)
        R.ref_rmsnorm.argtypes = [f32p, f32p, f32p, I64, I64, C.c_float]
        R.ref_matmul_transB_blocked.argtypes = [f32p, f32p, f32p, I64, I64, I64]
        R.ref_matmul_transB_naive.argtypes = [f32p, f32p, f32p, I64, I64, I64]
        R.ref_apply_rope.argtypes = [f32p, f32p, I64, I64, I64, I64, I64, C.c_float]
        R.ref_causal_gqa.argtypes = [f32p, f32p, f32p, f32p, I64, I64, I64, I64]
        R.ref_swiglu.argtypes = [f32p, f32p, f32p, I64]
        R.ref_embedding_lookup.argtypes = [i64p, f32p, f32p, I64, I64]
        R.ref_forward_cpu.argtypes = [I64, I64, I64, I64, I64, I64, I64, C.c_float, C.c_float,
                                      f32p, f32p, C.c_void_p, i64p, I64, f32p]
        R.ref_forward_cpu.restype = C.c_int
        R.ref_model_create.argtypes = [I64, I64, I64, I64, I64, I64, I64, C.c_float, C.c_float, f32p, f32p,
                                       C.c_void_p]
        R.ref_model_create.restype = C.c_void_p
        R.ref_model_forward.argtypes = [C.c_void_p, i64p, I64, C.c_void_p]
        R.ref_model_forward.restype = C.c_int
        R.ref_model_destroy.argtypes = [C.c_void_p]
        _REF = R
    return _REF


def set_threads(n: int) -> None:
    lib().ora_set_threads(int(n))


# --------------------------------------------------------------------------
# fp16 + seeded weights
# --------------------------------------------------------------------------

def f16(x) -> np.ndarray:
    """Round to fp16 and back to fp32 (the values the device sees)."""
    return np.asarray(x, np.float32).astype(np.float16).astype(np.float32)


def init_scale(std: float) -> float:
    return float(lib().ora_init_scale(std))


def init_tensor(seed: int, tensor_id: int, rows: int, cols: int, std: float,
                row_offset: int = 0, col_offset: int = 0, ld_global: int | None = None) -> np.ndarray:
    """fp16 block of the seeded tensor, bit-identical to the device generator."""
    out = np.empty((rows, cols), np.uint16)
    lib().ora_init_tensor(seed, tensor_id, rows, cols, row_offset, col_offset,
                          cols if ld_global is None else ld_global, init_scale(std), out)
    return out.view(np.float16)


def widen(h16: np.ndarray) -> np.ndarray:
    """fp16 array -> fp32 (multithreaded)."""
    h = np.ascontiguousarray(h16).view(np.uint16)
    out = np.empty(h.shape, np.float32)
    lib().ora_f16_to_f32_par(h.reshape(-1), out.reshape(-1), h.size)
    return out


# --------------------------------------------------------------------------
# ops (float32 numpy in / out)
# --------------------------------------------------------------------------

def _c(a, dt=np.float32):
    return np.ascontiguousarray(a, dtype=dt)


def rmsnorm(x, w, eps, ref=False):
    x = _c(x); w = _c(w)
    rows, dim = x.reshape(-1, x.shape[-1]).shape
    out = np.empty_like(x)
    (ref_lib().ref_rmsnorm if ref else lib().ora_rmsnorm)(x, w, out, rows, dim, eps)
    return out


def matmul_transB(A, B, ref=False, naive=False):
    A = _c(A); B = _c(B)
    M, K = A.shape
    N = B.shape[0]
    out = np.empty((M, N), np.float32)
    if ref:
        fn = ref_lib().ref_matmul_transB_naive if naive else ref_lib().ref_matmul_transB_blocked
    else:
        fn = lib().ora_matmul_transB_naive if naive else lib().ora_matmul_transB_blocked
    fn(A, B, out, M, K, N)
    return out


def apply_rope(q, k, S, nq, nkv, D, start_pos, theta, ref=False):
    q = _c(q).copy(); k = _c(k).copy()
    (ref_lib().ref_apply_rope if ref else lib().ora_apply_rope)(q, k, S, nq, nkv, D, start_pos, theta)
    return q, k


def rope_table(pos0, npos, D, theta):
    c = np.empty((npos, D // 2), np.float32)
    s = np.empty((npos, D // 2), np.float32)
    lib().ora_rope_table(pos0, npos, D, theta, c, s)
    return c, s


def causal_gqa(q, k, v, S, nq, nkv, D, ref=False):
    q = _c(q); k = _c(k); v = _c(v)
    out = np.zeros((S, nq * D), np.float32)
    (ref_lib().ref_causal_gqa if ref else lib().ora_causal_gqa)(q, k, v, out, S, nq, nkv, D)
    return out


def causal_gqa_rows(q, k, v, S, nq, nkv, D, q_begin):
    """causal_gqa's output rows [q_begin, S) only (rows are independent)."""
    q = _c(q); k = _c(k); v = _c(v)
    out = np.zeros((S, nq * D), np.float32)
    lib().ora_causal_gqa_rows(q, k, v, out, S, nq, nkv, D, q_begin)
    return out[q_begin:]


def swiglu(g, u, ref=False):
    g = _c(g); u = _c(u)
    out = np.empty_like(g)
    (ref_lib().ref_swiglu if ref else lib().ora_swiglu)(g, u, out, g.size)
    return out


def softmax(x):
    x = _c(x)
    out = np.empty_like(x)
    rows, cols = x.reshape(-1, x.shape[-1]).shape
    lib().ora_softmax(x, out, rows, cols)
    return out


def embedding_lookup(ids, table, ref=False):
    ids = _c(ids, np.int64); table = _c(table)
    out = np.empty((ids.size, table.shape[1]), np.float32)
    (ref_lib().ref_embedding_lookup if ref else lib().ora_embedding_lookup)(ids, table, out, ids.size, table.shape[1])
    return out


def decode_attention(q, k, v, strides, seq_lens, B, nq, nkv, D):
    """q [B,nq,D]; k/v flat float32 arrays addressed by element strides (b,h,s)."""
    q = _c(q); k = _c(k); v = _c(v)
    out = np.zeros((B, nq, D), np.float32)
    sb, sh, ss = strides
    lib().ora_decode_attention(q, k, v, sb, sh, ss, _c(seq_lens, np.int32), out, B, nq, nkv, D)
    return out


# --------------------------------------------------------------------------
# model
# --------------------------------------------------------------------------

@dataclass
class Config:
    vocab: int
    hidden: int
    inter: int
    layers: int
    nq: int
    nkv: int
    head_dim: int
    eps: float = 1e-5
    theta: float = 10000.0
    tied: bool = False
    has_bias: bool = False

    @property
    def qkv_rows(self):
        return (self.nq + 2 * self.nkv) * self.head_dim


class _OraConfig(C.Structure):
    _fields_ = [("vocab", I64), ("hidden", I64), ("inter", I64), ("layers", I64), ("nq", I64),
                ("nkv", I64), ("head_dim", I64), ("eps", C.c_float), ("theta", C.c_float),
                ("tied", C.c_int), ("has_bias", C.c_int)]


_LAYER_FIELDS = ["ln1", "ln2", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "wg", "wu", "wd"]


class _OraLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LAYER_FIELDS]


class _OraWeights(C.Structure):
    _fields_ = [("embed", C.c_void_p), ("final_norm", C.c_void_p), ("lm_head", C.c_void_p),
                ("layers", C.c_void_p)]


# Tensor ids of the seeded generator (shared with the device init kernel).
T_EMBED, T_LM_HEAD, T_FINAL_NORM = 1, 2, 3
LAYER_TID = {"wq": 0, "wk": 1, "wv": 2, "wo": 3, "wg": 4, "wu": 5, "wd": 6, "ln1": 7, "ln2": 8,
             "bq": 9, "bk": 10, "bv": 11}


def layer_tensor_id(layer: int, name: str) -> int:
    return 16 + 16 * layer + LAYER_TID[name]


def seeded_weights(cfg: Config, seed: int, std: float = 0.02) -> dict:
    """fp16 weights of the seeded model (float32 arrays holding fp16 values).
    Norm weights are 1.0; biases (when present) use the generator."""
    H, D, I, V = cfg.hidden, cfg.head_dim, cfg.inter, cfg.vocab
    qd, kvd = cfg.nq * D, cfg.nkv * D
    w = {"embed": widen(init_tensor(seed, T_EMBED, V, H, std)),
         "final_norm": np.ones(H, np.float32), "layers": []}
    if not cfg.tied:
        w["lm_head"] = widen(init_tensor(seed, T_LM_HEAD, V, H, std))
    shapes = {"wq": (qd, H), "wk": (kvd, H), "wv": (kvd, H), "wo": (H, qd), "wg": (I, H),
              "wu": (I, H), "wd": (H, I), "bq": (1, qd), "bk": (1, kvd), "bv": (1, kvd)}
    for l in range(cfg.layers):
        L = {"ln1": np.ones(H, np.float32), "ln2": np.ones(H, np.float32)}
        for n, (r, c) in shapes.items():
            if n.startswith("b"):
                L[n] = (widen(init_tensor(seed, layer_tensor_id(l, n), r, c, std)).reshape(-1)
                        if cfg.has_bias else np.zeros(c, np.float32))
            else:
                L[n] = widen(init_tensor(seed, layer_tensor_id(l, n), r, c, std))
        w["layers"].append(L)
    return w


def forward(cfg: Config, w: dict, ids, logit_row0: int = 0, want_final_norm: bool = False):
    """Full-recompute forward (restatement).  Returns logits [S - logit_row0, V]
    (and the final-norm hidden states [S, H] when asked)."""
    ids = _c(ids, np.int64)
    S = ids.size
    keep = []

    def p(a):
        a = _c(a)
        keep.append(a)
        return a.ctypes.data

    layers = (_OraLayer * cfg.layers)()
    for l, L in enumerate(w["layers"]):
        for n in _LAYER_FIELDS:
            setattr(layers[l], n, p(L[n]))
    W = _OraWeights(p(w["embed"]), p(w["final_norm"]), p(w["lm_head"]) if not cfg.tied else None,
                    C.cast(layers, C.c_void_p))
    oc = _OraConfig(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim,
                    cfg.eps, cfg.theta, int(cfg.tied), int(cfg.has_bias))
    logits = np.empty((S - logit_row0, cfg.vocab), np.float32)
    fn = np.empty((S, cfg.hidden), np.float32) if want_final_norm else None
    rc = lib().ora_forward(C.byref(oc), C.byref(W), ids, S, logit_row0,
                           logits.ctypes.data if S > logit_row0 else None,
                           fn.ctypes.data if fn is not None else None)
    if rc != 0:
        raise RuntimeError(f"ora_forward failed: {rc}")
    return (logits, fn) if want_final_norm else logits


class _RefLayer(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in _LAYER_FIELDS]


def ref_forward(cfg: Config, w: dict, ids):
    """The reference's own engine::forward_cpu (tied lm_head only)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("oracle/_ref/libref_cpu.so not built")
    assert cfg.tied, "the reference forward_cpu always ties lm_head to the embedding"
    ids = _c(ids, np.int64)
    keep = []

    def p(a):
        a = _c(a)
        keep.append(a)
        return a.ctypes.data

    layers = (_RefLayer * cfg.layers)()
    for l, L in enumerate(w["layers"]):
        for n in _LAYER_FIELDS:
            setattr(layers[l], n, p(L[n]))
    out = np.empty((ids.size, cfg.vocab), np.float32)
    rc = R.ref_forward_cpu(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim,
                           cfg.eps, cfg.theta, _c(w["embed"]), _c(w["final_norm"]),
                           C.cast(layers, C.c_void_p), ids, ids.size, out)
    if rc != 0:
        raise RuntimeError(f"ref_forward_cpu failed: {rc}")
    return out


# --------------------------------------------------------------------------
# sampler
# --------------------------------------------------------------------------

def argmax(logits) -> int:
    return int(lib().ora_argmax(_c(logits), np.asarray(logits).size))


def repetition_penalty(logits, history, penalty):
    lg = _c(logits).copy()
    h = _c(history, np.int64)
    lib().ora_repetition_penalty(lg, lg.size, h, h.size, penalty)
    return lg


class LCG:
    """Host LCG of the reference sampler (sampler.cu:186-200, 321-328)."""

    def __init__(self, state: int = 13374269):
        self.state = C.c_uint64(state)

    def reseed(self, seed: int):
        lib().ora_lcg_reseed(C.byref(self.state), seed)

    def next(self) -> float:
        return float(lib().ora_lcg_next(C.byref(self.state)))


def sample_topk_topp(logits, top_k, max_top_k, temperature, top_p, u) -> int:
    lg = _c(logits)
    return int(lib().ora_sample_topk_topp(lg, lg.size, top_k, max_top_k, temperature, top_p, u))


class Sampler:
    """SamplerGPU::sample semantics (sampler.cu:202-339) on the host."""

    def __init__(self, vocab: int, max_top_k: int = 1024):
        self.vocab, self.max_top_k = vocab, max_top_k
        self.lcg = LCG()

    def sample(self, logits, history, temperature=0.0, top_k=0, top_p=1.0, repetition_penalty=1.0, seed=42):
        lg = _c(logits)
        if repetition_penalty != 1.0 and len(history):
            lg = self.__class__._pen(lg, history, repetition_penalty)
        if temperature <= 1e-6:
            return argmax(lg)
        self.lcg.reseed(seed)
        u = self.lcg.next()
        return sample_topk_topp(lg, top_k, self.max_top_k, temperature, top_p, u)

    @staticmethod
    def _pen(lg, history, penalty):
        return repetition_penalty(lg, history, penalty)


class RefModel:
    """The reference's forward_cpu on weights converted once (for timing)."""

    def __init__(self, cfg: Config, w: dict):
        R = ref_lib()
        if R is None:
            raise RuntimeError("oracle/_ref/libref_cpu.so not built")
        assert cfg.tied
        self.cfg = cfg
        keep = []

        def p(a):
            a = _c(a)
            keep.append(a)
            return a.ctypes.data

        layers = (_RefLayer * max(cfg.layers, 1))()
        for l, L in enumerate(w["layers"]):
            for n in _LAYER_FIELDS:
                setattr(layers[l], n, p(L[n]))
        self.h = R.ref_model_create(cfg.vocab, cfg.hidden, cfg.inter, cfg.layers, cfg.nq, cfg.nkv, cfg.head_dim,
                                    cfg.eps, cfg.theta, _c(w["embed"]), _c(w["final_norm"]),
                                    C.cast(layers, C.c_void_p))

    def forward(self, ids, want_logits=False):
        ids = _c(ids, np.int64)
        out = np.empty((ids.size, self.cfg.vocab), np.float32) if want_logits else None
        ref_lib().ref_model_forward(self.h, ids, ids.size, out.ctypes.data if out is not None else None)
        return out

    def close(self):
        if getattr(self, "h", None):
            ref_lib().ref_model_destroy(self.h)
            self.h = None

    __del__ = close


# ---------------------------------------------------------------------------
# FP8 E4M3 weights (the quantised decode path).  The reference has no
# quantised path (its RESULTS.md:39-40 plans INT8/INT4 weights and FP8/INT8
# KV); this restates the OCP 8-bit floating-point format's E4M3 encoding
# (exponent bias 7, 3 mantissa bits, no infinities, largest finite 448) with
# round-to-nearest-even and saturation, and the per-row scaling that
# b2_quantize_fp8_rows documents: scale = max|w| / 448 (1 for a zero row),
# q = E4M3(w / scale) in float32 arithmetic.
# ---------------------------------------------------------------------------

def _e4m3_positive_values() -> np.ndarray:
    codes = np.arange(127)  # finite non-negative codes 0x00 .. 0x7e
    e, m = codes >> 3, codes & 7
    return np.where(e == 0, m / 8.0 * 2.0 ** -6, (1.0 + m / 8.0) * 2.0 ** (e - 7.0)).astype(np.float64)


_E4M3 = _e4m3_positive_values()


def e4m3_encode(x) -> np.ndarray:
    """float32 values -> E4M3 codes (uint8): nearest, ties to the even code,
    magnitudes above 448 saturated, the sign kept (also for zero).  Below
    2^-6 the codes are the multiples of 2^-9; above, 3 mantissa bits per
    binade (np.rint rounds halves to even; the scalings are exact)."""
    x = np.asarray(x, np.float32)
    a = np.minimum(np.abs(x), np.float32(448.0))
    sub = a < np.float32(2.0 ** -6)
    f, ex = np.frexp(np.where(sub, np.float32(1.0), a))      # a = f * 2^ex, f in [0.5, 1)
    m = np.rint(f * np.float32(16.0) - np.float32(8.0))       # 3-bit mantissa, 8 = carry
    e = ex.astype(np.int32) - 1 + (m == 8)
    m = np.where(m == 8, 0, m).astype(np.int32)
    code = np.where(sub, np.rint(a * np.float32(2.0 ** 9)).astype(np.int32), ((e + 7) << 3) | m)
    code = np.minimum(code, 126)
    return (code.astype(np.uint8) | (np.signbit(x).astype(np.uint8) << 7)).astype(np.uint8)


def e4m3_decode(q) -> np.ndarray:
    q = np.asarray(q, np.uint8)
    v = _E4M3[np.minimum(q & 0x7F, 126)].astype(np.float32)
    return np.where(q & 0x80, -v, v).astype(np.float32)


def quantize_e4m3_rows(w):
    """Per-row E4M3 codes and float32 scales of a [rows, K] matrix (in
    blocks of rows, to bound the temporaries of large matrices)."""
    w = np.asarray(w, np.float32)
    amax = np.max(np.abs(w), axis=1)
    scale = np.where(amax > 0, amax / np.float32(448.0), np.float32(1.0)).astype(np.float32)
    q = np.empty(w.shape, np.uint8)
    step = max(1, (1 << 23) // max(1, w.shape[1]))
    for r0 in range(0, w.shape[0], step):
        q[r0:r0 + step] = e4m3_encode((w[r0:r0 + step] / scale[r0:r0 + step, None]).astype(np.float32))
    return q, scale


def dequantize_e4m3_rows(q, scale) -> np.ndarray:
    return (e4m3_decode(q) * np.asarray(scale, np.float32)[:, None]).astype(np.float32)


I4_GROUP = 128                                         # weights per scale
_I4_SHIFT = np.array([16 * (j & 1) + 4 * (j >> 1) for j in range(8)], np.uint32)


def quantize_int4_rows(w):
    """4-bit codes of a [rows, K] matrix in the library's packed layout
    (include/b2engine.h, b2_quantize_int4_rows) and float32 group scales
    [rows, K/128]: scale = max|w| / 7 over each group of 128 (float32
    division), q = rint(w / scale) in [-7, 7] (0 for an all-zero group),
    stored as q + 8, weight j of each 8-weight word at bit
    16*(j & 1) + 4*(j >> 1)."""
    w = np.asarray(w, np.float32)
    rows, K = w.shape
    assert K % I4_GROUP == 0
    g = w.reshape(rows, K // I4_GROUP, I4_GROUP)
    scale = (np.max(np.abs(g), axis=2) / np.float32(7.0)).astype(np.float32)
    safe = np.where(scale > 0, scale, np.float32(1.0)).astype(np.float32)
    q = np.where(scale[..., None] > 0, np.rint(g / safe[..., None]), np.float32(0.0))
    u = (np.clip(q, -7, 7).astype(np.int32) + 8).astype(np.uint32).reshape(rows, K // 8, 8)
    words = np.bitwise_or.reduce(u << _I4_SHIFT, axis=2).astype("<u4")
    return words.view(np.uint8).reshape(rows, K // 2), scale


def int4_codes(packed) -> np.ndarray:
    """Packed 4-bit weights [rows, K/2] -> the signed codes q [rows, K]."""
    packed = np.ascontiguousarray(packed, np.uint8)
    rows = packed.shape[0]
    words = packed.view("<u4").reshape(rows, -1, 1)
    u = (words >> _I4_SHIFT) & np.uint32(0xF)
    return u.reshape(rows, -1).astype(np.int32) - 8


def dequantize_int4_rows(packed, scale) -> np.ndarray:
    q = int4_codes(packed).astype(np.float32)
    rows, K = q.shape
    s = np.repeat(np.asarray(scale, np.float32), I4_GROUP, axis=1)
    return (q * s).astype(np.float32)


def int4_weights(w: dict) -> dict:
    """The seeded weights with every projection and the lm_head replaced by
    their 4-bit round trip, rounded to fp16 (the oracle's weight type)."""
    out = dict(w)
    out["layers"] = []
    for L in w["layers"]:
        M = dict(L)
        for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            M[n] = f16(dequantize_int4_rows(*quantize_int4_rows(L[n])))
        out["layers"].append(M)
    if "lm_head" in w:
        out["lm_head"] = f16(dequantize_int4_rows(*quantize_int4_rows(w["lm_head"])))
    return out


def fp8_weights(w: dict) -> dict:
    """The seeded weights with every projection and the lm_head replaced by
    their per-row E4M3 round trip, rounded to fp16 (the oracle's weight
    type): what a model quantised with b2_model_quantize_weights decodes
    with, up to that fp16 rounding."""
    out = dict(w)
    out["layers"] = []
    for L in w["layers"]:
        M = dict(L)
        for n in ("wq", "wk", "wv", "wo", "wg", "wu", "wd"):
            M[n] = f16(dequantize_e4m3_rows(*quantize_e4m3_rows(L[n])))
        out["layers"].append(M)
    if "lm_head" in w:
        out["lm_head"] = f16(dequantize_e4m3_rows(*quantize_e4m3_rows(w["lm_head"])))
    return out
