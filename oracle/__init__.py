"""CPU oracle for the quantized decode path -- TEST INFRASTRUCTURE ONLY.

This package is the parity checker: a C++ restatement (oracle.cpp) of the
reference's CPU path (crates/beacon-format/src/dequant.rs,
crates/beacon-kernels/src/ops.rs, crates/beacon-core/src/cpu_backend.rs and
engine.rs, crates/beacon-scheduler/src/sampling.rs), loaded through ctypes.
Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import it. The CUDA product never does.

Parity is pinned by replaying the reference's own known-answer tests
(tests/test_oracle_kat.py). Q4_K has no known-answer test in the reference;
its restatement follows dequant.rs:289-365 line by line.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "liboracle.so")

# dtype tags (crates/beacon-format/src/dtype.rs:12-29)
F32, F16, BF16, I32, I8 = 0, 1, 2, 3, 4
Q4_0, Q4_K, Q5_K, Q6_K, Q8_0 = 100, 101, 102, 103, 104
Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q8_K = 105, 106, 107, 108, 109, 110
QUANTIZED = (Q4_0, Q4_K, Q5_K, Q6_K, Q8_0, Q4_1, Q5_0, Q5_1, Q2_K, Q3_K, Q8_K)

NIBBLE_REF_INTERLEAVED = 0
NIBBLE_GGUF_SPLIT = 1

W_EMBED, W_FINAL_NORM, W_LM_HEAD = 0, 1, 2
W_ATTN_NORM, W_Q, W_K, W_V, W_O = 10, 11, 12, 13, 14
W_FFN_NORM, W_GATE, W_UP, W_DOWN = 15, 16, 17, 18


def build() -> str:
    """Compile liboracle.so with the committed Makefile (g++, no GPU needed)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        c = ctypes
        P = c.c_void_p
        sig = {
            "orc_f16_to_f32": (c.c_float, [c.c_uint16]),
            "orc_f32_to_f16_rtz": (c.c_uint16, [c.c_float]),
            "orc_f32_to_f16_rne": (c.c_uint16, [c.c_float]),
            "orc_f32_to_f16_rtz_array": (None, [P, P, c.c_size_t]),
            "orc_f32_to_f16_rne_array": (None, [P, P, c.c_size_t]),
            "orc_block_size": (c.c_int64, [c.c_int]),
            "orc_block_bytes": (c.c_int64, [c.c_int]),
            "orc_dequantize_to_f16": (c.c_int, [P, c.c_int, c.c_uint64, c.c_int, P]),
            "orc_dequantize_to_f32": (c.c_int, [P, c.c_int, c.c_uint64, c.c_int, c.c_int, P]),
            "orc_quantize": (c.c_int, [P, c.c_int, c.c_uint64, c.c_int, P]),
            "orc_q4_dequantize_block": (None, [P, P]),
            "orc_q4_dot_f32": (c.c_float, [P, P, c.c_size_t]),
            "orc_q4_matmul_f32": (None, [P, P, P, c.c_size_t, c.c_size_t]),
            "orc_qgemv_f32": (c.c_int, [P, c.c_int, c.c_int, c.c_int, c.c_int64, c.c_int64,
                                        P, c.c_int64, P, c.c_int]),
            "orc_matmul_f32": (None, [P, P, P, c.c_size_t, c.c_size_t, c.c_size_t]),
            "orc_transpose_f32": (None, [P, P, c.c_size_t, c.c_size_t, c.c_size_t]),
            "orc_rms_norm": (None, [P, P, P, c.c_size_t, c.c_float]),
            "orc_silu_inplace": (None, [P, c.c_size_t]),
            "orc_softmax_inplace": (None, [P, c.c_size_t]),
            "orc_rope_inplace": (None, [P, c.c_size_t, c.c_size_t, c.c_size_t, c.c_float]),
            "orc_add": (None, [P, P, P, c.c_size_t]),
            "orc_mul": (None, [P, P, P, c.c_size_t]),
            "orc_attention": (c.c_int, [P, P, P, P, c.c_size_t, c.c_float, c.c_size_t, c.c_size_t,
                                        c.c_size_t, c.c_size_t, c.c_size_t, c.c_size_t, c.c_int, P]),
            "orc_argmax": (c.c_uint32, [P, c.c_size_t]),
            "orc_sample": (c.c_uint32, [P, c.c_size_t, P, c.c_size_t, P, c.c_float, P]),
            "orc_model_create": (P, [P]),
            "orc_model_set_weight": (c.c_int, [P, c.c_int, c.c_int, P, c.c_int, c.c_int]),
            "orc_model_forward": (c.c_int, [P, P, c.c_size_t, c.c_size_t, P]),
            "orc_model_reset": (None, [P]),
            "orc_model_destroy": (None, [P]),
            "orc_last_error": (c.c_char_p, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"], "oracle buffers must be C-contiguous"
    return a.ctypes.data


def _check(rc: int) -> None:
    if rc != 0:
        raise RuntimeError(lib().orc_last_error().decode())


def f32_to_f16_rtz_array(x: np.ndarray) -> np.ndarray:
    """Bit-preserving array form (signalling NaNs survive, unlike a Python float)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_rtz_array(_p(x), _p(out), x.size)
    return out


def f32_to_f16_rne_array(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_rne_array(_p(x), _p(out), x.size)
    return out


def block_size(dtype: int) -> int:
    return int(lib().orc_block_size(dtype))


def block_bytes(dtype: int) -> int:
    return int(lib().orc_block_bytes(dtype))


def row_bytes(dtype: int, k: int) -> int:
    return k // block_size(dtype) * block_bytes(dtype)


def f16_to_f32(bits: int) -> float:
    return float(lib().orc_f16_to_f32(bits))


def f32_to_f16_rtz(v: float) -> int:
    return int(lib().orc_f32_to_f16_rtz(v))


def f32_to_f16_rne(v: float) -> int:
    return int(lib().orc_f32_to_f16_rne(v))


def dequantize_to_f16(data: np.ndarray, dtype: int, n: int,
                      nibble_order: int = NIBBLE_REF_INTERLEAVED) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, dtype=np.uint16)
    _check(lib().orc_dequantize_to_f16(_p(data), dtype, n, nibble_order, _p(out)))
    return out


def dequantize_to_f32(data: np.ndarray, dtype: int, n: int,
                      nibble_order: int = NIBBLE_REF_INTERLEAVED, rtz: bool = False) -> np.ndarray:
    data = np.ascontiguousarray(data, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    _check(lib().orc_dequantize_to_f32(_p(data), dtype, n, nibble_order, int(rtz), _p(out)))
    return out


def quantize(x: np.ndarray, dtype: int, nibble_order: int = NIBBLE_REF_INTERLEAVED) -> np.ndarray:
    """Fixture quantizer: f32 values -> GGUF block bytes (row-major, blocks along K)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.size
    out = np.empty(n // block_size(dtype) * block_bytes(dtype), dtype=np.uint8)
    _check(lib().orc_quantize(_p(x), dtype, n, nibble_order, _p(out)))
    return out


def q4_dequantize_block(block: np.ndarray) -> np.ndarray:
    block = np.ascontiguousarray(block, dtype=np.uint8)
    out = np.empty(32, dtype=np.float32)
    lib().orc_q4_dequantize_block(_p(block), _p(out))
    return out


def q4_dot_f32(x: np.ndarray, w: np.ndarray) -> float:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    return float(lib().orc_q4_dot_f32(_p(x), _p(w), x.size))


def q4_matmul_f32(w: np.ndarray, x: np.ndarray, m: int) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.uint8)
    out = np.empty(m, dtype=np.float32)
    lib().orc_q4_matmul_f32(_p(w), _p(x), _p(out), m, x.size)
    return out


def qgemv(w: np.ndarray, dtype: int, n: int, k: int, x: np.ndarray,
          nibble_order: int = NIBBLE_REF_INTERLEAVED, rtz: bool = False,
          threads: int = 0) -> np.ndarray:
    """y[b, n] = sum_k deq(w)[n, k] * x[b, k], sequential f32 sum in ascending k."""
    w = np.ascontiguousarray(w, dtype=np.uint8)
    x2 = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    b = x2.shape[0]
    y = np.empty((b, n), dtype=np.float32)
    _check(lib().orc_qgemv_f32(_p(w), dtype, nibble_order, int(rtz), n, k, _p(x2), b, _p(y),
                               threads))
    return y


def matmul_f32(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    k2, n = b.shape
    assert k == k2
    c = np.empty((m, n), dtype=np.float32)
    lib().orc_matmul_f32(_p(a), _p(b), _p(c), m, k, n)
    return c


def transpose(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    m, n = x.shape[-2], x.shape[-1]
    batch = int(np.prod(x.shape[:-2])) if x.ndim > 2 else 1
    out = np.empty(x.shape[:-2] + (n, m), dtype=np.float32)
    lib().orc_transpose_f32(_p(x), _p(out), batch, m, n)
    return out


def rms_norm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """Per-row RMSNorm over the last dim (cpu_backend.rs:103-139)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    d = x.shape[-1]
    out = np.empty_like(x)
    xf, of = x.reshape(-1, d), out.reshape(-1, d)
    for r in range(xf.shape[0]):
        row = np.ascontiguousarray(xf[r])
        o = np.empty(d, dtype=np.float32)
        lib().orc_rms_norm(_p(row), _p(w), _p(o), d, eps)
        of[r] = o
    return out


def silu(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    lib().orc_silu_inplace(_p(y), y.size)
    return y


def softmax(x: np.ndarray) -> np.ndarray:
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    d = y.shape[-1]
    yf = y.reshape(-1, d)
    for r in range(yf.shape[0]):
        row = np.ascontiguousarray(yf[r])
        lib().orc_softmax_inplace(_p(row), d)
        yf[r] = row
    return y


def rope(x: np.ndarray, position_offset: int, theta: float, dim: int) -> np.ndarray:
    """RoPE over the last two dims, one group per leading index (cpu_backend.rs:141-180)."""
    y = np.array(x, dtype=np.float32, copy=True, order="C")
    seq_len = y.shape[-2] if y.ndim >= 2 else 1
    groups = y.size // (seq_len * dim)
    yf = y.reshape(groups, seq_len * dim)
    for g in range(groups):
        row = np.ascontiguousarray(yf[g])
        lib().orc_rope_inplace(_p(row), seq_len, dim, position_offset, theta)
        yf[g] = row
    return y


def add(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_add(_p(a), _p(b), _p(out), a.size)
    return out


def mul(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    out = np.empty_like(a)
    lib().orc_mul(_p(a), _p(b), _p(out), a.size)
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float,
              mask: np.ndarray | None = None, causal: bool = False) -> np.ndarray:
    q = np.ascontiguousarray(q, dtype=np.float32)
    k = np.ascontiguousarray(k, dtype=np.float32)
    v = np.ascontiguousarray(v, dtype=np.float32)
    b, nh, sq, hd = q.shape
    nkv, skv = k.shape[1], k.shape[2]
    out = np.empty_like(q)
    mp, mn = 0, 0
    if mask is not None:
        mask = np.ascontiguousarray(mask, dtype=np.float32)
        mp, mn = _p(mask), mask.size
    _check(lib().orc_attention(_p(q), _p(k), _p(v), mp, mn, scale, b, nh, sq, hd, nkv, skv,
                               int(causal), _p(out)))
    return out


def argmax(logits: np.ndarray) -> int:
    x = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_argmax(_p(x), x.size))


class SampleParams(ctypes.Structure):
    """GenerationParams' sampling fields (params.rs:6-31); has_* = Some(.)."""
    _fields_ = [("temperature", ctypes.c_float), ("has_top_k", ctypes.c_int32), ("top_k", ctypes.c_int32),
                ("has_top_p", ctypes.c_int32), ("top_p", ctypes.c_float), ("has_min_p", ctypes.c_int32),
                ("min_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float)]


def sample_params(temperature=0.0, top_k=None, top_p=None, min_p=None, repeat_penalty=1.0) -> SampleParams:
    return SampleParams(temperature, top_k is not None, top_k or 0, top_p is not None,
                        0.0 if top_p is None else top_p, min_p is not None, 0.0 if min_p is None else min_p,
                        repeat_penalty)


def sample(logits: np.ndarray, previous, params: SampleParams, r: float):
    """sampling::sample (sampling.rs:15-57) with the draw r given: (token, final distribution)."""
    x = np.ascontiguousarray(logits, dtype=np.float32)
    prev = np.ascontiguousarray(np.asarray(previous, dtype=np.uint32))
    probs = np.zeros(x.size, dtype=np.float32)
    tok = lib().orc_sample(_p(x), x.size, _p(prev) if prev.size else None, prev.size, ctypes.byref(params),
                           r, _p(probs))
    return int(tok), probs


class _Cfg(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "vocab_size", "hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim",
        "intermediate_size", "max_context")] + [
        ("rope_theta", ctypes.c_float), ("rms_norm_eps", ctypes.c_float),
        ("kv_persist", ctypes.c_int32), ("causal_prefill", ctypes.c_int32),
        ("weights_rtz", ctypes.c_int32), ("threads", ctypes.c_int32),
        ("ref_faithful", ctypes.c_int32)]


@dataclass
class OracleModelConfig:
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    max_context: int
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    kv_persist: bool = True
    causal_prefill: bool = True
    weights_rtz: bool = True
    threads: int = 0
    ref_faithful: bool = False   # the reference's transpose + column-strided matmul, one thread


class OracleModel:
    """engine.rs's forward pass over plain f32 weights (Engine::load_cpu path)."""

    def __init__(self, cfg: OracleModelConfig):
        self.cfg = cfg
        c = _Cfg(cfg.vocab_size, cfg.hidden_size, cfg.num_layers, cfg.num_heads,
                 cfg.num_kv_heads, cfg.head_dim, cfg.intermediate_size, cfg.max_context,
                 cfg.rope_theta, cfg.rms_norm_eps, int(cfg.kv_persist),
                 int(cfg.causal_prefill), int(cfg.weights_rtz), cfg.threads, int(cfg.ref_faithful))
        self._h = lib().orc_model_create(ctypes.byref(c))
        if not self._h:
            raise RuntimeError("orc_model_create failed")

    def set_weight(self, layer: int, which: int, data: np.ndarray, dtype: int,
                   nibble_order: int = NIBBLE_REF_INTERLEAVED) -> None:
        data = np.ascontiguousarray(data)
        _check(lib().orc_model_set_weight(self._h, layer, which, _p(data), dtype, nibble_order))

    def forward(self, tokens, position: int) -> np.ndarray:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        out = np.empty((toks.size, self.cfg.vocab_size), dtype=np.float32)
        _check(lib().orc_model_forward(self._h, _p(toks), toks.size, position, _p(out)))
        return out

    def reset(self) -> None:
        lib().orc_model_reset(self._h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            lib().orc_model_destroy(h)
            self._h = None
