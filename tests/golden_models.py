"""Seeded synthetic Llama-style weights shared by the oracle and CUDA tests.

Weights follow the bench's synthetic-data rule: linear weights N(0, 0.02)
quantized to a GGUF block format by the fixture quantizer (the reference ships
no GGUF quantizer), embeddings f16 N(0, 1), norm weights f16 near 1.0. Every
tensor has its own generator seeded from (seed, layer, slot), so any one tensor
can be regenerated alone.
"""
from __future__ import annotations

import numpy as np

import oracle as orc

LINEAR_SLOTS = (orc.W_Q, orc.W_K, orc.W_V, orc.W_O, orc.W_GATE, orc.W_UP, orc.W_DOWN)


def shape_of(cfg, which: int):
    H, F, V = cfg.hidden_size, cfg.intermediate_size, cfg.vocab_size
    QD, KD = cfg.num_heads * cfg.head_dim, cfg.num_kv_heads * cfg.head_dim
    return {
        orc.W_EMBED: (V, H), orc.W_LM_HEAD: (V, H), orc.W_FINAL_NORM: (H,),
        orc.W_ATTN_NORM: (H,), orc.W_FFN_NORM: (H,),
        orc.W_Q: (QD, H), orc.W_K: (KD, H), orc.W_V: (KD, H), orc.W_O: (H, QD),
        orc.W_GATE: (F, H), orc.W_UP: (F, H), orc.W_DOWN: (H, F),
    }[which]


def _rng(seed: int, layer: int, which: int) -> np.random.Generator:
    return np.random.default_rng([seed, layer + 1, which])


def make_tensor(cfg, layer: int, which: int, dtype: int, seed: int,
                nibble_order: int = orc.NIBBLE_REF_INTERLEAVED):
    """Returns (bytes-or-array, dtype) for one weight slot."""
    shape = shape_of(cfg, which)
    g = _rng(seed, layer, which)
    if which in (orc.W_FINAL_NORM, orc.W_ATTN_NORM, orc.W_FFN_NORM):
        return (1.0 + 0.1 * g.standard_normal(shape)).astype(np.float16), orc.F16
    if which == orc.W_EMBED:
        return g.standard_normal(shape).astype(np.float16), orc.F16
    w = (g.standard_normal(shape, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return orc.quantize(w, dtype, nibble_order), dtype


def make_weights(cfg, dtype: int, seed: int = 0, lm_head_dtype: int | None = None,
                 nibble_order: int = orc.NIBBLE_REF_INTERLEAVED):
    """All tensors of a model: {(layer, slot): (data, dtype)}; layer -1 = global."""
    out = {}
    for which in (orc.W_EMBED, orc.W_FINAL_NORM):
        out[(-1, which)] = make_tensor(cfg, -1, which, dtype, seed, nibble_order)
    out[(-1, orc.W_LM_HEAD)] = make_tensor(cfg, -1, orc.W_LM_HEAD,
                                           lm_head_dtype or dtype, seed, nibble_order)
    for layer in range(cfg.num_layers):
        for which in (orc.W_ATTN_NORM, orc.W_FFN_NORM) + LINEAR_SLOTS:
            out[(layer, which)] = make_tensor(cfg, layer, which, dtype, seed, nibble_order)
    return out


def build_oracle_model(cfg, weights, nibble_order: int = orc.NIBBLE_REF_INTERLEAVED):
    m = orc.OracleModel(cfg)
    for (layer, which), (data, dt) in weights.items():
        m.set_weight(max(layer, 0), which, data, dt, nibble_order)
    return m
