"""Seeded synthetic decoder weights generated on the device.

The benchmark configs are random-weight models (no checkpoints): linear
weights N(0, 0.02) quantized to GGUF blocks by the device quantizer
(beacon_cuda_quantize_blocks), embeddings f16 N(0, 1), norm weights 1.0.
Generation runs on the GPU so 8B- and 70B-shape models build in seconds.
torch provides the random numbers and the device buffers only.
"""
from __future__ import annotations

import ctypes

from . import _lib as L
from .model import CudaModel

QUANT_BLOCK = {L.DTYPE_Q4_0: (32, 18), L.DTYPE_Q8_0: (32, 34), L.DTYPE_Q4_K: (256, 144)}


def _gen(seed: int, layer: int, slot: int):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed((seed * 1_000_003 + (layer + 1) * 101 + slot) & 0x7FFFFFFFFFFF)
    return g


def quantize_on_device(backend, stream, n: int, k: int, dtype: int, seed: int, layer: int, slot: int,
                       row_chunk: int = 8192, scale: float = 0.02):
    """N(0, scale) [n, k] -> GGUF blocks in a torch uint8 device buffer
    (blocks along K, rows in order: the raw GGUF tensor bytes)."""
    import torch
    bs, bb = QUANT_BLOCK[dtype]
    out = torch.empty(n * (k // bs) * bb, dtype=torch.uint8, device="cuda")
    g = _gen(seed, layer, slot)
    row_bytes = k // bs * bb
    for r0 in range(0, n, row_chunk):
        r = min(row_chunk, n - r0)
        x = torch.randn((r, k), generator=g, device="cuda", dtype=torch.float32).mul_(scale)
        torch.cuda.synchronize()
        L.check(L.lib().beacon_cuda_quantize_blocks(backend.ctx, stream.handle,
                                                    ctypes.c_void_p(x.data_ptr()), r, k, dtype,
                                                    L.NIBBLE_REF_INTERLEAVED,
                                                    ctypes.c_void_p(out.data_ptr() + r0 * row_bytes)))
        stream.synchronize()
        del x
    torch.cuda.synchronize()
    return out


def quantized_tensor_on_device(model: CudaModel, n: int, k: int, dtype: int, seed: int, layer: int, slot: int,
                               row_chunk: int = 8192):
    """N(0, 0.02) [n, k] -> GGUF blocks in a torch uint8 device buffer."""
    return quantize_on_device(model.backend, model.stream, n, k, dtype, seed, layer, slot, row_chunk)


def load_synthetic(model: CudaModel, dtype: int, seed: int = 0) -> None:
    """Fill every weight slot of `model` (full tensors; each TP rank keeps its shard)."""
    import torch
    c = model.cfg
    H, F, V = c.hidden_size, c.intermediate_size, c.vocab_size
    QD, KD = c.num_heads * c.head_dim, c.num_kv_heads * c.head_dim
    emb = torch.randn((V, H), generator=_gen(seed, -1, L.W_EMBED), device="cuda").to(torch.float16)
    torch.cuda.synchronize()
    model.set_weight(-1, L.W_EMBED, emb.data_ptr(), L.DTYPE_F16)
    del emb
    ones = torch.ones(H, dtype=torch.float16, device="cuda")
    torch.cuda.synchronize()
    model.set_weight(-1, L.W_FINAL_NORM, ones.data_ptr(), L.DTYPE_F16)
    lm = quantized_tensor_on_device(model, V, H, dtype, seed, -1, L.W_LM_HEAD)
    model.set_weight(-1, L.W_LM_HEAD, lm.data_ptr(), dtype)
    del lm
    shapes = {L.W_Q: (QD, H), L.W_K: (KD, H), L.W_V: (KD, H), L.W_O: (H, QD), L.W_GATE: (F, H),
              L.W_UP: (F, H), L.W_DOWN: (H, F)}
    for li in range(c.num_layers):
        model.set_weight(li, L.W_ATTN_NORM, ones.data_ptr(), L.DTYPE_F16)
        model.set_weight(li, L.W_FFN_NORM, ones.data_ptr(), L.DTYPE_F16)
        for slot, (n, k) in shapes.items():
            w = quantized_tensor_on_device(model, n, k, dtype, seed, li, slot)
            model.set_weight(li, slot, w.data_ptr(), dtype)
            del w
    torch.cuda.synchronize()


LLAMA3_8B = dict(vocab_size=128256, hidden_size=4096, num_layers=32, num_heads=32, num_kv_heads=8, head_dim=128,
                 intermediate_size=14336, rope_theta=500000.0, rms_norm_eps=1e-5)
LLAMA3_70B = dict(vocab_size=128256, hidden_size=8192, num_layers=80, num_heads=64, num_kv_heads=8, head_dim=128,
                  intermediate_size=28672, rope_theta=500000.0, rms_norm_eps=1e-5)
TINYLLAMA = dict(vocab_size=32000, hidden_size=2048, num_layers=22, num_heads=32, num_kv_heads=4, head_dim=64,
                 intermediate_size=5632, rope_theta=10000.0, rms_norm_eps=1e-5)
