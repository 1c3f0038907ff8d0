"""Engine<CudaBackend>: engine.rs's forward pass driven op by op through the
ComputeBackend methods of CudaBackend.

This is what crates/beacon-core/src/engine.rs:135-456 does when it is
monomorphised over the CUDA backend: the same calls, in the same order, with
quantized projections going through `quantized_matmul`. It proves the trait
surface is complete; the fused runtime (model.CudaModel) is the fast path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .backend import ContextOverflow, CudaBackend, Stream, Tensor


@dataclass
class ModelConfig:
    """The fields of ModelConfig (crates/beacon-format/src/config.rs:43-66) the forward pass reads."""
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    max_position_embeddings: int
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5


@dataclass
class ProjectionWeight:
    """ProjectionWeight (weights.rs:19-36): `plain` (f32 [out, in]) or `quantized` (GGUF blocks)."""
    plain: Tensor | None = None
    quantized: Tensor | None = None


@dataclass
class LayerWeights:
    attn_norm: Tensor
    q_proj: ProjectionWeight
    k_proj: ProjectionWeight
    v_proj: ProjectionWeight
    o_proj: ProjectionWeight
    ffn_norm: Tensor
    gate_proj: ProjectionWeight
    up_proj: ProjectionWeight
    down_proj: ProjectionWeight


@dataclass
class KvCache:
    """KvCache (kv_cache.rs:13-21): [max_context, num_kv_heads, head_dim]."""
    cache_k: Tensor
    cache_v: Tensor
    current_length: int = 0


class Engine:
    def __init__(self, backend: CudaBackend, config: ModelConfig, embed_tokens: Tensor,
                 layers: list[LayerWeights], final_norm: Tensor, lm_head: ProjectionWeight,
                 kv_dtype: int = L.DTYPE_F32, kv_persist: bool = True, causal_prefill: bool = True):
        self.backend = backend
        self.config = config
        self.embed_tokens = embed_tokens
        self.layers = layers
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.kv_dtype = kv_dtype
        # kv_persist=False reproduces cpu_backend.rs:459-460 (the update lands
        # in a clone); causal_prefill=False reproduces engine.rs:418 (mask None)
        self.kv_persist = kv_persist
        self.causal_prefill = causal_prefill
        shape = (config.max_position_embeddings, config.num_kv_heads, config.head_dim)
        self.cache = [KvCache(backend.zeros(shape, kv_dtype), backend.zeros(shape, kv_dtype))
                      for _ in range(config.num_layers)]

    def proj_matmul(self, stream: Stream, x: Tensor, w: ProjectionWeight) -> Tensor:
        # engine.rs:143-170
        if w.quantized is not None:
            return self.backend.quantized_matmul(stream, x, w.quantized)
        wt = self.backend.transpose(stream, w.plain)
        return self.backend.matmul(stream, x, wt)

    def reset_cache(self) -> None:
        for kv in self.cache:
            kv.current_length = 0

    def forward(self, tokens, position: int) -> Tensor:
        # engine.rs:190-241
        b = self.backend
        stream = b.new_stream()
        seq_len = len(tokens)
        indices = b.create_token_tensor(tokens)
        h = b.embedding(stream, self.embed_tokens, indices)
        for i, layer in enumerate(self.layers):
            normed = b.rms_norm(stream, h, layer.attn_norm, self.config.rms_norm_eps)
            attn = self.attention_block(stream, normed, i, position, seq_len)
            h = b.add(stream, h, attn)
            normed = b.rms_norm(stream, h, layer.ffn_norm, self.config.rms_norm_eps)
            ffn = self.ffn_block(stream, normed, i)
            h = b.add(stream, h, ffn)
        h = b.rms_norm(stream, h, self.final_norm, self.config.rms_norm_eps)
        logits = self.proj_matmul(stream, h, self.lm_head)
        b.eval(logits, stream)
        for kv in self.cache:
            kv.current_length = position + seq_len
        return logits

    def generate_next_token(self, token: int, position: int) -> int:
        # engine.rs:249-264; argmax on the host exactly as the reference reads it
        logits = self.forward([token], position)
        vals = self.backend.read_f32(logits, self.config.vocab_size)
        best = 0
        for i in range(1, len(vals)):
            if not (vals[best] > vals[i]):
                best = i
        return best

    def attention_block(self, stream: Stream, hidden: Tensor, li: int, position: int, seq_len: int) -> Tensor:
        # engine.rs:277-429
        b, cfg, lw = self.backend, self.config, self.layers[li]
        q = self.proj_matmul(stream, hidden, lw.q_proj)
        k = self.proj_matmul(stream, hidden, lw.k_proj)
        v = self.proj_matmul(stream, hidden, lw.v_proj)
        q = b.swapaxes(stream, b.reshape(stream, q, [1, seq_len, cfg.num_heads, cfg.head_dim]), 1, 2)
        k = b.swapaxes(stream, b.reshape(stream, k, [1, seq_len, cfg.num_kv_heads, cfg.head_dim]), 1, 2)
        v = b.swapaxes(stream, b.reshape(stream, v, [1, seq_len, cfg.num_kv_heads, cfg.head_dim]), 1, 2)
        q = b.rope(stream, q, position, cfg.rope_theta, cfg.head_dim, None)
        k = b.rope(stream, k, position, cfg.rope_theta, cfg.head_dim, None)
        if position + seq_len > cfg.max_position_embeddings:
            raise ContextOverflow("context overflow: KV cache exhausted")
        k_sq = b.reshape(stream, b.swapaxes(stream, k, 1, 2), [seq_len, cfg.num_kv_heads, cfg.head_dim])
        v_sq = b.reshape(stream, b.swapaxes(stream, v, 1, 2), [seq_len, cfg.num_kv_heads, cfg.head_dim])
        cache = self.cache[li]
        if self.kv_persist:
            ck, cv = cache.cache_k, cache.cache_v
        else:
            shape = (cfg.max_position_embeddings, cfg.num_kv_heads, cfg.head_dim)
            ck, cv = b.zeros(shape, self.kv_dtype), b.zeros(shape, self.kv_dtype)
        k_cached, v_cached = b.kv_cache_update(stream, ck, cv, k_sq, v_sq, position)
        cached_len = position + seq_len
        k_full = b.swapaxes(stream, b.reshape(stream, k_cached, [1, cached_len, cfg.num_kv_heads, cfg.head_dim]), 1, 2)
        v_full = b.swapaxes(stream, b.reshape(stream, v_cached, [1, cached_len, cfg.num_kv_heads, cfg.head_dim]), 1, 2)
        scale = np.float32(1.0) / np.sqrt(np.float32(cfg.head_dim))  # f32 as engine.rs:415
        causal = -1 if self.causal_prefill else 0
        out = b.attention(stream, q, k_full, v_full, None, float(scale), causal)
        out = b.reshape(stream, b.swapaxes(stream, out, 1, 2), [seq_len, cfg.hidden_size])
        return self.proj_matmul(stream, out, lw.o_proj)

    def ffn_block(self, stream: Stream, hidden: Tensor, li: int) -> Tensor:
        # engine.rs:436-456
        b, lw = self.backend, self.layers[li]
        gate = b.silu(stream, self.proj_matmul(stream, hidden, lw.gate_proj))
        up = self.proj_matmul(stream, hidden, lw.up_proj)
        return self.proj_matmul(stream, b.mul(stream, gate, up), lw.down_proj)
