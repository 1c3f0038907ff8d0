"""CudaModel: the fused decoder runtime (beacon_cuda_model_*) from Python.

One object per GPU (per tensor-parallel rank). Weights go in as full GGUF
tensors (host or device bytes); each rank keeps its shard. `forward` is
Engine::forward (engine.rs:190-241) for one sequence; `decode_step` is one
greedy step for a batch (Engine::generate_next_token, engine.rs:249-264,
for batch 1) and runs as a replayed CUDA graph.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np

from . import _lib as L
from .backend import CudaBackend, Stream, _raise


@dataclass
class DecoderConfig:
    vocab_size: int
    hidden_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    intermediate_size: int
    max_context: int
    max_batch: int = 1
    rope_theta: float = 10000.0
    rms_norm_eps: float = 1e-5
    numerics: int = L.NUMERICS_FAST
    kv_dtype: int = L.DTYPE_F16
    kv_persist: bool = True
    causal_prefill: bool = True
    tp_size: int = 1
    tp_rank: int = 0

    def to_c(self) -> L.ModelConfig:
        return L.ModelConfig(self.vocab_size, self.hidden_size, self.num_layers, self.num_heads,
                             self.num_kv_heads, self.head_dim, self.intermediate_size, self.max_context,
                             self.max_batch, self.rope_theta, self.rms_norm_eps, self.numerics, self.kv_dtype,
                             int(self.kv_persist), int(self.causal_prefill), self.tp_size, self.tp_rank)


class CudaModel:
    def __init__(self, backend: CudaBackend, cfg: DecoderConfig):
        self.backend = backend
        self.cfg = cfg
        c = cfg.to_c()
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_model_create(backend.ctx, ctypes.byref(c), ctypes.byref(h)))
        self._h = h
        self.stream = backend.new_stream()

    def set_weight(self, layer: int, slot: int, data, dtype: int,
                   nibble_order: int = L.NIBBLE_REF_INTERLEAVED) -> None:
        """data: numpy array (host bytes) or an int device pointer."""
        if isinstance(data, int):
            _raise(L.lib().beacon_cuda_model_set_weight(self._h, layer, slot, ctypes.c_void_p(data), dtype,
                                                        nibble_order, 1))
        else:
            arr = np.ascontiguousarray(data)
            _raise(L.lib().beacon_cuda_model_set_weight(self._h, layer, slot, arr.ctypes.data, dtype,
                                                        nibble_order, 0))

    def load_gguf(self, gguf) -> None:
        """Every weight slot from a GGUF file (beacon_cuda.gguf.GgufFile)."""
        _raise(L.lib().beacon_cuda_model_load_gguf(self._h, gguf.handle))

    def reset(self) -> None:
        _raise(L.lib().beacon_cuda_model_reset(self._h))

    def forward(self, tokens, position: int, want_logits: bool = True) -> np.ndarray | None:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        out = np.empty((toks.size, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        _raise(L.lib().beacon_cuda_model_forward(self._h, self.stream.handle, toks.ctypes.data, toks.size,
                                                 position, out.ctypes.data if out is not None else None))
        return out

    def decode_step(self, tokens, position: int, want_logits: bool = False):
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        nxt = np.empty(toks.size, dtype=np.uint32)
        logits = np.empty((toks.size, self.cfg.vocab_size), dtype=np.float32) if want_logits else None
        _raise(L.lib().beacon_cuda_model_decode_step(self._h, self.stream.handle, toks.ctypes.data, toks.size,
                                                     position, nxt.ctypes.data,
                                                     logits.ctypes.data if logits is not None else None))
        return nxt, logits

    def decode_step_sampled(self, tokens, position: int, params: L.SamplingParams, uniforms,
                            previous=None) -> np.ndarray:
        """One step with the next tokens sampled on the device (no logits to the host).
        uniforms: [batch] draws in [0, 1); previous: [batch, n] generated tokens or None."""
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        u = np.ascontiguousarray(np.asarray(uniforms, dtype=np.float32))
        prev = None if previous is None else np.ascontiguousarray(np.asarray(previous, dtype=np.uint32))
        n_prev = 0 if prev is None else prev.shape[-1]
        nxt = np.empty(toks.size, dtype=np.uint32)
        _raise(L.lib().beacon_cuda_model_decode_step_sampled(
            self._h, self.stream.handle, toks.ctypes.data, toks.size, position, ctypes.byref(params), u.ctypes.data,
            prev.ctypes.data if n_prev else None, n_prev, nxt.ctypes.data))
        return nxt

    def decode_step_device(self, d_tokens: int | None, batch: int, position: int,
                           d_next: int | None = None, d_logits: int | None = None,
                           stream: Stream | None = None) -> None:
        """Enqueue one step on device buffers. d_tokens=None and position<0
        continues from the previous step (greedy feedback on the device)."""
        s = stream or self.stream
        _raise(L.lib().beacon_cuda_model_decode_step_device(
            self._h, s.handle, ctypes.c_void_p(d_tokens) if d_tokens else None, batch, position,
            ctypes.c_void_p(d_next) if d_next else None, ctypes.c_void_p(d_logits) if d_logits else None))

    def synchronize(self, stream: Stream | None = None) -> None:
        """Wait for the model's enqueued work; raises its device-side errors."""
        s = stream or self.stream
        _raise(L.lib().beacon_cuda_model_synchronize(self._h, s.handle))

    def profile_linear(self, slot: int, batch: int = 1, iters: int = 5) -> tuple[float, int]:
        """(mean microseconds per launch, algorithmic bytes per launch) of one projection."""
        us, nb = ctypes.c_float(), ctypes.c_uint64()
        _raise(L.lib().beacon_cuda_model_profile_linear(self._h, self.stream.handle, slot, batch, iters,
                                                        ctypes.byref(us), ctypes.byref(nb)))
        return us.value, nb.value

    def fill_kv_random(self, n_rows: int, seed: int = 0) -> None:
        _raise(L.lib().beacon_cuda_model_fill_kv_random(self._h, n_rows, seed))

    def launches_per_step(self, batch: int, continuing: bool) -> int:
        v = ctypes.c_int32()
        _raise(L.lib().beacon_cuda_model_launches_per_step(self._h, batch, int(continuing), ctypes.byref(v)))
        return v.value

    def memory_bytes(self) -> int:
        v = ctypes.c_uint64()
        _raise(L.lib().beacon_cuda_model_memory(self._h, ctypes.byref(v)))
        return v.value

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            L.lib().beacon_cuda_model_destroy(h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
