"""CudaBackend: beacon-core's ComputeBackend trait over the C ABI.

Method names, argument meaning and error behaviour follow
crates/beacon-core/src/backend.rs:14-167 (and CpuBackend,
crates/beacon-core/src/cpu_backend.rs, for the corner cases); every method
lands in one `beacon_cuda_op_*` call of libbeacon_cuda.so. Errors map to the
EngineError variants of crates/beacon-core/src/error.rs:7-32.
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L


class EngineError(RuntimeError):
    """EngineError::Backend (error.rs:11-12) and the base of the others."""


class ShapeMismatch(EngineError):
    """EngineError::ShapeMismatch (error.rs:20-21)."""


class ContextOverflow(EngineError):
    """EngineError::ContextOverflow (error.rs:24-25)."""


def _raise(status: int) -> None:
    if status == L.OK:
        return
    msg = L.lib().beacon_cuda_last_error_message()
    text = msg.decode() if msg else ""
    if status == L.ERR_SHAPE_MISMATCH:
        raise ShapeMismatch(text)
    if status == L.ERR_CONTEXT_OVERFLOW:
        raise ContextOverflow(text)
    err = EngineError(f"backend error [status {status}]: {text}")
    err.status = status
    raise err


_NP_DTYPE = {np.dtype(np.float32): L.DTYPE_F32, np.dtype(np.float16): L.DTYPE_F16,
             np.dtype(np.int32): L.DTYPE_I32, np.dtype(np.int8): L.DTYPE_I8}


class Tensor:
    """Owning handle of a BeaconCudaTensor (device memory)."""

    __slots__ = ("_h",)

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)

    @property
    def handle(self) -> ctypes.c_void_p:
        return self._h

    @property
    def shape(self) -> tuple:
        nd = ctypes.c_size_t(8)
        buf = (ctypes.c_int64 * 8)()
        _raise(L.lib().beacon_cuda_tensor_shape(self._h, buf, ctypes.byref(nd)))
        return tuple(buf[i] for i in range(nd.value))

    @property
    def dtype(self) -> int:
        d = ctypes.c_int32()
        _raise(L.lib().beacon_cuda_tensor_dtype(self._h, ctypes.byref(d)))
        return d.value

    @property
    def device_ptr(self) -> int:
        p = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_tensor_device_ptr(self._h, ctypes.byref(p)))
        return p.value or 0

    def numel(self) -> int:
        n = 1
        for d in self.shape:
            n *= d
        return n

    def read_raw(self, nbytes: int) -> np.ndarray:
        out = np.empty(nbytes, dtype=np.uint8)
        _raise(L.lib().beacon_cuda_tensor_read_raw(self._h, out.ctypes.data, nbytes))
        return out

    def numpy(self) -> np.ndarray:
        """Host copy as f32 (or the raw dtype for I32/F16 tensors)."""
        shape = self.shape
        n = self.numel()
        dt = self.dtype
        if dt == L.DTYPE_F16:
            return self.read_raw(2 * n).view(np.float16).reshape(shape)
        if dt == L.DTYPE_I32:
            return self.read_raw(4 * n).view(np.int32).reshape(shape)
        out = np.empty(n, dtype=np.float32)
        _raise(L.lib().beacon_cuda_tensor_read_f32(self._h, out.ctypes.data, n))
        return out.reshape(shape)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                L.lib().beacon_cuda_tensor_destroy(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p()


class Stream:
    __slots__ = ("_h",)

    def __init__(self, handle: int):
        self._h = ctypes.c_void_p(handle)

    @property
    def handle(self):
        return self._h

    def synchronize(self) -> None:
        _raise(L.lib().beacon_cuda_stream_synchronize(self._h))

    @property
    def cuda_stream(self) -> int:
        """The underlying cudaStream_t, e.g. for torch.cuda.ExternalStream."""
        p = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_stream_handle(self._h, ctypes.byref(p)))
        return p.value or 0

    def __del__(self):
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            try:
                L.lib().beacon_cuda_stream_destroy(h)
            except Exception:
                pass
            self._h = ctypes.c_void_p()


def _shape_arr(shape):
    arr = (ctypes.c_int64 * max(1, len(shape)))(*shape)
    return arr, len(shape)


class CudaBackend:
    """ComputeBackend implementation on one B200 (backend.rs:14-167)."""

    def __init__(self, device: int = 0, numerics: int = L.NUMERICS_FAST):
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_context_create(device, ctypes.byref(h)))
        self.ctx = h
        self.set_numerics(numerics)

    def set_numerics(self, numerics: int) -> None:
        _raise(L.lib().beacon_cuda_context_set_numerics(self.ctx, numerics))

    def set_wait_limit(self, cycles: int) -> None:
        """Limit (SM clock cycles) of the kernels' bounded waits; 0 = default."""
        _raise(L.lib().beacon_cuda_context_set_wait_limit(self.ctx, cycles))

    def close(self) -> None:
        if self.ctx and self.ctx.value:
            L.lib().beacon_cuda_context_destroy(self.ctx)
            self.ctx = ctypes.c_void_p()

    # --- tensor creation (beacon_shim.h:56-71) -------------------------------
    def upload(self, data: np.ndarray, shape=None, dtype: int | None = None,
               nibble_order: int = L.NIBBLE_REF_INTERLEAVED) -> Tensor:
        data = np.ascontiguousarray(data)
        if dtype is None:
            dtype = _NP_DTYPE[data.dtype]
        if shape is None:
            shape = data.shape
        arr, nd = _shape_arr(shape)
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_tensor_upload(self.ctx, data.ctypes.data, arr, nd, dtype, nibble_order,
                                                 ctypes.byref(h)))
        return Tensor(h.value)

    def from_device_blocks(self, device_ptr: int, shape, dtype: int,
                           nibble_order: int = L.NIBBLE_REF_INTERLEAVED) -> Tensor:
        """A quantized tensor from raw GGUF block bytes already in device memory."""
        arr, nd = _shape_arr(shape)
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_tensor_from_device_blocks(self.ctx, ctypes.c_void_p(device_ptr), arr, nd, dtype,
                                                             nibble_order, ctypes.byref(h)))
        return Tensor(h.value)

    def zeros(self, shape, dtype: int = L.DTYPE_F32) -> Tensor:
        arr, nd = _shape_arr(shape)
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_tensor_zeros(self.ctx, arr, nd, dtype, ctypes.byref(h)))
        return Tensor(h.value)

    # --- ComputeBackend ----------------------------------------------------------
    def new_stream(self) -> Stream:
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_stream_create(self.ctx, ctypes.byref(h)))
        return Stream(h.value)

    def _op(self, fn, *args) -> Tensor:
        out = ctypes.c_void_p()
        _raise(fn(self.ctx, *args, ctypes.byref(out)))
        return Tensor(out.value)

    def matmul(self, stream: Stream, a: Tensor, b: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_matmul, stream.handle, a.handle, b.handle)

    def quantized_matmul(self, stream: Stream, x: Tensor, w: Tensor, scales: Tensor | None = None,
                         biases: Tensor | None = None, group_size: int = 0, bits: int = 0) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_quantized_matmul, stream.handle, x.handle, w.handle,
                        scales.handle if scales else None, biases.handle if biases else None,
                        group_size, bits)

    def rms_norm(self, stream: Stream, x: Tensor, weight: Tensor, eps: float) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_rms_norm, stream.handle, x.handle, weight.handle, eps)

    def rope(self, stream: Stream, x: Tensor, position_offset: int, theta: float, dim: int,
             freqs: Tensor | None = None) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_rope, stream.handle, x.handle, position_offset, theta, dim,
                        freqs.handle if freqs else None)

    def attention(self, stream: Stream, q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None,
                  scale: float, causal: int = -1) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_attention, stream.handle, q.handle, k.handle, v.handle,
                        mask.handle if mask else None, scale, causal)

    def silu(self, stream: Stream, x: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_silu, stream.handle, x.handle)

    def softmax(self, stream: Stream, x: Tensor, axis: int = -1) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_softmax, stream.handle, x.handle, axis)

    def add(self, stream: Stream, a: Tensor, b: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_add, stream.handle, a.handle, b.handle)

    def mul(self, stream: Stream, a: Tensor, b: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_elementwise_mul, stream.handle, a.handle, b.handle)

    def reshape(self, stream: Stream, x: Tensor, shape) -> Tensor:
        arr, nd = _shape_arr(shape)
        return self._op(L.lib().beacon_cuda_op_reshape, stream.handle, x.handle, arr, nd)

    def swapaxes(self, stream: Stream, x: Tensor, axis1: int, axis2: int) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_swapaxes, stream.handle, x.handle, axis1, axis2)

    def transpose(self, stream: Stream, x: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_transpose, stream.handle, x.handle)

    def embedding(self, stream: Stream, weight: Tensor, indices: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_embedding, stream.handle, weight.handle, indices.handle)

    def eval(self, t: Tensor, stream: Stream) -> None:
        _raise(L.lib().beacon_cuda_tensor_eval(t.handle, stream.handle))

    def read_f32(self, t: Tensor, n: int) -> np.ndarray:
        out = np.empty(n, dtype=np.float32)
        _raise(L.lib().beacon_cuda_tensor_read_f32(t.handle, out.ctypes.data, n))
        return out

    def kv_cache_update(self, stream: Stream, cache_k: Tensor, cache_v: Tensor, new_k: Tensor,
                        new_v: Tensor, position: int):
        ok, ov = ctypes.c_void_p(), ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_op_kv_cache_update(self.ctx, stream.handle, cache_k.handle, cache_v.handle,
                                                      new_k.handle, new_v.handle, position,
                                                      ctypes.byref(ok), ctypes.byref(ov)))
        return Tensor(ok.value), Tensor(ov.value)

    def create_token_tensor(self, tokens) -> Tensor:
        toks = np.ascontiguousarray(np.asarray(tokens, dtype=np.uint32))
        out = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_create_token_tensor(self.ctx, toks.ctypes.data, toks.size, ctypes.byref(out)))
        return Tensor(out.value)

    # --- beyond the trait --------------------------------------------------------
    def argmax(self, stream: Stream, logits: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_argmax, stream.handle, logits.handle)

    def profile_quantized_matmul(self, stream: Stream, weights, x: Tensor, iters: int = 10) -> tuple[float, int]:
        """(mean microseconds per launch, algorithmic bytes per launch) of
        quantized_matmul's decode path, cycling over `weights` (copies)."""
        arr = (ctypes.c_void_p * len(weights))(*[w.handle.value for w in weights])
        us, nb = ctypes.c_float(), ctypes.c_uint64()
        _raise(L.lib().beacon_cuda_profile_quantized_matmul(self.ctx, stream.handle, arr, len(weights), x.handle,
                                                            iters, ctypes.byref(us), ctypes.byref(nb)))
        return us.value, nb.value

    def sample(self, stream: Stream, logits: Tensor, params: L.SamplingParams, uniforms: Tensor,
               previous: Tensor | None = None) -> Tensor:
        """sampling::sample (sampling.rs:15-57) per row on the device; I32 [rows]."""
        return self._op(L.lib().beacon_cuda_op_sample, stream.handle, logits.handle,
                        previous.handle if previous else None, ctypes.byref(params), uniforms.handle)

    def dequantize_to_f16(self, stream: Stream, w: Tensor) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_dequantize_to_f16, stream.handle, w.handle)

    def quantize(self, stream: Stream, x: Tensor, dtype: int,
                 nibble_order: int = L.NIBBLE_REF_INTERLEAVED) -> Tensor:
        return self._op(L.lib().beacon_cuda_op_quantize, stream.handle, x.handle, dtype, nibble_order)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
