"""GGUF v3 files through the C ABI (beacon_cuda_gguf_*): the reader of
crates/beacon-format/src/gguf and the weight loading of
crates/beacon-core/src/weights.rs for the fused decoder."""
from __future__ import annotations

import ctypes

import numpy as np

from . import _lib as L
from .backend import _raise


class GgufTensorInfo:
    __slots__ = ("index", "name", "dtype", "shape", "nbytes", "_ptr")

    def __init__(self, index, name, dtype, shape, nbytes, ptr):
        self.index, self.name, self.dtype, self.shape, self.nbytes, self._ptr = index, name, dtype, shape, nbytes, ptr

    def data(self) -> np.ndarray:
        """A copy of the tensor's bytes (GgufFile::tensor_data)."""
        return np.ctypeslib.as_array((ctypes.c_uint8 * self.nbytes).from_address(self._ptr)).copy()


class GgufFile:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        _raise(L.lib().beacon_cuda_gguf_open(str(path).encode(), ctypes.byref(h)))
        self._h = h

    @property
    def handle(self):
        return self._h

    @property
    def version(self) -> int:
        v = ctypes.c_uint32()
        _raise(L.lib().beacon_cuda_gguf_version(self._h, ctypes.byref(v)))
        return v.value

    @property
    def tensors(self) -> list[GgufTensorInfo]:
        n = ctypes.c_int64()
        _raise(L.lib().beacon_cuda_gguf_tensor_count(self._h, ctypes.byref(n)))
        out = []
        for i in range(n.value):
            name, dt, ptr, nb = ctypes.c_char_p(), ctypes.c_int32(), ctypes.c_void_p(), ctypes.c_uint64()
            shape, nd = (ctypes.c_int64 * 8)(), ctypes.c_size_t(8)
            _raise(L.lib().beacon_cuda_gguf_tensor_info(self._h, i, ctypes.byref(name), ctypes.byref(dt), shape,
                                                        ctypes.byref(nd), ctypes.byref(ptr), ctypes.byref(nb)))
            out.append(GgufTensorInfo(i, name.value.decode(), dt.value, tuple(shape[d] for d in range(nd.value)),
                                      nb.value, ptr.value or 0))
        return out

    def get_int(self, key: str) -> int:
        v = ctypes.c_int64()
        _raise(L.lib().beacon_cuda_gguf_get_int(self._h, key.encode(), ctypes.byref(v)))
        return v.value

    def get_float(self, key: str) -> float:
        v = ctypes.c_double()
        _raise(L.lib().beacon_cuda_gguf_get_float(self._h, key.encode(), ctypes.byref(v)))
        return v.value

    def get_string(self, key: str) -> str:
        v = ctypes.c_char_p()
        _raise(L.lib().beacon_cuda_gguf_get_string(self._h, key.encode(), ctypes.byref(v)))
        return v.value.decode()

    def get_array_len(self, key: str) -> int:
        v = ctypes.c_uint64()
        _raise(L.lib().beacon_cuda_gguf_get_array_len(self._h, key.encode(), ctypes.byref(v)))
        return v.value

    def model_config(self, max_context: int = 0) -> dict:
        """GgufFile::model_config (config_map.rs:14-100) as DecoderConfig fields."""
        c = L.ModelConfig()
        c.max_context = max_context
        _raise(L.lib().beacon_cuda_gguf_model_config(self._h, ctypes.byref(c)))
        keys = ("vocab_size", "hidden_size", "num_layers", "num_heads", "num_kv_heads", "head_dim",
                "intermediate_size", "max_context", "rope_theta", "rms_norm_eps")
        return {k: getattr(c, k) for k in keys}

    def close(self) -> None:
        h = getattr(self, "_h", None)
        if h is not None and h.value:
            L.lib().beacon_cuda_gguf_close(h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
