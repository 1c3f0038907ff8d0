"""B200 (sm_100a) backend for Beacon's quantized decode path.

- ``_lib``: ctypes binding of libbeacon_cuda.so (include/beacon_cuda.h);
- ``backend.CudaBackend``: the ComputeBackend trait (crates/beacon-core/src/backend.rs);
- ``engine.Engine``: engine.rs's forward pass driven op by op through the trait;
- ``model.CudaModel``: the fused, graph-captured decoder runtime (the fast path).
"""
from . import _lib
from .backend import ContextOverflow, CudaBackend, EngineError, ShapeMismatch, Stream, Tensor
from .model import CudaModel, DecoderConfig

__all__ = ["_lib", "CudaBackend", "CudaModel", "DecoderConfig", "EngineError", "ShapeMismatch",
           "ContextOverflow", "Stream", "Tensor"]
