"""The allocation-free quantized matvec (beacon_cuda_quantized_matvec_noalloc).

It exists for callers that must not have device memory allocated for them —
a serving process whose arena owns all of HBM, code running beside another
thread's graph capture, latency-critical loops that cannot wait in the
allocator. Its scratch is a fixed array in the library, shared by every call
and left dirty between calls, so the test calls it twice in a row on the same
output buffer and compares each result with the allocating entry point
(quantized_matmul) at the GEMV tolerance the other tests use. The shapes cover
a split-K plan (scratch in use), a plan without split, and the reduced-split
path. Kept in its own file so that pytest collects it last.
"""
import ctypes

import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3


def _rel(y, r):
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.mark.parametrize("dtype,n,k,batch,x16", [
    (orc.Q4_K, 4096, 4096, 1, False),     # split-K over CTAs: scratch in use
    (orc.Q4_0, 300, 2048, 3, True),       # ragged rows, f16 activations
    (orc.Q8_0, 1024, 14336, 4, False),
    (orc.Q4_K, 28672, 4096, 2, False),    # enough row groups: no split
    (orc.Q4_K, 2048, 28672, 16, False),   # shared-memory-forced 12-way split, 16 columns
])
def test_noalloc_matches_quantized_matmul_on_two_calls(be, dtype, n, k, batch, x16):
    from beacon_cuda import _lib as L
    rng = np.random.default_rng(n + k + batch)
    w = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), dtype)
    wt = be.upload(w, shape=(n, k), dtype=dtype)
    x = rng.standard_normal((batch, k)).astype(np.float16 if x16 else np.float32)
    xt = be.upload(x)
    s = be.new_stream()
    ref = be.quantized_matmul(s, xt, wt).numpy()
    orc_ref = orc.qgemv(w, dtype, n, k, x.astype(np.float32))
    yt = be.zeros((batch, n))
    for call in range(2):
        st = L.lib().beacon_cuda_quantized_matvec_noalloc(
            s.handle, wt.handle, ctypes.c_void_p(xt.device_ptr), L.DTYPE_F16 if x16 else L.DTYPE_F32, batch,
            ctypes.c_void_p(yt.device_ptr))
        L.check(st)
        s.synchronize()
        got = yt.numpy()
        assert _rel(got, ref) <= GEMV_TOL, (call, _rel(got, ref))
        assert _rel(got, orc_ref) <= GEMV_TOL, (call, _rel(got, orc_ref))


def test_noalloc_leaves_device_memory_unchanged(be):
    """After a first call on the device (which looks the scratch array up),
    repeated calls with the same and smaller shapes leave the device's free
    memory exactly where it was: the entry point allocates nothing."""
    import torch
    from beacon_cuda import _lib as L
    rng = np.random.default_rng(7)
    n, k = 4096, 4096
    w = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), orc.Q4_K)
    wt = be.upload(w, shape=(n, k), dtype=orc.Q4_K)
    x = rng.standard_normal((4, k)).astype(np.float32)
    xt, yt = be.upload(x), be.zeros((4, n))
    s = be.new_stream()

    def call(batch):
        L.check(L.lib().beacon_cuda_quantized_matvec_noalloc(s.handle, wt.handle, ctypes.c_void_p(xt.device_ptr),
                                                             L.DTYPE_F32, batch, ctypes.c_void_p(yt.device_ptr)))

    for batch in (1, 2, 4):  # every plan once: kernels loaded, scratch address looked up
        call(batch)
    s.synchronize()
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        for batch in (4, 1, 2):
            call(batch)
    s.synchronize()
    torch.cuda.synchronize()
    free1 = torch.cuda.mem_get_info()[0]
    assert free1 == free0, (free0, free1)
    got = yt.numpy()[:2]
    assert _rel(got, orc.qgemv(w, orc.Q4_K, n, k, x[:2])) <= GEMV_TOL


def test_noalloc_rejects_a_stream_of_another_context(be):
    from beacon_cuda import CudaBackend
    from beacon_cuda import _lib as L
    rng = np.random.default_rng(8)
    w = orc.quantize((rng.standard_normal((64, 256)) * 0.02).astype(np.float32), orc.Q4_K)
    wt = be.upload(w, shape=(64, 256), dtype=orc.Q4_K)
    xt, yt = be.zeros((1, 256)), be.zeros((1, 64))
    other = CudaBackend(0)
    try:
        s2 = other.new_stream()
        st = L.lib().beacon_cuda_quantized_matvec_noalloc(s2.handle, wt.handle, ctypes.c_void_p(xt.device_ptr),
                                                          L.DTYPE_F32, 1, ctypes.c_void_p(yt.device_ptr))
        assert st == L.ERR_INVALID_ARGUMENT
        assert b"another context" in L.lib().beacon_cuda_last_error_message()
        del s2
    finally:
        other.close()


def test_noalloc_rejects_bad_arguments(be):
    from beacon_cuda import _lib as L
    rng = np.random.default_rng(5)
    w = orc.quantize((rng.standard_normal((64, 256)) * 0.02).astype(np.float32), orc.Q4_K)
    wt = be.upload(w, shape=(64, 256), dtype=orc.Q4_K)
    xt, yt = be.zeros((17, 256)), be.zeros((17, 64))
    s = be.new_stream()
    lib = L.lib()
    st = lib.beacon_cuda_quantized_matvec_noalloc(s.handle, wt.handle, ctypes.c_void_p(xt.device_ptr),
                                                  L.DTYPE_F32, 17, ctypes.c_void_p(yt.device_ptr))
    assert st == L.ERR_INVALID_ARGUMENT and b"batch" in lib.beacon_cuda_last_error_message()
    st = lib.beacon_cuda_quantized_matvec_noalloc(s.handle, wt.handle, None, L.DTYPE_F32, 1,
                                                  ctypes.c_void_p(yt.device_ptr))
    assert st == L.ERR_INVALID_ARGUMENT
    st = lib.beacon_cuda_quantized_matvec_noalloc(s.handle, wt.handle, ctypes.c_void_p(xt.device_ptr),
                                                  L.DTYPE_I32, 1, ctypes.c_void_p(yt.device_ptr))
    assert st == L.ERR_UNSUPPORTED_DTYPE


def test_noalloc_rejects_shapes_beyond_the_fixed_scratch(be):
    """f32 activations at 16 columns force a 19-way K-split of a 28672-column
    weight; 19 x 16 x 2048 partial sums exceed the 2 MiB array."""
    from beacon_cuda import _lib as L
    rng = np.random.default_rng(6)
    n, k = 2048, 28672
    w = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), orc.Q4_K)
    wt = be.upload(w, shape=(n, k), dtype=orc.Q4_K)
    xt, yt = be.zeros((16, k)), be.zeros((16, n))
    s = be.new_stream()
    be.set_numerics(L.NUMERICS_EXACT)
    try:
        st = L.lib().beacon_cuda_quantized_matvec_noalloc(s.handle, wt.handle, ctypes.c_void_p(xt.device_ptr),
                                                          L.DTYPE_F32, 16, ctypes.c_void_p(yt.device_ptr))
        assert st == L.ERR_SHAPE_MISMATCH
        assert b"2 MiB" in L.lib().beacon_cuda_last_error_message()
    finally:
        be.set_numerics(L.NUMERICS_FAST)
