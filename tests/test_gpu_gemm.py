"""Prefill dequant-GEMM (tcgen05 tensor cores) against the CPU oracle.

quantized_matmul with more than 16 rows in the fast numerics runs one
tensor-core GEMM (f16 x f16 products, f32 accumulation): its outputs must
stay within max|y - r| / max|r| <= 1e-3 of the oracle's sequential f32 sums
of the exact dequantised weights (q4_dot_f32 order, ops.rs:38-56), for every
block format, f32 and f16 activations, and ragged M, N and K (tails of the
128 x 256 x 64 tiling). The exact and CPU-reproducing numerics keep the
GEMV path at any row count; they are held to the GEMV's f32 bound.
"""
import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu

GEMM_TOL = 1e-3  # relative to max|reference|


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.fixture(scope="module")
def stream(be):
    return be.new_stream()


def _rel(y, r):
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


def _case(be, stream, rng, dtype, m, n, k, f16=False):
    w = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), dtype, orc.NIBBLE_REF_INTERLEAVED)
    x = rng.standard_normal((m, k)).astype(np.float16 if f16 else np.float32)
    y = be.quantized_matmul(stream, be.upload(x), be.upload(w, shape=(n, k), dtype=dtype, nibble_order=orc.NIBBLE_REF_INTERLEAVED)).numpy()
    r = orc.qgemv(w, dtype, n, k, x.astype(np.float32))
    return y, r


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
@pytest.mark.parametrize("m,n,k", [(17, 256, 256), (64, 300, 2048), (130, 1024, 4096), (200, 520, 1280)])
def test_tc_gemm_parity(be, stream, dtype, m, n, k):
    rng = np.random.default_rng(7000 + 100 * dtype + m)
    y, r = _case(be, stream, rng, dtype, m, n, k)
    assert y.shape == (m, n)
    assert _rel(y, r) <= GEMM_TOL, (m, n, k, _rel(y, r))


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0])
def test_tc_gemm_k_not_a_tile_multiple(be, stream, dtype):
    """K = 800: 25 blocks of 32, so the last 64-column slice is partly padding."""
    rng = np.random.default_rng(31 + dtype)
    y, r = _case(be, stream, rng, dtype, 40, 96, 800)
    assert _rel(y, r) <= GEMM_TOL


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
def test_tc_gemm_f16_activations(be, stream, dtype):
    rng = np.random.default_rng(55 + dtype)
    y, r = _case(be, stream, rng, dtype, 96, 512, 4096, f16=True)
    assert _rel(y, r) <= GEMM_TOL


def test_tc_gemm_full_tiles_multi_cta(be, stream):
    """Several 128-row and 256-column tiles: every CTA of the grid writes its own block."""
    rng = np.random.default_rng(99)
    y, r = _case(be, stream, rng, orc.Q4_K, 384, 768, 1024)
    assert _rel(y, r) <= GEMM_TOL
    assert np.all(np.isfinite(y))


@pytest.mark.parametrize("numerics", [1, 2])   # EXACT, REF_RTZ: the GEMV path at any row count
def test_exact_numerics_keep_the_gemv_for_many_rows(be, stream, numerics):
    rng = np.random.default_rng(400 + numerics)
    n, k, m = 96, 1024, 40
    w = orc.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), orc.Q4_K, orc.NIBBLE_REF_INTERLEAVED)
    x = rng.standard_normal((m, k)).astype(np.float32)
    be.set_numerics(numerics)
    try:
        y = be.quantized_matmul(stream, be.upload(x), be.upload(w, shape=(n, k), dtype=orc.Q4_K, nibble_order=orc.NIBBLE_REF_INTERLEAVED)).numpy()
    finally:
        be.set_numerics(0)
    r = orc.qgemv(w, orc.Q4_K, n, k, x, rtz=(numerics == 2))
    assert _rel(y, r) <= 2e-5
