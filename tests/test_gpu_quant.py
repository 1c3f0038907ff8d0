"""GPU parity of the GGUF kernels against the CPU oracle, through the C ABI.

- dequantize_to_f16: bit-exact (dequant.rs:33-60), including NaN/Inf/
  subnormal block scales and both Q4_0 nibble orders;
- the device quantizer writes the same bytes as the oracle's;
- dequant-GEMV: max|y - r| / max|r| <= 1e-3 against the oracle's sequential
  f32 sum (q4_dot_f32 order, ops.rs:38-56), for every numerics mode, batch
  1..16, f32 and f16 activations, ragged N and K.
"""
import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu

GEMV_TOL = 1e-3  # relative to max|reference|, the bound the reference path is held to


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.fixture(scope="module")
def stream(be):
    return be.new_stream()


def quant_bytes(rng, dtype, n, k, nibble=orc.NIBBLE_REF_INTERLEAVED, scale=0.02):
    return orc.quantize((rng.standard_normal((n, k)) * scale).astype(np.float32), dtype, nibble)


def upload_q(be, data, dtype, n, k, nibble=orc.NIBBLE_REF_INTERLEAVED):
    return be.upload(data, shape=(n, k), dtype=dtype, nibble_order=nibble)


def random_blocks(rng, dtype, nblocks):
    """Arbitrary block bytes with hostile scales: 0, subnormal, large, Inf, NaN."""
    bb = orc.block_bytes(dtype)
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    special = np.array([0x0000, 0x0001, 0x03FF, 0x7BFF, 0x7C00, 0xFC00, 0x7E00, 0x7D01, 0x3C00, 0x8000],
                       dtype=np.uint16)
    sc = special[rng.integers(0, special.size, nblocks)]
    pick = rng.random(nblocks) < 0.3
    raw[pick, 0] = (sc[pick] & 0xFF).astype(np.uint8)
    raw[pick, 1] = (sc[pick] >> 8).astype(np.uint8)
    if dtype == orc.Q4_K:  # dmin too
        sc2 = special[rng.integers(0, special.size, nblocks)]
        pick2 = rng.random(nblocks) < 0.3
        raw[pick2, 2] = (sc2[pick2] & 0xFF).astype(np.uint8)
        raw[pick2, 3] = (sc2[pick2] >> 8).astype(np.uint8)
    return raw.reshape(-1)


@pytest.mark.parametrize("dtype,nibble", [(orc.Q4_0, orc.NIBBLE_REF_INTERLEAVED), (orc.Q4_0, orc.NIBBLE_GGUF_SPLIT),
                                          (orc.Q8_0, orc.NIBBLE_REF_INTERLEAVED), (orc.Q4_K, orc.NIBBLE_REF_INTERLEAVED)])
@pytest.mark.parametrize("n,k", [(64, 512), (37, 768), (1, 256), (130, 2560)])
def test_dequant_bit_exact_random_bytes(be, stream, dtype, nibble, n, k):
    if k % orc.block_size(dtype):
        pytest.skip("K not a whole number of blocks")
    rng = np.random.default_rng(n * 7919 + k + dtype)
    raw = random_blocks(rng, dtype, n * k // orc.block_size(dtype))
    t = upload_q(be, raw, dtype, n, k, nibble)
    got = be.dequantize_to_f16(stream, t).numpy().view(np.uint16).reshape(-1)
    ref = orc.dequantize_to_f16(raw, dtype, n * k, nibble)
    bad = np.nonzero(got != ref)[0]
    assert bad.size == 0, f"{bad.size} mismatches, first at {bad[:5]}: got {got[bad[:5]]} ref {ref[bad[:5]]}"


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
def test_dequant_known_answers_on_device(be, stream, dtype):
    """The reference's KAT blocks, dequantized on the GPU."""
    if dtype == orc.Q4_0:
        blk = np.array([0x00, 0x3C] + [0xAA] * 16, np.uint8)       # dequant.rs:633-649 -> 2.0
        want = 2.0
    elif dtype == orc.Q8_0:
        blk = np.array([0x00, 0x38] + [4] * 32, np.uint8)          # dequant.rs:651-667 -> 2.0
        want = 2.0
    else:
        blk = np.zeros(144, np.uint8)                               # d = 1, sc = 1, nibbles 3 -> 3.0
        blk[1] = 0x3C
        blk[4:8] = 1
        blk[8:12] = 0
        blk[12:16] = 0x01
        blk[16:] = 0x33
        want = 3.0
    bs = orc.block_size(dtype)
    blocks = np.tile(blk, 32)                                       # one 32-row group
    t = upload_q(be, blocks, dtype, 32, bs)
    got = be.dequantize_to_f16(stream, t).numpy().astype(np.float32)
    assert np.all(got == want)


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
@pytest.mark.parametrize("nibble", [orc.NIBBLE_REF_INTERLEAVED, orc.NIBBLE_GGUF_SPLIT])
def test_device_quantizer_matches_oracle(be, stream, dtype, nibble):
    import ctypes

    import torch
    from beacon_cuda import _lib as L
    if dtype != orc.Q4_0 and nibble == orc.NIBBLE_GGUF_SPLIT:
        pytest.skip("nibble order only applies to Q4_0")
    rng = np.random.default_rng(dtype)
    n, k = 48, 1024
    x = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    x[3, :32] = 0.0                      # all-zero block
    x[5, 100] = 1e-30                    # tiny values
    x[7, :] *= 1e4                       # large values
    ref = orc.quantize(x, dtype, nibble)
    dx = torch.from_numpy(x).cuda()
    dout = torch.empty(ref.size, dtype=torch.uint8, device="cuda")
    torch.cuda.synchronize()
    st = L.lib().beacon_cuda_quantize_blocks(be.ctx, stream.handle, ctypes.c_void_p(dx.data_ptr()), n, k, dtype,
                                             nibble, ctypes.c_void_p(dout.data_ptr()))
    L.check(st)
    stream.synchronize()
    got = dout.cpu().numpy()
    assert np.array_equal(got, ref)


def _rel(y, r):
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
@pytest.mark.parametrize("numerics", [0, 1, 2])   # FAST, EXACT, REF_RTZ
@pytest.mark.parametrize("batch", [1, 2, 3, 4, 8, 16])
def test_gemv_parity(be, stream, dtype, numerics, batch):
    rng = np.random.default_rng(1000 * dtype + 10 * numerics + batch)
    n, k = 300, 2048                      # ragged N (not a multiple of 32)
    w = quant_bytes(rng, dtype, n, k)
    x = rng.standard_normal((batch, k)).astype(np.float32)
    be.set_numerics(numerics)
    try:
        y = be.quantized_matmul(stream, be.upload(x), upload_q(be, w, dtype, n, k)).numpy()
    finally:
        be.set_numerics(0)
    r = orc.qgemv(w, dtype, n, k, x, rtz=(numerics == 2))
    err = _rel(y, r)
    # FAST quantizes activations to int16 per 32; the f32 modes differ only in order of summation
    assert err <= (GEMV_TOL if numerics == 0 else 2e-5), err


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
def test_gemv_f16_activations_and_shapes(be, stream, dtype):
    """BASELINE op-sweep inputs: fp16 N(0,1) activations, several shapes incl. split-K ones."""
    rng = np.random.default_rng(dtype + 5)
    for n, k, b in [(4096, 4096, 1), (1024, 14336, 4), (96, 256, 16), (32, 8192, 2)]:
        w = quant_bytes(rng, dtype, n, k)
        x = rng.standard_normal((b, k)).astype(np.float16)
        y = be.quantized_matmul(stream, be.upload(x), upload_q(be, w, dtype, n, k)).numpy()
        r = orc.qgemv(w, dtype, n, k, x.astype(np.float32))
        assert _rel(y, r) <= GEMV_TOL, (n, k, b)


def test_gemv_q4_0_gguf_split_order(be, stream):
    rng = np.random.default_rng(77)
    n, k = 64, 1024
    w = quant_bytes(rng, orc.Q4_0, n, k, orc.NIBBLE_GGUF_SPLIT)
    x = rng.standard_normal((1, k)).astype(np.float32)
    y = be.quantized_matmul(stream, be.upload(x), upload_q(be, w, orc.Q4_0, n, k, orc.NIBBLE_GGUF_SPLIT)).numpy()
    r = orc.qgemv(w, orc.Q4_0, n, k, x, nibble_order=orc.NIBBLE_GGUF_SPLIT)
    assert _rel(y, r) <= GEMV_TOL


def test_q4_matmul_reference_kat_on_device(be, stream):
    """beacon-kernels tests.rs:93-109: two all-ones rows, scale 1 -> 32."""
    blk = np.array([0x00, 0x3C] + [0x99] * 16, np.uint8)        # nibbles 9 -> +1
    w = np.tile(blk, 32)                                          # 32 rows of K = 32
    y = be.quantized_matmul(stream, be.upload(np.ones((1, 32), np.float32)),
                            upload_q(be, w, orc.Q4_0, 32, 32)).numpy()
    assert np.allclose(y, 32.0, atol=1e-3)


def test_quantized_matmul_errors(be, stream):
    from beacon_cuda import EngineError, ShapeMismatch
    rng = np.random.default_rng(1)
    w = upload_q(be, quant_bytes(rng, orc.Q4_K, 32, 256), orc.Q4_K, 32, 256)
    with pytest.raises(ShapeMismatch):
        be.quantized_matmul(stream, be.upload(np.ones((1, 128), np.float32)), w)
    with pytest.raises(EngineError):
        be.quantized_matmul(stream, be.upload(np.ones((1, 256), np.float32)), w, group_size=32, bits=4)
    with pytest.raises(EngineError):   # not a BeaconDtype
        be.upload(np.zeros(210, np.uint8), shape=(1, 256), dtype=111)
