"""The GGUF block formats beyond Q4_0/Q8_0/Q4_K on the device, against the
oracle's restatement of crates/beacon-format/src/dequant.rs:182-254 (Q4_1,
Q5_0, Q5_1) and :377-597 (Q5_K, Q6_K, Q2_K, Q3_K, Q8_K), through the C ABI.

- dequantize_to_f16 is bit-exact on arbitrary block bytes, including NaN,
  Inf and subnormal scales (x86 NaN propagation reproduced);
- quantized_matmul is within 1e-3 (fast numerics, which compute these formats
  in f32) and 2e-5 (exact and CPU-reproducing numerics) of the oracle's
  sequential f32 sum, at batch 1..16 and ragged shapes;
- a small decoder whose linears use these formats matches the oracle engine.
The reference ships no quantizer for these types; weights are random block
bytes with finite scales of realistic size (the GEMV and model cases).
"""
import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu

FORMATS = [orc.Q4_1, orc.Q5_0, orc.Q5_1, orc.Q2_K, orc.Q3_K, orc.Q5_K, orc.Q6_K, orc.Q8_K]
# byte offsets of the f16 scale fields of a block (Q8_K: an f32 scale at 0)
F16_SCALES = {orc.Q4_1: (0, 2), orc.Q5_0: (0,), orc.Q5_1: (0, 2), orc.Q2_K: (80, 82), orc.Q3_K: (108,),
              orc.Q5_K: (0, 2), orc.Q6_K: (208,)}


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.fixture(scope="module")
def stream(be):
    return be.new_stream()


def sane_blocks(rng, dtype, n, k, scale=0.002):
    """Random codes with finite scales: f16 scales |s| ~ scale, Q8_K f32."""
    bb, bs = orc.block_bytes(dtype), orc.block_size(dtype)
    nb = n * k // bs
    raw = rng.integers(0, 256, size=(nb, bb), dtype=np.uint8)
    if dtype == orc.Q8_K:
        d = (rng.random(nb) * scale).astype(np.float32)
        raw[:, 0:4] = d.view(np.uint8).reshape(nb, 4)
    else:
        for off in F16_SCALES[dtype]:
            s = (rng.random(nb) * scale + scale / 10).astype(np.float16)
            raw[:, off:off + 2] = s.view(np.uint8).reshape(nb, 2)
    return raw.reshape(-1)


def _rel(y, r):
    return float(np.abs(y - r).max() / max(np.abs(r).max(), 1e-30))


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("n,k", [(37, 256), (64, 768), (3, 2560)])
def test_dequant_bit_exact_arbitrary_bytes(be, stream, dtype, n, k):
    if k % orc.block_size(dtype):
        pytest.skip("not a whole number of blocks")
    rng = np.random.default_rng(dtype * 7 + n + k)
    raw = rng.integers(0, 256, size=n * k // orc.block_size(dtype) * orc.block_bytes(dtype), dtype=np.uint8)
    w = be.upload(raw, shape=(n, k), dtype=dtype)
    got = be.dequantize_to_f16(stream, w).numpy().view(np.uint16).reshape(-1)
    ref = orc.dequantize_to_f16(raw, dtype, n * k)
    assert np.array_equal(got, ref), int(np.count_nonzero(got != ref))


@pytest.mark.parametrize("dtype", [orc.Q4_1, orc.Q5_0, orc.Q5_1])
def test_dequant_ragged_last_tile(be, stream, dtype):
    """32-element formats with K not a multiple of 256 (a partial last tile)."""
    rng = np.random.default_rng(dtype)
    n, k = 33, 32 * 11
    raw = sane_blocks(rng, dtype, n, k)
    got = be.dequantize_to_f16(stream, be.upload(raw, shape=(n, k), dtype=dtype)).numpy().view(np.uint16)
    assert np.array_equal(got.reshape(-1), orc.dequantize_to_f16(raw, dtype, n * k))


@pytest.mark.parametrize("dtype", FORMATS)
@pytest.mark.parametrize("numerics", [0, 1, 2])
def test_gemv_parity(be, stream, dtype, numerics):
    rng = np.random.default_rng(100 * dtype + numerics)
    cases = [(300, 2048, 1), (300, 2048, 3), (96, 4096, 8), (4096, 4096, 16), (64, 1024, 5)]
    be.set_numerics(numerics)
    try:
        for n, k, b in cases:
            w = sane_blocks(rng, dtype, n, k)
            x = rng.standard_normal((b, k)).astype(np.float32)
            y = be.quantized_matmul(stream, be.upload(x), be.upload(w, shape=(n, k), dtype=dtype)).numpy()
            r = orc.qgemv(w, dtype, n, k, x, rtz=(numerics == 2))
            assert _rel(y, r) <= (1e-3 if numerics == 0 else 2e-5), (n, k, b, _rel(y, r))
    finally:
        be.set_numerics(0)


def test_quantized_matmul_bits_per_format(be, stream):
    from beacon_cuda import EngineError
    rng = np.random.default_rng(3)
    bits = {orc.Q2_K: 2, orc.Q3_K: 3, orc.Q4_1: 4, orc.Q5_0: 5, orc.Q5_1: 5, orc.Q5_K: 5, orc.Q6_K: 6, orc.Q8_K: 8}
    for dtype, nb in bits.items():
        gs = orc.block_size(dtype)
        w = be.upload(sane_blocks(rng, dtype, 32, 256), shape=(32, 256), dtype=dtype)
        x = be.upload(np.ones((1, 256), np.float32))
        be.quantized_matmul(stream, x, w, group_size=gs, bits=nb)
        with pytest.raises(EngineError):
            be.quantized_matmul(stream, x, w, group_size=gs, bits=nb + 1)


@pytest.mark.parametrize("dtype", [orc.Q6_K, orc.Q5_K, orc.Q3_K, orc.Q5_0])
def test_decoder_with_format_matches_oracle(be, dtype):
    """A decoder whose linears are all of one of these formats: prefill and
    greedy decode logits match the oracle engine in the exact numerics."""
    from beacon_cuda import CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from golden_models import make_tensor
    c = dict(vocab_size=1000, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64,
             intermediate_size=1024, max_context=32, rope_theta=10000.0, rms_norm_eps=1e-5)
    ocfg = orc.OracleModelConfig(**c, weights_rtz=False)
    om = orc.OracleModel(ocfg)
    m = CudaModel(be, DecoderConfig(**c, numerics=L.NUMERICS_EXACT, kv_dtype=L.DTYPE_F32))
    rng = np.random.default_rng(dtype)
    H, F, V = 512, 1024, 1000
    shapes = {orc.W_Q: (H, H), orc.W_K: (128, H), orc.W_V: (128, H), orc.W_O: (H, H), orc.W_GATE: (F, H),
              orc.W_UP: (F, H), orc.W_DOWN: (H, F), orc.W_LM_HEAD: (V, H)}
    slots = [(-1, orc.W_EMBED), (-1, orc.W_FINAL_NORM), (-1, orc.W_LM_HEAD)] + [
        (li, s) for li in range(2) for s in (orc.W_ATTN_NORM, orc.W_FFN_NORM) + tuple(shapes)[:-1]]
    for li, s in slots:
        if s in shapes:
            n, k = shapes[s]
            data, dt = sane_blocks(rng, dtype, n, k, scale=0.001), dtype
        else:
            data, dt = make_tensor(ocfg, li, s, orc.Q4_K, seed=5)
        om.set_weight(max(li, 0), s, data, dt)
        m.set_weight(li, s, data, dt)
    prompt = [3, 14, 159, 265, 358]
    assert np.abs(m.forward(prompt, 0) - om.forward(prompt, 0)).max() <= 1e-3
    tok = 42
    for pos in range(len(prompt), len(prompt) + 4):
        nxt, lg = m.decode_step([tok], pos, want_logits=True)
        lo = om.forward([tok], pos)[0]
        assert np.abs(lg[0] - lo).max() <= 1e-3
        tok = int(nxt[0])
    m.close()
