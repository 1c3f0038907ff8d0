"""Pins the CPU oracle to the reference's own known-answer tests.

Every case below is a replay of a reference unit test (file:line cited) or a
value that follows directly from the reference function's definition
(dequant.rs:116-152 for the round-toward-zero f16 conversion). The oracle is
only trusted as the CUDA parity checker once these pass.
"""
import math
import struct

import numpy as np
import pytest

import oracle as orc


def f32_to_f16_approx(v: float) -> int:
    """beacon-kernels/src/tests.rs:36-50 (the test helper that packs scales)."""
    bits = struct.unpack("<I", struct.pack("<f", v))[0]
    sign = (bits >> 16) & 0x8000
    exp = ((bits >> 23) & 0xFF) - 127 + 15
    man = (bits >> 13) & 0x3FF
    if exp <= 0:
        return sign
    if exp >= 31:
        return sign | 0x7C00
    return sign | (exp << 10) | man


def build_q4_block(scale: float, weights) -> np.ndarray:
    """beacon-kernels/src/tests.rs:14-28."""
    blk = np.zeros(18, dtype=np.uint8)
    s = f32_to_f16_approx(scale)
    blk[0], blk[1] = s & 0xFF, s >> 8
    for i in range(16):
        lo = (weights[2 * i] + 8) & 0xFF
        hi = (weights[2 * i + 1] + 8) & 0xFF
        blk[2 + i] = ((hi << 4) | (lo & 0x0F)) & 0xFF
    return blk


# --- f16 conversions -------------------------------------------------------

def test_f16_known_values():  # q4.rs:256-264
    assert orc.f16_to_f32(0x0000) == 0.0
    assert orc.f16_to_f32(0x3C00) == 1.0
    assert orc.f16_to_f32(0xBC00) == -1.0
    assert orc.f16_to_f32(0x4000) == 2.0
    assert orc.f16_to_f32(0x3800) == 0.5


def test_f16_subnormal_and_special():  # dequant.rs:85-104
    assert orc.f16_to_f32(0x0001) == 2.0 ** -24
    assert orc.f16_to_f32(0x03FF) == 1023 * 2.0 ** -24
    assert orc.f16_to_f32(0x7C00) == math.inf
    assert orc.f16_to_f32(0xFC00) == -math.inf
    assert math.isnan(orc.f16_to_f32(0x7E00))


def test_f32_f16_roundtrip():  # dequant.rs:620-631
    for v in [0.0, 1.0, -1.0, 0.5, -0.5, 42.0, 0.001]:
        back = orc.f16_to_f32(orc.f32_to_f16_rtz(v))
        assert abs(back - v) < 0.01 or abs(back - v) / max(abs(v), 1e-6) < 0.01


@pytest.mark.parametrize("v,bits", [
    (1.0 + 2.0 ** -10, 0x3C01),
    (1.0 + 3 * 2.0 ** -12, 0x3C00),   # truncates where nearest-even would round up
    (-(1.0 + 3 * 2.0 ** -12), 0xBC00),
    (65519.0, 0x7BFF),
    (65536.0, 0x7C00),                # overflow goes to Inf, not 65504
    (1e6, 0x7C00),
    (-1e6, 0xFC00),
    (2.0 ** -24, 0x0001),             # smallest subnormal
    (1.5 * 2.0 ** -24, 0x0001),
    (2.0 ** -25, 0x0000),             # flushed
    (-1e-8, 0x8000),
    (2.0 ** -14, 0x0400),
    (math.inf, 0x7C00),
])
def test_f32_to_f16_rtz_definition(v, bits):  # dequant.rs:116-152
    assert orc.f32_to_f16_rtz(v) == bits


def test_f32_to_f16_rtz_nan_payload():  # dequant.rs:122-128
    bits = np.array([0x7FC00000, 0x7F800001, 0xFF800010, 0x7F802000], dtype=np.uint32)
    out = orc.f32_to_f16_rtz_array(bits.view(np.float32))
    # payload >> 13, clamped to at least 1 so a NaN never becomes Inf
    assert list(out) == [0x7E00, 0x7C01, 0xFC01, 0x7C01]


def test_rtz_matches_numpy_truncation_on_random_values():
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(20000) * 10.0).astype(np.float32)
    ours = orc.f32_to_f16_rtz_array(x)
    # numpy rounds to nearest: the truncated value never has a larger magnitude
    rne = x.astype(np.float16).view(np.uint16)
    assert np.all(np.abs(ours.view(np.float16).astype(np.float32)) <= np.abs(x))
    assert np.all((ours == rne) | (np.abs(ours.astype(np.int32) - rne.astype(np.int32)) == 1))


def test_rne_matches_numpy():
    rng = np.random.default_rng(1)
    x = np.concatenate([(rng.standard_normal(20000) * s).astype(np.float32)
                        for s in (1e-6, 1e-3, 1.0, 1e3, 2e4)])
    ours = orc.f32_to_f16_rne_array(x)
    assert np.array_equal(ours, x.astype(np.float16).view(np.uint16))


# --- dequantization --------------------------------------------------------

def test_dequant_q4_0_aa():  # dequant.rs:633-649
    blk = np.array([0x00, 0x3C] + [0xAA] * 16, dtype=np.uint8)
    out = orc.dequantize_to_f16(blk, orc.Q4_0, 32)
    assert np.all(out.view(np.float16).astype(np.float32) == 2.0)


def test_dequant_q8_0():  # dequant.rs:651-667
    blk = np.array([0x00, 0x38] + [4] * 32, dtype=np.uint8)
    out = orc.dequantize_to_f16(blk, orc.Q8_0, 32)
    assert np.all(out.view(np.float16).astype(np.float32) == 2.0)


def test_dequant_q4_0_zeros():  # dequant.rs:669-684, q4.rs:266-285
    blk = np.array([0x00, 0x3C] + [0x88] * 16, dtype=np.uint8)
    assert np.all(orc.dequantize_to_f16(blk, orc.Q4_0, 32) == 0)
    assert np.all(orc.q4_dequantize_block(blk) == 0.0)


def test_q4_dequantize_known_values():  # beacon-kernels/src/tests.rs:52-77
    out = orc.q4_dequantize_block(build_q4_block(0.5, [1] * 32))
    assert np.all(np.abs(out - 0.5) < 0.01)
    w = [0] * 32
    w[:5] = [-7, -3, 0, 3, 7]
    out = orc.q4_dequantize_block(build_q4_block(2.0, w))
    assert abs(out[0] + 14) < 0.1 and abs(out[1] + 6) < 0.1 and abs(out[2]) < 0.1
    assert abs(out[3] - 6) < 0.1 and abs(out[4] - 14) < 0.1


def test_q4_nibble_order_interleaved_vs_split():  # dequant.rs:170-176
    blk = np.array([0x00, 0x3C] + [(i & 0xF) | ((15 - (i & 0xF)) << 4) for i in range(16)],
                   dtype=np.uint8)
    inter = orc.dequantize_to_f32(blk, orc.Q4_0, 32, orc.NIBBLE_REF_INTERLEAVED)
    split = orc.dequantize_to_f32(blk, orc.Q4_0, 32, orc.NIBBLE_GGUF_SPLIT)
    for i in range(16):
        assert inter[2 * i] == i - 8 and inter[2 * i + 1] == (15 - i) - 8
        assert split[i] == i - 8 and split[i + 16] == (15 - i) - 8


def pack_k_scales(sc, mn) -> list:
    """Inverse of decode_k_scales_mins (dequant.rs:289-307), written from its doc."""
    q = [0] * 12
    for j in range(4):
        q[j] = sc[j] | ((sc[j + 4] >> 4) << 6)
        q[j + 4] = mn[j] | ((mn[j + 4] >> 4) << 6)
        q[j + 8] = (sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4)
    return q


def test_dequant_q4_k_hand_computed():  # dequant.rs:318-365
    sc = [1, 2, 3, 63, 17, 33, 48, 5]
    mn = [0, 1, 62, 3, 20, 40, 1, 63]
    qs = [((j % 16) | ((15 - j % 16) << 4)) for _ in range(4) for j in range(32)]
    blk = np.array([0x00, 0x3C, 0x00, 0x38] + pack_k_scales(sc, mn) + qs, dtype=np.uint8)
    out = orc.dequantize_to_f16(blk, orc.Q4_K, 256).view(np.float16).astype(np.float32)
    for p in range(4):
        for j in range(32):
            assert out[64 * p + j] == (j % 16) * sc[2 * p] * 1.0 - mn[2 * p] * 0.5
            assert out[64 * p + 32 + j] == (15 - j % 16) * sc[2 * p + 1] * 1.0 - mn[2 * p + 1] * 0.5


def test_block_tables():  # dtype.rs:56-82
    assert (orc.block_size(orc.Q4_0), orc.block_bytes(orc.Q4_0)) == (32, 18)
    assert (orc.block_size(orc.Q8_0), orc.block_bytes(orc.Q8_0)) == (32, 34)
    assert (orc.block_size(orc.Q4_K), orc.block_bytes(orc.Q4_K)) == (256, 144)
    assert orc.block_bytes(orc.Q6_K) == 210 and orc.block_bytes(orc.Q8_K) == 292


@pytest.mark.parametrize("dtype", [orc.Q4_0, orc.Q8_0, orc.Q4_K])
def test_quantizer_roundtrip(dtype):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(4096) * 0.02).astype(np.float32)
    q = orc.quantize(x, dtype)
    assert q.size == 4096 // orc.block_size(dtype) * orc.block_bytes(dtype)
    back = orc.dequantize_to_f32(q, dtype, 4096)
    err = np.abs(back - x).max() / np.abs(x).max()
    assert err < {orc.Q4_0: 0.1, orc.Q8_0: 0.005, orc.Q4_K: 0.08}[dtype]


# --- GEMV / matmul -----------------------------------------------------------

def test_q4_dot_scalar():  # beacon-kernels/src/tests.rs:83-91
    assert abs(orc.q4_dot_f32(np.ones(32, np.float32), build_q4_block(1.0, [1] * 32)) - 32) < 1


def test_q4_matmul_scalar():  # beacon-kernels/src/tests.rs:93-109
    w = np.concatenate([build_q4_block(1.0, [1] * 32)] * 2)
    out = orc.q4_matmul_f32(w, np.ones(32, np.float32), 2)
    assert np.all(np.abs(out - 32) < 1)


def test_qgemv_matches_q4_matmul_bitwise():  # ops.rs:38-70 order
    rng = np.random.default_rng(5)
    w = orc.quantize((rng.standard_normal(64 * 256) * 0.02).astype(np.float32), orc.Q4_0)
    x = rng.standard_normal(256).astype(np.float32)
    a = orc.q4_matmul_f32(w, x, 64)
    b = orc.qgemv(w, orc.Q4_0, 64, 256, x)[0]
    assert np.array_equal(a, b)


def test_matmul_f32_known():  # beacon-kernels/src/tests.rs:115-128
    c = orc.matmul_f32(np.array([[1, 2, 3], [4, 5, 6]], np.float32),
                       np.array([[7, 8], [9, 10], [11, 12]], np.float32))
    assert np.array_equal(c, np.array([[58, 64], [139, 154]], np.float32))


def test_cpu_matmul_2x2_and_non_square():  # beacon-core/src/tests.rs:67-94
    c = orc.matmul_f32(np.array([[1, 2], [3, 4]], np.float32), np.array([[5, 6], [7, 8]], np.float32))
    assert np.array_equal(c, np.array([[19, 22], [43, 50]], np.float32))
    c = orc.matmul_f32(np.array([[1, 2, 3]], np.float32), np.array([[4], [5], [6]], np.float32))
    assert abs(c[0, 0] - 32) < 1e-6


# --- element-wise ops ----------------------------------------------------------

def test_rms_norm_known():  # beacon-kernels/src/tests.rs:135-151; beacon-core tests.rs:96-117
    x = np.array([1, 2, 3, 4], np.float32)
    out = orc.rms_norm(x, np.ones(4, np.float32), 1e-5)
    rms = np.sqrt(np.float32(7.5) + np.float32(1e-5))
    assert np.all(np.abs(out - x / rms) < 1e-5)


def test_rms_norm_2d():  # beacon-core/src/tests.rs:119-131
    out = orc.rms_norm(np.array([[3, 4], [1, 0]], np.float32), np.ones(2, np.float32), 1e-5)
    assert out.shape == (2, 2)


def test_silu_known():  # beacon-kernels/src/tests.rs:153-163; beacon-core tests.rs:133-145
    x = np.array([0.0, 1.0, -1.0, 2.0], np.float32)
    exp = x * (1.0 / (1.0 + np.exp(-x)))
    assert np.all(np.abs(orc.silu(x) - exp) < 1e-6)
    y = orc.silu(np.array([0.0, 1.0, -1.0], np.float32))
    assert abs(y[0]) < 1e-6 and abs(y[1] - 0.7311) < 1e-3 and abs(y[2] + 0.2689) < 1e-3


def test_softmax_known():  # beacon-kernels/src/tests.rs:166-178
    y = orc.softmax(np.array([1.0, 2.0, 3.0], np.float32))
    assert abs(y.sum() - 1) < 1e-6 and y[0] < y[1] < y[2]


def test_rope_known():  # beacon-kernels/src/tests.rs:180-197
    y = orc.rope(np.array([[1.0, 0.0, 1.0, 0.0]], np.float32), 0, 10000.0, 4)[0]
    assert np.allclose(y, [1, 0, 1, 0], atol=1e-6)
    y = orc.rope(np.array([[1.0, 0.0, 1.0, 0.0]], np.float32), 1, 10000.0, 4)[0]
    assert abs(y[0] - math.cos(1.0)) < 1e-5 and abs(y[1] - math.sin(1.0)) < 1e-5


def test_add_mul_known():  # beacon-kernels/src/tests.rs:199-227; beacon-core tests.rs:163-183
    assert np.array_equal(orc.add(np.array([1, 2, 3], np.float32), np.array([10, 20, 30], np.float32)),
                          np.array([11, 22, 33], np.float32))
    assert np.array_equal(orc.mul(np.array([2, 3, 4], np.float32), np.array([5, 6, 7], np.float32)),
                          np.array([10, 18, 28], np.float32))


# --- attention -----------------------------------------------------------------

def test_attention_single_head():  # beacon-core/src/tests.rs:224-257
    q = np.array([1.0, 0.0], np.float32).reshape(1, 1, 1, 2)
    k = np.array([1.0, 0.0, 0.0, 1.0], np.float32).reshape(1, 1, 2, 2)
    v = np.array([1.0, 2.0, 3.0, 4.0], np.float32).reshape(1, 1, 2, 2)
    out = orc.attention(q, k, v, 1.0)
    s0 = math.exp(1) / (math.exp(1) + 1)
    s1 = 1 - s0
    assert abs(out[0, 0, 0, 0] - (s0 + 3 * s1)) < 1e-4
    assert abs(out[0, 0, 0, 1] - (2 * s0 + 4 * s1)) < 1e-4


def test_attention_gqa():  # beacon-core/src/tests.rs:259-282
    q = np.array([1.0, 0.0, 0.0, 1.0], np.float32).reshape(1, 2, 1, 2)
    k = np.array([1.0, 1.0], np.float32).reshape(1, 1, 1, 2)
    v = np.array([2.0, 3.0], np.float32).reshape(1, 1, 1, 2)
    out = orc.attention(q, k, v, 1.0)
    assert np.allclose(out.reshape(-1), [2, 3, 2, 3], atol=1e-5)


def test_attention_causal_masks_future_keys():
    rng = np.random.default_rng(7)
    q = rng.standard_normal((1, 2, 3, 4)).astype(np.float32)
    k = rng.standard_normal((1, 1, 5, 4)).astype(np.float32)
    v = rng.standard_normal((1, 1, 5, 4)).astype(np.float32)
    out = orc.attention(q, k, v, 0.5, causal=True)
    # query row s (of 3) sees keys [0, s + 2]
    for s in range(3):
        ref = orc.attention(q[:, :, s:s + 1], k[:, :, :s + 3], v[:, :, :s + 3], 0.5)
        assert np.allclose(out[:, :, s], ref[:, :, 0], atol=1e-6)


# --- argmax -------------------------------------------------------------------

def test_argmax_basic():  # beacon-scheduler/src/tests.rs:21-28, 10-19
    assert orc.argmax(np.array([1.0, 5.0, 3.0])) == 1
    assert orc.argmax(np.array([9.0, 1.0, 2.0])) == 0
    assert orc.argmax(np.array([0.0, 0.0, 1.0])) == 2
    assert orc.argmax(np.array([1.0, 3.0, 2.0, 0.5])) == 1


def test_argmax_tie_and_nan_rules():  # sampling.rs:60-66 (Iterator::max_by semantics)
    assert orc.argmax(np.array([3.0, 1.0, 3.0, 2.0])) == 2      # last of equal maxima
    assert orc.argmax(np.array([1.0, np.nan, 0.5])) == 2        # NaN compares Equal
    assert orc.argmax(np.array([5.0, np.nan])) == 1
    assert orc.argmax(np.array([], np.float32)) == 0


# --- engine ---------------------------------------------------------------------

def tiny_cfg(**kw):
    base = dict(vocab_size=64, hidden_size=32, num_layers=2, num_heads=4, num_kv_heads=2,
                head_dim=8, intermediate_size=64, max_context=16)
    base.update(kw)
    return orc.OracleModelConfig(**base)


def test_engine_decode_matches_prefill_when_persisting():
    """With the intended semantics, prefill logits of row s equal the logits
    of decoding the same tokens one at a time (engine.rs:190-241)."""
    from golden_models import build_oracle_model, make_weights
    cfg = tiny_cfg()
    w = make_weights(cfg, orc.Q8_0, seed=11)
    m = build_oracle_model(cfg, w)
    toks = [3, 17, 42, 5, 9]
    pre = m.forward(toks, 0)
    m.reset()
    rows = [m.forward([t], i)[0] for i, t in enumerate(toks)]
    assert np.allclose(pre, np.stack(rows), atol=2e-5)


def test_engine_literal_mode_differs_from_intended():
    """ref-literal (kv not persisted, no causal mask) vs ref-intended."""
    from golden_models import build_oracle_model, make_weights
    w = make_weights(tiny_cfg(num_layers=1), orc.Q8_0, seed=12)
    lit = build_oracle_model(tiny_cfg(num_layers=1, kv_persist=False, causal_prefill=False), w)
    intended = build_oracle_model(tiny_cfg(num_layers=1), w)
    toks = [1, 2, 3, 4]
    a, b = lit.forward(toks, 0), intended.forward(toks, 0)
    assert np.allclose(a[-1], b[-1], atol=1e-6)        # one layer: last row sees all keys either way
    assert not np.allclose(a[0], b[0], atol=1e-4)      # first row differs without the mask
    a1, b1 = lit.forward([7], 4), intended.forward([7], 4)
    assert not np.allclose(a1, b1, atol=1e-4)          # decode differs without the cache


def test_engine_context_overflow():  # engine.rs:366-368
    from golden_models import build_oracle_model, make_weights
    cfg = tiny_cfg(max_context=4)
    m = build_oracle_model(cfg, make_weights(cfg, orc.Q4_0, seed=1))
    with pytest.raises(RuntimeError, match="overflow"):
        m.forward([1, 2, 3, 4, 5], 0)


# --- sampling (crates/beacon-scheduler/src/tests.rs:10-75) -----------------------------

def test_sample_greedy_kat():
    """tests.rs:11-20: temperature 0 picks the highest logit."""
    assert orc.sample([1.0, 3.0, 2.0, 0.5], [], orc.sample_params(0.0), 0.5)[0] == 1


def test_sample_argmax_kat():
    """tests.rs:23-27."""
    assert orc.argmax(np.array([1.0, 5.0, 3.0], np.float32)) == 1
    assert orc.argmax(np.array([9.0, 1.0, 2.0], np.float32)) == 0
    assert orc.argmax(np.array([0.0, 0.0, 1.0], np.float32)) == 2


def test_sample_low_temperature_kat():
    """tests.rs:30-40: temperature 0.01 behaves like greedy, for any draw."""
    for r in (1e-6, 0.3, 0.999999):
        assert orc.sample([1.0, 10.0, 2.0], [], orc.sample_params(0.01), r)[0] == 1
    # r = 0.0 (rng.random() can return it) takes index 0 whatever its probability: cumulative >= r
    assert orc.sample([1.0, 10.0, 2.0], [], orc.sample_params(0.01), 0.0)[0] == 0


def test_sample_repeat_penalty_kat():
    """tests.rs:43-57: penalty 2 halves token 1's positive logit (5.0 -> 2.5)."""
    assert orc.sample([4.9, 5.0, 1.0], [1], orc.sample_params(0.0, repeat_penalty=2.0), 0.5)[0] == 0


def test_sample_top_k_kat():
    """tests.rs:60-75: top_k 2 keeps only tokens 1 and 2."""
    for r in np.linspace(1e-6, 0.999, 7):
        assert orc.sample([1.0, 10.0, 5.0, 0.1], [], orc.sample_params(0.001, top_k=2), float(r))[0] in (1, 2)


def test_sample_pipeline_definitions():
    """Values that follow from sampling.rs's definitions: top_k = Some(k) keeps
    every value >= the k-th largest (0-based), so k = 1 keeps two tokens; top_p
    keeps the smallest descending prefix whose mass exceeds p; min_p drops
    probabilities below min_p * max; the draw takes the first index whose
    cumulative probability reaches r; a repeated token is penalised once per
    occurrence; negative logits are multiplied by the penalty."""
    lg = np.log(np.array([0.1, 0.4, 0.2, 0.3], np.float32))
    _, p = orc.sample(lg, [], orc.sample_params(1.0, top_k=1), 0.5)
    assert (p > 0).tolist() == [False, True, False, True]
    _, p = orc.sample(lg, [], orc.sample_params(1.0, top_p=0.65), 0.5)    # 0.4 + 0.3 > 0.65
    assert (p > 0).tolist() == [False, True, False, True]
    _, p = orc.sample(lg, [], orc.sample_params(1.0, min_p=0.6), 0.5)     # 0.4 * 0.6 = 0.24: keeps 0.3, 0.4
    assert (p > 0).tolist() == [False, True, False, True]
    probs = np.array([0.1, 0.4, 0.2, 0.3], np.float32)
    assert orc.sample(lg, [], orc.sample_params(1.0), 0.05)[0] == 0
    assert orc.sample(lg, [], orc.sample_params(1.0), 0.45)[0] == 1
    assert orc.sample(lg, [], orc.sample_params(1.0), 0.65)[0] == 2
    assert orc.sample(lg, [], orc.sample_params(1.0), 0.95)[0] == 3
    _, p2 = orc.sample(lg, [1, 1], orc.sample_params(1.0, repeat_penalty=2.0), 0.5)
    _, p1 = orc.sample(lg, [1], orc.sample_params(1.0, repeat_penalty=4.0), 0.5)
    assert np.allclose(p2, p1, rtol=0, atol=1e-7)     # log(0.4) < 0: *2 *2 == *4
    assert np.isclose(probs.sum(), 1.0)
