"""GPU parity of the non-GEMV ComputeBackend methods against the oracle
(cpu_backend.rs / ops.rs semantics), replaying the reference's own op tests
(crates/beacon-core/src/tests.rs:67-333) on the device plus seeded cases.
Float tolerances are stated per test; copies and indices are exact."""
import math

import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.fixture(scope="module")
def s(be):
    return be.new_stream()


def up(be, a):
    return be.upload(np.ascontiguousarray(a, dtype=np.float32))


def test_matmul_known_and_random(be, s):
    c = be.matmul(s, up(be, [[1, 2], [3, 4]]), up(be, [[5, 6], [7, 8]])).numpy()
    assert np.array_equal(c, np.array([[19, 22], [43, 50]], np.float32))   # tests.rs:67-80
    rng = np.random.default_rng(0)
    a, b = rng.standard_normal((7, 33)).astype(np.float32), rng.standard_normal((33, 5)).astype(np.float32)
    assert np.allclose(be.matmul(s, up(be, a), up(be, b)).numpy(), orc.matmul_f32(a, b), atol=1e-5)


def test_rms_norm(be, s):
    x = np.array([1, 2, 3, 4], np.float32)
    got = be.rms_norm(s, up(be, x), up(be, np.ones(4)), 1e-5).numpy()
    assert np.allclose(got, orc.rms_norm(x, np.ones(4, np.float32), 1e-5), atol=1e-6)   # tests.rs:96-117
    rng = np.random.default_rng(1)
    x = rng.standard_normal((5, 2048)).astype(np.float32)
    w = (1 + 0.1 * rng.standard_normal(2048)).astype(np.float32)
    assert np.allclose(be.rms_norm(s, up(be, x), up(be, w), 1e-5).numpy(), orc.rms_norm(x, w, 1e-5),
                       rtol=1e-5, atol=1e-6)


def test_rope(be, s):
    x = np.array([[1.0, 0.0, 1.0, 0.0]], np.float32)
    g = be.rope(s, up(be, x), 1, 10000.0, 4).numpy()[0]
    assert abs(g[0] - math.cos(1.0)) < 1e-5 and abs(g[1] - math.sin(1.0)) < 1e-5   # ops tests.rs:180-197
    rng = np.random.default_rng(2)
    x = rng.standard_normal((1, 4, 9, 64)).astype(np.float32)
    for pos, theta in [(0, 10000.0), (37, 10000.0), (4090, 500000.0)]:
        got = be.rope(s, up(be, x), pos, theta, 64).numpy()
        # libm and CUDA powf/sinf/cosf may differ by an ulp; the f32 angle
        # pos*freq then carries ~pos * 2^-23 absolute error, so the bound
        # grows with the position.
        tol = 2e-5 + 4 * (pos + 1) * 2.0 ** -23 * np.abs(x).max()
        assert np.allclose(got, orc.rope(x, pos, theta, 64), atol=tol), pos


def test_silu_softmax_add_mul(be, s):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((3, 100)) * 4).astype(np.float32)
    y = rng.standard_normal((3, 100)).astype(np.float32)
    assert np.allclose(be.silu(s, up(be, x)).numpy(), orc.silu(x), rtol=1e-6, atol=1e-6)
    assert np.allclose(be.softmax(s, up(be, x), -1).numpy(), orc.softmax(x), rtol=1e-5, atol=1e-7)
    assert np.array_equal(be.add(s, up(be, x), up(be, y)).numpy(), orc.add(x, y))
    assert np.array_equal(be.mul(s, up(be, x), up(be, y)).numpy(), orc.mul(x, y))


def test_silu_known(be, s):   # beacon-core tests.rs:133-145
    r = be.silu(s, up(be, [0.0, 1.0, -1.0])).numpy()
    assert abs(r[0]) < 1e-6 and abs(r[1] - 0.7311) < 1e-3 and abs(r[2] + 0.2689) < 1e-3


def test_add_length_mismatch(be, s):
    from beacon_cuda import ShapeMismatch
    with pytest.raises(ShapeMismatch):
        be.add(s, up(be, [1, 2, 3]), up(be, [1, 2]))


def test_reshape_swapaxes_transpose(be, s):
    from beacon_cuda import ShapeMismatch
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2, 3, 4, 5)).astype(np.float32)
    t = up(be, x)
    assert np.array_equal(be.reshape(s, t, [6, 20]).numpy(), x.reshape(6, 20))
    assert np.array_equal(be.swapaxes(s, t, 1, 2).numpy(), np.swapaxes(x, 1, 2))
    assert np.array_equal(be.swapaxes(s, t, -1, 0).numpy(), np.swapaxes(x, -1, 0))
    assert np.array_equal(be.transpose(s, t).numpy(), np.swapaxes(x, -1, -2))
    with pytest.raises(ShapeMismatch):                                    # tests.rs:196-204
        be.reshape(s, up(be, [1, 2, 3]), [2, 2])


def test_embedding(be, s):
    from beacon_cuda import ShapeMismatch
    w = up(be, [[0.1, 0.2], [0.3, 0.4], [0.5, 0.6]])
    r = be.embedding(s, w, be.create_token_tensor([2, 0])).numpy()      # tests.rs:206-222
    assert np.allclose(r, [[0.5, 0.6], [0.1, 0.2]])
    wf16 = np.random.default_rng(5).standard_normal((50, 64)).astype(np.float16)
    r = be.embedding(s, be.upload(wf16), be.create_token_tensor([49, 7, 7])).numpy()
    assert np.array_equal(r, wf16[[49, 7, 7]].astype(np.float32))
    with pytest.raises(ShapeMismatch):
        be.embedding(s, w, be.create_token_tensor([3]))


def test_kv_cache_update_in_place(be, s):
    from beacon_cuda import ContextOverflow
    ck, cv = be.zeros((4, 1, 2)), be.zeros((4, 1, 2))
    kk, vv = be.kv_cache_update(s, ck, cv, up(be, [[[1.0, 2.0]]]), up(be, [[[3.0, 4.0]]]), 0)
    assert kk.shape == (1, 1, 2) and np.array_equal(kk.numpy().reshape(-1), [1, 2])   # tests.rs:295-316
    assert np.array_equal(vv.numpy().reshape(-1), [3, 4])
    kk, vv = be.kv_cache_update(s, ck, cv, up(be, [[[5.0, 6.0]]]), up(be, [[[7.0, 8.0]]]), 1)
    # persisted: the first row is still there (the MLX semantics)
    assert np.array_equal(kk.numpy().reshape(-1), [1, 2, 5, 6])
    assert np.array_equal(ck.numpy().reshape(-1), [1, 2, 5, 6, 0, 0, 0, 0])
    with pytest.raises(ContextOverflow):
        be.kv_cache_update(s, ck, cv, up(be, [[[1.0, 1.0]]]), up(be, [[[1.0, 1.0]]]), 4)
    # f16 cache, f32 rows
    ck16, cv16 = be.zeros((3, 2, 4), 1), be.zeros((3, 2, 4), 1)
    rows = np.random.default_rng(6).standard_normal((2, 2, 4)).astype(np.float32)
    kk, _ = be.kv_cache_update(s, ck16, cv16, up(be, rows), up(be, rows), 1)
    assert np.array_equal(kk.numpy()[1:], rows.astype(np.float16))


@pytest.mark.parametrize("case", ["single", "gqa", "random", "causal", "mask"])
def test_attention(be, s, case):
    rng = np.random.default_rng(8)
    if case == "single":                                                   # tests.rs:224-257
        q = np.array([1.0, 0.0], np.float32).reshape(1, 1, 1, 2)
        k = np.array([1.0, 0.0, 0.0, 1.0], np.float32).reshape(1, 1, 2, 2)
        v = np.array([1.0, 2.0, 3.0, 4.0], np.float32).reshape(1, 1, 2, 2)
        scale, mask, causal = 1.0, None, 0
    elif case == "gqa":                                                    # tests.rs:259-282
        q = np.array([1.0, 0.0, 0.0, 1.0], np.float32).reshape(1, 2, 1, 2)
        k = np.array([1.0, 1.0], np.float32).reshape(1, 1, 1, 2)
        v = np.array([2.0, 3.0], np.float32).reshape(1, 1, 1, 2)
        scale, mask, causal = 1.0, None, 0
    else:
        q = rng.standard_normal((2, 8, 5, 64)).astype(np.float32)
        k = rng.standard_normal((2, 2, 13, 64)).astype(np.float32)
        v = rng.standard_normal((2, 2, 13, 64)).astype(np.float32)
        scale = 0.125
        mask = (rng.standard_normal((5, 13)) * 3).astype(np.float32) if case == "mask" else None
        causal = 1 if case == "causal" else 0
    got = be.attention(s, up(be, q), up(be, k), up(be, v), up(be, mask) if mask is not None else None,
                       scale, causal).numpy()
    ref = orc.attention(q, k, v, scale, mask=mask, causal=bool(causal))
    assert np.allclose(got, ref, atol=2e-5, rtol=1e-5)


def test_attention_default_causal_rule(be, s):
    """causal=-1: causal exactly when no mask and seq_q > 1 (shim/src/ops.cpp:216-223)."""
    rng = np.random.default_rng(9)
    q = rng.standard_normal((1, 2, 4, 32)).astype(np.float32)
    k = rng.standard_normal((1, 2, 6, 32)).astype(np.float32)
    got = be.attention(s, up(be, q), up(be, k), up(be, k), None, 0.2, -1).numpy()
    assert np.allclose(got, orc.attention(q, k, k, 0.2, causal=True), atol=2e-5)


@pytest.mark.parametrize("vals", [
    [1.0, 5.0, 3.0], [9.0, 1.0, 2.0], [0.0, 0.0, 1.0],                   # scheduler tests.rs:21-28
    [3.0, 1.0, 3.0, 2.0], [1.0, np.nan, 0.5], [5.0, np.nan], [np.nan, np.nan, np.nan],
    [-0.0, 0.0, -0.0], [-np.inf, -np.inf],
])
def test_argmax_reference_rule(be, s, vals):
    x = np.array(vals, np.float32)
    got = int(be.argmax(s, up(be, x)).numpy()[0])
    assert got == orc.argmax(x)


def test_argmax_large_rows_with_ties(be, s):
    rng = np.random.default_rng(10)
    x = rng.integers(-5, 5, size=(4, 128256)).astype(np.float32)   # many exact ties
    x[2, 1000] = np.nan
    got = be.argmax(s, up(be, x)).numpy()
    assert [int(g) for g in got] == [orc.argmax(r) for r in x]
