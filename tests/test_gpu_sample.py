"""Device sampling against the oracle's restatement of sampling::sample
(crates/beacon-scheduler/src/sampling.rs:15-186), through the C ABI.

Each row's draw r is given to both sides (the reference draws it from an
unseeded thread RNG). The device sums the vocabulary in parallel, so a token
may differ from the oracle's only when r lies within rounding of a cumulative
boundary between the two tokens (checked on the oracle's final distribution,
tolerance 1e-5), or at a top-p cut within rounding of p; every other case
must pick the oracle's token.
"""
import numpy as np
import pytest

import oracle as orc

pytestmark = pytest.mark.gpu

BOUNDARY_TOL = 1e-5


@pytest.fixture(scope="module")
def be(cuda_lib):
    from beacon_cuda import CudaBackend
    return CudaBackend(0)


@pytest.fixture(scope="module")
def stream(be):
    return be.new_stream()


CASES = [
    dict(temperature=0.0),
    dict(temperature=0.0, repeat_penalty=1.3),
    dict(temperature=1.0),
    dict(temperature=0.7, top_k=40),
    dict(temperature=1.0, top_k=0),
    dict(temperature=1.3, top_p=0.9),
    dict(temperature=1.0, top_p=0.5),
    dict(temperature=1.0, min_p=0.05),
    dict(temperature=0.8, top_k=50, top_p=0.95, min_p=0.02, repeat_penalty=1.1),
    dict(temperature=1.2, top_p=1.0, min_p=0.0, repeat_penalty=0.9),
]


def _check(label, got, o_tok, probs, r):
    """A different token is allowed only when r lies between the reference's
    sequential f32 cumulative sum and the exact one at a boundary between the
    two tokens (the f32 sum drifts by ~1e-5 over 10^5 terms), with
    BOUNDARY_TOL of slack for the device's own rounding."""
    if got == o_tok:
        return False
    c32 = np.cumsum(probs, dtype=np.float32).astype(np.float64)   # sequential, as sampling.rs:176-183
    c64 = np.cumsum(probs.astype(np.float64))
    lo, hi = min(got, o_tok), max(got, o_tok)
    a, b = np.minimum(c32[lo:hi], c64[lo:hi]), np.maximum(c32[lo:hi], c64[lo:hi])
    gap = float(np.maximum(np.maximum(a - r, r - b), 0.0).min()) if hi > lo else 1.0
    assert gap <= BOUNDARY_TOL, f"{label}: device {got} vs oracle {o_tok}, r={r} is {gap:.2e} from a boundary"
    return True


@pytest.mark.parametrize("V", [1000, 32000, 128256])
@pytest.mark.parametrize("case", range(len(CASES)))
def test_sample_matches_oracle(be, stream, V, case):
    from beacon_cuda import _lib as L
    params = CASES[case]
    rows = 4
    rng = np.random.default_rng(1000 * case + V % 997)
    logits = (rng.standard_normal((rows, V)) * 3.0).astype(np.float32)
    prev = rng.integers(0, V, size=(rows, 12)).astype(np.int32)
    prev[:, 6:] = prev[:, :6]                      # repeated tokens are penalised once per occurrence
    r = rng.random(rows).astype(np.float32)
    got = be.sample(stream, be.upload(logits), L.sampling_params(**params), be.upload(r), be.upload(prev)).numpy()
    near = 0
    for i in range(rows):
        o_tok, probs = orc.sample(logits[i], prev[i].astype(np.uint32), orc.sample_params(**params), float(r[i]))
        near += _check(f"V={V} case {case} row {i}", int(got[i]), o_tok, probs, float(r[i]))
    assert near <= 1


def test_sample_edge_cases(be, stream):
    """Draw 0 takes index 0 (cumulative >= r holds at once); top_k = Some(k)
    keeps every value >= the k-th largest (ties included); penalties skip
    out-of-range ids; a row of one token."""
    from beacon_cuda import _lib as L
    lg = np.array([[1.0, 3.0, 3.0, 2.0, 0.5], [0.0, 1.0, 2.0, 3.0, 4.0]], np.float32)
    prev = np.array([[7, -1], [4, 4]], np.int32)   # out of range ids are skipped
    p = dict(temperature=1.0, top_k=1, repeat_penalty=1.5)
    for r in (0.0, 0.3, 0.7, 0.9999):
        got = be.sample(stream, be.upload(lg), L.sampling_params(**p), be.upload(np.array([r, r], np.float32)),
                        be.upload(prev)).numpy()
        for i in range(2):
            o_tok, probs = orc.sample(lg[i], prev[i].astype(np.uint32), orc.sample_params(**p), r)
            _check(f"edge row {i} r={r}", int(got[i]), o_tok, probs, r)
    one = be.sample(stream, be.upload(np.array([[5.0]], np.float32)), L.sampling_params(temperature=1.0),
                    be.upload(np.array([0.5], np.float32))).numpy()
    assert one.tolist() == [0]


def test_decode_step_sampled_matches_host_sampling(be):
    """The sampled decode step picks what the oracle's sampler picks from
    the same step's logits (read back through the host path)."""
    from beacon_cuda import CudaModel, DecoderConfig
    from beacon_cuda import _lib as L
    from golden_models import make_weights
    c = dict(vocab_size=1000, hidden_size=512, num_layers=2, num_heads=8, num_kv_heads=2, head_dim=64,
             intermediate_size=1024, max_context=64, rope_theta=10000.0, rms_norm_eps=1e-5)
    w = make_weights(orc.OracleModelConfig(**c), orc.Q4_K, seed=91)
    m = CudaModel(be, DecoderConfig(**c, numerics=L.NUMERICS_FAST, kv_dtype=L.DTYPE_F16, max_batch=4))
    for (layer, which), (data, dt) in w.items():
        m.set_weight(layer, which, data, dt)
    rng = np.random.default_rng(92)
    toks = [5, 77, 300, 999]
    prev = rng.integers(0, 1000, size=(4, 8)).astype(np.uint32)
    params = dict(temperature=0.9, top_k=60, top_p=0.92, repeat_penalty=1.15)
    near = 0
    for pos in range(6):
        r = rng.random(4).astype(np.float32)
        _, lg = m.decode_step(toks, pos, want_logits=True)       # same inputs, same cache row: same logits
        nxt = m.decode_step_sampled(toks, pos, L.sampling_params(**params), r, prev)
        for b in range(4):
            o_tok, probs = orc.sample(lg[b], prev[b], orc.sample_params(**params), float(r[b]))
            near += _check(f"step {pos} seq {b}", int(nxt[b]), o_tok, probs, float(r[b]))
        toks = [int(t) for t in nxt]
    assert near <= 1
    m.close()
