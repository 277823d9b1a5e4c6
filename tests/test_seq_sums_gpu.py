"""The device sampler's summation against the reference's sequential f32
loops (src/ops.rs:1219-1223, src/sampler.rs:107-113, :140-148).

The device adds a window of terms at once while the running sum stays in
one binade and adds ties, binade crossings, infinities and NaNs one at a
time; every running sum must equal the sequential loop's bit for bit. The
inputs below reach each of those cases: ties (powers of two, small
integers, dyadic fractions), subnormal terms and sums, zeros, terms far
above the running sum, and a window boundary in the middle of a run."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _sequential(x):
    return np.add.accumulate(np.asarray(x, np.float32), dtype=np.float32)


def _cases():
    rng = np.random.default_rng(7)
    yield "uniform", rng.random(151_936, dtype=np.float32)
    yield "exps", np.exp(-rng.random(151_936) * 20).astype(np.float32)
    yield "powers_of_two", np.ldexp(1.0, rng.integers(-30, 10, 40_000)).astype(np.float32)
    yield "small_ints", rng.integers(0, 8, 40_000).astype(np.float32)
    yield "subnormals", rng.integers(0, 1 << 23, 30_000).astype(np.uint32).view(np.float32)
    big = rng.random(50_000).astype(np.float32) * np.float32(1e-3)
    big[rng.random(50_000) < 0.02] = np.float32(1e6)
    yield "rare_large", big
    yield "dyadic", (rng.integers(0, 1000, 60_000) / 1024.0).astype(np.float32)
    z = rng.random(20_000).astype(np.float32)
    z[rng.random(20_000) < 0.3] = 0.0
    yield "zeros", z
    yield "one_term", np.array([0.375], np.float32)
    yield "window_edge", np.full(8192 * 3 + 5, 1.0, np.float32)
    w = rng.random(9_000).astype(np.float32)
    w[4_000] = np.inf
    yield "infinity", w
    # a flat softmax of the headline vocabulary: what the top-p sampler adds
    logits = rng.standard_normal(151_936).astype(np.float32) * np.float32(0.5)
    e = np.exp(logits - logits.max()).astype(np.float32)
    p = (e * (np.float32(1) / _sequential(e)[-1])).astype(np.float32)
    yield "sorted_probs", np.sort(p)[::-1].copy()


@pytest.mark.parametrize("name,x", list(_cases()), ids=[c[0] for c in _cases()])
def test_seq_sums_bit_exact(name, x):
    import cosxamix_b200 as cx
    got = cx.seq_sums(x)
    want = _sequential(x)
    np.testing.assert_array_equal(got.view(np.uint32), want.view(np.uint32))
