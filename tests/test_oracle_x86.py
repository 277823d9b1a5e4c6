"""The oracle's x86 backend and its thread pool (CPU only).

The x86 backend runs what the reference runs on an AVX2/FMA/F16C host
(src/kernels/x86.rs, chosen by src/kernels/mod.rs:136-163). Only the timed CPU
baseline uses it; parity stays on the scalar backend. These tests pin its
kernels against the scalar restatement and against the reference's own
compiled kernels (live when oracle/_ref was built, and through the golden
vectors those kernels produced), the way the reference tests its AVX2 kernels
against its scalar ones (src/kernels/mod.rs:808-970, src/ops.rs:1567-1606).
"""
import os
import threading

import numpy as np
import pytest

from oracle import oracle as O
from tests.golden.make_golden import finite_row

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_dots.npz")


def _term_scale(t, row, xq, xe, xs):
    """Sum of the magnitudes of the row's sub-block terms (from the unpacked
    row: value scale, offset, activation scale and sum per sub-block). Two
    float orders of the same terms differ by a few ulps of this, whatever
    the row total cancels to."""
    sub = O.SUB[t]
    q, e, d = O.unpack_i8(t, row, xq.size)
    prod = np.abs(q.astype(np.float64) * xq.astype(np.float64)).reshape(-1, sub).sum(1)
    mag = np.abs(e.astype(np.float64) * xe) * prod + np.abs(d.astype(np.float64) * xe * xs)
    return max(float(mag.sum()), 1e-30)


def _x86_dot(t, row, xq, xe, xs):
    f = {O.Q4K: O.lib().orc_x86_dot_q4k, O.Q6K: O.lib().orc_x86_dot_q6k}[t]
    return f(O.ptr(row), O.ptr(xq), O.ptr(xe), O.ptr(xs), xq.size // 256)


@pytest.mark.parametrize("t", [O.Q4K, O.Q6K])
def test_avx2_fused_matches_scalar_on_reference_pattern(t):
    # the byte pattern and input of src/kernels/mod.rs:808-902: relative 1e-4
    nb = 8
    row = np.array([(i * 131 + 17) % 251 for i in range(nb * O.BLOCK_BYTES[t])], np.uint8)
    x = np.sin(np.arange(nb * 256, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    xq, xe, xs = O.quantize_i8(x, O.SUB[t])
    want = O.dot_row(t, row, xq, xe, xs)
    got = _x86_dot(t, row, xq, xe, xs)
    assert abs(got - want) / max(abs(want), 1.0) < 1e-4


@pytest.mark.parametrize("t", [O.Q4K, O.Q6K])
def test_avx2_fused_matches_scalar_on_random_rows(t):
    rng = np.random.default_rng(40 + t)
    for nb in (1, 3, 8, 43):
        for _ in range(20):
            row = finite_row(rng, t, nb)
            xq, xe, xs = O.quantize_i8(rng.standard_normal(nb * 256).astype(np.float32), O.SUB[t])
            want = O.dot_row(t, row, xq, xe, xs)
            got = _x86_dot(t, row, xq, xe, xs)
            assert abs(got - want) / _term_scale(t, row, xq, xe, xs) < 1e-6, (nb, got, want)


def test_avx2_q4k_matches_reference_golden():
    # the Q4_K outputs of the reference's own assembly kernel
    g = np.load(GOLDEN)
    seen = 0
    for i in range(int(g["n"][0])):
        if int(g[f"c{i}_type"][0]) != O.Q4K:
            continue
        row, xq, xe, xs = g[f"c{i}_row"], g[f"c{i}_xq"], g[f"c{i}_xe"], g[f"c{i}_xs"]
        got = _x86_dot(O.Q4K, row, xq, xe, xs)
        for ref in g[f"c{i}_ref"]:
            assert abs(got - float(ref)) / _term_scale(O.Q4K, row, xq, xe, xs) < 1e-6
            seen += 1
    assert seen >= 3


def test_avx2_q4k_scales_equal_the_readable_unpack():
    # src/kernels/mod.rs:913-970: the word-mask unpack of the eight 6-bit
    # scales gives d*scale*xe bit for bit over 5000 xorshift blocks; the mins
    # (through one FMA) within 1e-5
    state = 0x9E3779B97F4A7C15
    mask = (1 << 64) - 1

    def azar():
        nonlocal state
        state ^= (state << 13) & mask
        state ^= state >> 7
        state ^= (state << 17) & mask
        return state

    L = O.lib()
    sc, mn = np.zeros(8, np.float32), np.zeros(8, np.float32)
    for _ in range(5000):
        block = np.array([azar() & 0xFF for _ in range(144)], np.uint8)
        d = np.float32(0.001) + np.float32(azar() % 1000) * np.float32(1e-5)
        dmin = np.float32(0.0005) + np.float32(azar() % 1000) * np.float32(1e-5)
        block[0:2] = np.frombuffer(np.uint16(O.f32_to_f16(float(d))).tobytes(), np.uint8)
        block[2:4] = np.frombuffer(np.uint16(O.f32_to_f16(float(dmin))).tobytes(), np.uint8)
        xe = np.array([np.float32(azar() % 1000) * np.float32(1e-3) for _ in range(8)], np.float32)
        xs = np.array([np.float32(azar() % 4000) - np.float32(2000) for _ in range(8)], np.float32)
        L.orc_x86_q4k_scales(O.ptr(block), O.ptr(xe), O.ptr(xs), O.ptr(sc), O.ptr(mn))
        _, e, off = O.unpack_i8(O.Q4K, block, 256)  # e = d*scale, off = -(dmin*min)
        np.testing.assert_array_equal(sc.view(np.uint32), (e * xe).astype(np.float32).view(np.uint32))
        want = np.float32(0)
        for j in range(8):
            want = np.float32(want + np.float32(np.float32(-off[j] * xe[j]) * xs[j]))
        got = np.float32(0)
        for v in mn:  # the lanes summed in order, in f32, as the reference's check does
            got = np.float32(got + v)
        assert abs(float(got) - float(want)) <= abs(float(want)) * 1e-5 + 1e-6


def test_x86_backend_takes_reference_kernels_when_built():
    used = O.set_backend("x86")
    try:
        rng = np.random.default_rng(7)
        for t in (O.Q2K, O.Q3K, O.Q4K, O.Q5K, O.Q6K):
            row = finite_row(rng, t, 4)
            xq, xe, xs = O.quantize_i8(rng.standard_normal(1024).astype(np.float32), O.SUB[t])
            got = O.lib().orc_x86_dot_row(t, O.ptr(row), O.ptr(xq), O.ptr(xe), O.ptr(xs), 4)
            want = O.dot_row(t, row, xq, xe, xs)
            assert abs(got - want) / _term_scale(t, row, xq, xe, xs) < 1e-6, (t, used[t])
        if O.ref_lib() is not None:
            assert used[O.Q4K] == "reference cosxamix_q4k_completo"
            assert used[O.Q5K].startswith("reference ")
        assert used[O.Q6K].startswith("AVX2 restatement")
    finally:
        O.set_backend("scalar")
    assert O.backend() == "scalar"


@pytest.mark.parametrize("n", [1, 7, 8, 31, 32, 33, 128, 4097])
def test_avx2_dot_f32_odd_lengths(n):
    # the tail handling the reference tests with odd lengths (src/kernels/mod.rs:588-620)
    rng = np.random.default_rng(n)
    a, b = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    got = O.lib().orc_x86_dot_f32(O.ptr(a), O.ptr(b), n)
    want = float(a.astype(np.float64) @ b.astype(np.float64))
    assert abs(got - want) <= 1e-5 * float(np.abs(a.astype(np.float64) * b).sum()) + 1e-7


@pytest.mark.parametrize("n", [1, 8, 15, 16, 17, 2048, 2051])
def test_avx2_rmsnorm_matches_scalar(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    w = rng.uniform(0.5, 1.5, n).astype(np.float32)
    a, b = np.zeros(n, np.float32), np.zeros(n, np.float32)
    O.lib().orc_x86_rmsnorm(O.ptr(a), O.ptr(x), O.ptr(w), n, 1e-6)
    O.lib().orc_rmsnorm(O.ptr(b), O.ptr(x), O.ptr(w), n, 1e-6)
    np.testing.assert_allclose(a, b, rtol=2e-6, atol=1e-7)


def _tiny(tmp_path):
    import cosxamix_b200 as cx
    p = str(tmp_path / "tiny.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42, n_layer=2))
    return p


def test_x86_forward_close_to_scalar_and_scalar_untouched(tmp_path):
    m = O.Model(_tiny(tmp_path))
    prompt = [3, 1, 4, 1, 5, 9, 2, 6]
    ref = m.forward(O.Cache(m), prompt)
    O.set_backend("x86")
    try:
        fast = m.forward(O.Cache(m), prompt)
    finally:
        O.set_backend("scalar")
    # float order only: a flipped activation rounding moves logits by ~1e-3 of the range
    assert float(np.max(np.abs(fast - ref)) / (ref.max() - ref.min())) <= 1e-2
    np.testing.assert_array_equal(m.forward(O.Cache(m), prompt), ref)


def _matmul(x, w, t, k, n):
    out = np.zeros(n, np.float32)
    assert O.lib().orc_matmul_auto(1, k, n, O.ptr(x), O.ptr(w), w.size, t, O.ptr(out)) == 0
    return out


@pytest.mark.parametrize("backend", ["scalar", "x86"])
def test_pool_results_independent_of_thread_count(backend):
    rng = np.random.default_rng(3)
    k, n = 1024, 1000  # 32-row tasks with a ragged last one
    w = np.concatenate([finite_row(rng, O.Q4K, k // 256) for _ in range(n)])
    x = rng.standard_normal(k).astype(np.float32)
    O.set_backend(backend)
    try:
        O.set_threads(1)
        want = _matmul(x, w, O.Q4K, k, n)
        for th in (2, 3, 8, 5, 1, 8):
            O.set_threads(th)
            for _ in range(3):
                np.testing.assert_array_equal(_matmul(x, w, O.Q4K, k, n), want)
    finally:
        O.set_backend("scalar")
        O.set_threads(0)
    assert O.threads() == len(os.sched_getaffinity(0))  # 0: one per CPU this process may use


def test_pool_serialises_callers_on_several_threads():
    rng = np.random.default_rng(4)
    k, n = 512, 700
    w = np.concatenate([finite_row(rng, O.Q4K, k // 256) for _ in range(n)])
    xs = [rng.standard_normal(k).astype(np.float32) for _ in range(4)]
    O.set_threads(1)
    want = [_matmul(x, w, O.Q4K, k, n) for x in xs]
    O.set_threads(4)
    got = [None] * 4
    errors = []

    def run(i):
        try:
            for _ in range(5):
                got[i] = _matmul(xs[i], w, O.Q4K, k, n)
                np.testing.assert_array_equal(got[i], want[i])
        except Exception as e:  # noqa: BLE001 - reported below
            errors.append(e)

    ths = [threading.Thread(target=run, args=(i,)) for i in range(4)]
    for t in ths:
        t.start()
    for t in ths:
        t.join()
    O.set_threads(0)
    assert not errors, errors


@pytest.mark.parametrize("backend", ["scalar", "x86"])
def test_projections_in_one_region_equal_separate_calls(tmp_path, backend):
    # src/ops.rs:1613-1670: q/k/v (and gate/up) in one parallel region with the
    # input quantized once give the separate calls' values bit for bit; the
    # Q6_K model mixes sub-blocks of 16 and 32 in one region
    import cosxamix_b200 as cx
    paths = [_tiny(tmp_path)]
    p6 = str(tmp_path / "q6.gguf")
    cx.synth_write(p6, cx.synth_spec("tiny", seed=5, n_layer=2, mix=cx.MIX_Q4_K_M))  # Q6_K attn_v in layer 0
    paths.append(p6)
    O.set_backend(backend)
    try:
        for p in paths:
            m = O.Model(p)
            out = {}
            for varias in (1, 0):
                O.lib().orc_set_varias(varias)
                c = O.Cache(m)
                lg = [m.forward(c, [3, 1, 4, 1, 5])]
                for _ in range(4):
                    lg.append(m.forward(c, [int(np.argmax(lg[-1]))]))
                out[varias] = np.stack(lg)
            np.testing.assert_array_equal(out[1].view(np.uint32), out[0].view(np.uint32))
    finally:
        O.lib().orc_set_varias(1)
        O.set_backend("scalar")
