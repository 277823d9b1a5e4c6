"""The CPU oracle against the reference's known-answer tests and golden vectors.

Each test restates one of the reference's own unit tests (cited); the golden
vectors in tests/golden/ref_dots.npz are outputs of the reference's compiled C
and assembly kernels (see tests/golden/make_golden.py).
"""
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ref_dots.npz")


# ── f16 (src/quant.rs:812-826, :937-971) ──

def test_f16_special_values():
    assert O.f16_to_f32(0x0000) == 0.0
    assert math.copysign(1.0, O.f16_to_f32(0x8000)) == -1.0
    assert O.f16_to_f32(0x3C00) == 1.0
    assert O.f16_to_f32(0xBC00) == -1.0
    assert O.f16_to_f32(0x4000) == 2.0
    assert O.f16_to_f32(0x7BFF) == 65504.0
    assert math.isinf(O.f16_to_f32(0x7C00))
    assert math.isnan(O.f16_to_f32(0x7E00))
    assert O.f16_to_f32(0x0001) == 2.0 ** -24
    assert O.f16_to_f32(0x03FF) == 1023.0 * 2.0 ** -24


def test_f16_round_trip_and_ties_to_even():
    for v in [0.0, -0.0, 1.0, -1.0, 0.5, 2.0, 65504.0, -65504.0, 6.1035156e-5, 5.9604645e-8, 1.0 / 1024.0]:
        v32 = np.float32(v)
        back = np.float32(O.f16_to_f32(O.f32_to_f16(float(v32))))
        assert back.tobytes() == v32.tobytes(), v
    assert math.isinf(O.f16_to_f32(O.f32_to_f16(1e30)))
    assert math.isinf(O.f16_to_f32(O.f32_to_f16(-1e30)))
    assert math.isnan(O.f16_to_f32(O.f32_to_f16(float("nan"))))
    mid = (np.float32(O.f16_to_f32(0x3C00)) + np.float32(O.f16_to_f32(0x3C01))) / np.float32(2)
    assert O.f32_to_f16(float(mid)) == 0x3C00


def test_f16_matches_numpy_on_every_half():
    h = np.arange(65536, dtype=np.uint16)
    ours = np.array([O.f16_to_f32(int(x)) for x in h[::97]], np.float32)
    ref = h[::97].view(np.float16).astype(np.float32)
    same = (ours == ref) | (np.isnan(ours) & np.isnan(ref))
    assert same.all()


# ── dequantization and unpacking (src/quant.rs:829-839, :891-928) ──

def test_q8_0_by_hand():
    b = np.zeros(34, np.uint8)
    b[0:2] = [0x00, 0x3C]
    b[2] = 5
    b[3] = np.uint8(253)  # -3
    y = O.dequantize(O.Q8_0, b, 32)
    assert y[0] == 5.0 and y[1] == -3.0


def test_dequantize_rejects_bad_sizes():
    with pytest.raises(ValueError):
        O.dequantize(O.Q8_0, np.zeros(34, np.uint8), 17)
    with pytest.raises(ValueError):
        O.dequantize(O.Q8_0, np.zeros(10, np.uint8), 32)


@pytest.mark.parametrize("t,bb,vals,sub", [
    (O.Q8_0, 34, 32, 32), (O.Q5_0, 22, 32, 32), (O.Q2K, 84, 256, 16), (O.Q3K, 110, 256, 16),
    (O.Q4K, 144, 256, 32), (O.Q5K, 176, 256, 32), (O.Q6K, 210, 256, 16)])
def test_unpack_reconstructs_dequantization_exactly(t, bb, vals, sub):
    n = 3
    data = np.array([(i * 97 + 13) % 251 for i in range(n * bb)], np.uint8)
    want = O.dequantize(t, data, n * vals)
    q, e, d = O.unpack_i8(t, data, n * vals)
    rec = e.repeat(sub) * q.astype(np.float32) + d.repeat(sub)
    np.testing.assert_array_equal(rec, want)


# ── activation quantization (src/ops.rs:178-198) ──

def test_quantize_round_half_away_and_zero_block():
    x = np.zeros(64, np.float32)
    x[32:] = np.linspace(-1, 1, 32, dtype=np.float32)
    q, e, s = O.quantize_i8(x, 32)
    assert e[0] == 0.0 and (q[:32] == 0).all() and s[0] == 0.0
    amax = np.float32(1.0)
    inv = np.float32(127.0) / amax
    want = np.array([int(math.copysign(math.floor(abs(float(v * inv)) + 0.5), float(v))) for v in x[32:]], np.int8)
    np.testing.assert_array_equal(q[32:], want)
    assert e[1] == np.float32(1.0) / np.float32(127.0)
    assert s[1] == float(int(want.astype(np.int32).sum()))
    assert q.min() >= -127 and q.max() <= 127


# ── dots ──

def test_dot_i8_exact_at_extremes():
    # src/kernels/mod.rs:630-667
    lib = O.lib()
    for n in [0, 1, 7, 31, 32, 33, 64, 100, 2048, 2049]:
        a = np.array([max(np.int8(np.int32((i * 37) % 255).astype(np.int8)), -127) for i in range(n)], np.int8)
        b = np.array([max(np.int8(((i * 53) % 255 - 127)), -127) for i in range(n)], np.int8)
        want = int(a.astype(np.int64) @ b.astype(np.int64)) if n else 0
        assert lib.orc_dot_i8(O.ptr(a) if n else None, O.ptr(b) if n else None, n) == want
    for x, y in [(127, 127), (-127, 127), (-127, -127), (127, -127)]:
        a = np.full(2048, x, np.int8)
        b = np.full(2048, y, np.int8)
        assert lib.orc_dot_i8(O.ptr(a), O.ptr(b), 2048) == x * y * 2048


def _unpacked_dot(t, row, xq, xe, xs):
    sub = O.SUB[t]
    q, e, d = O.unpack_i8(t, row, xq.size)
    lib = O.lib()
    total = lib.orc_dot_i8_scaled(O.ptr(q), O.ptr(xq), O.ptr(e), O.ptr(xe), xq.size, sub)
    total = np.float32(total)
    for b in range(xq.size // sub):
        total = np.float32(total + np.float32(np.float32(d[b] * xe[b]) * xs[b]))
    return float(total)


@pytest.mark.parametrize("t", [O.Q4K, O.Q3K, O.Q5K, O.Q6K, O.Q2K])
def test_fused_equals_unpack_then_multiply(t):
    # src/kernels/mod.rs:808-902 (Q4_K/Q3_K/Q5_K) and src/ops.rs:1567-1606 (Q6_K)
    nb = 8
    k = nb * 256
    row = np.array([(i * 131 + 17) % 251 for i in range(nb * O.BLOCK_BYTES[t])], np.uint8)
    x = np.sin(np.arange(k, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
    xq, xe, xs = O.quantize_i8(x, O.SUB[t])
    want = _unpacked_dot(t, row, xq, xe, xs)
    got = O.dot_row(t, row, xq, xe, xs)
    assert abs(got - want) / max(abs(want), 1.0) < 1e-4


def test_subblock_sums_rebuild_the_dot():
    rng = np.random.default_rng(5)
    for t in (O.Q4K, O.Q5K, O.Q6K, O.Q3K, O.Q2K):
        nb = 4
        row = rng.integers(0, 256, nb * O.BLOCK_BYTES[t], dtype=np.uint8)
        x = rng.standard_normal(nb * 256).astype(np.float32)
        xq, xe, xs = O.quantize_i8(x, O.SUB[t])
        sums = O.subblock_sums(t, row, xq)
        q, e, d = O.unpack_i8(t, row, xq.size)
        # the unpacked values are the fused kernel's values minus a per-format bias
        bias = {O.Q4K: 0, O.Q5K: 0, O.Q2K: 0, O.Q3K: 4, O.Q6K: 32}[t]
        sub = O.SUB[t]
        for s in range(xq.size // sub):
            seg = slice(s * sub, (s + 1) * sub)
            want = int((xq[seg].astype(np.int64) * (q[seg].astype(np.int64) + bias)).sum())
            assert sums[s] == want


def test_oracle_matches_reference_kernels_golden():
    g = np.load(GOLDEN)
    n = int(g["n"][0])
    assert n >= 20
    for i in range(n):
        t = int(g[f"c{i}_type"][0])
        got = O.dot_row(t, g[f"c{i}_row"], g[f"c{i}_xq"], g[f"c{i}_xe"], g[f"c{i}_xs"])
        for ref in g[f"c{i}_ref"]:
            # the reference's kernels sum in AVX2 lane order; relative to the
            # magnitude of the sub-block terms the difference is float noise
            xe, xs = g[f"c{i}_xe"], g[f"c{i}_xs"]
            scale = max(abs(float(ref)), float(np.abs(xe).sum() * 127 * O.SUB[t] * 0.01), 1.0)
            assert abs(got - float(ref)) / scale < 2e-5, (i, t, got, ref)


def test_oracle_matches_live_reference_kernels_when_built():
    if O.ref_lib() is None:
        pytest.skip("oracle/_ref not built here")
    rng = np.random.default_rng(99)
    from tests.golden.make_golden import KERNELS, finite_row
    for t, ks in KERNELS.items():
        row = finite_row(rng, t, 5)
        x = rng.standard_normal(5 * 256).astype(np.float32)
        xq, xe, xs = O.quantize_i8(x, O.SUB[t])
        mine = O.dot_row(t, row, xq, xe, xs)
        for k in ks:
            r = O.ref_dot(k, row, xq, xe, xs)
            assert abs(mine - r) / max(abs(mine), 1.0) < 1e-4


# ── elementwise (src/kernels/scalar.rs:345-376) ──

def test_rmsnorm_properties():
    s = O.rmsnorm(np.array([1, 2, 3, 4], np.float32), np.ones(4, np.float32), 1e-6)
    assert abs(math.sqrt(float((s * s).sum()) / 4) - 1.0) < 1e-4
    p = np.array([2, 3, 4, 5], np.float32)
    np.testing.assert_allclose(O.rmsnorm(np.ones(4, np.float32), p, 1e-6), p, atol=1e-4)
    z = O.rmsnorm(np.zeros(8, np.float32), np.ones(8, np.float32), 1e-6)
    assert np.isfinite(z).all()


def test_silu():
    x = np.sin(np.arange(1024) * 0.37).astype(np.float32) * 40
    y = O.silu(x)
    np.testing.assert_allclose(y, x / (1 + np.exp(-x.astype(np.float64))), rtol=1e-5, atol=1e-6)


# ── softmax / RoPE / attention properties (src/ops.rs:1763-1845, :1959-2062) ──

def test_softmax_properties():
    x = O.softmax(np.array([1, 2, 3, 4], np.float32), 4)
    assert abs(x.sum() - 1) < 1e-6 and x[3] > x[2] > x[1]
    y = O.softmax(np.array([101, 102, 103, 104], np.float32), 4)
    np.testing.assert_allclose(x, y, atol=1e-6)
    z = O.softmax(np.array([90, 0, -90], np.float32), 3)
    assert np.isfinite(z).all() and abs(z[0] - 1) < 1e-6
    m = O.softmax(np.full(4, -np.inf, np.float32), 4)
    np.testing.assert_allclose(m, 0.25, atol=1e-6)
    two = O.softmax(np.array([0, 10, 10, 0], np.float32), 2)
    assert abs(two[0] + two[1] - 1) < 1e-6 and two[1] > two[0] and two[2] > two[3]
    with pytest.raises(ValueError):
        O.softmax(np.zeros(3, np.float32), 2)


def test_rope_identity_at_zero_and_norm_preserving():
    heads, dim, tokens = 2, 8, 3
    c, s = O.rope_tables(dim, 10000.0, 16)
    orig = np.sin(np.arange(tokens * heads * dim) * 0.37).astype(np.float32)
    x = O.rope(orig[: heads * dim], 1, heads, dim, c, s, 0)
    np.testing.assert_allclose(x, orig[: heads * dim], atol=1e-6)
    x = O.rope(orig, tokens, heads, dim, c, s, 5)
    half = dim // 2
    for t in range(tokens):
        for h in range(heads):
            b = t * heads * dim + h * dim
            before = orig[b:b + half] ** 2 + orig[b + half:b + dim] ** 2
            after = x[b:b + half] ** 2 + x[b + half:b + dim] ** 2
            np.testing.assert_allclose(before, after, atol=1e-5)
    assert (np.abs(x - orig) > 1e-3).any()
    with pytest.raises(ValueError):
        O.rope(orig, tokens, heads, dim, c, s, 14)


def test_rope_tables_f64_angle():
    c, s = O.rope_tables(128, 1e6, 4096)
    half = 64
    j = np.arange(half)
    import ctypes
    libm = ctypes.CDLL("libm.so.6")
    libm.powf.restype = ctypes.c_float
    libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]
    # f32 powf as Rust's f32::powf calls it, then the angle in f64
    freq = np.array([np.float32(1.0) / np.float32(libm.powf(1e6, float(np.float32(2.0 * jj) / np.float32(128))))
                     for jj in j], np.float32)
    p = 4095
    ang = p * freq.astype(np.float64)
    np.testing.assert_allclose(c[p * half:(p + 1) * half], np.cos(ang).astype(np.float32), atol=2e-7)
    np.testing.assert_allclose(s[p * half:(p + 1) * half], np.sin(ang).astype(np.float32), atol=2e-7)


def test_attention_properties():
    heads, kvh, dim = 4, 2, 8
    wq, wkv = heads * dim, kvh * dim
    q = np.sin(np.arange(wq) * 0.3).astype(np.float32)
    k = np.cos(np.arange(wkv) * 0.7).astype(np.float32)
    v = np.arange(wkv, dtype=np.float32)
    out = O.attention(q, k, v, 1, 1, heads, kvh, dim)
    for h in range(heads):
        g = h // (heads // kvh)
        np.testing.assert_allclose(out[h * dim:(h + 1) * dim], v[g * dim:(g + 1) * dim], atol=1e-5)
    total, tokens = 6, 3
    k = np.sin(np.arange(total * wkv) * 0.21).astype(np.float32)
    v = np.cos(np.arange(total * wkv) * 0.13).astype(np.float32)
    q = np.sin(np.arange(tokens * wq) * 0.37).astype(np.float32)
    out = O.attention(q, k, v, tokens, total, heads, kvh, dim)
    for h in range(heads):
        g = h // (heads // kvh)
        for d in range(dim):
            col = v[np.arange(total) * wkv + g * dim + d]
            for t in range(tokens):
                x = out[t * wq + h * dim + d]
                assert col.min() - 1e-5 <= x <= col.max() + 1e-5
    v2 = v.copy()
    v2[(total - 1) * wkv:] += 100
    out2 = O.attention(q, k, v2, tokens, total, heads, kvh, dim)
    np.testing.assert_allclose(out[: (tokens - 1) * wq], out2[: (tokens - 1) * wq], atol=1e-5)
    assert (np.abs(out[(tokens - 1) * wq:] - out2[(tokens - 1) * wq:]) > 1e-3).any()
    with pytest.raises(ValueError):
        O.attention(q, k, v, tokens, total, 4, 3, dim)
    with pytest.raises(ValueError):
        O.attention(q, k, v, 7, 6, heads, kvh, dim)


# ── sampler (src/sampler.rs:160-237) ──

def test_greedy_is_first_max():
    s = O.Sampler(0, 0.0, 1.0)
    assert s.pick(np.array([0.1, 3.0, 2.0, 3.0], np.float32)) == 1
    assert s.pick(np.array([-5.0, -1.0, -3.0], np.float32)) == 1
    assert O.lib().orc_argmax(O.ptr(np.array([1.0], np.float32)), 1) == 0


def test_nucleus_cuts_the_tail():
    logits = np.zeros(5000, np.float32)
    logits[42] = 10.0
    s = O.Sampler(7, 1.0, 0.5)
    assert all(s.pick(logits) == 42 for _ in range(200))


def test_frequencies_follow_probabilities():
    logits = np.log(np.array([0.5, 0.3, 0.2], np.float32))
    s = O.Sampler(12345, 1.0, 1.0)
    n = 30000
    counts = np.bincount([s.pick(logits) for _ in range(n)], minlength=3) / n
    np.testing.assert_allclose(counts, [0.5, 0.3, 0.2], atol=0.015)


def test_flat_distribution_uses_full_order():
    s = O.Sampler(3, 1.0, 0.9)
    logits = np.ones(5000, np.float32)
    seen = {s.pick(logits) for _ in range(3000)}
    assert len(seen) > 1024


def test_seed_determinism():
    logits = np.sin(np.arange(300) * 0.07).astype(np.float32)
    a = O.Sampler(99, 0.8, 0.9)
    b = O.Sampler(99, 0.8, 0.9)
    assert [a.pick(logits) for _ in range(50)] == [b.pick(logits) for _ in range(50)]


# ── Azar (src/daiss.rs:750-803) ──

def test_azar_seed_and_sigma():
    a, b, c = O.Azar(7), O.Azar(7), O.Azar(8)
    xa = [a.next() for _ in range(8)]
    assert xa == [b.next() for _ in range(8)]
    assert xa != [c.next() for _ in range(8)]
    z = O.Azar(0)
    assert z.next() != 0 and z.next() != 0
    r = O.Azar(1234)
    v = np.array([x for _ in range(10000) for x in r.normals(0.02)], np.float32)
    assert abs(v.mean()) < 0.001 and abs(v.std() - 0.02) < 0.001


def test_azar_known_first_outputs():
    # xorshift64* on seed 7 computed from the published recurrence
    st = 7
    out = []
    for _ in range(3):
        x = st
        x ^= x >> 12
        x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 27
        st = x
        out.append((x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF)
    a = O.Azar(7)
    assert [a.next() for _ in range(3)] == out


@pytest.mark.parametrize("t", [O.Q2K, O.Q3K, O.Q4K, O.Q5K, O.Q6K])
def test_fused_dot_equals_dequantize_then_multiply(t):
    # src/kernels/q2k.rs:325-340, src/kernels/q5k.rs:195-250: the fused dot
    # against the definition, sum of dequant(w)_i * xq_i * xe[i / sub] in f64
    from tests.golden.make_golden import finite_row
    rng = np.random.default_rng(30 + t)
    sub = O.SUB[t]
    for nb in (1, 2, 8):
        row = finite_row(rng, t, nb)
        xq, xe, xs = O.quantize_i8(rng.standard_normal(nb * 256).astype(np.float32), sub)
        w = O.dequantize(t, row, nb * 256).astype(np.float64)
        want = float((w * xq.astype(np.float64) * np.repeat(xe.astype(np.float64), sub)).sum())
        got = O.dot_row(t, row, xq, xe, xs)
        assert abs(got - want) / max(abs(want), 1.0) < 1e-3, (nb, got, want)


# ── dispatch (src/ops.rs:1706-1758) ──

@pytest.mark.parametrize("t", [O.Q4K, O.Q3K, O.Q2K, O.F32, O.F16])
def test_quantized_matmul_within_3pct_of_f32(t):
    # the integer path quantizes the input and the f32 path does not: within
    # 3 % of the f32 result's range, for each row count either side of the
    # reference's blocked-path threshold (24)
    k, n = 256, 64
    if t == O.F32:
        w = np.sin(np.arange(n * k, dtype=np.float32) * np.float32(0.019)).astype(np.float32).view(np.uint8)
    elif t == O.F16:
        vals = np.sin(np.arange(n * k, dtype=np.float32) * np.float32(0.019)).astype(np.float32)
        w = np.array([O.f32_to_f16(float(v)) for v in vals], np.uint16).view(np.uint8)
    else:
        w = np.array([(i * 97 + 29) % 251 for i in range(n * O.BLOCK_BYTES[t])], np.uint8)
    dense = np.stack([O.dequantize(t, w[r * (w.size // n):(r + 1) * (w.size // n)], k) for r in range(n)])
    lib = O.lib()
    for m in (1, 2, 4, 8, 23, 24, 37):
        x = np.cos(np.arange(m * k, dtype=np.float32) * np.float32(0.021)).astype(np.float32)
        ref = (x.reshape(m, k).astype(np.float64) @ dense.T.astype(np.float64)).astype(np.float32)
        got = np.zeros(m * n, np.float32)
        assert lib.orc_matmul_auto(m, k, n, O.ptr(x), O.ptr(w), w.size, t, O.ptr(got)) == 0
        # the byte pattern gives some blocks NaN/Inf scales; the reference's
        # folds with f32::max skip NaN, and so do these
        with np.errstate(invalid="ignore"):
            rng = float(np.nanmax(ref) - np.nanmin(ref))
            worst = float(np.nanmax(np.abs(got.reshape(m, n) - ref)))
        assert worst < 0.03 * rng, (t, m, worst, rng)
        # non-finite exactly where the f32 path is (the blocks with NaN/Inf scales)
        np.testing.assert_array_equal(np.isfinite(got.reshape(m, n)), np.isfinite(ref))


# ── KV cache (src/forward.rs:62-127; the reference's test :587-603) ──

def test_cache_prefix_copies_first_tokens_and_equals_truncate(tmp_path):
    import cosxamix_b200 as cx
    p = str(tmp_path / "tiny.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42, n_layer=2))
    m = O.Model(p)
    cfg = m.config
    w = cfg.n_head_kv * cfg.head_dim
    c = O.Cache(m)
    m.forward(c, [7, 3, 9, 1])
    k_all, v_all = c.layer(1, False), c.layer(0, True)
    pre = c.prefix(2)
    assert len(pre) == 2
    np.testing.assert_array_equal(pre.layer(1, False), k_all[: 2 * w])
    np.testing.assert_array_equal(pre.layer(0, True), v_all[: 2 * w])
    assert len(c) == 4, "the original is untouched"
    assert len(c.prefix(10)) == 4, "asking for more than there is keeps it all"
    c.truncate(2)
    for layer in range(cfg.n_layer):
        for v in (False, True):
            np.testing.assert_array_equal(c.layer(layer, v), pre.layer(layer, v))
    c.truncate(5)  # longer than the cache: nothing changes
    assert len(c) == 2
    # continuing from the prefix equals computing the whole prompt afresh
    np.testing.assert_array_equal(m.forward(pre, [9, 1, 4]), m.forward(O.Cache(m), [7, 3, 9, 1, 4]))
    c.clear()
    assert len(c) == 0


# ── matmul_auto's dispatch (src/ops.rs:1056-1093, :837-858, :599-606) ──

def test_matmul_path_follows_matmul_auto_on_each_backend():
    F, B, BL, F32 = O.PATH_FUSED, O.PATH_BUFFERED, O.PATH_BLOCKED, O.PATH_F32
    # COSXAMIX_KERNEL=escalar: only Q4_K and Q3_K have a fused kernel in use;
    # Q3_K's is taken up to 4 rows, Q4_K's below the blocked threshold; the
    # blocked path needs AVX2, so from 24 rows every format is buffered
    scalar = {
        O.Q4K: {1: F, 4: F, 5: F, 23: F, 24: B, 512: B},
        O.Q3K: {1: F, 4: F, 5: B, 23: B, 24: B},
        O.Q6K: {1: B, 4: B, 5: B, 24: B},
        O.Q5K: {1: B, 24: B},
        O.Q2K: {1: B, 24: B},
        O.F32: {1: F32, 24: F32},
        O.F16: {1: F32, 37: F32},
    }
    x86 = {
        O.Q4K: {1: F, 23: F, 24: BL, 512: BL},
        O.Q3K: {1: F, 4: F, 5: B, 24: BL},
        O.Q6K: {1: F, 4: F, 5: B, 23: B, 24: BL},
        O.Q5K: {1: F, 5: B, 24: BL},
        O.Q2K: {1: F, 4: F, 5: B, 24: BL},
    }
    for backend, table in (("scalar", scalar), ("x86", x86)):
        O.set_backend(backend)
        try:
            for t, rows in table.items():
                for m, want in rows.items():
                    assert O.matmul_path(m, 2048, t) == want, (backend, t, m)
        finally:
            O.set_backend("scalar")


def _pattern_weights(t, n, k):
    """The reference tests' byte pattern (i*97+29)%251 (src/ops.rs:1536-1540);
    Q8_0 as its identity-plus-pattern helper (:1526-1534, :1336-1351)."""
    if t == O.Q8_0:
        b = np.zeros(n * (k // 32) * 34, np.uint8)
        for r in range(n):
            for bl in range(k // 32):
                o = (r * (k // 32) + bl) * 34
                b[o:o + 2] = np.frombuffer(np.uint16(0x3C00).tobytes(), np.uint8)
                for j in range(32):
                    b[o + 2 + j] = 1 if bl * 32 + j == r else 0
        i = np.arange(b.size)
        body = (i % 34) >= 2
        b[body] = (((i[body] * 29) % 253) - 126).astype(np.int8).view(np.uint8)
        return b
    return ((np.arange(n * k // 256 * O.BLOCK_BYTES[t]) * 97 + 29) % 251).astype(np.uint8)


@pytest.mark.parametrize("t", [O.Q3K, O.Q4K, O.Q5K, O.Q6K, O.Q2K, O.Q8_0])
def test_blocked_matches_buffered(t):
    # src/ops.rs:1517-1561 `por_bloques_coincide_con_el_de_buffer`: the AVX2
    # blocked path and the buffered one agree within 1e-4 of the buffered
    # result's largest magnitude; 37 rows leave a partial 4-row tile, 70 and
    # 71 columns a last tramo of 6 and 7
    k = 512
    O.set_backend("x86")
    try:
        for n in (70, 71):
            w = _pattern_weights(t, n, k)
            for m in (4, 37):
                x = np.cos(np.arange(m * k, dtype=np.float32) * np.float32(0.021)).astype(np.float32)
                buf = O.matmul(x, w, t, k, n, path=O.PATH_BUFFERED)
                blk = O.matmul(x, w, t, k, n, path=O.PATH_BLOCKED)
                with np.errstate(invalid="ignore"):
                    scale = float(np.nanmax(np.abs(buf)))
                    worst = float(np.nanmax(np.abs(buf - blk)))
                assert worst <= scale * 1e-4, (t, m, n, worst, scale)
                np.testing.assert_array_equal(np.isnan(buf), np.isnan(blk))
    finally:
        O.set_backend("scalar")


@pytest.mark.parametrize("t", [O.Q2K, O.Q3K, O.Q4K, O.Q5K, O.Q6K])
def test_buffered_row_is_unpack_then_scaled_dot_then_offsets(t):
    # src/ops.rs:383-405 restated from its parts: dot_i8_escalado of the
    # unpacked row, then des*xe*xs per sub-block when any des is nonzero
    from tests.golden.make_golden import finite_row
    rng = np.random.default_rng(t)
    nb = 8
    row = finite_row(rng, t, nb)
    x = rng.standard_normal(nb * 256).astype(np.float32)
    sub = O.SUB[t]
    xq, xe, xs = O.quantize_i8(x, sub)
    q, esc, des = O.unpack_i8(t, row, nb * 256)
    total = np.float32(0.0)
    for b in range(nb * 256 // sub):
        part = int(np.dot(q[b * sub:(b + 1) * sub].astype(np.int32), xq[b * sub:(b + 1) * sub].astype(np.int32)))
        total = np.float32(total + np.float32(np.float32(esc[b] * xe[b]) * np.float32(part)))
    if np.any(des != 0):
        for b in range(nb * 256 // sub):
            total = np.float32(total + np.float32(np.float32(des[b] * xe[b]) * xs[b]))
    assert O.dot_row_buffered(t, row, xq, xe, xs) == total
    # the fused kernel forms the same integer sums: within the reference's 1e-4
    fused = O.dot_row(t, row, xq, xe, xs)
    assert abs(fused - total) <= 1e-4 * max(abs(total), 1.0)


def test_scalar_prompt_paths_agree_within_float_order(tmp_path):
    # A prompt of 24+ tokens takes the buffered path for every matrix and a
    # shorter one the fused path for Q4_K: the same integer sums in another
    # float order, so the KV rows agree closely but not bit for bit
    import cosxamix_b200 as cx
    p = str(tmp_path / "tiny.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42, n_layer=2))
    m = O.Model(p)
    prompt = [(i * 37 + 11) % 8192 for i in range(24)]
    whole = O.Cache(m)
    a = m.forward(whole, prompt)
    split = O.Cache(m)
    m.forward(split, prompt[:12])
    b = m.forward(split, prompt[12:])
    assert float(np.max(np.abs(a - b)) / (a.max() - a.min())) <= 1e-2
    assert not np.array_equal(whole.layer(1, False), split.layer(1, False))
