"""CPU tests of the host side: the C ABI library loads and exports what
include/cxm.h declares, refuses to run without a GPU, and its synthetic-model
writer produces GGUF files and k-quant blocks that the oracle reads back within
the reference's error bounds (src/quant_kquants.rs:425-503)."""
import os
import re

import numpy as np
import pytest

import cosxamix_b200 as cx
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "cxm.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cxm_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    L = cx.lib()
    syms = header_symbols()
    assert len(syms) >= 20
    for s in syms:
        assert hasattr(L, s), s


def test_library_is_built_for_sm100a_only():
    # the recipe compiles and links every CUDA source for sm_100a alone
    from cosxamix_b200 import build as b
    assert b.ARCH == ["-gencode", "arch=compute_100a,code=sm_100a"]
    assert all(f in b.CUDA_FLAGS for f in b.ARCH)
    assert not any("compute_" in f and "100a" not in f for f in b.CUDA_FLAGS)


def header_prototypes():
    """name -> number of parameters, for every function include/cxm.h declares"""
    text = open(os.path.join(ROOT, "include", "cxm.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = re.sub(r"//[^\n]*", "", text)
    out = {}
    for name, params in re.findall(r"\b(cxm_[a-z0-9_]+)\s*\(([^)]*)\)\s*;", text, flags=re.S):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_python_binding_matches_header_arity():
    # every declared entry point is bound with as many arguments as the header gives it
    protos = header_prototypes()
    assert len(protos) >= 20
    L = cx.lib()
    for name, n in protos.items():
        f = getattr(L, name)
        assert f.argtypes is not None, f"{name} has no ctypes signature"
        assert len(f.argtypes) == n, (name, len(f.argtypes), n)


def test_no_cpu_fallback_without_gpu(tmp_path):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = str(tmp_path / "t.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", n_layer=1, vocab=512))
    with pytest.raises(ValueError, match="no CUDA device"):
        cx.Modelo(p)
    with pytest.raises(ValueError, match="no CUDA device"):
        cx.matvec(cx.Q4_K, np.zeros(2 * 144, np.uint8), 2, 256, np.zeros(256, np.float32))


def rmse(a, b):
    return float(np.sqrt(np.mean((a.astype(np.float64) - b) ** 2)))


def round_trip(t, x):
    b = cx.quantize(t, x)
    assert b.size == x.size // 256 * O.BLOCK_BYTES[t]
    return O.dequantize(t, b, x.size)


def normals(n, sigma, seed=7):
    a = O.Azar(seed)
    return np.array([a.normals(sigma)[0] for _ in range(n)], np.float32)


def test_writer_error_matches_bits():
    # src/quant_kquants.rs:427-437 (Q6_K added: fewer bits of error than Q5_K)
    x = normals(256 * 64, 0.02)
    e = {t: rmse(x, round_trip(t, x)) / 0.02 for t in (cx.Q2_K, cx.Q3_K, cx.Q4_K, cx.Q5_K, cx.Q6_K)}
    assert e[cx.Q4_K] < e[cx.Q3_K] < e[cx.Q2_K]
    assert e[cx.Q5_K] < e[cx.Q4_K] / 1.6
    assert e[cx.Q6_K] < e[cx.Q5_K]
    assert e[cx.Q4_K] < 0.09 and e[cx.Q3_K] < 0.2 and e[cx.Q2_K] < 0.42 and e[cx.Q6_K] < 0.03


@pytest.mark.parametrize("t", [cx.Q2_K, cx.Q3_K, cx.Q4_K, cx.Q5_K, cx.Q6_K])
def test_writer_zero_and_uneven_blocks(t):
    # src/quant_kquants.rs:439-477
    z = np.zeros(256, np.float32)
    np.testing.assert_array_equal(round_trip(t, z), z)
    x = normals(256, 0.5)
    x[32:64] = 0
    y = round_trip(t, x)
    assert rmse(x, y) < 0.3 and np.isfinite(y).all()
    x = normals(256, 0.001)
    x[:16] *= 1000
    y = round_trip(t, x)
    assert rmse(x[:16], y[:16]) < 0.5 and np.isfinite(y).all()
    pos = np.abs(normals(256, 0.1))
    assert rmse(pos, round_trip(t, pos)) < 0.05
    assert rmse(-pos, round_trip(t, -pos)) < 0.05


@pytest.mark.parametrize("t,sub", [(cx.Q2_K, 16), (cx.Q3_K, 16), (cx.Q4_K, 32), (cx.Q5_K, 32), (cx.Q6_K, 16)])
def test_writer_each_subblock_keeps_its_scale(t, sub):
    # src/quant_kquants.rs:481-503
    n = 256 // sub
    x = np.zeros(256, np.float32)
    for j in range(n):
        amp = 0.1 * (1 + j / n)
        x[j * sub:(j + 1) * sub] = [amp if i % 2 == 0 else -amp for i in range(sub)]
    y = round_trip(t, x)
    for j in range(n):
        assert rmse(x[j * sub:(j + 1) * sub], y[j * sub:(j + 1) * sub]) < 0.06


def test_q6k_writer_output_is_read_by_the_reference_layout():
    # the fused dot of the oracle (the reference's reading of Q6_K) agrees with
    # dequantize-then-dot on the writer's bytes
    x = normals(256 * 8, 0.02, seed=3)
    b = cx.quantize(cx.Q6_K, x)
    act = np.sin(np.arange(x.size) * 0.013).astype(np.float32)
    xq, xe, xs = O.quantize_i8(act, 16)
    fused = O.dot_row(cx.Q6_K, b, xq, xe, xs)
    w = O.dequantize(cx.Q6_K, b, x.size)
    ref = float(np.sum(w.astype(np.float64) * xq * np.repeat(xe, 16)))
    assert abs(fused - ref) / max(abs(ref), 1e-3) < 1e-4


def test_synthetic_gguf_reads_back(tmp_path):
    p = str(tmp_path / "tiny.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42))
    m = O.Model(p)
    c = m.config
    assert (c.n_layer, c.dim, c.n_head, c.n_head_kv, c.vocab, c.ffn, c.tied) == (6, 256, 8, 8, 8192, 768, 0)
    assert abs(c.eps - 1e-6) < 1e-12 and c.rope_base == 10000.0


def test_synthetic_gguf_is_deterministic_and_seeded(tmp_path):
    a, b, c = (str(tmp_path / f"{n}.gguf") for n in "abc")
    cx.synth_write(a, cx.synth_spec("tiny", seed=42, n_layer=1, threads=3))
    cx.synth_write(b, cx.synth_spec("tiny", seed=42, n_layer=1, threads=1))
    cx.synth_write(c, cx.synth_spec("tiny", seed=43, n_layer=1))
    assert open(a, "rb").read() == open(b, "rb").read()
    assert open(a, "rb").read() != open(c, "rb").read()


def test_synthetic_rows_follow_the_seed_rule(tmp_path):
    # row r of tensor `name` is Azar(semilla_de(seed, name, r)) Box-Muller
    # pairs, then quantized (src/daiss.rs:364-379, :551-567)
    p = str(tmp_path / "t.gguf")
    cx.synth_write(p, cx.synth_spec("tiny", seed=42, n_layer=1))

    def semilla_de(model, name, row):
        h = 0xcbf29ce484222325
        for ch in name.encode():
            h ^= ch
            h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
        h ^= row
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
        return h ^ (((model << 17) | (model >> 47)) & 0xFFFFFFFFFFFFFFFF)

    for name, row in [("blk.0.ffn_up.weight", 5), ("token_embd.weight", 8191)]:
        az = O.Azar(semilla_de(42, name, row))
        vals = np.array([v for _ in range(128) for v in az.normals(0.02)], np.float32)
        want = cx.quantize(cx.Q4_K, vals)
        m = O.Model(p)
        # read the row bytes from the file through the oracle's mmap
        data = open(p, "rb").read()
        # locate by searching the unique 144-byte row
        assert data.find(want.tobytes()) > 0, name
