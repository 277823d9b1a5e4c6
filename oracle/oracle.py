"""ctypes wrapper of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by __graft_entry__.smoke() as the
checker, and by bench.py's CPU-baseline leg. The product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libcxm_ref.so")

F32, F16, Q8_0, Q5_0 = 0, 1, 8, 6
Q2K, Q3K, Q4K, Q5K, Q6K = 10, 11, 12, 13, 14
BLOCK_BYTES = {Q2K: 84, Q3K: 110, Q4K: 144, Q5K: 176, Q6K: 210, Q8_0: 34, Q5_0: 22}
SUB = {Q2K: 16, Q3K: 16, Q6K: 16, Q4K: 32, Q5K: 32, Q8_0: 32, Q5_0: 32}

_lib = None


def build() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p


def _declare(L: C.CDLL) -> None:
    sig = {
        "orc_f16_to_f32": (C.c_float, [C.c_uint16]),
        "orc_f32_to_f16": (C.c_uint16, [C.c_float]),
        "orc_dequantize": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, P]),
        "orc_unpack_i8": (C.c_int, [C.c_int, P, C.c_size_t, C.c_size_t, P, P, P]),
        "orc_quantize_i8": (None, [P, C.c_size_t, C.c_int, P, P, P]),
        "orc_dot_i8": (C.c_int32, [P, P, C.c_size_t]),
        "orc_dot_i8_scaled": (C.c_float, [P, P, P, P, C.c_size_t, C.c_int]),
        "orc_dot_f32": (C.c_float, [P, P, C.c_size_t]),
        "orc_dot_row": (C.c_float, [C.c_int, P, P, P, P, C.c_size_t]),
        "orc_subblock_sums": (C.c_int, [C.c_int, P, P, C.c_size_t, P]),
        "orc_rmsnorm": (None, [P, P, P, C.c_size_t, C.c_float]),
        "orc_silu": (None, [P, P, C.c_size_t]),
        "orc_rope_tables": (None, [C.c_int, C.c_float, C.c_int, P, P]),
        "orc_rope": (C.c_int, [P, C.c_int, C.c_int, C.c_int, P, P, C.c_int, C.c_int]),
        "orc_softmax": (C.c_int, [P, C.c_size_t, C.c_size_t]),
        "orc_attention": (C.c_int, [P, P, P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, P]),
        "orc_matmul_auto": (C.c_int, [C.c_int, C.c_int, C.c_int, P, P, C.c_size_t, C.c_int, P]),
        "orc_matmul_path": (C.c_int, [C.c_int, C.c_int, C.c_int]),
        "orc_matmul_by_path": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_int, P, P, C.c_size_t, C.c_int, P]),
        "orc_dot_row_buffered": (C.c_float, [C.c_int, P, P, P, P, C.c_size_t]),
        "orc_x86_dot_i8_scaled": (C.c_float, [P, P, P, P, C.c_size_t, C.c_int]),
        "orc_x86_tile_out": (C.c_float, [P, P, P, P, C.c_size_t, C.c_int]),
        "orc_azar_next": (C.c_uint64, [P]),
        "orc_azar_normals": (None, [P, C.c_float, P, P]),
        "orc_azar_seed": (C.c_uint64, [C.c_uint64]),
        "orc_sampler_new": (P, [C.c_uint64, C.c_float, C.c_float]),
        "orc_sampler_free": (None, [P]),
        "orc_sampler_pick": (C.c_uint32, [P, P, C.c_size_t]),
        "orc_sampler_state": (C.c_uint64, [P]),
        "orc_argmax": (C.c_uint32, [P, C.c_size_t]),
        "orc_model_open": (P, [C.c_char_p]),
        "orc_last_error": (C.c_char_p, []),
        "orc_model_close": (None, [P]),
        "orc_model_config": (None, [P, P]),
        "orc_cache_new": (P, [P]),
        "orc_cache_free": (None, [P]),
        "orc_cache_len": (C.c_int, [P]),
        "orc_cache_truncate": (None, [P, C.c_int]),
        "orc_cache_prefix": (P, [P, C.c_int]),
        "orc_cache_clear": (None, [P]),
        "orc_cache_layer": (P, [P, C.c_int, C.c_int]),
        "orc_forward": (C.c_int, [P, P, P, C.c_int, P]),
        "orc_generate": (C.c_int, [P, P, P, C.c_int, C.c_int, P, P, P]),
        "orc_cache_fill": (None, [P, C.c_int, C.c_uint64]),
        "orc_expf": (None, [P, P, C.c_size_t]),
        "orc_set_threads": (None, [C.c_int]),
        "orc_get_threads": (C.c_int, []),
        "orc_set_varias": (None, [C.c_int]),
        "orc_set_backend": (None, [C.c_int]),
        "orc_get_backend": (C.c_int, []),
        "orc_set_dot_kernel": (C.c_int, [C.c_int, P]),
        "orc_set_q4k_acc_kernel": (None, [P]),
        "orc_x86_dot_f32": (C.c_float, [P, P, C.c_size_t]),
        "orc_x86_rmsnorm": (None, [P, P, P, C.c_size_t, C.c_float]),
        "orc_x86_dot_q4k": (C.c_float, [P, P, P, P, C.c_size_t]),
        "orc_x86_dot_q6k": (C.c_float, [P, P, P, P, C.c_size_t]),
        "orc_x86_dot_row": (C.c_float, [C.c_int, P, P, P, P, C.c_size_t]),
        "orc_x86_q4k_scales": (None, [P, P, P, P, P]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args


def ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def err() -> str:
    return lib().orc_last_error().decode()


# ───────────── thin numpy helpers ─────────────

def f16_to_f32(h: int) -> float:
    return lib().orc_f16_to_f32(h)


def f32_to_f16(x: float) -> int:
    return lib().orc_f32_to_f16(x)


def dequantize(t: int, blocks: np.ndarray, n: int) -> np.ndarray:
    out = np.zeros(n, np.float32)
    b = np.ascontiguousarray(blocks, np.uint8)
    if lib().orc_dequantize(t, ptr(b), b.size, n, ptr(out)):
        raise ValueError(err())
    return out


def unpack_i8(t: int, blocks: np.ndarray, n: int):
    sub = SUB[t]
    q = np.zeros(n, np.int8)
    e = np.zeros(n // sub, np.float32)
    d = np.zeros(n // sub, np.float32)
    b = np.ascontiguousarray(blocks, np.uint8)
    r = lib().orc_unpack_i8(t, ptr(b), b.size, n, ptr(q), ptr(e), ptr(d))
    if r < 0:
        raise ValueError(err())
    return q, e, d


def quantize_i8(x: np.ndarray, sub: int):
    x = np.ascontiguousarray(x, np.float32)
    nb = (x.size + sub - 1) // sub
    q = np.zeros(x.size, np.int8)
    e = np.zeros(nb, np.float32)
    s = np.zeros(nb, np.float32)
    lib().orc_quantize_i8(ptr(x), x.size, sub, ptr(q), ptr(e), ptr(s))
    return q, e, s


def dot_row(t: int, row: np.ndarray, xq, xe, xs) -> float:
    row = np.ascontiguousarray(row, np.uint8)
    return lib().orc_dot_row(t, ptr(row), ptr(xq), ptr(xe), ptr(xs), xq.size // 256)


def subblock_sums(t: int, row: np.ndarray, xq: np.ndarray) -> np.ndarray:
    row = np.ascontiguousarray(row, np.uint8)
    out = np.zeros(xq.size // SUB[t], np.int32)
    if lib().orc_subblock_sums(t, ptr(row), ptr(xq), xq.size // 256, ptr(out)):
        raise ValueError(err())
    return out


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.zeros_like(x)
    lib().orc_rmsnorm(ptr(out), ptr(x), ptr(w), x.size, eps)
    return out


def silu(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().orc_silu(ptr(out), ptr(x), x.size)
    return out


def rope_tables(hd: int, base: float, ctx: int):
    c = np.zeros(ctx * (hd // 2), np.float32)
    s = np.zeros_like(c)
    lib().orc_rope_tables(hd, base, ctx, ptr(c), ptr(s))
    return c, s


def rope(x: np.ndarray, tokens: int, heads: int, hd: int, cos, sin, pos: int) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    ctx = cos.size // (hd // 2)
    if lib().orc_rope(ptr(x), tokens, heads, hd, ptr(cos), ptr(sin), ctx, pos):
        raise ValueError(err())
    return x


def softmax(x: np.ndarray, width: int) -> np.ndarray:
    x = np.array(x, np.float32, copy=True)
    if lib().orc_softmax(ptr(x), x.size, width):
        raise ValueError(err())
    return x


def attention(q, k, v, tokens, total, heads, heads_kv, hd) -> np.ndarray:
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.zeros(tokens * heads * hd, np.float32)
    if lib().orc_attention(ptr(q), ptr(k), ptr(v), tokens, total, heads, heads_kv, hd, ptr(out)):
        raise ValueError(err())
    return out


PATH_F32, PATH_FUSED, PATH_BUFFERED, PATH_BLOCKED = 0, 1, 2, 3
BLOCKED_FROM = 24


def matmul_path(m: int, k: int, t: int) -> int:
    """The path ops::matmul_auto takes for m activation rows on this backend."""
    return lib().orc_matmul_path(m, k, t)


def dot_row_buffered(t: int, row: np.ndarray, xq, xe, xs) -> float:
    """One output of the buffered path (src/ops.rs:383-405)."""
    row = np.ascontiguousarray(row, np.uint8)
    return lib().orc_dot_row_buffered(t, ptr(row), ptr(xq), ptr(xe), ptr(xs), xq.size // 256)


def matmul(lhs: np.ndarray, w: np.ndarray, t: int, k: int, n: int, path: int | None = None) -> np.ndarray:
    """ops::matmul_auto: the rows of `lhs` (m x k) times W (n x k) by the
    path the reference takes for m rows (or the one `path` forces)."""
    lhs = np.ascontiguousarray(lhs, np.float32)
    m = lhs.size // k
    w = np.ascontiguousarray(w, np.uint8)
    out = np.zeros(m * n, np.float32)
    if path is None:
        rc = lib().orc_matmul_auto(m, k, n, ptr(lhs), ptr(w), w.size, t, ptr(out))
    else:
        rc = lib().orc_matmul_by_path(path, m, k, n, ptr(lhs), ptr(w), w.size, t, ptr(out))
    if rc:
        raise ValueError(err())
    return out.reshape(m, n)


class Azar:
    """xorshift64* of src/daiss.rs:317-357."""

    def __init__(self, seed: int):
        self.state = np.array([lib().orc_azar_seed(seed)], np.uint64)

    def next(self) -> int:
        return lib().orc_azar_next(ptr(self.state))

    def normals(self, sigma: float):
        a = np.zeros(1, np.float32)
        b = np.zeros(1, np.float32)
        lib().orc_azar_normals(ptr(self.state), sigma, ptr(a), ptr(b))
        return float(a[0]), float(b[0])


class Sampler:
    def __init__(self, seed: int, temperature: float, top_p: float):
        self.h = lib().orc_sampler_new(seed, temperature, top_p)

    def pick(self, logits: np.ndarray) -> int:
        logits = np.ascontiguousarray(logits, np.float32)
        return lib().orc_sampler_pick(self.h, ptr(logits), logits.size)

    @property
    def state(self) -> int:
        return lib().orc_sampler_state(self.h)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_sampler_free(self.h)
            self.h = None


class Config(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("n_layer", "dim", "n_head", "n_head_kv", "head_dim", "vocab", "ctx", "ffn")] + [
        ("eps", C.c_float), ("rope_base", C.c_float), ("tied", C.c_int)]


class Cache:
    def __init__(self, model: "Model", handle=None):
        self.model = model
        self.h = handle if handle is not None else lib().orc_cache_new(model.h)

    def __len__(self) -> int:
        return lib().orc_cache_len(self.h)

    def truncate(self, n: int) -> None:
        lib().orc_cache_truncate(self.h, n)

    def clear(self) -> None:
        lib().orc_cache_clear(self.h)

    def prefix(self, n: int) -> "Cache":
        return Cache(self.model, lib().orc_cache_prefix(self.h, n))

    def fill(self, n: int, seed: int = 1) -> None:
        lib().orc_cache_fill(self.h, n, seed)

    def layer(self, l: int, v: bool) -> np.ndarray:
        cfg = self.model.config
        n = len(self) * cfg.n_head_kv * cfg.head_dim
        p = lib().orc_cache_layer(self.h, l, int(v))
        return np.ctypeslib.as_array((C.c_float * n).from_address(p)).copy() if n else np.zeros(0, np.float32)

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_cache_free(self.h)
            self.h = None


class Model:
    def __init__(self, path: str):
        self.h = lib().orc_model_open(path.encode())
        if not self.h:
            raise ValueError(err())
        self.config = Config()
        lib().orc_model_config(self.h, C.byref(self.config))

    def cache(self) -> Cache:
        return Cache(self)

    def forward(self, cache: Cache, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros(self.config.vocab, np.float32)
        if lib().orc_forward(self.h, cache.h, ptr(toks), toks.size, ptr(out)):
            raise ValueError(err())
        return out

    def generate(self, cache: Cache, prompt, max_new: int, sampler: Sampler):
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_new, 1), np.uint32)
        n = C.c_int(0)
        if lib().orc_generate(self.h, cache.h, ptr(p), p.size, max_new, sampler.h, ptr(out), C.byref(n)):
            raise ValueError(err())
        return out[: n.value].tolist()

    def __del__(self):
        if getattr(self, "h", None):
            lib().orc_model_close(self.h)
            self.h = None


def set_threads(n: int) -> None:
    lib().orc_set_threads(n)


def threads() -> int:
    return lib().orc_get_threads()


SCALAR, X86 = 0, 1
# the reference's own compiled kernels (oracle/_ref) the X86 backend takes when
# they were built: GGML type -> (symbol, "dot" = kernel ABI | "acc" = 16 floats out)
REF_KERNELS = {Q4K: ("cosxamix_q4k_completo", "acc"), Q5K: ("cosxamix_q5k_asm", "dot"),
               Q3K: ("cosxamix_q3k_completo", "dot"), Q2K: ("cosxamix_q2k_asm", "dot")}


def set_backend(name: str, reference_kernels: bool = True) -> dict:
    """Kernel backend of Model.forward: "scalar" (the parity restatement, the
    default) or "x86" (what the reference runs on an AVX2/FMA/F16C host; for
    timing only). With `reference_kernels`, "x86" runs the reference's own
    compiled kernels of oracle/_ref where they were built. Returns, per GGML
    type, the kernel in use."""
    L = lib()
    for t in range(16):
        L.orc_set_dot_kernel(t, None)
    L.orc_set_q4k_acc_kernel(None)
    if name == "scalar":
        L.orc_set_backend(SCALAR)
        return {t: "scalar restatement" for t in (Q2K, Q3K, Q4K, Q5K, Q6K)}
    if name != "x86":
        raise ValueError(f"unknown backend {name!r}")
    L.orc_set_backend(X86)
    used = {Q4K: "AVX2 restatement (x86.rs)", Q6K: "AVX2 restatement (x86.rs)",
            Q5K: "scalar restatement", Q3K: "scalar restatement", Q2K: "scalar restatement"}
    R = ref_lib() if reference_kernels else None
    if R is not None:
        for t, (sym, abi) in REF_KERNELS.items():
            addr = C.cast(getattr(R, sym), C.c_void_p).value
            if abi == "acc":
                L.orc_set_q4k_acc_kernel(addr)
            else:
                L.orc_set_dot_kernel(t, addr)
            used[t] = f"reference {sym}"
    return used


def backend() -> str:
    return "x86" if lib().orc_get_backend() == X86 else "scalar"


# ───────────── the reference's own kernels (oracle/_ref) ─────────────

_ref = None


def ref_lib():
    """The reference's C/asm dot kernels, or None when not built."""
    global _ref
    if _ref is None and os.path.exists(REF_PATH):
        _ref = C.CDLL(REF_PATH)
        for n in ("cosxamix_q2k_c", "cosxamix_q3k_c", "cosxamix_q5k_c", "cosxamix_q2k_asm",
                  "cosxamix_q3k_completo", "cosxamix_q5k_asm"):
            f = getattr(_ref, n)
            f.restype = C.c_float
            f.argtypes = [P, P, P, P, C.c_size_t]
        _ref.cosxamix_q4k_completo.restype = None
        _ref.cosxamix_q4k_completo.argtypes = [P, P, P, P, C.c_size_t, P]
    return _ref


def ref_dot(kernel: str, row, xq, xe, xs) -> float:
    """Run one of the reference's kernels; for q4k_completo apply the final
    reduction its Rust bridge does (src/kernels/q4k_asm.rs:214-235)."""
    L = ref_lib()
    row = np.ascontiguousarray(row, np.uint8)
    n = xq.size // 256
    if kernel == "cosxamix_q4k_completo":
        acc = np.zeros(16, np.float32)
        L.cosxamix_q4k_completo(ptr(row), ptr(xq), ptr(xe), ptr(xs), n, ptr(acc))
        return float(np.float32(acc[:8].sum(dtype=np.float32)) - np.float32(acc[8:].sum(dtype=np.float32)))
    return getattr(L, kernel)(ptr(row), ptr(xq), ptr(xe), ptr(xs), n)
