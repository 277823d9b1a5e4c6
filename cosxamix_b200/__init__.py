"""cosxamix_b200 — B200-native (sm_100a) decode path of Cosxamix.

Python mirror of the reference's decode interface, over the C ABI of
include/cxm.h (libcxm.so, built in-tree by cosxamix_b200/build.py):

    Modelo.abrir(path)              src/forward.rs:187      Model.open
    Modelo.forward(tokens, cache)   src/forward.rs:375      Model.forward
    Modelo.generar(prompt, max, m, cache)  src/forward.rs:533  Model.generate
    Cache.largo/truncar/prefijo/limpiar    src/forward.rs:62-137
    Muestreador(semilla, temperatura, top_p)  src/sampler.rs:40

Errors raise ValueError with the library's message, like the reference's
Err(String). There is no CPU fallback: without the library or a CUDA device
every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libcxm.so")

Q2_K, Q3_K, Q4_K, Q5_K, Q6_K = 10, 11, 12, 13, 14
TP_HANDLE_BYTES = 64  # CXM_TP_HANDLE_BYTES
MIX_UNIFORM, MIX_Q4_K_M = 0, 1

_lib = None
P = C.c_void_p


class Config(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("n_layer", "dim", "n_head", "n_head_kv", "head_dim", "vocab", "ctx", "ffn")] + [
        ("eps", C.c_float), ("rope_base", C.c_float), ("tied", C.c_int32), ("has_eos", C.c_int32), ("eos", C.c_uint32)]


class SynthSpec(C.Structure):
    _fields_ = [(n, C.c_int32) for n in ("vocab", "dim", "n_layer", "n_head", "n_head_kv", "ffn", "ctx")] + [
        ("eps", C.c_float), ("rope_base", C.c_float), ("tied", C.c_int32), ("mix", C.c_int32), ("type", C.c_int32),
        ("seed", C.c_uint64), ("sigma", C.c_float), ("threads", C.c_int32), ("has_eos", C.c_int32),
        ("eos", C.c_uint32)]


def lib() -> C.CDLL:
    """Load libcxm.so; raise (never fall back) when it is missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m cosxamix_b200.build`")
        L = C.CDLL(LIB_PATH)
        sig = {
            "cxm_last_error": (C.c_char_p, []),
            "cxm_model_open": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(P)]),
            "cxm_model_open_tp": (C.c_int, [C.c_char_p, C.c_int, C.c_int, C.c_int, C.POINTER(P)]),
            "cxm_tp_handle": (C.c_int, [P, P]),
            "cxm_tp_connect": (C.c_int, [P, P]),
            "cxm_model_tp_info": (C.c_int, [P, C.POINTER(C.c_int), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                            C.POINTER(C.c_int)]),
            "cxm_model_config": (C.c_int, [P, C.POINTER(Config)]),
            "cxm_model_weight_bytes": (C.c_uint64, [P]),
            "cxm_model_set_prefill": (C.c_int, [P, C.c_int]),
            "cxm_model_close": (None, [P]),
            "cxm_cache_new": (C.c_int, [P, C.c_uint32, C.POINTER(P)]),
            "cxm_cache_free": (None, [P]),
            "cxm_cache_len": (C.c_uint32, [P]),
            "cxm_cache_truncate": (C.c_int, [P, C.c_uint32]),
            "cxm_cache_clear": (C.c_int, [P]),
            "cxm_cache_copy_prefix": (C.c_int, [P, C.c_uint32, P]),
            "cxm_cache_share_prefix": (C.c_int, [P, C.c_uint32, P]),
            "cxm_generate_batch": (C.c_int, [P, P, P, P, C.c_uint32, C.c_uint32, P, P]),
            "cxm_cache_read": (C.c_int, [P, C.c_uint32, C.c_int, P]),
            "cxm_forward": (C.c_int, [P, P, P, C.c_uint32, P]),
            "cxm_sampler_new": (C.c_int, [C.c_uint64, C.c_float, C.c_float, C.POINTER(P)]),
            "cxm_sampler_free": (None, [P]),
            "cxm_sampler_state": (C.c_uint64, [P]),
            "cxm_sample": (C.c_int, [P, P, C.POINTER(C.c_uint32)]),
            "cxm_generate": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32, P, P, C.POINTER(C.c_uint32)]),
            "cxm_debug_subblock_sums": (C.c_int, [C.c_int, P, P, C.c_uint32, P]),
            "cxm_debug_matvec": (C.c_int, [C.c_int, P, C.c_uint32, C.c_uint32, P, P]),
            "cxm_debug_matmul": (C.c_int, [C.c_int, P, C.c_uint32, C.c_uint32, P, C.c_uint32, P]),
            "cxm_debug_attention": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P]),
            "cxm_debug_expf": (C.c_int, [P, P, C.c_uint64]),
            "cxm_debug_seq_sums": (C.c_int, [P, P, C.c_uint64]),
            "cxm_attention_noalloc": (C.c_int, [P, P, P, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32, P, P]),
            "cxm_bench_decode": (C.c_int, [P, P, C.c_uint32, C.POINTER(C.c_float)]),
            "cxm_bench_decode_sampled": (C.c_int, [P, P, P, C.c_uint32, C.POINTER(C.c_float)]),
            "cxm_bench_matvec": (C.c_int, [P, C.c_uint32, C.POINTER(C.c_float), C.POINTER(C.c_uint64)]),
            "cxm_bench_sample": (C.c_int, [P, P, C.c_uint32, C.POINTER(C.c_float), P, C.c_uint32]),
            "cxm_arm_gemm_stamps": (C.c_int, [C.c_int]),
            "cxm_read_gemm_stamps": (C.c_int, [P, C.c_uint32]),
            "cxm_step_launches": (C.c_int, [P]),
            "cxm_synth_write": (C.c_int, [C.POINTER(SynthSpec), C.c_char_p]),
            "cxm_quantize": (C.c_int64, [C.c_int, P, C.c_uint64, P, C.c_uint64]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _err() -> str:
    return lib().cxm_last_error().decode(errors="replace")


def _check(rc: int) -> None:
    if rc != 0:
        raise ValueError(_err())


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


# ───────────── synthetic models (src/daiss.rs) ─────────────

CONFIGS = {
    # the tiny parity configuration: Llama-style decoder, untied, all Q4_K
    "tiny": dict(vocab=8192, dim=256, n_layer=6, n_head=8, n_head_kv=8, ffn=768, ctx=256, eps=1e-6,
                 rope_base=10000.0, tied=0, mix=MIX_UNIFORM, type=Q4_K),
    # the headline configuration: Qwen2.5-3B shape, Q4_K_M-style, tied embeddings
    "qwen3b": dict(vocab=151936, dim=2048, n_layer=36, n_head=16, n_head_kv=2, ffn=11008, ctx=4096, eps=1e-6,
                   rope_base=1e6, tied=1, mix=MIX_Q4_K_M, type=Q4_K),
    # the uniform-format configurations: the Qwen2.5-3B shape re-quantized uniformly (output included)
    "qwen3b_q5k": dict(vocab=151936, dim=2048, n_layer=36, n_head=16, n_head_kv=2, ffn=11008, ctx=4096, eps=1e-6,
                       rope_base=1e6, tied=1, mix=MIX_UNIFORM, type=Q5_K),
    "qwen3b_q3k": dict(vocab=151936, dim=2048, n_layer=36, n_head=16, n_head_kv=2, ffn=11008, ctx=4096, eps=1e-6,
                       rope_base=1e6, tied=1, mix=MIX_UNIFORM, type=Q3_K),
    "qwen3b_q2k": dict(vocab=151936, dim=2048, n_layer=36, n_head=16, n_head_kv=2, ffn=11008, ctx=4096, eps=1e-6,
                       rope_base=1e6, tied=1, mix=MIX_UNIFORM, type=Q2_K),
    # a small Llama-style shape that splits over 2 or 4 tensor-parallel ranks
    # (whole heads, o/down K slices of whole super-blocks): the TP tests' model
    "tp_small": dict(vocab=8192, dim=1024, n_layer=4, n_head=8, n_head_kv=4, ffn=2048, ctx=512, eps=1e-5,
                     rope_base=5e5, tied=0, mix=MIX_Q4_K_M, type=Q4_K),
    # the tensor-parallel configuration: Llama-3-8B shape, Q4_K_M-style, untied
    "llama8b": dict(vocab=128256, dim=4096, n_layer=32, n_head=32, n_head_kv=8, ffn=14336, ctx=8192, eps=1e-5,
                    rope_base=5e5, tied=0, mix=MIX_Q4_K_M, type=Q4_K),
}


def synth_spec(name: str = "tiny", seed: int = 42, sigma: float = 0.02, threads: int = 0, eos: int | None = None,
               **over) -> SynthSpec:
    """`eos`: write tokenizer.ggml.eos_token_id (the benchmark models have
    none, so generation never stops early)."""
    cfg = dict(CONFIGS[name])
    cfg.update(over)
    return SynthSpec(seed=seed, sigma=sigma, threads=threads, has_eos=int(eos is not None), eos=eos or 0, **cfg)


def synth_write(path: str, spec: SynthSpec) -> str:
    """Write a seeded random-init GGUF (src/daiss.rs:494-586 generation rule)."""
    _check(lib().cxm_synth_write(C.byref(spec), path.encode()))
    return path


def quantize(ggml_type: int, x: np.ndarray) -> np.ndarray:
    """The library's k-quant writers (src/quant_kquants.rs; Q6_K own)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros(x.size * 2 + 1024, np.uint8)
    n = lib().cxm_quantize(ggml_type, _ptr(x), x.size, _ptr(out), out.size)
    if n < 0:
        raise ValueError(_err())
    return out[:n].copy()


# ───────────── the decode path ─────────────

class Muestreador:
    """Muestreador::nuevo(semilla, temperatura, top_p), src/sampler.rs:40-48."""

    def __init__(self, semilla: int = 42, temperatura: float = 0.0, top_p: float = 1.0):
        h = P()
        _check(lib().cxm_sampler_new(semilla, temperatura, top_p, C.byref(h)))
        self.h = h
        self.temperatura = temperatura
        self.top_p = top_p

    @classmethod
    def voraz(cls) -> "Muestreador":
        return cls(0, 0.0, 1.0)

    @property
    def estado(self) -> int:
        return lib().cxm_sampler_state(self.h)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.cxm_sampler_free(self.h)
            self.h = None


Sampler = Muestreador


class Cache:
    """The KV cache of one conversation, resident in HBM (src/forward.rs:62-137)."""

    def __init__(self, modelo: "Modelo", max_tokens: int | None = None):
        self.modelo = modelo
        n = max_tokens or modelo.cfg.ctx
        h = P()
        _check(lib().cxm_cache_new(modelo.h, n, C.byref(h)))
        self.h = h
        self.max_tokens = n

    def largo(self) -> int:
        return lib().cxm_cache_len(self.h)

    __len__ = largo

    def truncar(self, n: int) -> None:
        _check(lib().cxm_cache_truncate(self.h, n))

    def limpiar(self) -> None:
        _check(lib().cxm_cache_clear(self.h))

    def prefijo(self, n: int) -> "Cache":
        """Cache::prefijo: a copy of the first n tokens (device to device)."""
        other = Cache(self.modelo, self.max_tokens)
        _check(lib().cxm_cache_copy_prefix(self.h, n, other.h))
        return other

    def copiar_prefijo(self, src: "Cache", n: int) -> None:
        """Become a copy of the first n tokens of `src` (Cache::prefijo into
        this cache's own buffers, which keeps its captured decode graphs)."""
        _check(lib().cxm_cache_copy_prefix(src.h, n, self.h))

    def compartir_prefijo(self, src: "Cache", n: int) -> None:
        """Borrow the first n tokens of `src` as a shared prefix, held once
        (include/cxm.h: cxm_cache_share_prefix)."""
        _check(lib().cxm_cache_share_prefix(src.h, n, self.h))

    share_prefix = compartir_prefijo

    def capa(self, layer: int, v: bool = False) -> np.ndarray:
        """Layer `layer`'s K (or V) rows [0, len): this rank's KV heads."""
        cfg = self.modelo.cfg
        out = np.zeros(len(self) * (cfg.n_head_kv // self.modelo.tp_size) * cfg.head_dim, np.float32)
        _check(lib().cxm_cache_read(self.h, layer, int(v), _ptr(out)))
        return out

    truncate, clear, prefix, layer = truncar, limpiar, prefijo, capa

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.cxm_cache_free(self.h)
            self.h = None


class Modelo:
    """Modelo::abrir(ruta) on a CUDA device (src/forward.rs:187-266)."""

    def __init__(self, ruta: str, device: int = 0, tp: tuple[int, int] | None = None):
        """`tp=(rank, size)`: this process's share of a tensor-parallel model
        (one process per GPU); it runs after `tp_connect`."""
        h = P()
        if tp is None:
            _check(lib().cxm_model_open(ruta.encode(), device, C.byref(h)))
        else:
            _check(lib().cxm_model_open_tp(ruta.encode(), device, int(tp[0]), int(tp[1]), C.byref(h)))
        self.h = h
        self.cfg = Config()
        _check(lib().cxm_model_config(h, C.byref(self.cfg)))
        self.ruta = ruta
        r, n, lo, vn = (C.c_int() for _ in range(4))
        _check(lib().cxm_model_tp_info(h, C.byref(r), C.byref(n), C.byref(lo), C.byref(vn)))
        self.tp_rank, self.tp_size, self.vocab_lo, self.vocab_n = r.value, n.value, lo.value, vn.value

    # ── tensor parallelism ──
    def tp_handle(self) -> bytes:
        """The CUDA IPC handle of this rank's exchange area."""
        buf = (C.c_uint8 * TP_HANDLE_BYTES)()
        _check(lib().cxm_tp_handle(self.h, buf))
        return bytes(buf)

    def tp_connect(self, handles: list[bytes]) -> None:
        """Map every rank's exchange area (handles in rank order)."""
        if len(handles) != self.tp_size or any(len(x) != TP_HANDLE_BYTES for x in handles):
            raise ValueError(f"need {self.tp_size} handles of {TP_HANDLE_BYTES} bytes")
        buf = (C.c_uint8 * (TP_HANDLE_BYTES * self.tp_size)).from_buffer_copy(b"".join(handles))
        _check(lib().cxm_tp_connect(self.h, buf))

    abrir = classmethod(lambda cls, ruta, device=0: cls(ruta, device))
    open = abrir

    @property
    def weight_bytes(self) -> int:
        return lib().cxm_model_weight_bytes(self.h)

    def set_prefill(self, tensor_cores: bool) -> None:
        """Prompts of 24+ tokens on the tensor cores (default) or replayed
        through the decode step; the same results either way."""
        _check(lib().cxm_model_set_prefill(self.h, int(tensor_cores)))

    def cache(self, max_tokens: int | None = None) -> Cache:
        return Cache(self, max_tokens)

    def forward(self, tokens, cache: Cache) -> np.ndarray:
        """Logits of the last token; extends `cache` (src/forward.rs:375-505).
        A tensor-parallel rank returns its vocabulary rows
        [vocab_lo, vocab_lo + vocab_n)."""
        t = np.ascontiguousarray(tokens, np.uint32)
        out = np.zeros(self.vocab_n, np.float32)
        _check(lib().cxm_forward(self.h, cache.h, _ptr(t) if t.size else None, t.size, _ptr(out)))
        return out

    def elegir(self, muestreador: Muestreador) -> int:
        """Muestreador::elegir on the device logits of the last forward."""
        tok = C.c_uint32(0)
        _check(lib().cxm_sample(self.h, muestreador.h, C.byref(tok)))
        return tok.value

    def generar(self, prompt, max_nuevos: int, muestreador: Muestreador, cache: Cache) -> list[int]:
        """Modelo::generar (src/forward.rs:533-559)."""
        p = np.ascontiguousarray(prompt, np.uint32)
        out = np.zeros(max(max_nuevos, 1), np.uint32)
        n = C.c_uint32(0)
        _check(lib().cxm_generate(self.h, cache.h, _ptr(p) if p.size else None, p.size, max_nuevos, muestreador.h,
                                  _ptr(out), C.byref(n)))
        return out[: n.value].tolist()

    generate = generar

    def generar_lote(self, prompts, max_nuevos: int, caches: "list[Cache]") -> list[list[int]]:
        """Greedy Modelo::generar for several conversations at once, one cache
        each (include/cxm.h: cxm_generate_batch)."""
        n = len(caches)
        ps = [np.ascontiguousarray(p, np.uint32) for p in prompts]
        if len(ps) != n:
            raise ValueError("one prompt per cache")
        hs = (P * n)(*[c.h for c in caches])
        pp = (P * n)(*[p.ctypes.data_as(P) for p in ps])
        lens = np.array([p.size for p in ps], np.uint32)
        out = np.zeros((n, max(max_nuevos, 1)), np.uint32)
        n_out = np.zeros(n, np.uint32)
        _check(lib().cxm_generate_batch(self.h, hs, pp, _ptr(lens), n, max_nuevos, _ptr(out), _ptr(n_out)))
        return [out[z, : n_out[z]].tolist() for z in range(n)]

    generate_batch = generar_lote

    # measurement hooks (device-timed; include/cxm.h)
    def bench_decode(self, cache: Cache, steps: int, sampler: "Muestreador | None" = None) -> float:
        """Device time (ms) of `steps` decode steps replayed from the cache's
        end: greedy, or sampled with `sampler` (temperature > 0)."""
        ms = C.c_float(0)
        if sampler is None:
            _check(lib().cxm_bench_decode(self.h, cache.h, steps, C.byref(ms)))
        else:
            _check(lib().cxm_bench_decode_sampled(self.h, cache.h, sampler.h, steps, C.byref(ms)))
        return ms.value

    def bench_sample(self, sampler: "Muestreador", reps: int):
        """Device time (ms) of `reps` runs of the device sampler on the logits
        of the last step, the last run's step ends (ns from its start), then
        the passes of its two sums."""
        ms = C.c_float(0)
        ph = np.zeros(78, np.uint64)
        _check(lib().cxm_bench_sample(self.h, sampler.h, reps, C.byref(ms), _ptr(ph), ph.size))
        return ms.value, ph.tolist()

    def bench_matvec(self, reps: int):
        ms = C.c_float(0)
        nb = C.c_uint64(0)
        _check(lib().cxm_bench_matvec(self.h, reps, C.byref(ms), C.byref(nb)))
        return ms.value, nb.value

    @property
    def step_launches(self) -> int:
        return lib().cxm_step_launches(self.h)

    def __del__(self):
        if getattr(self, "h", None) and _lib is not None:
            _lib.cxm_model_close(self.h)
            self.h = None


Model = Modelo


# ───────────── kernel-level entry points ─────────────

def subblock_sums(ggml_type: int, row: np.ndarray, xq: np.ndarray) -> np.ndarray:
    row = np.ascontiguousarray(row, np.uint8)
    xq = np.ascontiguousarray(xq, np.int8)
    sub = 32 if ggml_type in (Q4_K, Q5_K) else 16
    out = np.zeros(xq.size // sub, np.int32)
    _check(lib().cxm_debug_subblock_sums(ggml_type, _ptr(row), _ptr(xq), xq.size // 256, _ptr(out)))
    return out


def matvec(ggml_type: int, w: np.ndarray, rows: int, k: int, x: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros(rows, np.float32)
    _check(lib().cxm_debug_matvec(ggml_type, _ptr(w), rows, k, _ptr(x), _ptr(y)))
    return y


def matmul(ggml_type: int, w: np.ndarray, rows: int, k: int, x: np.ndarray) -> np.ndarray:
    """ops::matmul_auto on the device: x (m x k) times W (rows x k), each
    output in the order the reference's path for m rows gives it."""
    w = np.ascontiguousarray(w, np.uint8)
    x = np.ascontiguousarray(x, np.float32)
    m = x.size // k
    y = np.zeros(m * rows, np.float32)
    _check(lib().cxm_debug_matmul(ggml_type, _ptr(w), rows, k, _ptr(x), m, _ptr(y)))
    return y.reshape(m, rows)


def expf(x: np.ndarray) -> np.ndarray:
    """The device exp of the decode path (matches the host libm expf)."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    _check(lib().cxm_debug_expf(_ptr(x), _ptr(y), x.size))
    return y


def arm_gemm_stamps(launch: int) -> None:
    """Measurement: the launch-th prompt GEMM from now records its CTA
    (0, 0)'s step times (include/cxm.h, cxm_arm_gemm_stamps)."""
    _check(lib().cxm_arm_gemm_stamps(launch))


def read_gemm_stamps() -> list:
    out = np.zeros(100, np.uint64)
    _check(lib().cxm_read_gemm_stamps(_ptr(out), out.size))
    return out.tolist()


def seq_sums(x: np.ndarray) -> np.ndarray:
    """The running f32 sums of x, rounded one addition at a time as the
    reference's loops round them, by the device sampler's summation."""
    x = np.ascontiguousarray(x, np.float32)
    y = np.zeros_like(x)
    _check(lib().cxm_debug_seq_sums(_ptr(x), _ptr(y), x.size))
    return y


def attention(q, k, v, total: int, heads: int, heads_kv: int, head_dim: int) -> np.ndarray:
    q, k, v = (np.ascontiguousarray(a, np.float32) for a in (q, k, v))
    out = np.zeros(heads * head_dim, np.float32)
    _check(lib().cxm_debug_attention(_ptr(q), _ptr(k), _ptr(v), total, heads, heads_kv, head_dim, _ptr(out)))
    return out


def attention_noalloc(q_dev: int, k_dev: int, v_dev: int, total: int, heads: int, heads_kv: int, head_dim: int,
                      out_dev: int, stream: int = 0) -> None:
    """Attention on caller-owned device buffers (addresses as ints), without
    any device allocation inside the library; see cxm_attention_noalloc in
    include/cxm.h for its scratch limit and its sharing rule."""
    _check(lib().cxm_attention_noalloc(q_dev, k_dev, v_dev, total, heads, heads_kv, head_dim, out_dev,
                                       stream or None))
