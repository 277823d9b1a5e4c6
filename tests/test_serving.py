"""Host logic of data-parallel serving (the shared-prefix configuration) on CPU: the
conversation shards, the shared-prefix reuse and the job reduction, run as
world_size-2 gloo process groups (no GPU)."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from cosxamix_b200 import serving


def test_shards_cover_every_conversation_once():
    for world in (1, 2, 3, 4, 8):
        seen = []
        for r in range(world):
            seen += serving.shard(64, r, world)
        assert sorted(seen) == list(range(64))
    assert serving.shard(5, 1, 2) == [1, 3]
    with pytest.raises(ValueError):
        serving.shard(4, 2, 2)


def test_seeded_tokens_follow_the_reference_generator():
    # Azar::con_semilla(42).siguiente() (src/daiss.rs:317-337), modulo vocab
    st = 42
    x = st
    x ^= x >> 12
    x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
    x ^= x >> 27
    assert serving.seeded_tokens(42, 1, 1 << 62)[0] == ((x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF) % (1 << 62)
    w = serving.Workload()
    assert len(w.prefix_tokens(151936)) == 1024 and len(w.suffix_tokens(3, 151936)) == 64
    assert w.suffix_tokens(3, 151936) != w.suffix_tokens(4, 151936)


class _Cfg:
    vocab = 1000


class _Cache:
    def __init__(self):
        self.toks = []
        self.lender = None

    def copiar_prefijo(self, src, n):
        self.toks = list(src.toks[:n])

    def compartir_prefijo(self, src, n):  # borrowed, not copied: read through the lender
        self.lender = (src, n)
        self.toks = []

    def all_toks(self):
        return (list(self.lender[0].toks[: self.lender[1]]) if self.lender else []) + self.toks


class _Model:
    """CPU stand-in with the Modelo interface serve() uses: the next token
    is a function of everything in the cache, like a decoder."""
    cfg = _Cfg()

    def __init__(self):
        self.prefills = 0

    def cache(self, n):
        return _Cache()

    def forward(self, toks, c):
        self.prefills += 1
        c.toks += list(toks)

    def generar(self, prompt, n, sampler, c):
        c.toks += list(prompt)
        out = []
        for _ in range(n):
            t = (sum(c.all_toks()) * 31 + len(c.all_toks())) % self.cfg.vocab
            out.append(t)
            c.toks.append(t)
        return out

    def generar_lote(self, prompts, n, caches):
        self.batches = getattr(self, "batches", 0) + 1
        return [self.generar(p, n, None, c) for p, c in zip(prompts, caches)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        work = serving.Workload(conversations=10, prefix=16, suffix=4, new_tokens=6)
        model = _Model()
        mine = serving.shard(work.conversations, rank, world)
        out, secs, n = serving.serve(model, work, mine, lambda: None)
        job_s, job_n = serving.reduce_job(0.5 + rank, n)
        q.put((rank, out, job_s, job_n, model.prefills))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_serve_the_same_conversations_as_one():
    work = serving.Workload(conversations=10, prefix=16, suffix=4, new_tokens=6)
    single, _, n1 = serving.serve(_Model(), work, list(range(10)), lambda: None)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    merged = {}
    for rank, out, job_s, job_n, prefills in res:
        assert set(out) == set(serving.shard(10, rank, 2))
        merged.update(out)
        assert job_s == 1.5        # the slowest rank's time
        assert job_n == n1         # every rank's tokens
        assert prefills == 1       # the shared prefix once per rank
    assert merged == single


def test_batched_serving_borrows_the_prefix_and_matches_one_at_a_time():
    work = serving.Workload(conversations=10, prefix=16, suffix=4, new_tokens=6)
    single, _, n1 = serving.serve(_Model(), work, list(range(10)), lambda: None)
    model = _Model()
    batched, _, n2 = serving.serve_batched(model, work, list(range(10)), max_batch=4)
    assert batched == single and n2 == n1
    assert model.prefills == 1 and model.batches == 3  # groups of 4, 4 and 2
