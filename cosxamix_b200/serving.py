"""Shared-prefix serving across GPUs (the data-parallel configuration).

Independent conversations, replicated weights, no collective on the data
path: rank r of N serves conversations r, r + N, r + 2N, ... Each rank
prefills the shared system prefix once into a cache. `serve_batched` (the
served path) has every conversation borrow that prefix (held once,
cxm_cache_share_prefix) and decodes all of the rank's conversations
together, one read of the weights per step for all of them
(cxm_generate_batch); `serve` starts each conversation from a
device-to-device copy of the prefix (Cache::prefijo, src/forward.rs:115-127,
which is what MotorPropio's reuse/borrow of a prefix does for a new chat,
src/engine_own.rs:198-245) and decodes the conversations one after another.
Both give every conversation the tokens the reference gives it alone.

The only cross-rank operations are host bookkeeping: the slowest rank's time
(max) and the total generated tokens (sum), over any torch.distributed
process group (NCCL on the GPUs, gloo in the CPU tests).
"""
from __future__ import annotations

import time
from dataclasses import dataclass


def shard(n_items: int, rank: int, world: int) -> list[int]:
    """The conversations rank `rank` serves: every world-th, from `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    return list(range(rank, n_items, world))


def seeded_tokens(seed: int, n: int, vocab: int) -> list[int]:
    """Uniform token ids from the reference's xorshift64* (src/daiss.rs:317-337)."""
    st = seed if seed else 0x9E3779B97F4A7C15
    out = []
    for _ in range(n):
        x = st
        x ^= x >> 12
        x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 27
        st = x
        out.append(((x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF) % vocab)
    return out


@dataclass
class Workload:
    """One shared prefix, a suffix per conversation, greedy decode."""
    conversations: int = 64
    prefix: int = 1024
    suffix: int = 64
    new_tokens: int = 128
    seed: int = 42

    def prefix_tokens(self, vocab: int) -> list[int]:
        return seeded_tokens(self.seed, self.prefix, vocab)

    def suffix_tokens(self, conv: int, vocab: int) -> list[int]:
        return seeded_tokens(self.seed * 1000003 + conv + 1, self.suffix, vocab)


def serve(model, work: Workload, convs: list[int], sampler_factory, clock=time.perf_counter):
    """Run this rank's conversations; returns ({conv: tokens}, seconds, tokens).

    `model` is a cosxamix_b200.Modelo (or anything with the same cache /
    generar interface); the prefix is prefilled once, then each conversation
    copies it and generates from its own suffix."""
    vocab = model.cfg.vocab
    total = work.prefix + work.suffix + work.new_tokens
    base = model.cache(total)
    model.forward(work.prefix_tokens(vocab), base)
    c = model.cache(total)  # one working cache per rank: its decode graphs are reused
    out = {}
    generated = 0
    t0 = clock()
    for conv in convs:
        c.copiar_prefijo(base, work.prefix)
        toks = model.generar(work.suffix_tokens(conv, vocab), work.new_tokens, sampler_factory(), c)
        out[conv] = toks
        generated += len(toks)
    return out, clock() - t0, generated


def serve_batched(model, work: Workload, convs: list[int], max_batch: int = 512, clock=time.perf_counter):
    """This rank's conversations decoded together (up to max_batch at once),
    each borrowing the prefix prefilled once; returns ({conv: tokens},
    seconds, tokens)."""
    vocab = model.cfg.vocab
    total = work.prefix + work.suffix + work.new_tokens
    base = model.cache(total)
    model.forward(work.prefix_tokens(vocab), base)
    out = {}
    generated = 0
    t0 = clock()
    for i in range(0, len(convs), max_batch):
        group = convs[i:i + max_batch]
        caches = []
        for _ in group:
            c = model.cache(total)
            c.compartir_prefijo(base, work.prefix)
            caches.append(c)
        toks = model.generar_lote([work.suffix_tokens(conv, vocab) for conv in group], work.new_tokens, caches)
        for conv, t in zip(group, toks):
            out[conv] = t
            generated += len(t)
    return out, clock() - t0, generated


def reduce_job(seconds: float, tokens: int, group=None) -> tuple[float, int]:
    """The job's time (the slowest rank) and its generated tokens (all ranks)."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return seconds, tokens
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([seconds], dtype=torch.float64, device=dev)
    n = torch.tensor([tokens], dtype=torch.int64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    dist.all_reduce(n, op=dist.ReduceOp.SUM, group=group)
    return float(t.item()), int(n.item())
