"""Tensor parallelism on 2 GPUs (one process per GPU, gloo for the host-side
handle exchange): the TP=2 model against the same model on one GPU, and a
rank that never launches its step. Skipped with fewer than two GPUs."""
import os
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


needs2 = pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.fixture(scope="module")
def tp_model(tmp_path_factory):
    import cosxamix_b200 as cx
    path = str(tmp_path_factory.mktemp("tp") / "tp_small.gguf")
    cx.synth_write(path, cx.synth_spec("tp_small", seed=11))
    return path


def _seeded(seed, n, vocab):
    from cosxamix_b200 import serving
    return serving.seeded_tokens(seed, n, vocab)


def _parity_rank(rank, world, port, path, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    import cosxamix_b200 as cx
    from cosxamix_b200 import tensor_parallel as tpm
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = cx.Modelo(path, device=rank, tp=(rank, world))
        tpm.connect(m)
        V = m.cfg.vocab
        prompt = _seeded(5, 40, V)
        c = m.cache(256)
        logits = tpm.gather_logits(m, m.forward(prompt, c))
        c2 = m.cache(256)
        toks = m.generar(_seeded(9, 24, V), 64, cx.Muestreador.voraz(), c2)
        res = {"rank": rank, "logits": logits, "toks": toks}
        if rank == 0:  # the same model on one GPU
            s = cx.Modelo(path, device=0)
            res["logits1"] = s.forward(prompt, s.cache(256))
            res["toks1"] = s.generar(_seeded(9, 24, V), 64, cx.Muestreador.voraz(), s.cache(256))
            # the CPU oracle with the same split: o_proj / ffn_down as two
            # K-slice partial sums added in rank order
            from oracle import oracle as orc
            orc.set_tp(world)
            om = orc.Model(path)
            res["logits_orc"] = om.forward(orc.Cache(om), prompt)
            res["toks_orc"] = om.generate(orc.Cache(om), _seeded(9, 24, V), 64, orc.Sampler(0, 0.0, 1.0))
            orc.set_tp(1)
        q.put(res)
        dist.barrier()
    finally:
        dist.destroy_process_group()


@needs2
def test_tp2_logits_and_greedy_tokens_match_one_gpu(tp_model):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_parity_rank, args=(r, 2, port, tp_model, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {r["rank"]: r for r in (q.get(timeout=600) for _ in procs)}
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    a, b = res[0]["logits"], res[0]["logits1"]
    np.testing.assert_array_equal(res[0]["logits"], res[1]["logits"])  # both ranks see the same gathered logits
    # bit-exact against the oracle's emulation of the same two-rank split
    np.testing.assert_array_equal(a, res[0]["logits_orc"])
    assert res[0]["toks"] == res[1]["toks"] == list(res[0]["toks_orc"])
    # Against the single-rank order: the split sums round differently, and a
    # changed rounding can flip an i8 activation downstream. On this model the
    # oracle itself moves by 6.5e-3 of the logit range between 1 and 2 ranks,
    # and its greedy picks from the second prompt differ from the first token
    # on (the random-init logits are nearly flat), so only the logits are
    # bounded here.
    rel = float(np.max(np.abs(a - b)) / (b.max() - b.min()))
    assert rel <= 2e-2, rel


def _stall_rank(rank, world, port, path, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    import torch.distributed as dist
    import cosxamix_b200 as cx
    from cosxamix_b200 import tensor_parallel as tpm
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = cx.Modelo(path, device=rank, tp=(rank, world))
        tpm.connect(m)
        c = m.cache(64)
        if rank == 0:  # rank 1 never launches: the exchange wait runs out
            t = time.time()
            try:
                m.forward([1, 2, 3], c)
                q.put((rank, "no error", time.time() - t))
            except ValueError as e:
                q.put((rank, str(e), time.time() - t))
        dist.barrier()  # rank 1 stays alive (its exchange area mapped) until rank 0 is done
        if rank == 1:
            q.put((rank, "idle", 0.0))
    finally:
        dist.destroy_process_group()


@needs2
def test_tp_rank_that_never_launches_ends_the_step_with_an_error(tp_model):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_stall_rank, args=(r, 2, port, tp_model, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict((r, (msg, dt)) for r, msg, dt in (q.get(timeout=600) for _ in procs))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    msg, dt = res[0]
    assert "timed out" in msg, msg
    assert dt < 60, dt
