"""Host logic of tensor parallelism (the 8B-shape configuration) on CPU: the row
shares, the exchange of the ranks' IPC handles and the gather of the logits
slices, run as world_size-2 gloo process groups (no GPU)."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from cosxamix_b200 import CONFIGS, tensor_parallel as tpm


def _cover(total, spans):
    seen = np.zeros(total, np.int32)
    for lo, n in spans:
        seen[lo:lo + n] += 1
    return bool((seen == 1).all())


@pytest.mark.parametrize("name,sizes", [("llama8b", (1, 2, 4, 8)), ("tp_small", (1, 2, 4))])
def test_shares_cover_every_row_once(name, sizes):
    c = CONFIGS[name]
    for n in sizes:
        sh = [tpm.shares(c["dim"], c["ffn"], c["vocab"], r, n) for r in range(n)]
        assert _cover(c["ffn"], [s["ffn_rows"] for s in sh])
        assert _cover(c["dim"], [s["down_rows"] for s in sh])
        assert _cover(c["vocab"], [s["vocab_rows"] for s in sh])
        for s in sh:  # the attention block is whole on every rank; exchange slices of 16-byte units
            assert s["attention"] == (0, c["dim"])
            assert s["ffn_rows"][1] % 4 == 0 and s["down_rows"][1] % 4 == 0
            assert s["vocab_rows"][1] % 2 == 0


def test_shares_reject_what_does_not_split():
    with pytest.raises(ValueError):
        tpm.shares(1000, 2048, 8192, 0, 8)   # 1000 / 8 = 125 hidden rows: not a multiple of 4
    with pytest.raises(ValueError):
        tpm.shares(1024, 3000, 8192, 0, 4)   # FFN 3000 / 4 = 750
    with pytest.raises(ValueError):
        tpm.shares(1024, 2048, 8192, 2, 2)   # rank out of range


class _FakeModel:
    """The Modelo surface connect/gather use."""

    def __init__(self, rank, size, vocab=10):
        self.tp_rank, self.tp_size = rank, size
        self.connected = None

        class _C:
            pass
        self.cfg = _C()
        self.cfg.vocab = vocab
        self.vocab_lo = 0 if rank == 0 else 4
        self.vocab_n = 4 if rank == 0 else vocab - 4

    def tp_handle(self):
        return bytes([self.tp_rank + 1]) * 64

    def tp_connect(self, handles):
        self.connected = handles


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m = _FakeModel(rank, world)
        tpm.connect(m)
        local = np.arange(m.vocab_lo, m.vocab_lo + m.vocab_n, dtype=np.float32) * 0.5
        full = tpm.gather_logits(m, local)
        q.put((rank, m.connected, full.tolist()))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_exchange_handles_and_gather_logits():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, handles, full in res:
        assert handles == [bytes([1]) * 64, bytes([2]) * 64]  # rank order, own included
        assert full == [0.5 * i for i in range(10)]
