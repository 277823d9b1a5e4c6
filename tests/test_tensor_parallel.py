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
    hd = c["dim"] // c["n_head"]
    for n in sizes:
        sh = [tpm.shares(c["n_head"], c["n_head_kv"], hd, c["ffn"], c["vocab"], r, n) for r in range(n)]
        assert _cover(c["dim"], [s["q_rows"] for s in sh])
        assert _cover(c["n_head_kv"] * hd, [s["kv_rows"] for s in sh])
        assert _cover(c["ffn"], [s["ffn_rows"] for s in sh])
        assert _cover(c["dim"], [s["o_k"] for s in sh])
        assert _cover(c["vocab"], [s["vocab_rows"] for s in sh])
        for s in sh:  # K slices of whole super-blocks; even vocabulary shares (output row pairs)
            assert s["o_k"][0] % 256 == 0 and s["o_k"][1] % 256 == 0
            assert s["down_k"][0] % 256 == 0 and s["down_k"][1] % 256 == 0
            assert s["vocab_rows"][1] % 2 == 0


def test_shares_reject_what_does_not_split():
    with pytest.raises(ValueError):
        tpm.shares(8, 4, 64, 1024, 8192, 0, 4)   # 2 heads x 64 = 128: not a super-block
    with pytest.raises(ValueError):
        tpm.shares(8, 4, 128, 768, 8192, 0, 2)   # FFN 768 = 3 super-blocks
    with pytest.raises(ValueError):
        tpm.shares(8, 8, 128, 2048, 8192, 2, 2)  # rank out of range


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


def test_oracle_tp_emulation_is_deterministic_and_bounded(tmp_path):
    # the oracle's emulation of N ranks (o_proj / ffn_down as N K-slice
    # partial sums added in rank order), which the GPU's tensor-parallel
    # path matches bit for bit: repeatable, 1 rank = the reference exactly,
    # and within the bound the GPU test uses against the single-rank order
    import cosxamix_b200 as cx
    from cosxamix_b200 import serving
    from oracle import oracle as O
    p = str(tmp_path / "tp_small.gguf")
    cx.synth_write(p, cx.synth_spec("tp_small", seed=11, n_layer=2))
    m = O.Model(p)
    prompt = serving.seeded_tokens(5, 16, 8192)
    try:
        ref = m.forward(O.Cache(m), prompt)
        out = {}
        for n in (2, 4):
            O.set_tp(n)
            a, b = m.forward(O.Cache(m), prompt), m.forward(O.Cache(m), prompt)
            np.testing.assert_array_equal(a, b)
            out[n] = a
        O.set_tp(1)
        np.testing.assert_array_equal(m.forward(O.Cache(m), prompt), ref)
        for n, a in out.items():
            assert not np.array_equal(a, ref)  # the split rounds differently
            assert float(np.max(np.abs(a - ref)) / (ref.max() - ref.min())) <= 2e-2
    finally:
        O.set_tp(1)
