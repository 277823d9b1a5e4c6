"""Tensor parallelism across the GPUs of one box (the 8B-shape configuration).

One process per GPU. Rank r of N opens its share of the model
(`Modelo(path, device, tp=(r, N))`): the attention block whole (q/k/v of
every head, the whole KV cache, o_proj), the gate/up rows of its FFN slice
[r·F/N, (r+1)·F/N), the ffn_down rows of its hidden slice [r·D/N, (r+1)·D/N)
over the whole FFN vector, its vocabulary rows, and the embedding and norms.
Every decode step gathers the FFN's hidden vector and the residual stream
from the ranks' slices and picks the argmax over their vocabulary slices,
over peer memory inside the decode kernel (no NCCL on the data path). Each
value is computed by one rank exactly as one GPU computes it, so the model's
logits and tokens do not depend on N. This module only wires the ranks
together: the CUDA IPC handles of the exchange areas travel over any
torch.distributed process group (gloo or NCCL).
"""
from __future__ import annotations


def shares(dim: int, ffn: int, vocab: int, rank: int, size: int) -> dict:
    """This rank's rows, as the library splits them (model.cu's
    cxm_model_open_tp): FFN rows and hidden rows in equal slices (multiples
    of 4, the exchanges' 16-byte units), an even share of the vocabulary rows
    (the last rank takes the rest); the attention block is every rank's."""
    if size < 1 or not 0 <= rank < size:
        raise ValueError(f"rank {rank} of {size}")
    if dim % (4 * size) or ffn % (4 * size):
        raise ValueError(f"hidden {dim} / FFN {ffn} do not split over {size} ranks in groups of 4")
    fl, dl = ffn // size, dim // size
    vn = vocab if size == 1 else (vocab // size) & ~1
    vlo = rank * vn
    if rank == size - 1:
        vn = vocab - vlo
    return {"attention": (0, dim), "ffn_rows": (rank * fl, fl), "down_rows": (rank * dl, dl),
            "vocab_rows": (vlo, vn)}


def connect(model, group=None) -> None:
    """Exchange the ranks' IPC handles over `group` and map them."""
    import torch.distributed as dist
    handles = [None] * dist.get_world_size(group)
    dist.all_gather_object(handles, model.tp_handle(), group=group)
    model.tp_connect(handles)


def gather_logits(model, local, group=None):
    """The whole vocabulary's logits from the ranks' slices (host arrays)."""
    import numpy as np
    import torch.distributed as dist
    parts = [None] * dist.get_world_size(group)
    dist.all_gather_object(parts, (model.vocab_lo, np.asarray(local)), group=group)
    out = np.zeros(model.cfg.vocab, np.float32)
    for lo, v in parts:
        out[lo:lo + len(v)] = v
    return out
