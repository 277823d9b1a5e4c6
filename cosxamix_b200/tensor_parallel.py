"""Tensor parallelism across the GPUs of one box (the 8B-shape configuration).

One process per GPU. Rank r of N opens its share of the model
(`Modelo(path, device, tp=(r, N))`): the q/k/v rows of its heads, the
gate/up rows of its FFN slice, the K slice of o_proj and ffn_down, its
vocabulary rows, and the full embedding and norms. Every decode step
exchanges the o_proj and ffn_down partial sums and the per-slice argmax over
peer memory inside the decode kernel (no NCCL on the data path); this module
only wires the ranks together: the CUDA IPC handles of the exchange areas
travel over any torch.distributed process group (gloo or NCCL).
"""
from __future__ import annotations


def shares(n_head: int, n_head_kv: int, head_dim: int, ffn: int, vocab: int, rank: int, size: int) -> dict:
    """This rank's rows, as the library splits them (model.cu's
    cxm_model_open_tp): whole heads and KV heads, FFN rows and o/down K
    slices in whole 256-value super-blocks, an even share of the vocabulary
    rows (the last rank takes the rest)."""
    if size < 1 or not 0 <= rank < size:
        raise ValueError(f"rank {rank} of {size}")
    if n_head % size or n_head_kv % size or (size > 1 and (n_head // size * head_dim) % 256):
        raise ValueError(f"{n_head} heads / {n_head_kv} KV heads do not split over {size} ranks")
    if ffn % (256 * size):
        raise ValueError(f"FFN of {ffn} rows does not split over {size} ranks in super-blocks")
    hl, kl, fl = n_head // size, n_head_kv // size, ffn // size
    vn = vocab if size == 1 else (vocab // size) & ~1
    vlo = rank * vn
    if rank == size - 1:
        vn = vocab - vlo
    return {"q_rows": (rank * hl * head_dim, hl * head_dim), "kv_rows": (rank * kl * head_dim, kl * head_dim),
            "ffn_rows": (rank * fl, fl), "o_k": (rank * hl * head_dim, hl * head_dim), "down_k": (rank * fl, fl),
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
