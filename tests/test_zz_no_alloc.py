"""cxm_attention_noalloc: the attention kernels on caller-owned device buffers,
with their scratch in a static device array instead of a per-call
allocation. Checked against the allocating entry point (cxm_debug_attention,
itself bit-exact with the oracle's ops::atencion restatement) on two calls in
a row, which must both match exactly.

Collected last (file name) so it runs both after the rest of the suite and,
alone, in a fresh process."""
import numpy as np
import pytest

import cosxamix_b200 as cx

pytestmark = pytest.mark.gpu


def _inputs(heads, kvh, hd, total, seed):
    rng = np.random.default_rng(seed)
    q = rng.standard_normal(heads * hd).astype(np.float32)
    k = rng.standard_normal(total * kvh * hd).astype(np.float32)
    v = rng.standard_normal(total * kvh * hd).astype(np.float32)
    return q, k, v


@pytest.mark.parametrize("heads,kvh,hd,total", [(16, 2, 128, 640), (8, 8, 32, 96), (4, 2, 64, 1),
                                               (16, 2, 128, 4096)])
def test_noalloc_matches_allocating_entry_point_twice(heads, kvh, hd, total):
    import torch
    q, k, v = _inputs(heads, kvh, hd, total, seed=total + heads)
    want = cx.attention(q, k, v, total, heads, kvh, hd)
    dev = torch.device("cuda:0")
    dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    for call in range(2):
        out = torch.full((heads * hd,), float("nan"), dtype=torch.float32, device=dev)
        torch.cuda.synchronize()
        cx.attention_noalloc(dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), total, heads, kvh, hd, out.data_ptr())
        got = out.cpu().numpy()
        np.testing.assert_array_equal(got, want, err_msg=f"call {call + 1}")


def test_noalloc_takes_no_device_memory():
    import torch
    heads, kvh, hd, total = 16, 2, 128, 640
    q, k, v = _inputs(heads, kvh, hd, total, seed=7)
    dev = torch.device("cuda:0")
    dq, dk, dv = (torch.from_numpy(a).to(dev) for a in (q, k, v))
    out = torch.empty(heads * hd, dtype=torch.float32, device=dev)
    args = (dq.data_ptr(), dk.data_ptr(), dv.data_ptr(), total, heads, kvh, hd, out.data_ptr())
    cx.attention_noalloc(*args)  # first call on the device: scratch address lookup
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        cx.attention_noalloc(*args)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_sizes_beyond_its_scratch():
    import torch
    heads, kvh, hd = 32, 8, 64
    total = 65536 // heads + 1  # one position more than the scratch holds
    dev = torch.device("cuda:0")
    dq = torch.zeros(heads * hd, device=dev)
    dkv = torch.zeros(total * kvh * hd, device=dev)
    out = torch.zeros(heads * hd, device=dev)
    with pytest.raises(ValueError, match="attention scratch holds 65536 scores"):
        cx.attention_noalloc(dq.data_ptr(), dkv.data_ptr(), dkv.data_ptr(), total, heads, kvh, hd, out.data_ptr())
