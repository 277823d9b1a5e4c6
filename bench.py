"""Decode benchmark: batch-1 greedy decode of the Qwen2.5-3B-shaped Q4_K_M
synthetic model (the headline configuration: 512-token prompt) through the
C ABI.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
                    [--config tiny|qwen3b|...] [--workload decode|formats|shared-prefix|tp]

One process per GPU (torchrun for N > 1). Every rank decodes its own
conversation with replicated weights — independent conversations, no
collective on the data path — so `value` is the sum over ranks (weak scaling).
A step is one decode token: the forward of one token plus the greedy pick.

The other workloads (each prints its own one-line JSON): `formats`
(the 3B shape uniform in Q5_K, Q3_K, Q2_K, sampled decode),
`shared-prefix` (64 conversations sharded over the ranks, one shared
1024-token prefix prefilled once per GPU), `tp` (one Llama-3-8B-shaped
conversation, tensor-parallel over the ranks).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s bs=1, 3B-shape Q4_K_M; weight-stream HBM GB/s vs ~8 TB/s peak"
WORKLOAD = "qwen2.5-3B-shape Q4_K_M (Q6_K tied output, half of attn_v/ffn_down), synthetic N(0,0.02), " \
           "512-token seeded prompt, greedy decode bs=1"
FALLBACK_HBM_GBS = 6650.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def model_path(config: str, seed: int) -> str:
    d = os.environ.get("CXM_MODEL_DIR", tempfile.gettempdir())
    return os.path.join(d, f"cxm_{config}_s{seed}.gguf")


def ensure_model(config: str, seed: int, separate_process: bool = False) -> str:
    """The seeded synthetic GGUF of `config` (written once per box). The
    writer is this library's; `separate_process` writes it from a child
    process, so a process that times the reference never loads the library."""
    p = model_path(config, seed)
    if not os.path.exists(p):
        t = time.time()
        if separate_process:
            code = ("import sys; sys.path.insert(0, %r); import cosxamix_b200 as cx; "
                    "cx.synth_write(%r, cx.synth_spec(%r, seed=%d))" % (ROOT, p, config, seed))
            subprocess.run([sys.executable, "-c", code], check=True)
        else:
            import cosxamix_b200 as cx
            cx.synth_write(p, cx.synth_spec(config, seed=seed))
        print(f"[bench] wrote {p} in {time.time() - t:.1f}s", file=sys.stderr)
    return p


def decode_config(args, world: int) -> dict:
    """The `config` of the decode workload's line, the same in both arms."""
    return {"workload": workload_of(args), "prompt": args.prompt, "decode_steps": args.steps,
            "parallelism": f"dp{world} (independent conversations, replicated weights)",
            "l2": "inputs larger than L2: 1.92 GB of weights streamed per step vs 126 MB L2"}


def workload_of(args) -> str:
    """The workload label: the headline configuration's, or the named synthetic shape."""
    if args.config == "qwen3b":
        return WORKLOAD
    return f"{args.config}-shape synthetic model, {args.prompt}-token seeded prompt, greedy decode bs=1"


def seeded_prompt(seed: int, n: int, vocab: int):
    # uniform token ids from the reference's xorshift64* (src/daiss.rs:317-337)
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


class Clocks:
    """nvidia-smi samples during the timed region (clocks + throttle reasons)."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, device: int):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                       "-lms", "200", "-i", str(device)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self) -> dict:
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        self.p.wait()
        self.f.flush()
        rows = []
        with open(self.f.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) == 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        smax = max(int(r[2]) for r in rows)
        loaded = [int(r[1]) for r in rows if float(r[3] or 0) > 200] or [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": smax, "reasons": reasons, "samples": len(rows)}


def reference_cpu_path() -> tuple:
    """Put the oracle on the kernels the reference runs on an AVX2 host and
    describe them: (kind, text). The Q4_K/Q5_K/Q3_K/Q2_K rows go through the
    reference's own compiled kernels when oracle/_ref was built (the kernel
    whose speed decides the baseline is then the reference's code), Q6_K,
    RMSNorm and attention's dot products through AVX2 restatements of
    src/kernels/x86.rs; the loop around them is the C restatement of
    src/forward.rs:375-505 on a persistent thread pool (32-row tasks, as
    src/ops.rs:486-506)."""
    from oracle import oracle as O
    used = O.set_backend("x86")
    names = {O.Q4K: "Q4_K", O.Q6K: "Q6_K", O.Q5K: "Q5_K", O.Q3K: "Q3_K", O.Q2K: "Q2_K"}
    kernels = ", ".join(f"{names[t]}: {used[t]}" for t in (O.Q4K, O.Q6K))
    return "port", (f"C restatement of the reference's engine_own decode on its x86 AVX2 path ({kernels}; "
                    f"RMSNorm and attention dots: AVX2 restatements of x86.rs), reference Rust not buildable here")


def cpu_baseline(path: str, prompt_len: int, budget_s: float, threads: int = 0) -> dict:
    """The reference's decode on the host cores (its C restatement on the
    reference's x86 kernels, reference_cpu_path): decode tokens at context
    `prompt_len` for about `budget_s`."""
    from oracle import oracle as O
    if threads:
        O.set_threads(threads)
    kind, text = reference_cpu_path()
    m = O.Model(path)
    c = m.cache()
    c.fill(prompt_len, seed=1)
    tok = 17
    t0 = time.perf_counter()
    logits = m.forward(c, [tok])
    first = time.perf_counter() - t0
    n = max(2, min(200, int(budget_s / max(first, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(n):
        tok = int(O.lib().orc_argmax(O.ptr(logits), logits.size))
        logits = m.forward(c, [tok])
    dt = time.perf_counter() - t0
    O.set_backend("scalar")
    return {"value": n / dt, "unit": "tok/s", "cores": O.threads(), "kind": kind,
            "sample": f"{n} greedy decode tokens at context {prompt_len}..{prompt_len + n} "
                      f"(KV prefix filled with seeded values instead of a CPU prefill); {text}"}


def run_reference(args, rank: int, world: int) -> None:
    """`--impl reference`: the reference's CPU implementation of the path
    (its C restatement on the reference's x86 kernels, reference_cpu_path),
    timed on this box's host cores."""
    if rank != 0:
        return
    path = ensure_model(args.config, args.seed, separate_process=True)
    from oracle import oracle as O
    kind, text = reference_cpu_path()
    m = O.Model(path)
    c = m.cache()
    c.fill(args.prompt, seed=1)
    tok = 17
    logits = None
    for _ in range(args.warmup):
        logits = m.forward(c, [tok])
        tok = int(O.lib().orc_argmax(O.ptr(logits), logits.size))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        logits = m.forward(c, [tok])
        tok = int(O.lib().orc_argmax(O.ptr(logits), logits.size))
    dt = time.perf_counter() - t0
    v = args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": round(v, 4), "unit": "tok/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1000 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8-dot/f32", "data": "synthetic",
        "config": decode_config(args, world),
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": O.threads(), "kind": kind,
                         "sample": f"{args.steps} greedy decode tokens per step-set at context {args.prompt} (KV "
                                   f"prefix seeded instead of a CPU prefill), all host threads; {text}"},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_shared_prefix(args, rank: int, world: int, local: int) -> None:
    """`--workload shared-prefix` (the data-parallel configuration): 64 conversations
    sharing a 1024-token seeded system prefix, each with its own 64-token
    suffix and 128 greedy tokens, sharded over the ranks (replicated weights,
    no collective). Each rank prefills the prefix once (untimed setup), then
    serves its conversations through the public API: each borrows the prefix
    (cxm_cache_share_prefix) and all of them decode together
    (cxm_generate_batch). value = all ranks' generated tokens / the slowest
    rank's time."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import cosxamix_b200 as cx
    from cosxamix_b200 import serving

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))
    if rank == 0:
        ensure_model(args.config, args.seed)
    if world > 1:
        dist.barrier()
    m = cx.Modelo(model_path(args.config, args.seed), device=local)
    work = serving.Workload(conversations=args.conversations, seed=args.seed)
    mine = serving.shard(work.conversations, rank, world)
    # warm-up: one conversation's worth, outside the timed region
    serving.serve_batched(m, serving.Workload(conversations=2, prefix=16, suffix=4, new_tokens=4, seed=args.seed + 7),
                          [0, 1])
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    _, secs, n = serving.serve_batched(m, work, mine)
    torch.cuda.synchronize()
    secs, n = serving.reduce_job(secs, n)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    v = n / secs
    line = {
        "metric": "shared-prefix serving tok/s (generated), 3B-shape Q4_K_M", "value": round(v, 3), "unit": "tok/s",
        "n_gpus": world, "steps": work.conversations, "warmup": 1, "ms_per_step": round(secs * 1000 / max(1, len(mine)), 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-dot/f32",
        "data": "synthetic",
        "config": {"workload": f"{work.conversations} conversations, shared {work.prefix}-token seeded "
                               f"prefix (prefilled once per GPU, held once), {work.suffix}-token suffix each, "
                               f"{work.new_tokens} greedy tokens each, decoded together",
                   "parallelism": f"dp{world} (conversations sharded, replicated weights, no collective)"},
        "generated_tokens": n,
        "e2e": {"value": round(v, 3), "unit": "tok/s", "h2d_bytes_per_step": 4 * work.suffix,
                "d2h_bytes_per_step": 4 * work.new_tokens,
                "api": "cxm_cache_share_prefix per conversation + cxm_generate_batch"},
    }
    print(json.dumps(line), flush=True)


def run_formats(args, rank: int, world: int, local: int) -> None:
    """`--workload formats` (the uniform-format configuration): the Qwen2.5-3B shape
    re-quantized uniformly to Q5_K, Q3_K and Q2_K, one model after the other:
    128-token seeded prompt (untimed prefill), then sampled decode at
    temperature 0.7, top-p 0.9 (seed 42), every step the decode kernel plus
    the device sampler. Per format: device-timed tok/s and weight-stream GB/s.
    Each rank runs its own conversation (replicated weights, no collective).
    The greedy decode step is timed as well, K more steps on the same cache:
    its weight-stream GB/s is the format's figure, the sampled step's extra
    time is the device sampler's (sequential sums over the whole vocabulary
    in the reference's order)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import cosxamix_b200 as cx

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=900), device_id=torch.device("cuda", local))
    peak, peak_kind = peaks()
    out = {}
    total_ms = 0.0
    for fmt in ("q5k", "q3k", "q2k"):
        name = f"qwen3b_{fmt}"
        if rank == 0:
            ensure_model(name, args.seed)
        if world > 1:
            dist.barrier()
        m = cx.Modelo(model_path(name, args.seed), device=local)
        cache = m.cache(args.prompt + args.warmup + 2 * args.steps + 8)
        m.forward(seeded_prompt(args.seed + rank, args.prompt, m.cfg.vocab), cache)
        samp = cx.Muestreador(42, 0.7, 0.9)
        m.bench_decode(cache, args.warmup, samp)
        clocks = Clocks(local)
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        ms = m.bench_decode(cache, args.steps, samp)
        # the decode kernel alone (greedy steps), for the format's weight stream
        ms_k = m.bench_decode(cache, args.steps)
        clk = clocks.stop()
        if world > 1:
            t = torch.tensor([ms, ms_k], device="cuda")
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, ms_k = (float(v) for v in t.tolist())
        tok_s = world * args.steps / (ms / 1000.0)
        gbs = m.weight_bytes / (ms_k / args.steps / 1000.0) / 1e9
        out[fmt] = {"tok_s": round(tok_s, 3), "ms_per_step": round(ms / args.steps, 4),
                    "decode_kernel_ms_per_step": round(ms_k / args.steps, 4),
                    "sampler_ms_per_step": round((ms - ms_k) / args.steps, 4),
                    "weight_bytes": m.weight_bytes, "weight_gbs_per_gpu": round(gbs, 1),
                    "frac": round(gbs / peak, 4), "clocks": clk}
        total_ms += ms
        del cache, m
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    value = world * 3 * args.steps / (total_ms / 1000.0)
    line = {
        "metric": "decode tok/s bs=1, 3B-shape uniform Q5_K/Q3_K/Q2_K, top-p 0.9 T 0.7; weight-stream GB/s per format",
        "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / (3 * args.steps), 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8-dot/f32", "data": "synthetic",
        "config": {"workload": f"configs[2]: qwen2.5-3B shape, uniform Q5_K, Q3_K, Q2_K (three models), "
                               f"{args.prompt}-token seeded prompt, sampled decode (seed 42, T 0.7, top-p 0.9)",
                   "parallelism": f"dp{world} (independent conversations, replicated weights)",
                   "l2": "inputs larger than L2: 1.0-2.1 GB of weights streamed per step vs 126 MB L2"},
        "formats": out, "peak_gbs": peak, "peak_kind": peak_kind,
        "gpu_launches": 3 * args.steps * 2,
    }
    print(json.dumps(line), flush=True)


def run_tp(args, rank: int, world: int, local: int) -> None:
    """`--workload tp` (the tensor-parallel configuration): one Llama-3-8B-shaped Q4_K_M
    conversation, tensor-parallel over the ranks (torchrun, one process per
    GPU): each rank holds its heads / FFN rows / vocabulary rows, and every
    step exchanges the o_proj and ffn_down partial sums and the argmax over
    peer memory inside the decode kernel. Untimed prefill of a seeded prompt,
    then K greedy steps timed with CUDA events; value = tokens of the one
    conversation / the slowest rank's time (strong scaling)."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import cosxamix_b200 as cx
    from cosxamix_b200 import tensor_parallel as tpm

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("gloo", timeout=timedelta(seconds=1200))
    if rank == 0:
        ensure_model(args.config, args.seed)
    if world > 1:
        dist.barrier()
    m = cx.Modelo(model_path(args.config, args.seed), device=local, tp=(rank, world))
    if world > 1:
        tpm.connect(m)
    cache = m.cache(min(args.prompt + args.warmup + args.steps + 8, m.cfg.ctx))
    m.forward(seeded_prompt(args.seed, args.prompt, m.cfg.vocab), cache)  # prefill (untimed)
    m.bench_decode(cache, args.warmup)
    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = m.bench_decode(cache, args.steps)
    clk = clocks.stop()
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    nccl = nccl_exchange_baseline(m, world, local) if world > 1 else None
    peak, peak_kind = peaks()
    wbytes = m.weight_bytes  # this rank's share
    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return
    value = args.steps / (ms / 1000.0)
    line = {
        "metric": "decode tok/s bs=1, 8B-shape Q4_K_M, tensor-parallel", "value": round(value, 3), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8-dot/f32",
        "data": "synthetic",
        "config": {"workload": f"{args.config} shape Q4_K_M, {args.prompt}-token seeded prompt, "
                               f"greedy decode bs=1", "parallelism": f"tp{world} (attention replicated, FFN rows "
                               f"split; the hidden vector, the residual and the argmax gathered from the peers' "
                               f"memory inside the decode kernel)",
                   "l2": "inputs larger than L2: the weight shares stream from HBM every step"},
        "weight_stream": {"bytes_per_token_rank0": wbytes,
                          "gbs_per_gpu_rank0": round(wbytes / (ms / args.steps / 1000.0) / 1e9, 1),
                          "peak_gbs": peak, "peak_kind": peak_kind},
        "gpu_launches": args.steps * m.step_launches, "clocks": clk,
    }
    if nccl:
        line["nccl_baseline"] = nccl
    print(json.dumps(line), flush=True)


def nccl_exchange_baseline(m, world: int, local: int, reps: int = 20) -> dict:
    """The same exchanges as NCCL collectives: per token, per layer an
    all-gather of the FFN hidden vector and one of the residual stream (the
    ranks' slices), and one all-gather of the argmax keys; timed alone with
    CUDA events over `reps` tokens' worth (max over ranks). What a step with
    NCCL between kernel launches would spend in collectives, against the
    in-kernel peer-memory gathers."""
    import torch
    import torch.distributed as dist
    g = dist.new_group(backend="nccl")
    dev = torch.device("cuda", local)
    F, D, L = m.cfg.ffn, m.cfg.dim, m.cfg.n_layer
    hs = torch.zeros(F // world, device=dev)
    hb = torch.zeros(F, device=dev)
    xs = torch.zeros(D // world, device=dev)
    xb = torch.zeros(D, device=dev)
    ks = torch.zeros(1, dtype=torch.int64, device=dev)
    kb = torch.zeros(world, dtype=torch.int64, device=dev)

    def token():
        for _ in range(L):
            dist.all_gather_into_tensor(hb, hs, group=g)
            dist.all_gather_into_tensor(xb, xs, group=g)
        dist.all_gather_into_tensor(kb, ks, group=g)

    for _ in range(3):
        token()
    torch.cuda.synchronize()
    dist.barrier(group=g)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        token()
    e1.record()
    e1.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / reps], dtype=torch.float64, device=dev)
    dist.all_reduce(ms, op=dist.ReduceOp.MAX, group=g)
    dist.barrier(group=g)
    dist.destroy_process_group(g)
    return {"collectives_per_token": 2 * L + 1, "ms_per_token": round(float(ms.item()), 4),
            "what": "NCCL all_gather_into_tensor of the same slices (hidden vector and residual per layer, argmax "
                    "keys), collectives only, CUDA-event timed, max over ranks"}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3b")
    ap.add_argument("--prompt", type=int, default=512)
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "shared-prefix", "formats", "tp"])
    ap.add_argument("--conversations", type=int, default=64)
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if args.workload == "shared-prefix":
        run_shared_prefix(args, rank, world, local)
        return
    if args.workload == "tp":
        if args.config == "qwen3b":  # the tensor-parallel configuration is the 8B shape with a 4096-token prompt
            args.config = "llama8b"
            if args.prompt == 512:
                args.prompt = 4096
        run_tp(args, rank, world, local)
        return
    if args.workload == "formats":
        if args.prompt == 512:  # the default of the main workload; the uniform-format configuration prompts with 128
            args.prompt = 128
        run_formats(args, rank, world, local)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import cosxamix_b200 as cx

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    if rank == 0:
        path = ensure_model(args.config, args.seed)
    if world > 1:
        dist.barrier()
    path = model_path(args.config, args.seed)

    m = cx.Modelo(path, device=local)
    cfg = m.cfg
    e2e_steps = max(8, min(args.steps, 64))
    need = args.prompt + args.warmup + args.steps + e2e_steps + 8
    cache = m.cache(min(need, cfg.ctx))
    prompt = seeded_prompt(args.seed + rank, args.prompt, cfg.vocab)
    m.forward(prompt, cache)                           # prefill (untimed)
    m.bench_decode(cache, args.warmup)                 # warm-up steps (untimed)

    # timed: K decode steps, inputs resident, device events on the model stream
    clocks = Clocks(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = m.bench_decode(cache, args.steps)
    torch.cuda.synchronize()
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clk = clocks.stop()
    value = world * args.steps / (ms / 1000.0)

    # end to end through the public API: host token in, host token out
    pinned = torch.zeros(1, dtype=torch.int32, pin_memory=True)
    sampler = cx.Muestreador.voraz()
    tok = m.elegir(sampler)
    import ctypes
    lib = cx.lib()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        pinned[0] = tok
        rc = lib.cxm_forward(m.h, cache.h, pinned.data_ptr(), 1, None)
        if rc:
            raise ValueError(cx._err())
        tok = m.elegir(sampler)
    dt = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([dt], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    e2e = world * e2e_steps / dt

    # The dominant (only) kernel: k_decode, one launch per decode step. Its
    # algorithmic bytes: every weight once, the KV prefix read by attention at
    # the timed steps' mean context, the new K/V row written.
    peak, peak_kind = peaks()
    kvd = cfg.n_head_kv * cfg.head_dim
    ctx_mean = args.prompt + args.warmup + (args.steps + 1) / 2.0
    kv_read = 2 * cfg.n_layer * ctx_mean * kvd * 4
    kv_write = 2 * cfg.n_layer * kvd * 4
    step_bytes = m.weight_bytes + kv_read + kv_write
    achieved = step_bytes / (ms / args.steps / 1000.0) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "decode_step_qwen3b.md")) as f:
            for line in f:
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    traffic = int(line.split(":")[1].strip().split()[0])
    except OSError:
        pass
    # the largest matvec phase alone: gate|up, cycled over the layers
    mv_ms, mv_bytes = m.bench_matvec(3 * cfg.n_layer)

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    cpu = None
    if world == 1 and not args.no_cpu:
        cpu = cpu_baseline(path, args.prompt, args.cpu_budget)
    wbytes = m.weight_bytes
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "int8-dot/f32", "data": "synthetic",
        "config": decode_config(args, world),
        "weight_stream": {"bytes_per_token": wbytes, "gbs_per_gpu": round(value / world * wbytes / 1e9, 1),
                          "frac": round(value / world * wbytes / 1e9 / peak, 4), "peak_gbs": peak,
                          "peak_kind": peak_kind},
        "roofline": {"kernel": "k_decode (one launch = one greedy decode step)", "bound": "hbm",
                     "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s", "frac": round(achieved / peak, 4),
                     "traffic": traffic, "algorithmic_bytes_per_launch": int(step_bytes),
                     "launch_ms": round(ms / args.steps, 5), "peak_kind": peak_kind,
                     "gateup_phase": {"algorithmic_bytes": mv_bytes, "ms": round(mv_ms, 5),
                                      "gbs": round(mv_bytes / (mv_ms / 1000.0) / 1e9, 1)}},
        "cpu_baseline": cpu,
        "e2e": {"value": round(e2e, 3), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 12,
                "api": "cxm_forward([token]) + cxm_sample per step, pinned host token"},
        "gpu_launches": args.steps * m.step_launches,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
