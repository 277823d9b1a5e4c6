"""Kernel micro-benchmarks on a synthetic model (device-timed, CUDA events).

    python -m cosxamix_b200.kernel_bench [--config qwen3b] [--reps 108]
                                         [--layers N] [--vocab V]
                                         [--decode STEPS --prompt P [--sample]]
                                         [--sampler RUNS]
                                         [--prefill P [--gemm-stamps LAUNCH]]

Times the gate|up matvec phase of the decode kernel: `reps` such phases in
one launch, behind grid barriers as in the step, cycling over the model's
layers so every phase streams its own weights (36 layers x 25 MB > L2).
Prints the per-phase time and the algorithmic weight bytes per second.
With --decode: prefills a seeded P-token prompt (one decode-kernel launch
per token), then times STEPS greedy decode steps (one launch each), or with
--sample STEPS sampled steps (the decode kernel, then k_sample). With
--sampler RUNS: the device sampler alone, RUNS times on the prompt's
logits (T 0.7, top-p 0.9), with CTA 0's step ends of the last run. With
--prefill P: the forward of a seeded P-token prompt into an empty cache
(wall clock around the call, which returns once the logits are on the host;
best of 3 after a warm-up); with --gemm-stamps LAUNCH, one more forward in
which that prompt-GEMM launch (0-based, in launch order) records CTA (0, 0)'s
step times per role.
`--layers` / `--vocab` shrink the synthetic model (same matrix shapes) so an
ncu capture holds little device memory; keep layers x 25 MB above the 126 MB
L2 for DRAM figures to mean something.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="qwen3b")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--reps", type=int, default=108)
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--vocab", type=int, default=0)
    ap.add_argument("--decode", type=int, default=0)
    ap.add_argument("--prompt", type=int, default=16)
    ap.add_argument("--sample", action="store_true", help="--decode with the device top-p sampler (T 0.7, top-p 0.9)")
    ap.add_argument("--prefill", type=int, default=0, help="time the forward of a seeded prompt of this many tokens")
    ap.add_argument("--gemm-stamps", type=int, default=-1, help="with --prefill: step times of this GEMM launch")
    ap.add_argument("--sampler", type=int, default=0, help="time RUNS of the device sampler alone on the prompt's logits")
    args = ap.parse_args()
    import bench
    import cosxamix_b200 as cx

    if args.layers or args.vocab:
        over = {}
        if args.layers:
            over["n_layer"] = args.layers
        if args.vocab:
            over["vocab"] = args.vocab
        d = os.environ.get("CXM_MODEL_DIR", tempfile.gettempdir())
        path = os.path.join(d, f"cxm_{args.config}_s{args.seed}_l{args.layers}_v{args.vocab}.gguf")
        if not os.path.exists(path):
            t = time.time()
            cx.synth_write(path, cx.synth_spec(args.config, seed=args.seed, **over))
            print(f"[kernel_bench] wrote {path} in {time.time() - t:.1f}s", file=sys.stderr)
    else:
        path = bench.ensure_model(args.config, args.seed)
    m = cx.Modelo(path)
    if args.prefill:
        prompt = bench.seeded_prompt(args.seed, args.prefill, m.cfg.vocab)
        c = m.cache(min(m.cfg.ctx, args.prefill + 8))
        m.forward(prompt, c)  # warm-up: programs, graphs, workspaces
        times = []
        for _ in range(3):
            c.limpiar()
            t = time.perf_counter()
            m.forward(prompt, c)  # returns the last token's logits: the device work is done
            times.append((time.perf_counter() - t) * 1000)
        out = {"kernel": "prompt forward (tensor-core GEMMs)", "config": args.config,
               "layers": args.layers or None, "tokens": args.prefill,
               "ms": round(min(times), 2), "ms_all": [round(x, 2) for x in times]}
        if args.gemm_stamps >= 0:  # one more forward with a GEMM launch's step times
            c.limpiar()
            cx.arm_gemm_stamps(args.gemm_stamps)
            m.forward(prompt, c)
            st = [round(v / 1000, 2) for v in cx.read_gemm_stamps()]
            out["gemm_stamps_us"] = {"launch": args.gemm_stamps, "mma_in": st[16:32], "prod_in": st[32:48],
                                     "prod_out": st[48:64], "epi_in": st[64:80], "epi_out": st[80:96],
                                     "offsets_done": st[96], "end": st[97], "barrier": st[98],
                                     "chains_8": st[99]}
        print(json.dumps(out))
        return
    if args.sampler:
        c = m.cache(min(m.cfg.ctx, args.prompt + 8))
        m.forward(bench.seeded_prompt(args.seed, args.prompt, m.cfg.vocab), c)
        ms, ph = m.bench_sample(cx.Muestreador(42, 0.7, 0.9), args.sampler)
        names = ["max", "exps", "total", "keys", "radix0", "radix8", "radix16", "radix24", "gather", "cumsum", "end"]
        print(json.dumps({"kernel": "k_sample", "config": args.config, "layers": args.layers or None,
                          "vocab": m.cfg.vocab, "us_per_run": round(ms * 1000 / args.sampler, 2),
                          "step_end_us": {n: round(v / 1000, 2) for n, v in zip(names, ph[1:12])},
                          "sum_passes": {"total": ph[12], "cumsum": ph[13]},
                          "total_pass_start_us": [round(v / 1000, 2) for v in ph[14:14 + min(64, ph[12])]]}))
        return
    if args.decode:
        c = m.cache(min(m.cfg.ctx, args.prompt + args.decode + 8))
        m.forward(bench.seeded_prompt(args.seed, args.prompt, m.cfg.vocab), c)
        samp = cx.Muestreador(42, 0.7, 0.9) if args.sample else None
        ms = m.bench_decode(c, args.decode, samp) / args.decode
        print(json.dumps({"kernel": "k_decode step" + (" + k_sample" if args.sample else ""), "config": args.config,
                          "layers": args.layers or None,
                          "vocab": m.cfg.vocab, "prompt": args.prompt, "step_ms": round(ms, 4),
                          "weight_gbs": round(m.weight_bytes / (ms / 1000) / 1e9, 1)}))
        return
    ms, nbytes = m.bench_matvec(args.reps)
    print(json.dumps({"kernel": "k_decode gate|up phase", "config": args.config, "layers": args.layers or None,
                      "phase_us": round(ms * 1000, 3), "bytes_per_phase": nbytes,
                      "gbs": round(nbytes / (ms / 1000) / 1e9, 1)}))


if __name__ == "__main__":
    main()
