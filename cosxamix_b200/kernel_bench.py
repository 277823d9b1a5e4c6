"""Kernel micro-benchmarks on a synthetic model (device-timed, CUDA events).

    python -m cosxamix_b200.kernel_bench [--config qwen3b] [--reps 108]

Times the gate/up k-quant matvec of the model, cycling over its layers so
every launch streams its own weights from HBM (36 layers x 25 MB > L2), and
prints the per-launch time and the algorithmic weight bytes per second. Used
for the ncu captures summarised under profiles/.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="qwen3b")
    ap.add_argument("--seed", type=int, default=42)
    ap.add_argument("--reps", type=int, default=108)
    args = ap.parse_args()
    import bench
    import cosxamix_b200 as cx

    path = bench.ensure_model(args.config, args.seed)
    m = cx.Modelo(path)
    ms, nbytes = m.bench_matvec(args.reps)
    print(json.dumps({"kernel": "k_matvec gate/up", "config": args.config, "launch_us": round(ms * 1000, 3),
                      "bytes_per_launch": nbytes, "gbs": round(nbytes / (ms / 1000) / 1e9, 1)}))


if __name__ == "__main__":
    main()
