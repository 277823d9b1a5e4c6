"""Generate tests/golden/ref_dots.npz from the reference's own kernels.

Runs ONLY in a container where the reference sources exist: it needs
oracle/_ref/libcxm_ref.so, which `make -C oracle ref` builds straight from the
reference's kernels/q{2,3,5}k_avx2.c and kernels/q{2,3,4,5}k_avx2_sysv.s.

Each case stores the inputs of one fused row·activation dot (the raw GGUF row
bytes, the i8 activation with its per-sub-block scales and sums) and the value
the reference's kernel returned for it. The GPU box has no reference tree, so
the committed fixture is what the tests there read.

Cases:
  * seeded random rows (finite f16 d/dmin) with sin() activations, for
    1, 2, 8, 17 and 43 super-blocks (1 row of 256 .. an FFN row of the 3B);
  * the exact inputs of the reference's own unit test
    `el_fusionado_coincide_con_desempaquetar_y_multiplicar`
    (src/kernels/mod.rs:808-902): bytes (i*131+17)%251, x = sin(0.013 i), K=2048;
  * extreme activations (+127/-127 alternating), as src/kernels/q2k.rs:351-354.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
from oracle import oracle as O  # noqa: E402

KERNELS = {
    O.Q2K: ["cosxamix_q2k_c", "cosxamix_q2k_asm"],
    O.Q3K: ["cosxamix_q3k_c", "cosxamix_q3k_completo"],
    O.Q4K: ["cosxamix_q4k_completo"],
    O.Q5K: ["cosxamix_q5k_c", "cosxamix_q5k_asm"],
}
D_OFFSETS = {O.Q2K: [80, 82], O.Q3K: [108], O.Q4K: [0, 2], O.Q5K: [0, 2], O.Q6K: [208]}


def finite_row(rng, t, nb):
    bb = O.BLOCK_BYTES[t]
    row = rng.integers(0, 256, nb * bb, dtype=np.uint8)
    for b in range(nb):
        for off in D_OFFSETS[t]:
            h = O.f32_to_f16(float(rng.uniform(0.0005, 0.01)))
            row[b * bb + off] = h & 255
            row[b * bb + off + 1] = h >> 8
    return row


def main() -> None:
    if O.ref_lib() is None:
        raise SystemExit("oracle/_ref/libcxm_ref.so missing: run `make -C oracle ref` where the reference exists")
    rng = np.random.default_rng(20261201)
    cases = []
    for t, kernels in KERNELS.items():
        sub = O.SUB[t]
        for nb in (1, 2, 8, 17, 43):
            row = finite_row(rng, t, nb)
            x = np.sin(np.arange(nb * 256) * 0.017 + nb).astype(np.float32)
            cases.append((t, "random", row, x))
        # the reference's own unit-test inputs (src/kernels/mod.rs:820-824)
        nb = 8
        row = np.array([(i * 131 + 17) % 251 for i in range(nb * O.BLOCK_BYTES[t])], np.uint8)
        x = np.sin(np.arange(nb * 256, dtype=np.float32) * np.float32(0.013)).astype(np.float32)
        cases.append((t, "reference-test", row, x))
        # extremes of the i8 contract: +127/-127 alternating
        row = finite_row(rng, t, 3)
        x = np.where(np.arange(3 * 256) % 2 == 0, 1.0, -1.0).astype(np.float32)
        cases.append((t, "extremes", row, x))

    out = {}
    for i, (t, kind, row, x) in enumerate(cases):
        sub = O.SUB[t]
        xq, xe, xs = O.quantize_i8(x, sub)
        vals = np.array([O.ref_dot(k, row, xq, xe, xs) for k in KERNELS[t]], np.float32)
        out[f"c{i}_type"] = np.array([t], np.int32)
        out[f"c{i}_kind"] = np.array([kind])
        out[f"c{i}_row"] = row
        out[f"c{i}_xq"] = xq
        out[f"c{i}_xe"] = xe
        out[f"c{i}_xs"] = xs
        out[f"c{i}_ref"] = vals
        out[f"c{i}_kernels"] = np.array(KERNELS[t])
    out["n"] = np.array([len(cases)], np.int32)
    np.savez_compressed(os.path.join(HERE, "ref_dots.npz"), **out)
    print(f"wrote {len(cases)} cases")


if __name__ == "__main__":
    main()
