"""The device exp restates glibc's expf (the function the reference's
f32::exp calls). Its host compilation is checked here against the host libm
over a sampled sweep of every float bit pattern; the device side is checked in
tests/test_gpu_parity.py."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def checker(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("expf") / "expf_exhaustive")
    subprocess.run(["g++", "-O2", "-ffp-contract=off", "-o", exe, os.path.join(ROOT, "tests", "expf_exhaustive.cpp"),
                    "-lm"], check=True)
    return exe


def test_expf_restatement_matches_libm_on_a_sweep_of_all_floats(checker):
    # every 13th bit pattern with two phases: ~660M inputs incl. subnormal
    # results, overflow/underflow thresholds, infinities and NaNs
    for phase in (0, 6):
        out = subprocess.run([checker, "13", str(phase)], capture_output=True, text=True, check=True).stdout.split()
        n, bad = int(out[0]), int(out[1])
        assert n > 300_000_000
        assert bad == 0, f"{bad} mismatches"
