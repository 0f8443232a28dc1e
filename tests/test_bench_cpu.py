"""bench.py host logic on CPU: the algorithmic FLOP per unit of each workload
(the figures the roofline divides by), the synthetic input generators, and
the reference arm's JSON line."""

import json
import os
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import bench  # noqa: E402


class _Args:
    mode = "bf16"

    def __init__(self, workload):
        self.workload = workload


@pytest.mark.parametrize("workload,flop", [
    ("forward", 2_573_047_296),        # default 9-layer, one track
    ("multitask", 2_726_647_296),      # 9 profile tracks
    ("variant", 13_468_422_144),       # 12 layers, n_filters 256, per forward
])
def test_flop_per_seq(workload, flop):
    m = bench.build_model(_Args(workload))
    assert bench.flop_per_seq(m) == flop


def test_multitask_inputs_gc_fraction():
    (bases,) = bench.make_bases("multitask", 64, 2)
    assert bases.shape == (64, bench.L) and int(bases.min()) >= 0 and int(bases.max()) <= 3
    gc = ((bases == 1) | (bases == 2)).double().mean(1)
    assert float(gc.min()) > 0.3 and float(gc.max()) < 0.7
    # per-sequence fractions spread over the range, not one shared value
    assert float(gc.max() - gc.min()) > 0.1


def test_variant_pairs_differ_at_centre_only():
    ref, alt = bench.make_bases("variant", 32, 3)
    diff = ref != alt
    c = bench.L // 2
    assert bool(diff[:, c].all())
    diff[:, c] = False
    assert not bool(diff.any())


def test_reference_arm_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "0", "--ref-sample", "1"],
                         capture_output=True, text=True, timeout=600, check=True).stdout
    line = json.loads(out.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "seqs/s" and line["value"] > 0
    from oracle import upstream
    # the upstream package itself when it is installed, else the oracle port
    assert line["cpu_baseline"]["kind"] == ("reference" if upstream.available() else "port")
    assert line["e2e"]["h2d_bytes_per_step"] == 0
