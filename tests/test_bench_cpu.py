"""Host-side pieces of bench.py that shape its JSON line: the algorithmic
byte count behind ``roofline``, the sample the reference arm times, and the
reference arm itself on a small workload (skipped when the reference package
is not installed under baseline/_ref)."""
import os

import pytest

import bench
from scao_b200 import workloads


def _numel(spec):
    n = 1
    for d in spec.shape:
        n *= d
    return n


def test_algorithmic_bytes_llama_headline():
    w = workloads.c4()
    phase1 = sum(_numel(s) for s in w.params if s.adam_only)
    phase2 = sum(_numel(s) for s in w.params if not s.adam_only)
    got = bench.algorithmic_bytes(w, lambda s: 1 if s.adam_only else 2)
    # bf16 p/g, fp32 moments: 38 B/elem in Phase 2, 26 B/elem in Phase 1
    assert got == 38 * phase2 + 26 * phase1
    assert got == 38683488256


@pytest.mark.parametrize("make", [workloads.c4, workloads.c2, workloads.c5])
def test_sample_split_partitions_the_workload(make):
    w = make()
    w_e, w_l, n_layers = bench.sample_split(w, 1)
    names = [p.name for p in w.params]
    layer_names = [n for n in names if bench._layer_of(n) is not None]
    assert n_layers == 1 + max(bench._layer_of(n) for n in layer_names)
    # the non-layer part and every layer are disjoint and cover the set
    assert sorted(p.name for p in w_e.params) == sorted(n for n in names if bench._layer_of(n) is None)
    assert all(bench._layer_of(p.name) == 0 for p in w_l.params)
    # layers are alike: n_layers x (layer 0) has the element count of all layers
    per_layer = sum(_numel(p) for p in w_l.params)
    all_layers = sum(_numel(p) for p in w.params if bench._layer_of(p.name) is not None)
    assert n_layers * per_layer == all_layers
    # the samples keep the workload's optimizer settings
    assert w_e.scao_kwargs == w.scao_kwargs and w_l.scao_kwargs == w.scao_kwargs


def test_reference_arm_small_workload():
    ref = os.path.join(bench.ROOT, "baseline", "_ref", "scao", "__init__.py")
    if not os.path.isfile(ref):
        pytest.skip("reference package not installed under baseline/_ref")
    r = bench.reference_arm(workloads.c1(), steps=2, warmup=0)
    assert r is not None
    assert r["ms_per_step"] > 0 and r["cores"] >= 1
    assert r["steps"] == 2 and r["warmup"] == 0
    assert "1 of 4 transformer layers" in r["sample"]


def test_reference_line_contract():
    """``bench.py --impl reference`` prints one JSON line with the arm's own
    metric, config, cpu_baseline and a zero-copy e2e (GPT-2-small set, one
    timed step, the GPU fallback leg off)."""
    import json
    import subprocess
    import sys
    ref = os.path.join(bench.ROOT, "baseline", "_ref", "scao", "__init__.py")
    if not os.path.isfile(ref):
        pytest.skip("reference package not installed under baseline/_ref")
    out = subprocess.run(
        [sys.executable, os.path.join(bench.ROOT, "bench.py"), "--impl", "reference",
         "--workload", "gpt2-small", "--steps", "1", "--warmup", "3", "--no-gpu-fallback"],
        capture_output=True, text=True, timeout=600, check=True).stdout
    d = json.loads(out.strip().splitlines()[-1])
    assert d["impl"] == "reference" and d["steps"] == 1 and d["warmup"] == 3
    assert d["unit"] == "ms" and d["higher_is_better"] is False and d["value"] > 0
    assert d["config"]["workload"] == "c2-gpt2-small"
    cb = d["cpu_baseline"]
    assert cb["kind"] == "reference" and cb["cores"] >= 1 and cb["value"] == d["value"]
    assert "1 of 12 transformer layers" in cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "ms",
                        "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
