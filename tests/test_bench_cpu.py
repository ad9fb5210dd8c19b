"""CPU checks of bench.py's host-side arithmetic: the algorithmic bytes and
flops its rooflines divide by, the peaks it reads, and the per-launch DRAM
traffic it takes from the committed ncu summaries."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_module", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_algorithmic_bytes_count_codes_scales_activations_outputs(bench):
    # decode 1 x 4096 x 4096, 4-bit g64: 8 MiB of codes, 4 bytes of scale+bias per
    # group of 64, the bf16 activation row and the bf16 output row
    assert bench.algo_bytes(1, 4096, 4096) == 4096 * 4096 // 2 + 4096 * 64 * 4 + 4096 * 2 + 4096 * 2
    assert bench.algo_bytes(2, 128, 256, bits=8, gs=32) == 128 * 256 + 128 * 8 * 4 + 2 * 256 * 2 + 2 * 128 * 2


def test_algorithmic_flops(bench):
    assert bench.algo_flops(2048, 14336, 4096) == 2 * 2048 * 14336 * 4096


def test_traffic_comes_from_the_committed_summary(bench):
    lines = dict(l.split()[:2] for l in open(os.path.join(ROOT, "profiles", "traffic.txt"))
                 if len(l.split()) >= 2)
    for workload, value in lines.items():
        assert bench.ncu_traffic(workload) == float(value)
    assert bench.ncu_traffic("no-such-workload") is None


def test_peaks_are_the_measured_ones(bench):
    import json
    pk = bench.peaks()
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        measured = json.load(open(path))
        assert pk["hbm_gbs"] == measured["hbm_gbs"]
        assert pk["bf16_tflops"] == measured["bf16_tflops"]
    assert pk["hbm_gbs"] > 0 and pk["bf16_tflops"] > 0


def test_headline_workload_is_the_prefill_config(bench):
    assert bench.WORKLOADS["prefill"] == dict(M=2048, N=14336, K=4096)
    assert bench.WORKLOADS["decode"] == dict(M=1, N=4096, K=4096)
