"""bench.py's contract pieces that need no GPU: the default run's flags,
the committed DRAM-traffic figure the roofline reports, the peak
denominator's fallback, the config block, the normalised-nnz count and the
CPU-baseline timer."""
import sys

import pytest
import torch

import bench


def _args(*argv):
    old = sys.argv
    sys.argv = ["bench.py", *argv]
    try:
        return bench.parse()
    finally:
        sys.argv = old


def test_default_run_is_one_gpu_with_enough_warmup():
    a = _args()
    assert a.gpus == 1 and a.impl == "ours" and a.workload == "gcn" and a.mode == "fast"
    assert a.warmup >= 3 and a.steps > 0
    assert not a.suite and a.micro is None


def test_committed_traffic_is_the_full_size_capture():
    t = bench.committed_traffic("gather-gcn-L1-full-p1")
    assert t == 2_943_328_256  # profiles/traffic.txt: both passes + hub-row kernel, full graph
    assert bench.committed_traffic("no-such-kernel") is None


def test_measured_peak_or_fallback(monkeypatch, tmp_path):
    hbm, kind = bench.measured_peaks()
    assert hbm > 1000 and kind in ("measured", "fallback")
    monkeypatch.setattr(bench, "ROOT", str(tmp_path))  # no MEASURED_PEAKS.json there
    assert bench.measured_peaks() == (6650.0, "fallback")


def test_config_block_names_the_workload():
    a = _args()
    c = bench.config_dict(a, bench.NODES, 114_848_857)
    assert c["workload"] == "gcn-reddit-shape" and c["nodes"] == 232_965 and c["nnz"] == 114_848_857
    assert (c["features"], c["hidden"], c["classes"]) == (602, 128, 41)
    assert "l2" in c and "partition" in c and "mode" in c
    a8 = _args("--gpus", "8")
    assert "NVLink" in bench.config_dict(a8, 10, 10, "peer", [True, False])["partition"]


def test_nnz_normalized_counts_missing_diagonals():
    rp = torch.tensor([0, 2, 3, 3, 5], dtype=torch.int32)
    ci = torch.tensor([0, 2, 0, 1, 3], dtype=torch.int32)  # rows 0 and 3 hold their diagonal
    assert bench.nnz_normalized(rp, ci, 4) == 5 + 2


def test_reference_timer_takes_the_median_after_a_warmup(monkeypatch):
    calls = []
    ticks = iter([0.0, 0.0, 1.0, 1.0, 4.0, 4.0, 5.0, 5.0, 9.0, 9.0, 10.0, 10.0, 30.0, 30.0, 31.0, 100.0])
    monkeypatch.setattr(bench.time, "perf_counter", lambda: next(ticks))
    med, reps = bench.time_reference(lambda: calls.append(1), budget_s=8.0)
    assert len(calls) == reps + 1  # one warm-up
    assert (med, reps) == (1.0, 3)  # calls of 1, 0 and 4 s; the budget ends the loop at t = 9 s


@pytest.mark.parametrize("impl", ["ours", "reference"])
def test_reference_arm_flag_parses(impl):
    assert _args("--impl", impl, "--steps", "3", "--warmup", "3").impl == impl
