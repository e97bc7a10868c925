"""Calibration on the host: the read/write-mix bandwidth interpolation agrees with the reference's
formula (tcenv/backends/metal/profile.py:233-248), the roofline uses it, the cache file takes
precedence over the shipped figures, and the probe kernels build for sm_100a and fit their launch."""

from __future__ import annotations

import json

import pytest

from shapeforge_b200 import calibrate, kernel_stats
from shapeforge_b200.backend import CudaBackend, LaunchStage
from shapeforge_b200.candidates import kernel_resources

CAL = {"copy_gbs": 6000.0, "read_gbs": 7000.0, "peak_tflops": {"fp16": 1600.0}}


@pytest.mark.parametrize("rd,wr,want", [(1.0, 0.0, 7000.0), (3.0, 1.0, 6500.0), (1.0, 1.0, 6000.0), (1.0, 3.0, 6000.0),
                                        (0.0, 0.0, 7000.0)])
def test_effective_peak_interpolates_on_the_write_fraction(rd, wr, want):
    assert calibrate.effective_peak_gbps(rd, wr, CAL) == pytest.approx(want)


def test_roofline_uses_the_mix_when_the_split_is_known():
    b = CudaBackend()
    r = b.roofline({"min_bytes": 4e9, "read_bytes": 3e9, "write_bytes": 1e9, "flops": 0, "dtype": "fp16"}, 1e-3, CAL)
    assert r["peak_gbps_measured"] == pytest.approx(6500.0) and r["bandwidth_fraction"] == pytest.approx(4000 / 6500)
    r = b.roofline({"min_bytes": 4e9, "flops": 0, "dtype": "fp16"}, 1e-3, CAL)
    assert r["peak_gbps_measured"] == pytest.approx(6000.0)


def test_calibration_cache_precedence(tmp_path, monkeypatch):
    from shapeforge_b200 import backend as bk

    monkeypatch.setattr(bk, "ROOT", tmp_path)  # no pool-measured peaks under this root
    (tmp_path / "targets" / "b200").mkdir(parents=True)
    (tmp_path / "targets" / "b200" / "calibration.json").write_text(json.dumps({"copy_gbs": 1.0, "source": "shipped"}))
    monkeypatch.setenv("SF_CALIBRATION", str(tmp_path / "cal.json"))
    assert CudaBackend().calibration("b200")["source"] == "shipped"
    (tmp_path / "cal.json").write_text(json.dumps({"copy_gbs": 2.0, "source": "calibrate"}))
    assert CudaBackend().calibration("b200")["source"] == "calibrate"


def test_probe_kernels_build_and_fit_their_launch():
    res = kernel_resources(calibrate.PROBE_SOURCE, name="calibrate")
    assert set(res) == {"copy4", "read4"}
    grid = (148 * calibrate.BLOCKS_PER_SM, 1, 1)
    stages = [LaunchStage(k, grid, (calibrate.THREADS, 1, 1)) for k in res]
    assert kernel_stats.check_stages(res, stages) == []
    assert all(r.spill_stores == 0 and r.static_smem == 0 for r in res.values())
