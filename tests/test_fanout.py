"""Portfolio shards one GPU per shard, on the host: spawned workers (one per device mask) each
measure the points the balance dealt them, and the parent merges the runs in domain order.

The workers here run a stand-in measurement (no GPU): it records the device mask it ran under,
which shows each worker was pinned to its own GPU before anything initialised CUDA."""

from __future__ import annotations

import os

import pytest

from shapeforge_b200 import fanout
from shapeforge_b200 import portfolio_pack as pp
from tests.test_portfolio_pack import GEMV_OPSPEC, WIDE_GUARD, GEMV_VEC, make_tree


def stand_in_recipe(fail_on: str = "") -> dict:
    return {"make_inputs": None, "baseline": None, "verify": fail_on}


def stand_in_measure(parent, opspec, points, *, make_inputs, baseline, verify, reps):
    runs = []
    for p in points:
        if verify and p.instance_key == verify:
            raise RuntimeError(f"planted failure on {p.instance_key}")
        cost = fanout.point_cost(p)
        runs.append(pp.ShardRun(p, "candidate", "stand-in", cost / 1e3, cost / 5e2, True,
                                detail=os.environ.get("CUDA_VISIBLE_DEVICES", "")))
    return runs


def _domain_with_sizes():
    doc = dict(GEMV_OPSPEC)
    doc["sizes"] = dict(doc["sizes"])
    doc["sizes"].update({f"extra{i}": {"M": 64 * (i + 1), "K": 512, "usage": ["benchmark"]} for i in range(5)})
    return doc


def test_points_are_balanced_and_each_runs_once_on_its_gpu(tmp_path):
    doc = _domain_with_sizes()
    points = pp.domain(doc, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    bench = [p for p in points if p.usage == "benchmark"]
    parts = fanout.balance(points, 3)
    assert sorted(i for p in parts for i in p) == list(range(len(bench)))
    runs = fanout.measure_on_gpus(parent, doc, points, recipe="tests.test_fanout:stand_in_recipe", devices=["4", "6", "7"],
                                  measure="tests.test_fanout:stand_in_measure", timeout_s=120)
    assert [r.point.instance_key for r in runs] == [p.instance_key for p in bench]
    where = {r.point.instance_key: r.detail for r in runs}
    for mask, part in zip(["4", "6", "7"], parts):
        for i in part:
            assert where[bench[i].instance_key] == mask
    report = pp.performance(runs)
    assert len(report.document()["shards"]) == len(bench)


def test_fewer_points_than_gpus_starts_one_worker_per_point(tmp_path):
    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    runs = fanout.measure_on_gpus(parent, GEMV_OPSPEC, points, recipe="tests.test_fanout:stand_in_recipe",
                                  devices=[str(i) for i in range(8)], measure="tests.test_fanout:stand_in_measure", timeout_s=120)
    assert sorted(r.detail for r in runs) == ["0", "1"]


def test_a_failing_worker_reports_its_traceback(tmp_path):
    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    bad = [p for p in points if p.usage == "benchmark"][0].instance_key
    with pytest.raises(fanout.FanoutError) as exc:
        fanout.measure_on_gpus(parent, GEMV_OPSPEC, points, recipe="tests.test_fanout:stand_in_recipe",
                               recipe_kwargs={"fail_on": bad}, devices=["0", "1"], measure="tests.test_fanout:stand_in_measure",
                               timeout_s=120)
    assert "planted failure" in str(exc.value)


def test_device_masks_follow_the_visible_devices(monkeypatch):
    monkeypatch.setenv("CUDA_VISIBLE_DEVICES", "2,5,7")
    assert fanout.device_masks() == ["2", "5", "7"]
    assert fanout.device_masks(2) == ["2", "5"]
    monkeypatch.delenv("CUDA_VISIBLE_DEVICES")
    assert fanout.device_masks(3) == ["0", "1", "2"]


def stalled_measure(parent, opspec, points, *, make_inputs, baseline, verify, reps):
    import time

    time.sleep(120)  # a worker that never answers; the parent kills it at the deadline
    return []


def test_silent_workers_share_one_deadline(tmp_path):
    import time

    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    t0 = time.monotonic()
    with pytest.raises(fanout.FanoutError) as exc:
        fanout.measure_on_gpus(parent, GEMV_OPSPEC, points, recipe="tests.test_fanout:stand_in_recipe", devices=["0", "1"],
                               measure="tests.test_fanout:stalled_measure", timeout_s=4)
    elapsed = time.monotonic() - t0
    assert str(exc.value).count("no answer within 4 s") == 2
    assert elapsed < 7.5  # one 4 s limit for both workers, not 4 s each
