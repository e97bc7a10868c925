"""Fresh confirmation and publication of portfolio shards, on the host (synthetic shard runs).

The verdict rules restate taic/portfolio_confirmation.py:66-116; each rejection reason is planted
once in an otherwise confirmable pair of runs.
"""

from __future__ import annotations

import dataclasses
import json

import pytest

from shapeforge_b200 import confirmation as cf
from shapeforge_b200 import portfolio_pack as pp

PAPER = pp.Point("fp16/paper/benchmark", "paper", "benchmark", {"M": 4096, "K": 4096})
SMALL = pp.Point("fp16/small/benchmark", "small", "benchmark", {"M": 256, "K": 512})
GOLD = pp.Point("fp16/small/golden", "small", "golden", {"M": 256, "K": 512})


def run(point, provider="candidate", **kw):
    base = dict(point=point, provider=provider, selected="wide" if provider == "candidate" else "cuda-sm100.fallback.gemv",
                candidate_us=6.0, baseline_us=14.0, correct=True, detail="ok", timing_uncertain=False,
                candidate_cv=0.01, baseline_cv=0.02, attempts=1, source_sha256="ab" * 32, cache_hit=False)
    base.update(kw)
    return pp.ShardRun(**base)


def test_fresh_seed_is_deterministic_distinct_and_never_the_search_seed():
    a = cf.fresh_seed(1234, "d" * 64, PAPER.instance_key)
    assert a == cf.fresh_seed(1234, "d" * 64, PAPER.instance_key)
    assert a != cf.fresh_seed(1234, "d" * 64, SMALL.instance_key)
    assert a != cf.fresh_seed(1235, "d" * 64, PAPER.instance_key)
    assert a != cf.SEARCH_SEED and 0 <= a <= cf.MAX_SAFE_INTEGER


def test_a_clean_pair_is_confirmed_and_verifies():
    s = cf.subject(run(PAPER), run(PAPER, candidate_us=6.1), confirmation_seed=99)
    assert (s["status"], s["reason"]) == ("confirmed", None)
    assert cf.verify_subject(json.loads(json.dumps(s))) == s
    g = cf.subject(run(GOLD, provider="fallback"), run(GOLD, provider="fallback"), confirmation_seed=5)
    assert g["status"] == "confirmed" and g["credits_variant"] is False and "benchmark" not in g["search_report"]


@pytest.mark.parametrize("plant, reason", [
    (dict(conf=dict(correct=False)), "confirmation_status_not_ok"),
    (dict(search=dict(correct=False)), "search_status_not_ok"),
    (dict(conf=dict(cache_hit=True)), "cache_hit"),
    (dict(conf=dict(source_sha256="cd" * 32)), "candidate_sha256_mismatch"),
    (dict(conf=dict(timing_uncertain=True)), "timing_uncertain"),
    (dict(conf=dict(candidate_cv=0.2)), "timing_uncertain"),
    (dict(conf=dict(attempts=0)), "invalid_attempt_count"),
    (dict(conf=dict(attempts=4)), "invalid_attempt_count"),
    (dict(conf=dict(provider="fallback", selected="x")), "provider_mismatch"),
    (dict(seed=cf.SEARCH_SEED), "not_fresh"),
])
def test_each_rejection_rule(plant, reason):
    search = run(PAPER, **plant.get("search", {}))
    conf = run(PAPER, **plant.get("conf", {}))
    s = cf.subject(search, conf, confirmation_seed=plant.get("seed", 99))
    assert (s["status"], s["reason"]) == ("rejected", reason)


def test_document_level_rules():
    s = cf.subject(run(PAPER), run(PAPER), confirmation_seed=99)
    bad = dict(s, search_seed=8)
    assert cf.subject_verdict(bad) == ("rejected", "seed_mismatch")
    bad = dict(s, credits_variant=False)
    assert cf.subject_verdict(bad) == ("rejected", "variant_credit_mismatch")
    bad = dict(s, target_id="h100")
    assert cf.subject_verdict(bad) == ("rejected", "target_mismatch")
    golden_as_full = dict(s, instance_key="fp16/paper/golden", usage="golden")
    assert cf.subject_verdict(golden_as_full) == ("rejected", "measurement_mode_mismatch")


def test_an_edited_archive_fails_verification():
    s = cf.subject(run(PAPER), run(PAPER), confirmation_seed=99)
    edited = json.loads(json.dumps(s))
    edited["confirmation_report"]["benchmark"]["candidate"]["median_us"] = 1.0
    with pytest.raises(ValueError, match="recomputed"):
        cf.verify_subject(edited)


def _parent(tmp_path):
    from tests.test_portfolio_pack import GEMV_OPSPEC, GEMV_VEC, WIDE_GUARD, make_tree

    points = pp.domain(GEMV_OPSPEC, "fp16")
    return pp.pack(make_tree(tmp_path / "src", {"wide": (WIDE_GUARD, GEMV_VEC)}), points)


def test_publish_writes_the_catalog_entry(tmp_path):
    parent = _parent(tmp_path)
    runs = [run(PAPER), run(SMALL, provider="fallback", candidate_us=4.0, baseline_us=9.0)]
    subjects = [cf.subject(r, dataclasses.replace(r), confirmation_seed=1000 + i) for i, r in enumerate(runs)]
    out = cf.publish(tmp_path / "kernels", "gemv", "fp16", parent, runs, subjects)
    assert out == tmp_path / "kernels" / "b200" / "gemv" / "fp16" / parent.sha256[:16]
    manifest = json.loads((out / "manifest.json").read_text())
    assert manifest["parent_sha256"] == parent.sha256 and set(manifest["subjects"]) == {PAPER.instance_key, SMALL.instance_key}
    assert manifest["effective_end_to_end_speedup"] == pytest.approx(23.0 / 10.0)
    perf = json.loads((out / "performance.json").read_text())
    assert perf["publishable"] and perf["fallback_count_fraction"] == 0.5
    for f in ("paper-benchmark.json", "small-benchmark.json"):
        cf.verify_subject(json.loads((out / "subjects" / f).read_text()))
    assert pp.Parent.from_json((out / "parent.json").read_text()).sha256 == parent.sha256


def test_publish_refuses_unconfirmed_or_unpublishable(tmp_path):
    parent = _parent(tmp_path)
    good = [run(PAPER), run(SMALL, provider="fallback")]
    subjects = [cf.subject(r, dataclasses.replace(r), confirmation_seed=1000 + i) for i, r in enumerate(good)]
    noisy = [cf.subject(good[0], dataclasses.replace(good[0], timing_uncertain=True), confirmation_seed=1000), subjects[1]]
    with pytest.raises(cf.PublicationRefused, match="timing_uncertain"):
        cf.publish(tmp_path / "k1", "gemv", "fp16", parent, good, noisy)
    slow = [run(PAPER, candidate_us=20.0), good[1]]
    with pytest.raises(cf.PublicationRefused, match="not publishable"):
        cf.publish(tmp_path / "k2", "gemv", "fp16", parent, slow, subjects)
    with pytest.raises(cf.PublicationRefused, match="without a subject"):
        cf.publish(tmp_path / "k3", "gemv", "fp16", parent, good, subjects[:1])
