"""The L2 capacity contract of the varlen tasks on the host, pinned on the reference's own capacity
vectors (tests/golden/ref_varlen_kda_capacity_*.npz from tasks/varlen_kda at its capacity size).
"""

from __future__ import annotations

import pytest

from shapeforge_b200 import capacity as cap
from tests import golden

# tasks/varlen_kda/opspec.json sizes.capacity (capacity block and workload profiles).
CAPACITY_SIZE = {
    "H": 2, "D": 8, "usage": ["golden", "benchmark"],
    "capacity": {"total_tokens": 16, "num_seqs": 4, "cu_seqlens_sentinel": -1, "padding_poison_byte": 90},
    "workload_profiles": [{"id": "a_full", "seq_lens": [4, 4, 4, 4]}, {"id": "b_tiny", "seq_lens": [1]},
                          {"id": "c_mid", "seq_lens": [5, 3, 1]}, {"id": "d_shrink", "seq_lens": [2, 1]}],
}
CASES = ("canonical", "permuted", "skewed", "all_unaligned_primes", "max_handoff_stress", "chunk_boundary", "zero_length",
         "single_sequence", "fresh_distribution")


def spec():
    return cap.CapacitySpec.from_size(CAPACITY_SIZE)


def test_profiles_cycle_over_the_declared_cases():
    s = spec()
    assert [pid for pid, _ in s.profiles] == ["a_full", "b_tiny", "c_mid", "d_shrink"]
    assert [s.profile_for_case(CASES, c)[0] for c in CASES] == ["a_full", "b_tiny", "c_mid", "d_shrink"] * 2 + ["a_full"]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_reference_capacity_vectors_follow_the_contract(dtype):
    """Every case the reference generated at the capacity size: its boundary is legal, resolves to
    its case's profile total/count (the task owns the split, the harness owns the totals), and its
    input padding holds the poison byte."""
    doc = golden.load(f"ref_varlen_kda_capacity_{dtype}")
    s = spec()
    assert [r["case"] for r in doc["records"]] == list(CASES)
    for rec in doc["records"]:
        cu = [int(v) for v in rec["inputs"]["cu_seqlens"]]
        resolved = cap.resolved_from_cu(cu, s)
        assert cap.cu_seqlens_problems(cu, resolved, s) == (), rec["case"]
        _, lens = s.profile_for_case(CASES, rec["case"])
        assert (resolved.total_tokens, resolved.num_seqs) == (sum(lens), len(lens)), rec["case"]
        q = rec["inputs"]["q"]
        pad = q[resolved.total_tokens:].view("uint8")
        assert (pad == 90).all(), rec["case"]
        # The reference's final_state rows past num_seqs are the poison bytes read as fp32.
        fin = rec["refs"]["final_state"][resolved.num_seqs:]
        assert (fin == 1.5365221879119872e16).all()


def test_boundary_problems_are_reported():
    s = spec()
    r = cap.ResolvedShape.of([5, 3, 1], s)
    assert cap.cu_seqlens(([5, 3, 1]), s) == [0, 5, 8, 9, -1]
    assert cap.cu_seqlens_problems([0, 5, 8, 9, -1], r, s) == ()
    assert "start at 0" in cap.cu_seqlens_problems([1, 5, 8, 9, -1], r, s)[0]
    assert "end at the resolved" in cap.cu_seqlens_problems([0, 5, 8, 10, -1], r, s)[0]
    assert "non-decreasing" in cap.cu_seqlens_problems([0, 5, 4, 9, -1], r, s)[0]
    assert "not the sentinel" in cap.cu_seqlens_problems([0, 5, 8, 9, 0], r, s)[0]
    assert "offsets" in cap.cu_seqlens_problems([0, 5, 8, 9], r, s)[0]
    for bad, why in (([17], "exceeds the capacity"), ([1] * 5, "exceeds the capacity"), ([0], "at least one token"), ([], "at least one")):
        with pytest.raises(cap.CapacityError, match=why):
            cap.ResolvedShape.of(bad, s)
    with pytest.raises(cap.CapacityError, match="no capacity"):
        cap.CapacitySpec.from_size({"H": 2, "D": 8, "seq_lens": [4]})


def test_padding_check_finds_written_rows():
    import torch

    s = spec()
    r = cap.ResolvedShape.of([5, 3, 1], s)
    out = torch.full((16, 2, 8), 0, dtype=torch.float16)
    out.view(torch.uint8).fill_(90)
    assert cap.padding_problems("output", out, r, 90) == ()
    out[12, 1, 3] = 1.0
    assert cap.padding_problems("output", out, r, 90) == ("output padding row 12 was written",)
    out[3] = 0.0  # logical rows may hold anything
    assert len(cap.padding_problems("output", out, r, 90)) == 1


def test_benchmark_mixture_order_and_evidence_rules():
    s = spec()
    assert cap.benchmark_mixture(CASES, 3, capacity=False) == ("canonical",) * 3
    mix = cap.benchmark_mixture(CASES, 3, capacity=True)
    assert mix == CASES  # at least one set per declared case
    assert len(cap.benchmark_mixture(CASES, 100, capacity=True, ring_max=20)) == 20

    def batch(i, case, **kw):
        pid, lens = s.profile_for_case(CASES, case)
        b = {"case": case, "provider": "candidate", "evaluation_input_digest": f"{i:064x}",
             "resolved_shape": {"total_tokens": sum(lens), "num_seqs": len(lens), "workload_profile_id": pid}}
        b.update(kw)
        return b

    good = [batch(i, c) for i, c in enumerate(mix)]
    assert cap.mixture_problems(s, CASES, good) == ()
    assert "declared order" in cap.mixture_problems(s, CASES, [good[1]] + good[1:])[0]
    assert any("not the candidate" in p for p in cap.mixture_problems(s, CASES, [dict(good[0], provider="fallback")] + good[1:]))
    assert any("digest" in p for p in cap.mixture_problems(s, CASES, [dict(good[0], evaluation_input_digest="x")] + good[1:]))
    shrunk = dict(good[0], resolved_shape={"total_tokens": 9, "num_seqs": 3, "workload_profile_id": "a_full"})
    assert any("declares [16 / 4]" in p for p in cap.mixture_problems(s, CASES, [shrunk] + good[1:]))
    only_full = [batch(0, "canonical")]
    probs = cap.mixture_problems(s, CASES, only_full)
    assert any("does not time the declared profiles" in p for p in probs)
    assert cap.mixture_problems(s, CASES, []) == ("a capacity benchmark published no continuous-batching mixture",)
