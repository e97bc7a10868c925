"""Shape portfolios of CUDA candidates on the host: the guard/geometry expression language, packing a
source tree, the coverage check, exact dispatch and the registered fallback providers.

The expression rules are cross-checked against the reference's own evaluator
(tcenv/track/expr.py) when the reference checkout is mounted.
"""

from __future__ import annotations

import json
import os
import random
from pathlib import Path

import pytest

from shapeforge_b200 import expr, fallbacks
from shapeforge_b200 import portfolio_pack as pp
from shapeforge_b200.backend import CudaBackend, parse_launch_templates

REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))

# tasks/gemv/opspec.json: tensors, spec_params and sizes (paper is golden + benchmark, small too).
GEMV_OPSPEC = {
    "tensors": {
        "A": {"role": "input", "dims": ["M", "K"], "dtype": "T"},
        "x": {"role": "input", "dims": ["K"], "dtype": "T"},
        "y": {"role": "output", "dims": ["M"], "dtype": "T"},
    },
    "symbols": {"M": {"min": 1}, "K": {"min": 1}},
    "spec_params": ["M", "K"],
    "sizes": {"paper": {"M": 4096, "K": 4096, "usage": ["golden", "benchmark"]},
              "small": {"M": 256, "K": 512, "usage": ["golden", "benchmark"]}},
}

# A vectorised gemv variant: warp per row, 16-byte loads; valid where K % 8 == 0.
GEMV_VEC = r'''#include <cuda_fp16.h>
extern "C" __global__ void gemv_vec(const __half* __restrict__ A, const __half* __restrict__ x, __half* __restrict__ y,
                                    long long M, long long K) {
    const long long r = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
    if (r >= M) return;
    const uint4* a = reinterpret_cast<const uint4*>(A + r * K);
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    float acc = 0.f;
    for (long long v = threadIdx.x & 31; v < K / 8; v += 32) {
        const uint4 pa = a[v], px = __ldg(xv + v);
        const __half2* ha = reinterpret_cast<const __half2*>(&pa);
        const __half2* hx = reinterpret_cast<const __half2*>(&px);
        for (int j = 0; j < 4; ++j) {
            const float2 fa = __half22float2(ha[j]), fx = __half22float2(hx[j]);
            acc = fmaf(fa.x, fx.x, acc);
            acc = fmaf(fa.y, fx.y, acc);
        }
    }
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) y[r] = __float2half_rn(acc);
}
/* taic-launch
kernel gemv_vec grid=ceil_div(M,8) threads=256
*/
'''

WIDE_GUARD = ["and", ["eq", ["rem", "K", 8], 0], ["ge", "M", 1024]]


def make_tree(root: Path, variants: dict, fallback: str | None = "gemv", coverage_extra: dict | None = None) -> Path:
    """A source tree: ``variants`` maps key -> (guard, source); fallback is a task name (the
    registered provider), or None for a refuse fallback."""
    for key, (_, src) in variants.items():
        (root / "variants" / key).mkdir(parents=True)
        (root / "variants" / key / "kernel.cu").write_text(src)
    fb = pp.write_fallback(root, fallback, "fp16") if fallback else {"kind": "refuse", "reasons": ["outside_candidate_coverage"]}
    doc = {"schema_id": pp.COVERAGE_SCHEMA_ID, "planner": {"id": "gemv-rows", "version": 1},
           "variants": [{"variant_key": k, "guard": g} for k, (g, _) in variants.items()], "fallback": fb}
    doc.update(coverage_extra or {})
    (root / "coverage.json").write_text(json.dumps(doc))
    return root


def points():
    return pp.domain(GEMV_OPSPEC, "fp16")


# ---- expressions --------------------------------------------------------------------------------


def test_expression_semantics():
    env = {"N": 37, "K": -12}
    assert expr.evaluate_term("ceil_div(N, 8) * 8 - N", env) == 3
    assert expr.evaluate_term({"ceil_div": ["N", 256]}, env) == 1
    assert expr.evaluate_term("rem(-7, 2)", {}) == -1 and expr.evaluate_term("trunc_div(-7, 2)", {}) == -3
    assert expr.evaluate_term(["and", ["ge", "N", 1], ["not", ["eq", "K", 0]]], env, expect=expr.BOOL) is True
    assert expr.evaluate_term("min(N, 4, K)", env) == -12
    for bad, why in (("N / 5", "exact"), ("rem(N, 0)", "zero"), ("ceil_div(N, 0)", "positive"), ("Q + 1", "not declared"),
                     ("frobnicate(N)", "unknown function"), ("N +", "ends early"), ("N $ 2", "unexpected")):
        with pytest.raises(expr.ExprError, match=why):
            expr.evaluate_term(bad, env)
    with pytest.raises(expr.ExprError):
        expr.parse(True)
    with pytest.raises(expr.ExprError, match="predicate"):
        expr.guard("N + 1")
    with pytest.raises(expr.ExprError, match="must be a predicate"):
        expr.evaluate_term(["and", "N", ["eq", "K", 1]], env, expect=expr.BOOL)
    with pytest.raises(expr.ExprError, match="must be an integer"):
        expr.evaluate_term(["+", ["eq", "K", 1], 2], env)
    # A guard with an operand that cannot be evaluated is an error even if another operand decides it.
    with pytest.raises(expr.ExprError):
        expr.evaluate(expr.guard(["and", ["eq", "N", 0], ["eq", ["rem", "K", 0], 0]]), env)


def test_guard_digest_is_canonical():
    a = expr.digest(["and", ["eq", "N", 1], ["and", ["eq", "K", 2], ["ge", "M", 3]]])
    b = expr.digest("and(ge(M, 3), eq(K, 2), eq(1, N))")
    assert a == b
    assert a != expr.digest("and(ge(M, 3), eq(K, 2), eq(2, N))")


@pytest.mark.skipif(not (REF / "tcenv").is_dir(), reason="the reference checkout is not mounted")
def test_expression_rules_match_the_reference_evaluator():
    import sys

    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.track import expr as rexpr

    rng = random.Random(3)
    funcs = ["ceil_div", "trunc_div", "rem", "min", "max", "+", "-", "*", "/"]

    def term(depth):
        if depth == 0 or rng.random() < 0.3:
            return rng.choice([rng.randint(-20, 20), "N", "K", "M"])
        f = rng.choice(funcs)
        n = rng.randint(1, 3) if f in ("min", "max") else 2
        return [f] + [term(depth - 1) for _ in range(n)]

    env = {"N": 37, "K": -12, "M": 5}
    for _ in range(2000):
        t = term(4)
        try:
            ours = expr.evaluate_term(t, env)
        except expr.ExprError:
            ours = "error"
        try:
            theirs = rexpr.evaluate_term(t, env, where="t")
        except Exception:  # noqa: BLE001 - GeometryError
            theirs = "error"
        assert ours == theirs, t
        # Text spelling of the same term.
        assert expr.evaluate_term("2 * (N - 3) / 2 + rem(K, 5)", env) == rexpr.evaluate_term("2 * (N - 3) / 2 + rem(K, 5)", env, where="t")


# ---- packing and checking -----------------------------------------------------------------------


def test_pack_and_check_a_two_provider_portfolio(tmp_path):
    src = make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)})
    parent = pp.pack(src, points())
    doc = parent.document
    assert doc["schema_id"] == pp.PORTFOLIO_SCHEMA_ID
    assert doc["fallback"]["implementation_id"] == "cuda-sm100.fallback.gemv"
    assert doc["variants"][0]["guard"]["digest"] == expr.digest(WIDE_GUARD)
    assert [e.path for e in parent.entries] == ["fallback/kernel.cu", "variants/wide/kernel.cu", pp.PORTFOLIO_ENTRY_PATH]
    report = pp.check(parent, points())
    assert report.ok, report.problems
    providers = {r.instance_key: (r.provider, r.variant_key) for r in report.rows}
    assert providers == {
        "fp16/paper/golden": ("candidate", "wide"), "fp16/paper/benchmark": ("candidate", "wide"),
        "fp16/small/golden": ("fallback", None), "fp16/small/benchmark": ("fallback", None),
    }
    # The parent survives its transport form unchanged.
    again = pp.Parent.from_json(parent.to_json())
    assert again.document == json.loads(json.dumps(doc)) and again.sha256 == parent.sha256
    # Dispatch reproduces the check.
    port = pp.to_portfolio(parent)
    assert port.resolve({"M": 4096, "K": 4096}).selected == "wide"
    assert port.resolve({"M": 256, "K": 512}).provider == "fallback"
    assert "fallback_gemv" in pp.selected_source(parent, port.resolve({"M": 3, "K": 5}))


def test_check_reports_overlap_empty_variants_and_uncovered_points(tmp_path):
    overlap = make_tree(tmp_path / "o", {"a": (WIDE_GUARD, GEMV_VEC), "b": (["ge", "M", 4096], GEMV_VEC.replace("gemv_vec", "gemv_b"))})
    rep = pp.check(pp.pack(overlap, points()), points())
    assert not rep.ok and any("more than one variant" in p for p in rep.problems)

    empty = make_tree(tmp_path / "e", {"a": (WIDE_GUARD, GEMV_VEC), "never": (["gt", "M", 10**9], GEMV_VEC)})
    rep = pp.check(pp.pack(empty, points()), points())
    assert any(p.startswith("never: matches no point") for p in rep.problems)

    refuse = make_tree(tmp_path / "r", {"a": (WIDE_GUARD, GEMV_VEC)}, fallback=None)
    rep = pp.check(pp.pack(refuse, points()), points())
    assert [p.split(":")[0] for p in rep.problems] == ["fp16/small/golden", "fp16/small/benchmark"]

    # A guard error at a point is a dispatch failure there, not a crash.
    unknown = make_tree(tmp_path / "u", {"a": (["eq", ["rem", "K", ["-", "M", 256]], 0], GEMV_VEC)})
    rep = pp.check(pp.pack(unknown, points()), points())
    assert any("cannot be evaluated" in p for p in rep.problems)

    # Packed for one set of sizes, checked against another.
    rep = pp.check(pp.pack(tmp_path / "r", points()), pp.domain(GEMV_OPSPEC, "fp16", ["paper"]))
    assert any("another domain" in p for p in rep.problems)


def test_check_reports_a_launch_that_does_not_resolve(tmp_path):
    bad = GEMV_VEC.replace("grid=ceil_div(M,8)", "grid=ceil_div(ROWS,8)")
    tree = make_tree(tmp_path, {"a": (WIDE_GUARD, bad)})
    rep = pp.check(pp.pack(tree, points()), points())
    assert any("does not resolve" in p for p in rep.problems)


@pytest.mark.parametrize("mutate, why", [
    (lambda d: d.update(extra=1), "keys must be exactly"),
    (lambda d: d.update(schema_id="x"), "schema_id"),
    (lambda d: d.update(planner={"id": "p"}), "planner"),
    (lambda d: d["variants"][0].update(variant_key="Bad Key"), "must match"),
    (lambda d: d["variants"][0].update(colour="red"), "allows only"),
    (lambda d: d["fallback"].update(reasons=["because"]), "reasons"),
    (lambda d: d["fallback"].update(implementation_version=0), "implementation_version"),
    (lambda d: d["variants"][0].update(guard="M + 1"), "predicate"),
])
def test_pack_refuses_malformed_coverage(tmp_path, mutate, why):
    tree = make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)})
    doc = json.loads((tree / "coverage.json").read_text())
    mutate(doc)
    (tree / "coverage.json").write_text(json.dumps(doc))
    with pytest.raises(pp.PortfolioError, match=why):
        pp.pack(tree, points())


def test_pack_refuses_bad_trees(tmp_path):
    t1 = make_tree(tmp_path / "1", {"wide": (WIDE_GUARD, GEMV_VEC)})
    (t1 / "variants" / "wide" / "extra.cu").write_text("// stray")
    with pytest.raises(pp.PortfolioError, match="exactly kernel.cu"):
        pp.pack(t1, points())
    t2 = make_tree(tmp_path / "2", {"wide": (WIDE_GUARD, GEMV_VEC)})
    (t2 / "variants" / "orphan").mkdir()
    with pytest.raises(pp.PortfolioError, match="do not match the directories"):
        pp.pack(t2, points())
    t3 = make_tree(tmp_path / "3", {"wide": (WIDE_GUARD, GEMV_VEC.replace("/* taic-launch", "/* none"))})
    with pytest.raises(pp.PortfolioError, match="taic-launch"):
        pp.pack(t3, points())
    t4 = make_tree(tmp_path / "4", {"a": (WIDE_GUARD, GEMV_VEC), "b": (["lt", "M", 8], GEMV_VEC)})
    doc = json.loads((t4 / "coverage.json").read_text())
    for v in doc["variants"]:
        v["bucket_key"] = "same"
    (t4 / "coverage.json").write_text(json.dumps(doc))
    with pytest.raises(pp.PortfolioError, match="two different guards"):
        pp.pack(t4, points())
    t5 = make_tree(tmp_path / "5", {"a": (WIDE_GUARD, GEMV_VEC)}, fallback=None)
    (t5 / "fallback").mkdir()
    with pytest.raises(pp.PortfolioError, match="no fallback directory"):
        pp.pack(t5, points())


# ---- the registered fallbacks -------------------------------------------------------------------

# Symbol values of each task's opspec sizes (tasks/<task>/opspec.json sizes.paper / sizes.small).
FALLBACK_SHAPES = {
    "relu": [{"N": 16777216}, {"N": 65536}, {"N": 1}], "sigmoid": [{"N": 16777216}, {"N": 65536}],
    "sigmoid_shift": [{"N": 16777216}], "silu": [{"N": 16777216}], "swiglu": [{"N": 16777216}], "lion": [{"N": 8388608}],
    "rmsnorm": [{"M": 4096, "H": 4096}, {"M": 64, "H": 512}], "softmax": [{"M": 8192, "N": 2048}],
    "reduction_sum": [{"M": 4096, "N": 4096}], "gemv": [{"M": 4096, "K": 4096}, {"M": 1, "K": 3}],
    "gemm": [{"M": 2048, "N": 2048, "K": 2048}, {"M": 3, "N": 5, "K": 7}], "gemm_silu": [{"M": 256, "N": 256, "K": 128}],
    "rope": [{"B": 2, "H": 32, "S": 1024, "D": 128}, {"B": 1, "H": 1, "S": 1, "D": 2}],
    "bitdelta_gemm": [{"M": 512, "N": 4096, "K": 4096}, {"M": 128, "N": 256, "K": 256}],
    "flash_attention": [{"B": 2, "H": 8, "S": 1024, "D": 64}, {"B": 1, "H": 2, "S": 128, "D": 64}],
    "mamba2_chunk_scan": [{"BATCH": 2, "SEQLEN": 2048, "NHEADS": 8, "HEADDIM": 64, "DSTATE": 64, "CHUNK": 64, "NCHUNKS": 32}],
    "kda": [{"N": 256, "H": 8, "D": 64}, {"N": 1, "H": 2, "D": 8}],
    "varlen_kda": [{"H": 64, "D": 128, "num_seqs": 6, "total_tokens": 8192}, {"H": 2, "D": 8, "num_seqs": 4, "total_tokens": 16}],
}


@pytest.mark.parametrize("task", fallbacks.TASKS)
def test_registered_fallbacks_render_check_and_resolve(task):
    from shapeforge_b200.track_factory import CudaTrackBuilder

    assert set(FALLBACK_SHAPES) == set(fallbacks.TASKS)
    for dtype in ("fp16", "bf16"):
        src = fallbacks.render(task, dtype)
        assert fallbacks.kernel_name(task) in src and fallbacks.implementation_id(task) in src
        CudaTrackBuilder().check(src)
        (tpl,) = parse_launch_templates(src)
        for names in FALLBACK_SHAPES[task]:
            stage = tpl.resolve(names)
            assert CudaBackend().validate_launch([stage], {}) == [], (task, names, stage)
    with pytest.raises(KeyError):
        fallbacks.render("no_such_task", "fp16")
    with pytest.raises(ValueError):
        fallbacks.render(task, "fp32")


def test_varlen_sizes_get_their_batch_symbols():
    opspec = {"sizes": {"mixed": {"H": 2, "D": 8, "seq_lens": [4, 8, 2], "usage": ["golden"]},
                        "capacity": {"H": 2, "D": 8, "usage": ["benchmark"],
                                     "capacity": {"total_tokens": 16, "num_seqs": 4, "cu_seqlens_sentinel": -1,
                                                  "padding_poison_byte": 90}}}}
    mixed, cap = pp.domain(opspec, "fp16")
    assert mixed.names == {"H": 2, "D": 8, "total_tokens": 14, "num_seqs": 3, "NSP1": 4}
    assert cap.names == {"H": 2, "D": 8, "total_tokens": 16, "num_seqs": 4, "NSP1": 5}


def test_fallback_attributes_are_rendered():
    src = fallbacks.render("lion", "bf16", {"LR": 0.5})
    assert "#define ATTR_LR (0.5)" in src and "#define ATTR_BETA2 (0.99)" in src
    assert "typedef __nv_bfloat16 T;" in src


def test_command_line_pack_and_check(tmp_path):
    import subprocess
    import sys

    root = Path(__file__).resolve().parents[1]
    (tmp_path / "task").mkdir()
    (tmp_path / "task" / "opspec.json").write_text(json.dumps(GEMV_OPSPEC))
    src = make_tree(tmp_path / "src", {"wide": (WIDE_GUARD, GEMV_VEC)})
    run = lambda *a: subprocess.run([sys.executable, "-m", "shapeforge_b200.portfolio_pack", *a], capture_output=True,  # noqa: E731
                                    text=True, cwd=root, timeout=120)
    out = tmp_path / "parent.json"
    r = run("pack", str(src), "--task-dir", str(tmp_path / "task"), "--dtype", "fp16", "--out", str(out))
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)["variants"] == ["wide"]
    r = run("check", str(out), "--task-dir", str(tmp_path / "task"), "--dtype", "fp16")
    assert r.returncode == 0 and json.loads(r.stdout)["ok"] is True
    r = run("check", str(out), "--task-dir", str(tmp_path / "task"), "--dtype", "fp16", "--sizes", "paper")
    assert r.returncode == 1 and "another domain" in r.stdout
    (src / "variants" / "stray").mkdir()
    r = run("pack", str(src), "--task-dir", str(tmp_path / "task"), "--dtype", "fp16", "--out", str(out))
    assert r.returncode == 2 and "do not match" in r.stderr


def test_output_specs_cover_every_task_dtype():
    """Outputs are allocated from the opspec: derived dims evaluate on the point's symbols (the
    varlen batch symbols included) and u32 is held as int32."""
    import torch

    opspec = {
        "tensors": {
            "q": {"role": "input", "dims": ["total_tokens", "H", "D"], "dtype": "T"},
            "output": {"role": "output", "dims": ["total_tokens", "H", "D"], "dtype": "T"},
            "final_state": {"role": "output", "dims": ["num_seqs", "H", "D", "D"], "dtype": "fp32"},
            "work_items": {"role": "output", "dims": ["num_seqs*H*3", "2"], "dtype": "u32"},
            "item_counts": {"role": "output", "dims": ["num_seqs*H*3"], "dtype": "i32"},
        },
        "sizes": {"mixed": {"H": 2, "D": 8, "seq_lens": [4, 8, 2], "usage": ["benchmark"]}},
    }
    (p,) = pp.domain(opspec, "bf16")
    specs = pp.output_specs(opspec, p)
    assert list(specs) == ["output", "final_state", "work_items", "item_counts"]
    assert specs["output"] == ((14, 2, 8), torch.bfloat16)
    assert specs["final_state"] == ((3, 2, 8, 8), torch.float32)
    assert specs["work_items"] == ((18, 2), torch.int32) and specs["item_counts"] == ((18,), torch.int32)
    with pytest.raises(pp.PortfolioError):
        pp.storage_dtype("f8", "fp16")
