"""Shape portfolios on the B200: the registered fallback of every task is correct, and a packed
portfolio dispatches, runs and is timed shard by shard with real fallback time in its accounts.

Tolerances are the tasks' OpSpec ones (fp16 rtol 2e-3 / atol_rel 1e-3, bf16 rtol 1.6e-2 /
atol_rel 8e-3; reduction_sum scales by sum |x| per row, lion by its error-scale hook).
"""

from __future__ import annotations

import ctypes
import json

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import cases, compare, fallbacks
from shapeforge_b200 import portfolio_pack as pp
from shapeforge_b200.track_factory import CudaTrackBuilder, CudaTrackEvaluator
from tests.test_portfolio_pack import GEMV_OPSPEC, GEMV_VEC, WIDE_GUARD, make_tree

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}
L = cases.LION_DEFAULTS


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _case(task, case, seed, names, dtype):
    """(inputs by ABI name, symbol order, outputs {name: shape}, oracle outputs, scales)."""
    if task in ("relu", "sigmoid", "sigmoid_shift", "silu", "swiglu"):
        inp = cases.membound_inputs(task, case, seed, (names["N"],), dtype)
        f = {k: _np(v) for k, v in inp.items()}
        ref = {"relu": lambda: oref.relu(f["x"]), "sigmoid": lambda: oref.sigmoid(f["x"]),
               "sigmoid_shift": lambda: oref.sigmoid_shift(f["x"]), "silu": lambda: oref.silu(f["x"]),
               "swiglu": lambda: oref.swiglu(f["gate"], f["up"])}[task]()
        return inp, ("N",), {"y": (names["N"],)}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task in ("softmax", "reduction_sum"):
        inp = cases.membound_inputs(task, case, seed, (names["M"], names["N"]), dtype)
        x = _np(inp["x"])
        if task == "softmax":
            ref = oref.softmax(x)
            return inp, ("M", "N"), {"y": x.shape}, {"y": ref}, {"y": compare.rms_scale(ref)}
        ref = oref.reduction_sum(x)
        return inp, ("M", "N"), {"y": (names["M"],)}, {"y": ref}, {"y": oref.reduction_sum_error_scale(x)}
    if task == "rmsnorm":
        inp = cases.rmsnorm_inputs(case, seed, names["M"], names["H"], dtype)
        ref = oref.rmsnorm(_np(inp["x"]), _np(inp["w"]), 1e-6)
        return inp, ("M", "H"), {"y": ref.shape}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task in ("gemm", "gemm_silu"):
        m, n, k = names["M"], names["N"], names["K"]
        inp = cases.gemm_inputs(case, seed, (m, k), (k, n), dtype)
        fn = oref.gemm_nn if task == "gemm" else oref.gemm_silu
        ref = fn(_np(inp["A"]), _np(inp["B"]))
        return inp, ("M", "N", "K"), {"C": (m, n)}, {"C": ref}, {"C": compare.rms_scale(ref)}
    if task == "gemv":
        inp = cases.gemv_inputs(case, seed, names["M"], names["K"], dtype)
        ref = oref.gemv(_np(inp["A"]), _np(inp["x"]))
        return inp, ("M", "K"), {"y": (names["M"],)}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task == "lion":
        inp = cases.lion_inputs(case, seed, names["N"], dtype)
        f = [_np(inp[k]) for k in ("p", "g", "m")]
        po, mo = oref.lion(*f, L["LR"], L["WD"], L["BETA1"], L["BETA2"])
        sp, sm = oref.lion_error_scale(*f, po, mo, L["LR"], L["BETA1"], TOL[dtype]["atol_rel"])
        return inp, ("N",), {"p_out": (names["N"],), "m_out": (names["N"],)}, {"p_out": po, "m_out": mo}, {"p_out": sp, "m_out": sm}
    if task == "rope":
        shape = (names["B"], names["H"], names["S"], names["D"])
        inp = cases.membound_inputs("rope", case, seed, shape, dtype)
        ref = oref.rope(_np(inp["x"]), 10000.0)
        return inp, ("B", "H", "S", "D"), {"y": shape}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task == "bitdelta_gemm":
        m, n, k = names["M"], names["N"], names["K"]
        inp = cases.bitdelta_inputs(case, seed, m, n, k, dtype)
        ref = oref.bitdelta_gemm(_np(inp["x"]), inp["bits"].numpy(), 0.02)
        return inp, ("M", "N", "K"), {"y": (m, n)}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task == "flash_attention":
        shape = (names["B"], names["H"], names["S"], names["D"])
        inp = cases.attention_inputs(case, seed, shape, dtype)
        ref = oref.attention(_np(inp["q"]), _np(inp["k"]), _np(inp["v"]), 0.125)
        return inp, ("B", "H", "S", "D"), {"o": shape}, {"o": ref}, {"o": compare.rms_scale(ref)}
    if task == "mamba2_chunk_scan":
        b, l, h, p, n, c = (names[k] for k in ("BATCH", "SEQLEN", "NHEADS", "HEADDIM", "DSTATE", "CHUNK"))
        inp = cases.mamba2_inputs(case, seed, b, l, h, p, n, c, dtype)
        ref = oref.mamba2_chunk_scan(*(_np(inp[k]) for k in ("x", "dt", "dA_cumsum", "Bmat", "Cmat", "Dskip", "states")))
        order = ("BATCH", "SEQLEN", "NHEADS", "HEADDIM", "DSTATE", "CHUNK", "NCHUNKS")
        return inp, order, {"y": (b, l, h, p)}, {"y": ref}, {"y": compare.rms_scale(ref)}
    if task == "kda":
        n, h, d = names["N"], names["H"], names["D"]
        inp = cases.kda_fixed_inputs(case, seed, n, h, d, dtype)
        f = [_np(inp[k]) for k in ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state")]
        ro, rf = oref.kda_fixed(*f, float(inp["scale"][0]), -5.0)
        outs = {"output": (n, h, d), "final_state": ((h, d, d), torch.float32), "work_items": ((3, 2), torch.int32),
                "item_counts": ((1,), torch.int32), "handoff_states": ((2, h, d, d), torch.float32)}
        return inp, ("N", "H", "D"), outs, {"output": ro, "final_state": rf}, {"output": compare.rms_scale(ro),
                                                                                 "final_state": compare.rms_scale(rf)}
    if task == "varlen_kda":
        lens, h, d = names["seq_lens"], names["H"], names["D"]
        inp = cases.kda_task_inputs(lens, h, d, dtype, seed)
        f = [_np(inp[k]) for k in ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state")]
        ro, rf = oref.varlen_kda(*f, inp["cu_seqlens"].numpy(), float(inp["scale"][0]), -5.0)
        t, ns = sum(lens), len(lens)
        outs = {"output": (t, h, d), "final_state": ((ns, h, d, d), torch.float32), "log_decay_tab": ((t, h, d), torch.float32),
                "token_stats": ((t, h, 3), torch.float32), "work_items": ((ns * h * 3, 2), torch.int32),
                "item_counts": ((ns * h * 3,), torch.int32), "handoff_flags": ((ns * h * 4,), torch.int32),
                "handoff_states": ((ns * h * 2, d, d), torch.float32)}
        return inp, ("H", "D"), outs, {"output": ro, "final_state": rf}, {"output": compare.rms_scale(ro),
                                                                          "final_state": compare.rms_scale(rf)}
    raise KeyError(task)


SHAPES = {
    "relu": {"N": 65537}, "sigmoid": {"N": 65536}, "sigmoid_shift": {"N": 1001}, "silu": {"N": 65536}, "swiglu": {"N": 4099},
    "lion": {"N": 65536}, "rmsnorm": {"M": 64, "H": 512}, "softmax": {"M": 64, "N": 515}, "reduction_sum": {"M": 64, "N": 1024},
    "gemv": {"M": 256, "K": 513}, "gemm": {"M": 130, "N": 72, "K": 128}, "gemm_silu": {"M": 64, "N": 256, "K": 128},
    "rope": {"B": 1, "H": 2, "S": 64, "D": 64},
    "bitdelta_gemm": {"M": 33, "N": 72, "K": 256},
    "flash_attention": {"B": 1, "H": 2, "S": 130, "D": 64},
    "mamba2_chunk_scan": {"BATCH": 1, "SEQLEN": 128, "NHEADS": 2, "HEADDIM": 64, "DSTATE": 64, "CHUNK": 64, "NCHUNKS": 2},
    "kda": {"N": 17, "H": 2, "D": 8},
    "varlen_kda": {"H": 2, "D": 64, "seq_lens": [5, 0, 19, 1], "num_seqs": 4, "total_tokens": 25},
}
CASES = {"reduction_sum": ("normal", "cancel", "ieee"), "softmax": ("normal", "large", "ieee"),
         "bitdelta_gemm": ("random", "edge_bits", "ieee"), "mamba2_chunk_scan": ("normal", "wide_range", "ieee"),
         "kda": ("normal", "wide_range", "outlier"), "varlen_kda": ("normal",)}
# The varlen_kda / kda tasks take the recurrence's looser opspec tolerance for varlen_kda.
TASK_TOL = {"varlen_kda": {"fp16": dict(rtol=1e-2, atol_rel=5e-3), "bf16": dict(rtol=3e-2, atol_rel=1.5e-2)}}


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", fallbacks.TASKS)
def test_registered_fallback_matches_the_oracle(cuda_device, task, dtype):
    names = SHAPES[task]
    build = CudaTrackBuilder().build(fallbacks.render(task, dtype))
    for ci, case in enumerate(CASES.get(task, ("normal", "large", "ieee"))):
        inp, order, outs, refs, scales = _case(task, case, cases.case_seed(0, ci), names, dtype)
        inp = {k: v.to(cuda_device) for k, v in inp.items()}
        out = {}
        for k, spec in outs.items():
            shape, tdt = spec if isinstance(spec[0], tuple) else (spec, TD[dtype])
            out[k] = torch.empty(shape, dtype=tdt, device=cuda_device)
        launch = CudaTrackEvaluator.launcher(build, [ctypes.c_longlong(names[s]) for s in order], names=names)
        launch([t.data_ptr() for t in (*inp.values(), *out.values())])
        torch.cuda.synchronize()
        for k, ref in refs.items():
            tol = dict(TOL[dtype], atol_rel=3e-6) if task == "reduction_sum" else TASK_TOL.get(task, TOL)[dtype]
            odt = "fp32" if out[k].dtype == torch.float32 else dtype
            v = compare.check(_np(out[k]), ref, scales[k], dtype=odt, **tol)
            assert v.ok, (task, case, k, v.summary())
        if task == "kda":
            n = names["N"]
            assert out["work_items"].cpu().tolist() == [[0, n], [n, 0], [n, 0]] and out["item_counts"].item() == 1


def test_gemv_portfolio_dispatch_run_and_accounts(cuda_device, tmp_path):
    """paper (4096 x 4096) dispatches to the vectorised variant, small (256 x 512) to the registered
    fallback; both are verified against the oracle and timed against torch.mv, and the report's
    shards carry both providers with their real times."""
    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    assert pp.check(parent, points).ok

    def make_inputs(p):
        return {k: v.to(cuda_device) for k, v in cases.gemv_inputs("normal", 7, p.names["M"], p.names["K"], "fp16").items()}

    def verify(p, inputs, outputs):
        ref = oref.gemv(_np(inputs["A"]), _np(inputs["x"]))
        v = compare.check(_np(outputs["y"]), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"])
        return v.ok, v.summary()

    runs = pp.measure(parent, GEMV_OPSPEC, points, make_inputs=make_inputs, baseline=torch.mv, verify=verify, reps=15)
    by_key = {r.point.instance_key: r for r in runs}
    assert set(by_key) == {"fp16/paper/benchmark", "fp16/small/benchmark"}
    assert by_key["fp16/paper/benchmark"].provider == "candidate" and by_key["fp16/paper/benchmark"].selected == "wide"
    assert by_key["fp16/small/benchmark"].provider == "fallback"
    assert by_key["fp16/small/benchmark"].selected == "cuda-sm100.fallback.gemv"
    for r in runs:
        assert r.correct, (r.point.instance_key, r.detail)
        assert r.candidate_us > 0 and r.baseline_us > 0
    report = pp.performance(runs)
    doc = report.document()
    assert {s["provider"] for s in doc["shards"]} == {"candidate", "fallback"}
    if report.publishable:
        total = sum(r.candidate_us for r in runs)
        assert report.fallback_time_fraction == pytest.approx(by_key["fp16/small/benchmark"].candidate_us / total)
        assert report.fallback_count_fraction == pytest.approx(0.5)
    print(json.dumps(doc, indent=1))


def gemv_recipe(seed: int = 7) -> dict:
    """What a portfolio worker needs for the gemv portfolio (called inside the worker, on its GPU)."""
    dev = torch.device("cuda", 0)

    def make_inputs(p):
        return {k: v.to(dev) for k, v in cases.gemv_inputs("normal", seed, p.names["M"], p.names["K"], "fp16").items()}

    def verify(p, inputs, outputs):
        ref = oref.gemv(_np(inputs["A"]), _np(inputs["x"]))
        v = compare.check(_np(outputs["y"]), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"])
        return v.ok, v.summary()

    return {"make_inputs": make_inputs, "baseline": torch.mv, "verify": verify}


def test_gemv_portfolio_one_gpu_per_shard(cuda_device, tmp_path):
    """The same portfolio with its shards dealt to every GPU of the machine, one worker process
    per GPU: every shard verified and timed, both providers in one report."""
    from shapeforge_b200 import fanout

    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path, {"wide": (WIDE_GUARD, GEMV_VEC)}), points)
    runs = fanout.measure_on_gpus(parent, GEMV_OPSPEC, points, recipe="tests.test_portfolio_gpu:gemv_recipe", reps=15,
                                  timeout_s=900)
    by_key = {r.point.instance_key: r for r in runs}
    assert set(by_key) == {"fp16/paper/benchmark", "fp16/small/benchmark"}
    assert by_key["fp16/paper/benchmark"].selected == "wide" and by_key["fp16/small/benchmark"].provider == "fallback"
    for r in runs:
        assert r.correct, (r.point.instance_key, r.detail)
        assert r.candidate_us > 0 and r.baseline_us > 0
    doc = pp.performance(runs).document()
    assert {s["provider"] for s in doc["shards"]} == {"candidate", "fallback"}
    print(json.dumps(doc, indent=1))


def test_gemv_portfolio_fresh_confirmation_and_publication(cuda_device, tmp_path):
    """Each point runs twice from a fresh nvcc build: on the search seed and on its fresh seed.
    Every subject is then correct on both runs, and a fully confirmed, publishable portfolio
    lands in the catalog with subjects that re-verify.  Timing noise is a legitimate rejection
    (the reference's rule); every other reason is a failure."""
    from shapeforge_b200 import confirmation as cf

    points = pp.domain(GEMV_OPSPEC, "fp16")
    parent = pp.pack(make_tree(tmp_path / "src", {"wide": (WIDE_GUARD, GEMV_VEC)}), points)

    def make_inputs(p, seed):
        return {k: v.to(cuda_device) for k, v in cases.gemv_inputs("normal", seed, p.names["M"], p.names["K"], "fp16").items()}

    def verify(p, inputs, outputs):
        ref = oref.gemv(_np(inputs["A"]), _np(inputs["x"]))
        v = compare.check(_np(outputs["y"]), ref, compare.rms_scale(ref), dtype="fp16", **TOL["fp16"])
        return v.ok, v.summary()

    runs, subjects = cf.confirm(parent, GEMV_OPSPEC, points, make_inputs=make_inputs, baseline=torch.mv, verify=verify,
                                master_seed=20260101)
    assert len(subjects) == 4 and len(runs) == 2
    for s in subjects:
        assert s["search_report"]["status"] == "ok" and s["confirmation_report"]["status"] == "ok", s["instance_key"]
        assert s["search_report"]["cache_hit"] is False and s["confirmation_report"]["seed"] != cf.SEARCH_SEED
        assert s["status"] == "confirmed" or s["reason"] == "timing_uncertain", (s["instance_key"], s["reason"])
    if all(s["status"] == "confirmed" for s in subjects) and pp.performance(runs).publishable:
        out = cf.publish(tmp_path / "kernels", "gemv", "fp16", parent, runs, subjects)
        manifest = json.loads((out / "manifest.json").read_text())
        assert len(manifest["subjects"]) == 4
        for f in (out / "subjects").iterdir():
            cf.verify_subject(json.loads(f.read_text()))
        print(json.dumps(manifest, indent=1))
