"""varlen_kda (task contract), kda (the fixed-length task) and varlen_kda_gated (the gated
workload) on the B200.

Tolerances: tasks/varlen_kda/opspec.json numerics — fp16 rtol 1e-2 / atol_rel 5e-3, bf16 rtol
3e-2 / atol_rel 1.5e-2 — for both the output and the final state, scaled by the RMS of each
finite reference.  Heads are independent chains, so large shapes are checked on a few heads.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

import oracle
from oracle import ops as oref
from shapeforge_b200 import cases, compare, ops
from tests import golden

pytestmark = pytest.mark.gpu

TOL = {"fp16": dict(rtol=1e-2, atol_rel=5e-3), "bf16": dict(rtol=3e-2, atol_rel=1.5e-2)}
TD = {"fp16": torch.float16, "bf16": torch.bfloat16}


def _np(t):
    return t.detach().cpu().to(torch.float64).numpy()


def _from_fixture(arr, dtype_name, dev):
    a = np.ascontiguousarray(arr)
    if dtype_name in ("fp16", "bf16"):
        return torch.from_numpy(a.view(np.int16)).view(TD[dtype_name]).to(dev)
    if dtype_name == "fp32":
        return torch.from_numpy(a.astype(np.float32)).to(dev)
    return torch.from_numpy(a.astype(np.int32)).to(dev)


def _verdict(got, ref, dtype, out_dtype):
    return compare.check(got, ref, compare.rms_scale(ref), dtype=out_dtype, **TOL[dtype])


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("tier", ["mixed", "fixed", "uniform"])
def test_reference_vectors(cuda_device, tier, dtype):
    """All 9 correctness cases of the reference's own varlen planner, on its own input bytes."""
    doc = golden.load(f"ref_varlen_kda_{tier}_{dtype}")
    tdt = doc["tensor_dtypes"]
    assert len(doc["records"]) == 9
    for rec in doc["records"]:
        d = {k: _from_fixture(v, tdt[k], cuda_device) for k, v in rec["inputs"].items()}
        out, fin = ops.varlen_kda(d["q"], d["k"], d["v"], d["g"], d["beta"], d["A_log"], d["dt_bias"], d["initial_state"],
                                  d["cu_seqlens"], d["scale"], lower_bound=-5.0)
        torch.cuda.synchronize()
        v1 = _verdict(_np(out), rec["refs"]["output"], dtype, dtype)
        v2 = _verdict(_np(fin), rec["refs"]["final_state"], dtype, "fp32")
        assert v1.ok, (tier, rec["case"], "output", v1.summary())
        assert v2.ok, (tier, rec["case"], "final_state", v2.summary())


def _oracle_task(inp, heads, lower_bound=-5.0):
    f = lambda n: _np(inp[n])  # noqa: E731
    sel = lambda a: a[:, heads]  # noqa: E731
    out, fin = oref.varlen_kda(
        sel(f("q")), sel(f("k")), sel(f("v")), sel(f("g")), sel(f("beta")), f("A_log")[heads],
        f("dt_bias").reshape(-1, inp["q"].shape[2])[heads].reshape(-1), f("initial_state")[:, heads],
        inp["cu_seqlens"].cpu().numpy(), float(f("scale")[0]), lower_bound)
    return out, fin


@pytest.mark.parametrize("variant", [1, 4])
@pytest.mark.parametrize("lower_bound", [-12.0, -60.0])
def test_task_op_chunked_strong_lower_bound(cuda_device, lower_bound, variant):
    """LOWER_BOUND beyond what the chunk factors can hold (cumulative decays down to -190 and -960
    per 16-token chunk): the 16-token chunked kernel (variant 1) and the two-pass 32-token kernels
    (variant 4) form those chunks pair by pair and still match the fp64 oracle."""
    lengths = [300, 0, 45, 16]
    heads = 2
    inp = cases.kda_task_inputs(lengths, heads, 128, "bf16", seed=cases.case_seed(12, 4))
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    out, fin = ops.varlen_kda(d["q"], d["k"], d["v"], d["g"], d["beta"], d["A_log"], d["dt_bias"], d["initial_state"],
                              d["cu_seqlens"], d["scale"], lower_bound=lower_bound, variant=variant)
    torch.cuda.synchronize()
    code, where = ops.kernel_status()
    assert code == 0, (code, where)
    ro, rf = _oracle_task(d, [0, 1], lower_bound)
    v1 = _verdict(_np(out), ro, "bf16", "bf16")
    v2 = _verdict(_np(fin), rf, "bf16", "fp32")
    assert v1.ok, ("output", lower_bound, v1.summary())
    assert v2.ok, ("final_state", lower_bound, v2.summary())


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("variant", [1, 2, 4])
def test_task_op_chunked_and_recurrent(cuda_device, dtype, variant):
    """The task op at D = 128 through the 16-token chunked tensor-core kernel (variant 1: in-op q/k
    norms, gates from A_log / dt_bias, sigmoid beta, initial state), the recurrent kernel (variant
    2) and the two-pass kernels (variant 4: every 32-token chunk prepared into a workspace, then
    the chains), all against the fp64 oracle; a 700-token sequence carries the state through 44
    chunks, a zero-length one is skipped."""
    lengths = [700, 0, 33, 16, 129]
    heads = 3
    inp = cases.kda_task_inputs(lengths, heads, 128, dtype, seed=cases.case_seed(11, 2))
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    out = torch.full_like(d["v"], float("nan"))
    out, fin = ops.varlen_kda(d["q"], d["k"], d["v"], d["g"], d["beta"], d["A_log"], d["dt_bias"], d["initial_state"],
                              d["cu_seqlens"], d["scale"], output=out, variant=variant)
    torch.cuda.synchronize()
    hs = list(range(heads))
    ro, rf = _oracle_task(d, hs)
    v1 = _verdict(_np(out), ro, dtype, dtype)
    v2 = _verdict(_np(fin), rf, dtype, "fp32")
    assert v1.ok, ("output", variant, v1.summary())
    assert v2.ok, ("final_state", variant, v2.summary())
    code, where = ops.kernel_status()
    assert code == 0, f"tensor-core kernel status {code} at wait {where}"


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("dim", [128, 64, 32])
def test_task_op_large_heads(cuda_device, dtype, dim):
    lengths = [130, 64, 1, 300, 0, 17]
    heads = 4
    inp = cases.kda_task_inputs(lengths, heads, dim, dtype, seed=cases.case_seed(0, 3))
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    out = torch.full_like(d["v"], float("nan"))
    out, fin = ops.varlen_kda(d["q"], d["k"], d["v"], d["g"], d["beta"], d["A_log"], d["dt_bias"], d["initial_state"],
                              d["cu_seqlens"], d["scale"], output=out)
    torch.cuda.synchronize()
    hs = [0, heads - 1]
    ro, rf = _oracle_task(d, hs)
    v1 = _verdict(_np(out)[:, hs], ro, dtype, dtype)
    v2 = _verdict(_np(fin)[:, hs], rf, dtype, "fp32")
    assert v1.ok, ("output", v1.summary())
    assert v2.ok, ("final_state", v2.summary())


def test_capacity_sentinel_leaves_padding(cuda_device):
    """cu_seqlens entries of -1 (the L2 capacity sentinel) end the batch: unused final-state rows
    and output rows past the resolved total keep their padding bytes."""
    lengths = [5, 3, 1]
    inp = cases.kda_task_inputs(lengths, 2, 8, "fp16", seed=11)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    cap_seqs, cap_tokens = 4, 16
    cu = torch.tensor([0, 5, 8, 9, -1], dtype=torch.int32, device=cuda_device)
    pad = lambda t, n: torch.cat([t, torch.zeros((n - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)])  # noqa: E731
    q, k, v, g = (pad(d[n], cap_tokens) for n in ("q", "k", "v", "g"))
    beta = pad(d["beta"], cap_tokens)
    s0 = torch.cat([d["initial_state"], torch.zeros((1, 2, 8, 8), device=cuda_device)])
    out = torch.full((cap_tokens, 2, 8), 7.0, dtype=torch.float16, device=cuda_device)
    fin = torch.full((cap_seqs, 2, 8, 8), 7.0, dtype=torch.float32, device=cuda_device)
    ops.varlen_kda(q, k, v, g, beta, d["A_log"], d["dt_bias"], s0, cu, d["scale"], output=out, final_state=fin)
    torch.cuda.synchronize()
    assert torch.all(out[9:] == 7.0)
    assert torch.all(fin[3] == 7.0)
    ro, rf = _oracle_task(d, [0, 1])
    assert _verdict(_np(out[:9]), ro, "fp16", "fp16").ok
    assert _verdict(_np(fin[:3]), rf, "fp16", "fp32").ok


def test_task_op_two_pass_capacity_sentinel(cuda_device):
    """The two-pass kernels at D = 128 under the capacity contract: entries of -1 after the resolved
    total end the batch, padding rows of the output and unused final-state rows keep their bytes,
    and the live sequences match the oracle."""
    lengths = [70, 33, 1]
    heads, dim = 2, 128
    inp = cases.kda_task_inputs(lengths, heads, dim, "bf16", seed=cases.case_seed(5, 9))
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    cap_seqs, cap_tokens = 5, 160
    cu = torch.tensor([0, 70, 103, 104, -1, -1], dtype=torch.int32, device=cuda_device)
    pad = lambda t, n: torch.cat([t, torch.zeros((n - t.shape[0],) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)])  # noqa: E731
    q, k, v, g, beta = (pad(d[n], cap_tokens) for n in ("q", "k", "v", "g", "beta"))
    s0 = pad(d["initial_state"], cap_seqs)
    out = torch.full((cap_tokens, heads, dim), 7.0, dtype=torch.bfloat16, device=cuda_device)
    fin = torch.full((cap_seqs, heads, dim, dim), 7.0, dtype=torch.float32, device=cuda_device)
    ops.varlen_kda(q, k, v, g, beta, d["A_log"], d["dt_bias"], s0, cu, d["scale"], output=out, final_state=fin, variant=4)
    torch.cuda.synchronize()
    code, where = ops.kernel_status()
    assert code == 0, (code, where)
    assert torch.all(out[104:] == 7.0)
    assert torch.all(fin[3:] == 7.0)
    ro, rf = _oracle_task(d, [0, 1])
    assert _verdict(_np(out[:104]), ro, "bf16", "bf16").ok
    assert _verdict(_np(fin[:3]), rf, "bf16", "fp32").ok


def test_task_op_two_pass_matches_chunked(cuda_device):
    """The two-pass kernels and the 16-token chunked kernel agree on a batch of many heads (all
    heads compared, each to the other's RMS scale at the task tolerance)."""
    lengths = [257, 96, 31, 512]
    inp = cases.kda_task_inputs(lengths, 8, 128, "bf16", seed=cases.case_seed(3, 7))
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    args = [d[n] for n in ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state", "cu_seqlens", "scale")]
    o4, f4 = ops.varlen_kda(*args, variant=4)
    o1, f1 = ops.varlen_kda(*args, variant=1)
    torch.cuda.synchronize()
    v1 = _verdict(_np(o4), _np(o1), "bf16", "bf16")
    v2 = _verdict(_np(f4), _np(f1), "bf16", "fp32")
    assert v1.ok, v1.summary()
    assert v2.ok, v2.summary()


def _oracle_gated(inp, heads, scale):
    f = lambda n: _np(inp[n])[:, heads]  # noqa: E731
    return oref.varlen_kda_gated(f("q"), f("k"), f("v"), f("g"), f("beta"), inp["cu_seqlens"].cpu().numpy(), scale)


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gated_workload(cuda_device, dtype):
    """The gated workload: 8 packed sequences of seeded U(256, 4096) lengths, H=16, D=128."""
    lengths = cases.kda_gated_lengths()
    heads, dim = 16, 128
    inp = cases.kda_gated_inputs(lengths, heads, dim, dtype)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    scale = 1.0 / math.sqrt(dim)
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], scale)
    torch.cuda.synchronize()
    hs = [0, 9, 15]
    ro, rf = _oracle_gated(d, hs, scale)
    v1 = _verdict(_np(out)[:, hs], ro, dtype, dtype)
    v2 = _verdict(_np(fin)[:, hs], rf, dtype, "fp32")
    assert v1.ok, ("output", v1.summary())
    assert v2.ok, ("final_state", v2.summary())
    assert not torch.isnan(out).any()


@pytest.mark.parametrize("decay", [("shift", -8.0), ("const", -6.0), ("const", -30.0)])
def test_gated_workload_strong_decay(cuda_device, decay):
    """The workload's lengths and shapes with strong decays, on the default (chunked) kernel:
    logits shifted by -8 (about -8 per token, cumulative -130 over a 16-token chunk), a constant
    -6 (-96), and a constant -30 (-480, past what per-token factors can hold, so every chunk takes
    the pairwise path).  Checked on three heads against the fp64 recurrence."""
    kind, val = decay
    lengths = cases.kda_gated_lengths()
    heads, dim = 16, 128
    kw = {"logit_shift": val} if kind == "shift" else {"g_const": val}
    inp = cases.kda_gated_inputs(lengths, heads, dim, "bf16", **kw)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    scale = 1.0 / math.sqrt(dim)
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], scale)
    torch.cuda.synchronize()
    code, where = ops.kernel_status()
    assert code == 0, (code, where)
    assert torch.isfinite(out.float()).all() and torch.isfinite(fin).all()
    hs = [0, 7, 15]
    ro, rf = _oracle_gated(d, hs, scale)
    v1 = _verdict(_np(out)[:, hs], ro, "bf16", "bf16")
    v2 = _verdict(_np(fin)[:, hs], rf, "bf16", "fp32")
    assert v1.ok, ("output", decay, v1.summary())
    assert v2.ok, ("final_state", decay, v2.summary())


@pytest.mark.parametrize("variant", [1, 4])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gated_chunked_mixed_decay_with_state(cuda_device, dtype, variant):
    """Chunks of ordinary, strong and infinite decay in one sequence, from a non-zero initial state,
    on the single-pass (variant 1) and two-pass (variant 4) chunked kernels: each chunk takes the
    factored or the pairwise path on its own."""
    lengths = [7, 48, 130, 0, 65]
    heads = 2
    inp = cases.kda_gated_inputs(lengths, heads, 128, dtype, seed=21)
    gen = torch.Generator().manual_seed(5)
    g = inp["g"].clone()
    t = g.shape[0]
    band = (torch.arange(t) // 16) % 3  # chunk bands: 0 ordinary, 1 strong, 2 extreme
    strong = -6.0 + torch.randn(g.shape, generator=gen)
    extreme = -40.0 + 10.0 * torch.randn(g.shape, generator=gen)
    g = torch.where((band == 1)[:, None, None], strong, g)
    g = torch.where((band == 2)[:, None, None], extreme, g)
    g[torch.rand(g.shape, generator=gen) < 0.005] = -math.inf
    inp["g"] = g.float()
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    s0 = (0.1 * torch.randn((len(lengths), heads, 128, 128), generator=gen)).to(cuda_device)
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 0.125, initial_state=s0,
                                    variant=variant)
    torch.cuda.synchronize()
    code, where = ops.kernel_status()
    assert code == 0, (code, where)
    f = lambda n: _np(d[n])  # noqa: E731
    ro, rf = oref.varlen_kda_gated(f("q"), f("k"), f("v"), f("g"), f("beta"), inp["cu_seqlens"].numpy(), 0.125, state0=_np(s0))
    v1 = _verdict(_np(out), ro, dtype, dtype)
    v2 = _verdict(_np(fin), rf, dtype, "fp32")
    assert v1.ok, ("output", v1.summary())
    assert v2.ok, ("final_state", v2.summary())


def test_gated_two_pass_matches_single_pass(cuda_device):
    """The two-pass kernels (the default at D = 128) against the single-pass 32-token kernel on the
    workload: the same chunk algebra, so the outputs agree to a few 16-bit ulps."""
    lengths = cases.kda_gated_lengths()
    inp = cases.kda_gated_inputs(lengths, 16, 128, "bf16")
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    args = (d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 1.0 / math.sqrt(128))
    o4, f4 = ops.varlen_kda_gated(*args, variant=4)
    o1, f1 = ops.varlen_kda_gated(*args, variant=1)
    torch.cuda.synchronize()
    assert ops.kernel_status()[0] == 0
    assert (o4.float() - o1.float()).abs().max().item() <= 0.02 * o1.float().abs().max().item()
    assert (f4 - f1).abs().max().item() <= 1e-3 * f1.abs().max().item()


def test_gated_two_pass_rejects_understated_token_count(cuda_device):
    """A total token count below cu_seqlens[-1] (which also sizes the workspace too small): the
    kernels skip all work and report it through the status word (code 2, where 96); no row past the
    stated count is read and the workspace bounds are never crossed."""
    from shapeforge_b200 import _native

    lengths = [100, 300]
    inp = cases.kda_gated_inputs(lengths, 2, 128, "bf16", seed=4)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    t_small = 40
    ws_bytes = ops.varlen_kda_gated_workspace_bytes(t_small, 2, 2, 128)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=cuda_device)
    out = torch.full_like(d["v"], 3.0)
    fin = torch.full((2, 2, 128, 128), 3.0, device=cuda_device)
    ptrs = [d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["g"].data_ptr(), d["beta"].data_ptr(), d["cu_seqlens"].data_ptr(),
            0, out.data_ptr(), fin.data_ptr(), ws.data_ptr()]
    desc = _native.op_desc("varlen_kda_gated", "bf16", dims=(2, 2, 128, t_small, ws_bytes), attrs=(0.125,), variant=4)
    _native.run_op(desc, ptrs, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert ops.kernel_status() == (2, 96)
    assert torch.all(out == 3.0) and torch.all(fin == 3.0)


def test_gated_small_ragged(cuda_device):
    lengths = [1, 0, 63, 64, 65, 200]
    inp = cases.kda_gated_inputs(lengths, 3, 64, "bf16", seed=3)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 0.125)
    torch.cuda.synchronize()
    ro, rf = _oracle_gated(d, [0, 1, 2], 0.125)
    assert _verdict(_np(out), ro, "bf16", "bf16").ok
    assert _verdict(_np(fin), rf, "bf16", "fp32").ok


@pytest.mark.parametrize("variant", [1, 4])
@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_gated_chunked_ragged_with_state(cuda_device, dtype, variant):
    """The chunked tensor-core kernels (variant 1 single-pass, 4 two-pass): lengths around the
    16- and 32-token chunk edges, an empty sequence, more chunks than ring stages, and a non-zero
    initial state, against the fp64 recurrence."""
    lengths = [1, 0, 15, 16, 17, 31, 32, 33, 64, 200]
    heads = 2
    inp = cases.kda_gated_inputs(lengths, heads, 128, dtype, seed=5)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    g = torch.Generator().manual_seed(11)
    s0 = (0.1 * torch.randn((len(lengths), heads, 128, 128), generator=g)).to(cuda_device)
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 0.125, initial_state=s0,
                                    variant=variant)
    torch.cuda.synchronize()
    code, where = ops.kernel_status()
    assert code == 0, (code, where)
    f = lambda n: _np(d[n])  # noqa: E731
    ro, rf = oref.varlen_kda_gated(f("q"), f("k"), f("v"), f("g"), f("beta"), inp["cu_seqlens"].numpy(), 0.125, state0=_np(s0))
    v1 = _verdict(_np(out), ro, dtype, dtype)
    v2 = _verdict(_np(fin), rf, dtype, "fp32")
    assert v1.ok, ("output", v1.summary())
    assert v2.ok, ("final_state", v2.summary())


def test_gated_recurrent_variant_still_matches(cuda_device):
    """variant=2 keeps the recurrent CUDA-core kernel reachable (and correct) for D = 128."""
    lengths = [40, 7]
    inp = cases.kda_gated_inputs(lengths, 2, 128, "bf16", seed=9)
    d = {k: v.to(cuda_device) for k, v in inp.items()}
    out, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 0.125, variant=2)
    torch.cuda.synchronize()
    ro, rf = _oracle_gated(d, [0, 1], 0.125)
    assert _verdict(_np(out), ro, "bf16", "bf16").ok
    assert _verdict(_np(fin), rf, "bf16", "fp32").ok


# ---- fixed-length kda (tasks/kda) -------------------------------------------------------------

# tasks/kda/opspec.json numerics (tighter than varlen_kda's).
FIXED_TOL = {"fp16": dict(rtol=2e-3, atol_rel=1e-3), "bf16": dict(rtol=1.6e-2, atol_rel=8e-3)}


def _fixed_run(d, lb, variant=0):
    n = d["q"].shape[0]
    wi = torch.full((3, 2), -7, dtype=torch.int32, device=d["q"].device)
    ic = torch.full((1,), -7, dtype=torch.int32, device=d["q"].device)
    out, fin = ops.kda(d["q"], d["k"], d["v"], d["g"], d["beta"], d["A_log"], d["dt_bias"], d["initial_state"], d["scale"],
                       lower_bound=lb, work_items=wi, item_counts=ic, variant=variant)
    torch.cuda.synchronize()
    # The host program's work list: one piece [0, N) and two empty ones.
    assert wi.cpu().tolist() == [[0, n], [n, 0], [n, 0]]
    assert ic.item() == 1
    return out, fin


def _fixed_oracle(d, lb):
    f = lambda n: _np(d[n])  # noqa: E731
    return oref.kda_fixed(f("q"), f("k"), f("v"), f("g"), f("beta"), f("A_log"), f("dt_bias"), f("initial_state"),
                          float(f("scale")[0]), lb)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("size", ["single", "small", "tail"])
def test_fixed_kda_reference_vectors(cuda_device, size, dtype):
    """The reference's own inputs and fp64 outputs (D = 8) with its recorded error scales."""
    doc = golden.load(f"ref_kda_{size}_{dtype}")
    tdt = doc["tensor_dtypes"]
    lb = float(doc["attrs"]["LOWER_BOUND"])
    assert [r["case"] for r in doc["records"]] == list(cases.KDA_FIXED_CASES)
    for rec in doc["records"]:
        d = {k: _from_fixture(v, tdt[k], cuda_device) for k, v in rec["inputs"].items()}
        out, fin = _fixed_run(d, lb)
        v1 = compare.check(_np(out), rec["refs"]["output"], rec["scales"]["output"], dtype=dtype, **FIXED_TOL[dtype])
        v2 = compare.check(_np(fin), rec["refs"]["final_state"], rec["scales"]["final_state"], dtype="fp32", **FIXED_TOL[dtype])
        assert v1.ok, (size, rec["case"], "output", v1.summary())
        assert v2.ok, (size, rec["case"], "final_state", v2.summary())


FIXED_SHAPES = [(256, 8, 64), (17, 2, 8), (100, 3, 32), (1, 1, 16), (300, 2, 128)]


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("shape", FIXED_SHAPES, ids=[f"n{n}h{h}d{d}" for n, h, d in FIXED_SHAPES])
def test_fixed_kda_against_oracle(cuda_device, dtype, shape):
    """The task's input stream at the paper size (N=256, H=8, D=64) and other head dims, every case,
    through the default dispatch (the recurrent fp32 kernel at every D: the chunked kernel's TF32
    products do not always meet this task's tighter tolerance) and the recurrent variant named."""
    n, h, dim = shape
    for ci, case in enumerate(cases.KDA_FIXED_CASES):
        inp = cases.kda_fixed_inputs(case, cases.case_seed(0, ci), n, h, dim, dtype)
        d = {k: v.to(cuda_device) for k, v in inp.items()}
        ref_out, ref_fin = _fixed_oracle(d, -5.0)
        for variant in (0, 2):
            out, fin = _fixed_run(d, -5.0, variant)
            v1 = compare.check(_np(out), ref_out, compare.rms_scale(ref_out), dtype=dtype, **FIXED_TOL[dtype])
            v2 = compare.check(_np(fin), ref_fin, compare.rms_scale(ref_fin), dtype="fp32", **FIXED_TOL[dtype])
            assert v1.ok, (shape, case, variant, "output", v1.summary())
            assert v2.ok, (shape, case, variant, "final_state", v2.summary())


# ---- L2 capacity tier: continuous batching on one set of buffers ------------------------------------


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_capacity_tier_continuous_batching(cuda_device, dtype):
    """The nine reference cases of the capacity size, in declared order, through ONE set of
    capacity-sized buffers (a continuous-batching sequence of totals 16, 1, 9, 3, 16, ...): each
    call's boundary is checked against the contract, its logical region matches the reference, and
    every padding byte of both outputs still holds the poison after the call.  Then the timed
    mixture covers every declared profile (``mixture_problems`` is empty)."""
    from shapeforge_b200 import capacity as cap
    from tests.test_capacity import CAPACITY_SIZE, CASES

    doc = golden.load(f"ref_varlen_kda_capacity_{dtype}")
    tdt = doc["tensor_dtypes"]
    s = cap.CapacitySpec.from_size(CAPACITY_SIZE)
    batch = cap.CapacityBatch(s, 2, 8, TD[dtype], cuda_device)
    names = ("q", "k", "v", "g", "beta", "A_log", "dt_bias", "initial_state", "scale")
    per_case = {}
    for rec in doc["records"]:
        d = {k: _from_fixture(v, tdt[k], cuda_device) for k, v in rec["inputs"].items()}
        cu = [int(v) for v in rec["inputs"]["cu_seqlens"]]
        inputs = {k: d[k] for k in names}
        per_case[rec["case"]] = (inputs, cu)
        resolved = batch.run(inputs, cu=cu)
        torch.cuda.synchronize()
        assert batch.check_padding(resolved) == (), rec["case"]
        ro = rec["refs"]["output"][resolved.logical("output")]
        rf = rec["refs"]["final_state"][resolved.logical("final_state")]
        v1 = _verdict(_np(batch.output[resolved.logical("output")]), ro, dtype, dtype)
        v2 = _verdict(_np(batch.final_state[resolved.logical("final_state")]), rf, dtype, "fp32")
        assert v1.ok, (rec["case"], "output", v1.summary())
        assert v2.ok, (rec["case"], "final_state", v2.summary())
    batches = cap.time_mixture(batch, s, CASES, lambda case: per_case[case], reps=5)
    assert cap.mixture_problems(s, CASES, batches) == ()
    assert all(b["device_us"] > 0 for b in batches)
