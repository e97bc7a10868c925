"""The workload variants as OpSpec v2 task directories (``tasks/<op>/``).

gemm_nt, bitdelta_gemm_base, flash_attention_causal and varlen_kda_gated each have an opspec.json
and a reference.py restated from the workload formulas.  CPU: every directory loads through the
reference's own ``load_task_contract`` (when the reference checkout is mounted), and each task's
reference agrees with the oracle on the task's own inputs.  GPU: the kernels reproduce each task's
reference on every declared case of the small size, within the tolerances of its opspec.json.
"""

from __future__ import annotations

import importlib.util
import json
import math
import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import ops as oref
from shapeforge_b200 import compare

ROOT = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
TASKS = ("gemm_nt", "bitdelta_gemm_base", "flash_attention_causal", "varlen_kda_gated")
STORAGE = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32, "i32": torch.int32, "u32": torch.int32}


def _module(task):
    spec = importlib.util.spec_from_file_location(f"variant_{task}", ROOT / "tasks" / task / "reference.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _opspec(task):
    return json.loads((ROOT / "tasks" / task / "opspec.json").read_text())


def _instance(task, size, dtype):
    """The fields of the harness instance a gen_inputs reads: symbols, dtype, canonical lengths."""
    doc = _opspec(task)
    sz = {k: v for k, v in doc["sizes"][size].items() if k != "usage"}
    lengths = sz.pop("seq_lens", None)
    symbols = dict(sz)
    if lengths is not None:
        symbols.update(total_tokens=sum(lengths), num_seqs=len(lengths), NSP1=len(lengths) + 1)
    return SimpleNamespace(symbols=symbols, dtype=dtype, canonical_seq_lens=tuple(lengths or ()))


def _stored(task, logical, dtype):
    """Inputs rounded to their storage dtypes (T -> the instance dtype)."""
    tensors = _opspec(task)["tensors"]
    out = {}
    for name, value in logical.items():
        dt = tensors[name]["dtype"]
        out[name] = value.to(STORAGE[dtype if dt == "T" else dt])
    return out


def _cases(task):
    return _opspec(task)["cases"]["names"]


@pytest.mark.parametrize("task", TASKS)
def test_task_directory_loads_with_reference_loader(task):
    if not REF.is_dir():
        pytest.skip("reference checkout not mounted")
    sys.path.append(str(REF))  # after this repository: the reference also has a `tests` package
    from tcenv.taskcontract import load_task_contract

    contract = load_task_contract(ROOT / "tasks" / task)
    assert contract.instance.reference_outputs
    assert contract.spec.op_name == task


@pytest.mark.parametrize("task", TASKS)
def test_task_reference_agrees_with_oracle(task):
    mod = _module(task)
    dtype = _opspec(task)["discovery"]["default_instance"]["dtype"]
    inst = _instance(task, "small", dtype)
    for ci, case in enumerate(_cases(task)):
        inp = _stored(task, mod.gen_inputs(case, 7919 * (ci + 1), inst), dtype)
        ref = {k: v.numpy() for k, v in mod.reference({k: (v.float() if v.is_floating_point() else v) for k, v in inp.items()}, {}).items()}
        f = lambda n: inp[n].double().numpy()  # noqa: E731
        if task == "gemm_nt":
            mine = {"C": oref.gemm_nt(f("A"), f("B"))}
        elif task == "bitdelta_gemm_base":
            mine = {"y": oref.bitdelta_gemm_base(f("x"), f("w_base"), inp["s_words"].numpy(), f("alpha"))}
        elif task == "flash_attention_causal":
            mine = {"o": oref.attention(f("q"), f("k"), f("v"), 1.0 / math.sqrt(inp["q"].shape[-1]), causal=True)}
        else:
            o, fin = oref.varlen_kda_gated(f("q"), f("k"), f("v"), f("g"), f("beta"), inp["cu_seqlens"].numpy(),
                                           1.0 / math.sqrt(inp["q"].shape[-1]))
            mine = {"output": o, "final_state": fin}
        for name, r in ref.items():
            assert np.array_equal(np.isnan(mine[name]), np.isnan(r)), (task, case, name)
            v = compare.check(mine[name], r, compare.rms_scale(r) or 1.0, rtol=1e-9, atol_rel=1e-9, dtype="fp64")
            assert v.ok, (task, case, name, v.summary())


def _kernel(task, inp, dev):
    from shapeforge_b200 import ops

    d = {k: v.to(dev) for k, v in inp.items()}
    if task == "gemm_nt":
        return {"C": ops.gemm_nt(d["A"], d["B"])}
    if task == "bitdelta_gemm_base":
        return {"y": ops.bitdelta_gemm_base(d["x"], d["w_base"], d["s_words"], d["alpha"])}
    if task == "flash_attention_causal":
        return {"o": ops.flash_attention(d["q"], d["k"], d["v"], 1.0 / math.sqrt(d["q"].shape[-1]), causal=True)}
    o, fin = ops.varlen_kda_gated(d["q"], d["k"], d["v"], d["g"], d["beta"], d["cu_seqlens"], 1.0 / math.sqrt(d["q"].shape[-1]))
    return {"output": o, "final_state": fin}


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("task", TASKS)
def test_kernels_reproduce_task_reference(cuda_device, task, dtype):
    mod = _module(task)
    doc = _opspec(task)
    tol = doc["numerics"]["tolerances"][dtype]
    inst = _instance(task, "small", dtype)
    for ci, case in enumerate(_cases(task)):
        inp = _stored(task, mod.gen_inputs(case, 7919 * (ci + 1), inst), dtype)
        ref = mod.reference({k: (v.float() if v.is_floating_point() else v) for k, v in inp.items()}, {})
        got = _kernel(task, inp, cuda_device)
        torch.cuda.synchronize()
        for name, r in ref.items():
            rn = r.numpy()
            out_dtype = dtype if doc["tensors"][name]["dtype"] == "T" else doc["tensors"][name]["dtype"]
            v = compare.check(got[name].double().cpu().numpy(), rn, compare.rms_scale(rn), rtol=tol["rtol"],
                              atol_rel=tol["atol_rel"], dtype=out_dtype)
            assert v.ok, (task, dtype, case, name, v.summary())
