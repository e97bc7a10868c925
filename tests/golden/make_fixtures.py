"""Generate the golden fixtures under ``tests/golden/`` from the reference project.

Run in a checkout that has the reference available (``REFERENCE_ROOT``, default
``/root/reference``)::

    python tests/golden/make_fixtures.py

Two sources, both produced by the reference itself:

* **G0 corpus** (``tests/support/golden/shared/跨硬件算子生成分工-G0/corpus``): the exact input bytes,
  fp64 reference bytes and error-scale bytes of the small tier, for rmsnorm, softmax,
  reduction_sum, silu, swiglu and gemm.  Read with the archive layout of
  ``tests/shared/test_v2_g0_reference_outputs.py:35-80`` (zlib ``TG0TENS1`` + JSON header).
* **Reference task modules** (``tasks/<t>/reference.py`` through
  ``tcenv.taskcontract.load_task_contract``): inputs from the task's own ``gen_inputs`` at the
  harness case seeds ``seed + 7919 * (i + 1)`` (``tcenv/backends/metal/v2_runtime.py:1602``), rounded
  to storage dtype, and the task's fp64 ``reference`` outputs, for bitdelta_gemm,
  flash_attention, rope, varlen_kda, mamba2_chunk_scan, relu, sigmoid, sigmoid_shift, lion, gemv,
  gemm_silu and kda (fixed length, sizes single/small/tail); varlen_kda also at its L2 capacity
  size (capacity-sized inputs with the padding poison, the cu_seqlens sentinel tail).  Where the task module has an ``error_scale`` hook (lion) the recorded scales are
  the hook's, otherwise the RMS of the finite reference.

``python tests/golden/make_fixtures.py relu lion`` rewrites only the named tasks' fixtures.

Large tensors are sliced to a few rows/columns (the slice is recorded) so the fixtures stay
small; the reference outputs of the kept rows/columns depend only on kept inputs.  Storage
dtypes are kept bit-exact (fp16/bf16 as their uint16 bit patterns).
"""

from __future__ import annotations

import functools
import json
import os
import struct
import sys
import zlib
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REF = Path(os.environ.get("REFERENCE_ROOT", "/root/reference"))
CORPUS = REF / "tests/support/golden/shared/跨硬件算子生成分工-G0/corpus"
MAGIC = b"TG0TENS1"
ROWS = [0, 1, 2, 3, -1]


def _storage(arr_f32: np.ndarray, dtype: str) -> np.ndarray:
    """float32 values already rounded to ``dtype`` -> storage bit patterns."""
    import torch

    if dtype == "i32":
        return np.asarray(arr_f32).astype(np.int64).astype(np.int32)
    if dtype == "u32":
        return (np.asarray(arr_f32).astype(np.int64) & 0xFFFFFFFF).astype(np.uint32)
    t = torch.from_numpy(np.ascontiguousarray(arr_f32, dtype=np.float32))
    if dtype == "fp16":
        return t.to(torch.float16).view(torch.int16).numpy().view(np.uint16)
    if dtype == "bf16":
        return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    if dtype == "fp32":
        return t.numpy().astype(np.float32)
    raise ValueError(dtype)


def _g0_archive(rel: str):
    raw = zlib.decompress((CORPUS / rel).read_bytes())
    assert raw.startswith(MAGIC), rel
    n = struct.unpack("<I", raw[8:12])[0]
    header = json.loads(raw[12 : 12 + n])
    payload = raw[12 + n :]
    out = {"input": {}, "reference": {}, "scale": {}}
    for e in header:
        out[e["role"]][e["name"]] = (payload[e["offset"] : e["offset"] + e["nbytes"]], e)
    return out


def _g0_np(piece: bytes, entry: dict, storage: str) -> np.ndarray:
    shape = tuple(entry["shape"])
    if entry["role"] == "input":
        if storage in ("fp16", "bf16"):
            return np.frombuffer(piece, dtype=np.uint16).reshape(shape).copy()
        return np.frombuffer(piece, dtype=np.float32).reshape(shape).copy()
    return np.frombuffer(piece, dtype=np.float64).reshape(shape).copy()


# Slicers: (inputs, refs, scales) -> same, smaller, plus a description.
def _rows(inputs, refs, scales, names_in, names_out):
    rows = np.array(ROWS)
    i2 = {k: (v[rows] if k in names_in else v) for k, v in inputs.items()}
    r2 = {k: (v[rows] if k in names_out else v) for k, v in refs.items()}
    s2 = {k: (v[rows] if (np.ndim(v) and k in names_out) else v) for k, v in scales.items()}
    return i2, r2, s2, {"rows": ROWS}


def _flat_head(inputs, refs, scales, n=1024):
    idx = np.concatenate([np.arange(n), [-1]])
    return (
        {k: v[idx] for k, v in inputs.items()},
        {k: v[idx] for k, v in refs.items()},
        scales,
        {"flat_index": f"0..{n - 1},-1"},
    )


def _gemm_slice(inputs, refs, scales, a="A", b="B", c="C"):
    rows = np.array(ROWS)
    cols = np.concatenate([np.arange(32), [-1]])
    i2 = dict(inputs)
    i2[a] = inputs[a][rows]
    i2[b] = inputs[b][:, cols]
    r2 = {c: refs[c][rows][:, cols]}
    return i2, r2, scales, {"rows": ROWS, "cols": "0..31,-1"}


G0_TASKS = {
    "rmsnorm": (lambda i, r, s: _rows(i, r, s, {"x"}, {"y"})),
    "softmax": (lambda i, r, s: _rows(i, r, s, {"x"}, {"y"})),
    "reduction_sum": (lambda i, r, s: _rows(i, r, s, {"x"}, {"y"})),
    "silu": _flat_head,
    "swiglu": _flat_head,
    "gemm": _gemm_slice,
}

ATTRS = {"rmsnorm": {"EPS": 1e-6}}


def from_g0(task: str, dtype: str) -> dict:
    index = json.loads((CORPUS / "index.json").read_text(encoding="utf-8"))
    combo = [c for c in index["combos"] if c["task"] == task and c["dtype"] == dtype and c["size"] == "small"]
    # Several gemm tile variants share task "gemm": take the plain one.
    combo = [c for c in combo if c["case_records"][0]["archive"].startswith(f"tensors/{task}/")]
    assert len(combo) == 1, (task, dtype, len(combo))
    combo = combo[0]
    records = []
    for ci, case in enumerate(combo["cases"]):
        seed = 7919 * (ci + 1)  # base seed 0 of the corpus's seed formula
        rec = [r for r in combo["case_records"] if r["case"] == case and r["seed"] == seed]
        assert len(rec) == 1, (task, case, seed)
        arch = _g0_archive(rec[0]["archive"])
        inputs = {k: _g0_np(p, e, dtype) for k, (p, e) in arch["input"].items()}
        refs = {k: _g0_np(p, e, dtype) for k, (p, e) in arch["reference"].items()}
        scales = {k: _g0_np(p, e, dtype) for k, (p, e) in arch["scale"].items()}
        full_shapes = {k: list(v.shape) for k, v in {**inputs, **refs}.items()}
        inputs, refs, scales, sl = G0_TASKS[task](inputs, refs, scales)
        records.append({"case": case, "seed": seed, "inputs": inputs, "refs": refs, "scales": scales, "slice": sl, "full_shapes": full_shapes})
    return {
        "task": task,
        "dtype": dtype,
        "size": "small",
        "source": f"G0 corpus {combo['case_records'][0]['archive'].split('/')[1]}",
        "tolerances": combo["tolerances"],
        "attrs": ATTRS.get(task, {}),
        "records": records,
    }


def from_reference(task: str, dtype: str, size: str, slicer=None, cases=None) -> dict:
    sys.path.insert(0, str(REF))
    from tcenv.taskcontract import load_task_contract
    from tcenv.tensors import round_to

    contract = load_task_contract(REF / "tasks" / task, dtype=dtype, size=size)
    inst = contract.instance
    tensors = {t.name: t for t in inst.tensors}
    records = []
    use_cases = list(cases or inst.case_domain.cases)
    for ci, case in enumerate(inst.case_domain.cases):
        if case not in use_cases:
            continue
        seed = 7919 * (ci + 1)
        logical = contract.reference.generate(inst, case, seed)
        rounded = {}
        for name, value in logical.items():
            if name not in tensors:
                continue
            rounded[name] = round_to(value.reshape(tuple(int(v) for v in tensors[name].shape)), tensors[name].dtype)
        ref = contract.reference.execute(inst, rounded)
        inputs = {k: _storage(v.numpy(), tensors[k].dtype) for k, v in rounded.items()}
        refs = {k: v.numpy().astype(np.float64) for k, v in ref.items()}
        scales = {}
        for k, v in refs.items():
            fin = np.where(np.isfinite(v), v, 0.0)
            scales[k] = np.float64(np.sqrt(np.mean(fin**2))) if fin.size else np.float64(0.0)
        hook = contract.reference.error_scale(inst, rounded, ref)
        for k, v in (hook or {}).items():
            scales[k] = np.asarray(v.numpy() if hasattr(v, "numpy") else v, dtype=np.float64)
        full_shapes = {k: list(v.shape) for k, v in {**inputs, **refs}.items()}
        sl = {}
        if slicer is not None:
            inputs, refs, scales, sl = slicer(inputs, refs, scales)
        records.append({"case": case, "seed": seed, "inputs": inputs, "refs": refs, "scales": scales, "slice": sl, "full_shapes": full_shapes})
    tol = inst.tolerances
    return {
        "task": task,
        "dtype": dtype,
        "size": size,
        "source": f"tasks/{task}/reference.py via load_task_contract",
        "tolerances": {"rtol": tol.rtol, "atol_rel": tol.atol_rel, "exact": tol.exact},
        "attrs": {k: (v if not hasattr(v, "item") else v.item())
                  for k, v in dict(getattr(inst, "attr_values", {}) or getattr(inst, "resolved_attrs", {}) or {}).items()},
        "tensor_dtypes": {k: t.dtype for k, t in tensors.items()},
        "symbols": {k: int(v) for k, v in inst.symbols.items()},
        "records": records,
    }


def _fa_slice(inputs, refs, scales):
    rows = np.array([0, 1, 2, 3, 64, -1])
    i2 = dict(inputs)
    i2["q"] = inputs["q"][:, :, rows]
    return i2, {"o": refs["o"][:, :, rows]}, scales, {"q_rows": [0, 1, 2, 3, 64, -1]}


def _bitdelta_slice(inputs, refs, scales):
    rows = np.array(ROWS)
    cols = np.concatenate([np.arange(32), [-1]])
    i2 = dict(inputs)
    i2["x"] = inputs["x"][rows]
    i2["bits"] = inputs["bits"][:, cols]
    return i2, {"y": refs["y"][rows][:, cols]}, scales, {"rows": ROWS, "cols": "0..31,-1"}


def _rope_slice(inputs, refs, scales):
    pos = [0, 1, 2, 3, 31, -1]
    return inputs, {"y": refs["y"][:, :, np.array(pos)]}, scales, {"ref_positions": pos}


def _mamba2_slice(inputs, refs, scales):
    """Keep the first and the last chunk (chunks are independent: y of chunk c reads only chunk c's
    rows of x/dt/B/C, cs[:, :, c] and states[:, c]) and a few output rows of each."""
    cs = inputs["dA_cumsum"]
    nc, chunk = cs.shape[2], cs.shape[3]
    keep = [0, nc - 1]
    rows = np.concatenate([np.arange(c * chunk, (c + 1) * chunk) for c in keep])
    i2 = dict(inputs)
    for k in ("x", "dt", "Bmat", "Cmat"):
        i2[k] = inputs[k][:, rows]
    i2["dA_cumsum"] = cs[:, :, keep]
    i2["states"] = inputs["states"][:, keep]
    local = [0, 1, 2, chunk // 2 - 1, chunk - 1, chunk, chunk + 1, 2 * chunk - 2, 2 * chunk - 1]
    y = refs["y"][:, rows][:, np.array(local)]
    return i2, {"y": y}, scales, {"chunks": keep, "ref_rows": local}


def _nonfinite_storage(bits: np.ndarray, dtype: str) -> np.ndarray:
    """Inf/NaN mask of storage values: the 16-bit formats by their all-ones exponent field
    (fp16 0x7C00, bf16 0x7F80), other arrays by value."""
    bits = np.asarray(bits)
    if bits.dtype == np.uint16:
        mask = 0x7C00 if dtype == "fp16" else 0x7F80
        return (bits & mask) == mask
    return ~np.isfinite(bits)


def _eltwise_slice(inputs, refs, scales, dtype, extra=1024):
    """Keep the first ``extra`` elements, the last one and every element where an input is
    non-finite (the ``ieee`` case's planted specials); element-wise outputs at those indices
    depend only on the inputs there.  Per-element scales are sliced alike."""
    n = next(iter(inputs.values())).size
    keep = set(range(min(extra, n))) | {n - 1}
    for v in inputs.values():
        keep |= set(np.flatnonzero(_nonfinite_storage(np.asarray(v).reshape(-1), dtype)).tolist())
    keep = np.array(sorted(keep), dtype=np.int64)
    i2 = {k: np.asarray(v).reshape(-1)[keep] for k, v in inputs.items()}
    r2 = {k: np.asarray(v).reshape(-1)[keep] for k, v in refs.items()}
    s2 = {k: (np.asarray(v).reshape(-1)[keep] if np.ndim(v) else v) for k, v in scales.items()}
    return i2, r2, s2, {"flat_indices": keep.tolist()}


def _rows_with_specials(a2d, dtype):
    bad = _nonfinite_storage(a2d, dtype).any(axis=1)
    rows = {r % a2d.shape[0] for r in ROWS} | set(np.flatnonzero(bad).tolist())
    return np.array(sorted(rows), dtype=np.int64)


def _gemv_slice(inputs, refs, scales, dtype):
    """Rows of A (the usual few plus every row holding a special) and the matching y; x whole."""
    rows = _rows_with_specials(inputs["A"], dtype)
    i2 = dict(inputs)
    i2["A"] = inputs["A"][rows]
    return i2, {"y": refs["y"][rows]}, scales, {"rows": rows.tolist()}


def _gemm_silu_slice(inputs, refs, scales, dtype):
    """Rows of A and columns of B (the usual few plus every row/column holding a special)."""
    rows = _rows_with_specials(inputs["A"], dtype)
    b = inputs["B"]
    bad_cols = np.flatnonzero(_nonfinite_storage(b, dtype).any(axis=0))
    cols = np.array(sorted(set(range(32)) | {b.shape[1] - 1} | set(bad_cols.tolist())), dtype=np.int64)
    i2 = {"A": inputs["A"][rows], "B": b[:, cols]}
    return i2, {"C": refs["C"][rows][:, cols]}, scales, {"rows": rows.tolist(), "cols": cols.tolist()}


def write(doc: dict, name: str) -> Path:
    arrays = {}
    meta = {k: v for k, v in doc.items() if k != "records"}
    meta["records"] = []
    for i, rec in enumerate(doc["records"]):
        m = {"case": rec["case"], "seed": rec["seed"], "slice": rec["slice"], "full_shapes": rec["full_shapes"], "inputs": {}, "refs": [], "scales": []}
        for k, v in rec["inputs"].items():
            arrays[f"{i}/in/{k}"] = np.asarray(v)
            m["inputs"][k] = str(np.asarray(v).dtype)
        for k, v in rec["refs"].items():
            arrays[f"{i}/ref/{k}"] = np.asarray(v, dtype=np.float64)
            m["refs"].append(k)
        for k, v in rec["scales"].items():
            arrays[f"{i}/scale/{k}"] = np.asarray(v, dtype=np.float64)
            m["scales"].append(k)
        meta["records"].append(m)
    arrays["meta"] = np.frombuffer(json.dumps(meta, sort_keys=True).encode(), dtype=np.uint8)
    path = HERE / f"{name}.npz"
    np.savez_compressed(path, **arrays)
    return path


def sem_int_program(task: str) -> dict:
    """The task's int32 program document (the ``_PROGRAM`` JSON of tasks/<t>/reference.py)."""
    import re

    text = (REF / "tasks" / task / "reference.py").read_text(encoding="utf-8")
    m = re.search(r"_PROGRAM = json\.loads\(r'''(.*?)'''\)", text, re.S)
    return json.loads(m.group(1))


NEW_TASKS = {
    "relu": _eltwise_slice,
    "sigmoid": _eltwise_slice,
    "sigmoid_shift": _eltwise_slice,
    "lion": _eltwise_slice,
    "gemv": _gemv_slice,
    "gemm_silu": _gemm_silu_slice,
}


def _new_task(task: str, dtype: str) -> Path:
    slicer = functools.partial(NEW_TASKS[task], dtype=dtype)
    return write(from_reference(task, dtype, "small", slicer), f"ref_{task}_{dtype}")


KDA_FIXED_SIZES = ("single", "small", "tail")


def _kda_fixed(dtype: str) -> list[Path]:
    """tasks/kda at its three golden sizes (D = 8; the paper size is covered by the oracle)."""
    return [write(from_reference("kda", dtype, size), f"ref_kda_{size}_{dtype}") for size in KDA_FIXED_SIZES]


def main(only=()) -> None:
    if not REF.is_dir():
        raise SystemExit(f"reference checkout not found at {REF}")
    outs = []
    if only:
        for task in only:
            for dtype in ("fp16", "bf16"):
                if task == "kda":
                    outs.extend(_kda_fixed(dtype))
                elif task == "varlen_kda_capacity":
                    outs.append(write(from_reference("varlen_kda", dtype, "capacity"), f"ref_varlen_kda_capacity_{dtype}"))
                else:
                    outs.append(_new_task(task, dtype))
        for p in outs:
            print(f"{p.name:40s} {p.stat().st_size:8d} B")
        return
    for task in ("sem_int_1", "sem_int_2", "sem_int_3", "sem_int_4", "sem_int_5", "sem_int_7"):
        doc = from_reference(task, "i32", "small")
        doc["program"] = sem_int_program(task)
        doc["attrs"] = {"SCALAR_K": 12345}
        outs.append(write(doc, f"ref_{task}_i32"))
    for task in G0_TASKS:
        for dtype in ("fp16", "bf16"):
            outs.append(write(from_g0(task, dtype), f"g0_{task}_{dtype}"))
    for dtype in ("fp16", "bf16"):
        outs.append(write(from_reference("bitdelta_gemm", dtype, "small", _bitdelta_slice), f"ref_bitdelta_gemm_{dtype}"))
        outs.append(write(from_reference("flash_attention", dtype, "small", _fa_slice), f"ref_flash_attention_{dtype}"))
        outs.append(write(from_reference("rope", dtype, "small", _rope_slice), f"ref_rope_{dtype}"))
        outs.append(write(from_reference("mamba2_chunk_scan", dtype, "small", _mamba2_slice), f"ref_mamba2_chunk_scan_{dtype}"))
        for size in ("mixed", "fixed", "uniform", "capacity"):
            outs.append(write(from_reference("varlen_kda", dtype, size), f"ref_varlen_kda_{size}_{dtype}"))
        for task in NEW_TASKS:
            outs.append(_new_task(task, dtype))
        outs.extend(_kda_fixed(dtype))
    total = 0
    for p in outs:
        total += p.stat().st_size
        print(f"{p.name:40s} {p.stat().st_size:8d} B")
    print(f"total {total} B")


if __name__ == "__main__":
    main(tuple(sys.argv[1:]))
