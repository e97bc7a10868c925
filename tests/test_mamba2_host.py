"""mamba2_chunk_scan on the CPU: the seeded case stream and properties of the oracle.

The stream of ``shapeforge_b200.cases.mamba2_inputs`` must reproduce the reference module's own
inputs bit for bit (the fixture holds the first and the last chunk of each case), and the oracle
must have the structure of the formula: chunks independent, linear in (x, states), the state term
vanishing with zero states, and a non-finite x element poisoning exactly its own chunk.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import oracle
from oracle import ops
from shapeforge_b200 import cases
from tests import golden

SMALL = dict(batch=1, seq=256, heads=2, headdim=64, dstate=64, chunk=64)
NAMES = ("x", "dt", "dA_cumsum", "Bmat", "Cmat", "Dskip", "states")


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
def test_case_stream_matches_reference_inputs(dtype):
    doc = golden.load(f"ref_mamba2_chunk_scan_{dtype}")
    assert [r["case"] for r in doc["records"]] == list(cases.MAMBA2_CASES)
    for ci, rec in enumerate(doc["records"]):
        assert rec["seed"] == cases.case_seed(0, ci)
        inp = cases.mamba2_inputs(rec["case"], rec["seed"], dtype=dtype, **SMALL)
        keep = rec["slice"]["chunks"]
        rows = np.concatenate([np.arange(c * 64, (c + 1) * 64) for c in keep])
        mine = {
            "x": inp["x"][:, rows], "dt": inp["dt"][:, rows], "Bmat": inp["Bmat"][:, rows], "Cmat": inp["Cmat"][:, rows],
            "dA_cumsum": inp["dA_cumsum"][:, :, keep], "states": inp["states"][:, keep], "Dskip": inp["Dskip"],
        }
        for n in NAMES:
            want = np.asarray(rec["inputs"][n]).view(np.uint16)
            assert np.array_equal(_bits(mine[n]), want), (rec["case"], n)


def _f64(inp):
    return [inp[n].to(torch.float64).numpy() for n in NAMES]


def test_chunks_are_independent_and_linear():
    inp = cases.mamba2_inputs("normal", 5, 2, 192, 3, 16, 8, 64, "fp16")
    a = _f64(inp)
    y = ops.mamba2_chunk_scan(*a)
    # Chunk 1 alone (as a one-chunk problem) gives the same rows.
    sl = slice(64, 128)
    one = [a[0][:, sl], a[1][:, sl], a[2][:, :, 1:2], a[3][:, sl], a[4][:, sl], a[5], a[6][:, 1:2]]
    np.testing.assert_allclose(ops.mamba2_chunk_scan(*one), y[:, sl], rtol=1e-12, atol=1e-12)
    # Linear in (x, states) jointly.
    b2 = list(a)
    b2[0], b2[6] = 2.5 * a[0], 2.5 * a[6]
    np.testing.assert_allclose(ops.mamba2_chunk_scan(*b2), 2.5 * y, rtol=1e-12, atol=1e-12)
    # Zero states: only the intra-chunk and skip terms remain; zero x as well: y == 0.
    z = list(a)
    z[6] = np.zeros_like(a[6])
    z[0] = np.zeros_like(a[0])
    assert not np.any(ops.mamba2_chunk_scan(*z))


def test_nonfinite_x_poisons_its_own_chunk_only():
    inp = cases.mamba2_inputs("normal", 9, 1, 192, 2, 8, 8, 64, "bf16")
    a = _f64(inp)
    a[0] = a[0].copy()
    a[0][0, 64 + 40, 1, 3] = np.inf  # chunk 1, head 1, column 3
    y = ops.mamba2_chunk_scan(*a)
    bad = ~np.isfinite(y)
    assert bad[0, 64:128, 1, 3].all()          # every row of the chunk (masked zeros still multiply inf)
    assert not bad[0, :64].any() and not bad[0, 128:].any()
    assert not bad[0, :, 0].any()
    assert bad.sum() == 64


def test_oracle_rejects_bad_chunking():
    inp = cases.mamba2_inputs("normal", 1, 1, 128, 1, 8, 8, 64, "fp16")
    a = _f64(inp)
    a[2] = a[2][:, :, :1]  # NC * CHUNK != SEQLEN
    with pytest.raises(ValueError):
        ops.mamba2_chunk_scan(*a)
