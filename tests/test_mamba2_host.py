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


def _sequential(x, dt, cs, bm, cm, d, st):
    """The SSM recurrence token by token: per chunk the state starts at states[b, c], each token
    decays it by exp(cs_t - cs_{t-1}) (cs_{-1} = 0), adds dt_t x_t B_t^T, and emits C_t . h + D x_t."""
    bsz, seq, heads, hd = x.shape
    nc, chunk = cs.shape[2], cs.shape[3]
    y = np.zeros((bsz, seq, heads, hd))
    for b in range(bsz):
        for c in range(nc):
            hs = st[b, c].copy()                         # [H, P, N]
            prev = np.zeros(heads)
            for l in range(chunk):
                t = c * chunk + l
                cur = cs[b, :, c, l]
                hs = np.exp(cur - prev)[:, None, None] * hs + dt[b, t][:, None, None] * x[b, t][:, :, None] * bm[b, t][None, None, :]
                y[b, t] = hs @ cm[b, t] + d[:, None] * x[b, t]
                prev = cur
    return y


@pytest.mark.parametrize("case", ["normal", "wide_range", "large", "outlier"])
def test_oracle_equals_the_sequential_state_recurrence(case):
    """The chunked form (intra-chunk C.B^T with decay mask + carried-in states) is the same
    operator as the token-by-token recurrence (the reference's own check, on the small size)."""
    inp = cases.mamba2_inputs(case, 21, dtype="fp16", **SMALL)
    a = _f64(inp)
    y = ops.mamba2_chunk_scan(*a)
    seq = _sequential(*a)
    np.testing.assert_allclose(seq, y, rtol=1e-9, atol=1e-9 * float(np.abs(y).max()))


def test_paper_flops_count_the_shared_bc_product_once():
    """Work accounting of the paper size: C.B^T once per (batch, chunk), W.x and C.states^T per head."""
    batch, seq, heads, headdim, dstate, chunk = 2, 2048, 8, 64, 64, 64
    chunks = seq // chunk
    shared = batch * chunks * (2 * chunk * chunk * dstate)
    per_head = batch * heads * chunks * (2 * chunk * chunk * headdim + 2 * chunk * headdim * dstate)
    assert shared + per_head == 570_425_344


@pytest.mark.parametrize("dtype", ["fp16", "bf16"])
@pytest.mark.parametrize("case", list(cases.MAMBA2_CASES))
def test_inputs_keep_the_ssm_invariants(dtype, case):
    """dt in [0.001, 0.05], dA_cumsum finite, non-increasing and <= 0 inside every chunk (every
    decay <= 1, and exp(cs) never flushes to zero); the ieee case puts specials only in states."""
    inp = cases.mamba2_inputs(case, 5, dtype=dtype, **SMALL)
    dt, cs = inp["dt"].double(), inp["dA_cumsum"].double()
    assert bool((dt > 0).all()) and float(dt.min()) >= 0.001 * 0.99 and float(dt.max()) <= 0.05 * 1.01
    assert bool(torch.isfinite(cs).all()) and bool((cs[..., 1:] <= cs[..., :-1]).all()) and bool((cs <= 0).all())
    assert float(cs.min()) > -8.0 * 0.05 * 64 * 1.01
    others = [inp[n] for n in NAMES if n != "states"]
    assert all(bool(torch.isfinite(t).all()) for t in others)
    assert bool(torch.isfinite(inp["states"]).all()) == (case != "ieee")
