"""The C-ABI library loads and exports every symbol ``include/sfcuda.h`` declares (no GPU needed)."""

from __future__ import annotations

import re
from pathlib import Path

import pytest

from shapeforge_b200 import _native

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols() -> set[str]:
    names = set()
    for header in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", header.read_text(), flags=re.S)
        names |= set(re.findall(r"SF_API\s+[\w\s\*]+?\b(sf_\w+)\s*\(", text))
    return names


def test_header_declares_entry_points():
    names = declared_symbols()
    assert {"sf_rmsnorm", "sf_run_op", "sf_run_batch", "sf_device_info_get"} <= names


def test_library_exports_every_declared_symbol():
    lib = _native.load()
    missing = [n for n in sorted(declared_symbols()) if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert declared_symbols() == set(_native.SIGNATURES)


def test_version_string():
    assert _native.version().endswith("sm_100a")


def test_op_table_matches_library():
    lib = _native.load()
    for name, op in _native.OPS.items():
        assert lib.sf_op_nargs(op) > 0, name
    assert lib.sf_op_nargs(9999) == 0


def test_invalid_arguments_are_rejected_without_a_device():
    """Argument validation happens before any CUDA call: status 2 and a message."""
    with pytest.raises(_native.SfError) as exc:
        _native.call("sf_rmsnorm", None, None, None, 4, 0, 1e-6, 0, None)
    assert exc.value.code == _native.SF_EINVAL
    assert "hidden" in exc.value.message
    with pytest.raises(_native.SfError) as exc:
        _native.call("sf_rmsnorm", 16, 16, 16, 4, 8, 1e-6, 7, None)
    assert exc.value.code == _native.SF_EINVAL
    d = _native.op_desc("rmsnorm", "fp16", dims=(4, 8), attrs=(1e-6,))
    with pytest.raises(_native.SfError) as exc:
        _native.run_op(d, [16, 16], 0)
    assert exc.value.code == _native.SF_EINVAL


def test_lion_attribute_domains_are_enforced_without_a_device():
    """tasks/lion/opspec.json attrs: LR > 0, WD >= 0, 0 < BETA1 < 1, 0 < BETA2 < 1; anything else is
    status 2 before any CUDA call (pointers are never touched)."""
    good = dict(lr=1e-3, wd=0.1, b1=0.9, b2=0.99)
    for bad in (dict(lr=0.0), dict(lr=-1.0), dict(wd=-0.1), dict(b1=0.0), dict(b1=1.0), dict(b2=1.5), dict(lr=float("nan"))):
        a = dict(good, **bad)
        with pytest.raises(_native.SfError) as exc:
            _native.call("sf_lion", 16, 16, 16, 16, 16, 8, a["lr"], a["wd"], a["b1"], a["b2"], 0, None)
        assert exc.value.code == _native.SF_EINVAL, bad
        assert "lion" in exc.value.message


def test_missing_library_fails_loudly(tmp_path, monkeypatch):
    monkeypatch.setattr(_native, "LIB_PATH", tmp_path / "nope.so")
    monkeypatch.setattr(_native, "_lib", None)
    with pytest.raises(_native.NativeUnavailable):
        _native.load()


def test_kda_workspace_sizes_without_a_device():
    """The two-pass KDA workspace: a 1 KB-aligned header of nseq + 1 int32 chunk offsets, then one
    49,664-byte slot per (32-token chunk, head) bound, floor((T + 31 N) / 32) * H slots; the task op
    and the gated workload use the same layout; 0 when the shape does not qualify (D != 128)."""
    lib = _native.load()
    slot = 49664
    for t, n, h in ((8192, 6, 64), (16552, 8, 16), (1, 1, 1), (0, 3, 2), (1000, 1025, 4)):
        header = ((4 * (n + 1) + 1023) // 1024) * 1024
        want = header + ((t + 31 * n) // 32) * h * slot
        assert lib.sf_varlen_kda_workspace_bytes(t, n, h, 128) == want, (t, n, h)
        assert lib.sf_varlen_kda_gated_workspace_bytes(t, n, h, 128) == want, (t, n, h)
    for d in (64, 32, 256):
        assert lib.sf_varlen_kda_workspace_bytes(8192, 6, 64, d) == 0
    assert lib.sf_varlen_kda_workspace_bytes(8192, 0, 64, 128) == 0


def test_kda_op_takes_a_workspace_argument():
    """SF_OP_KDA carries the two-pass workspace as its 13th tensor argument (NULL: single pass)."""
    lib = _native.load()
    assert lib.sf_op_nargs(_native.OPS["varlen_kda"]) == 13
    assert lib.sf_op_nargs(_native.OPS["varlen_kda_gated"]) == 10


def _on(index: int):
    """Stand-in for a CUDA tensor on GPU ``index`` on a machine without a GPU: only ``is_cuda`` and
    ``device`` are read before an operator reaches the library."""
    import torch

    class FakeCuda(torch.Tensor):
        @property
        def is_cuda(self):
            return True

        @property
        def device(self):
            return self._fake_device

    t = torch.Tensor._make_subclass(FakeCuda, torch.zeros(4))
    t._fake_device = torch.device("cuda", index)
    return t


def test_operators_run_with_their_tensors_device_current(monkeypatch):
    import contextlib

    import torch

    from shapeforge_b200 import ops

    entered = []

    @contextlib.contextmanager
    def device(d):
        entered.append(d)
        yield

    monkeypatch.setattr(torch.cuda, "device", device)
    body = ops._tensor_device(lambda *a, **k: "ran")
    assert body(_on(1), w=_on(1), eps=1e-6) == "ran" and entered == [torch.device("cuda", 1)]
    assert body(torch.zeros(1), 3) == "ran" and len(entered) == 1  # CPU tensors: the operator's own check refuses them
    # Tensors on two GPUs are refused before anything reaches the library.
    for call in (lambda: ops.rmsnorm(_on(0), _on(1)), lambda: ops.gemm_nt(_on(0), _on(1)),
                 lambda: ops.flash_attention(_on(1), _on(1), _on(0), 0.125)):
        with pytest.raises(ValueError, match="more than one device"):
            call()
    assert len(entered) == 1
