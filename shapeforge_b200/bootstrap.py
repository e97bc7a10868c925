"""Install the B200 backend into a ShapeForge checkout without editing it.

The reference resolves backends and targets from roots fixed to its own file location
(tcenv/backends/registry.py:16-17 ``BACKENDS``, tcenv/target.py:13-15 ``TARGETS``/``BACKENDS``), and
``load_backend`` only accepts entry points under ``tcenv.backends.`` (registry.py:57-62).  This
module, called once at start-up of a harness process:

* registers ``tcenv.backends.cuda_sm100`` / ``tcenv.backends.cuda_sm100.backend`` as aliases of
  :mod:`shapeforge_b200` / :mod:`shapeforge_b200.backend`, so the entry point in
  ``backends/cuda-sm100/backend.toml`` imports;
* rebinds the backend and target roots to this repository's ``backends/`` and ``targets/``
  (which hold ``cuda-sm100`` and ``b200``) and clears the registry's cache.

A maintainer who vendors the backend instead copies the two directories into the checkout and
adds ``tcenv/backends/cuda_sm100/__init__.py`` re-exporting this package; no rebinding is needed.
"""

from __future__ import annotations

import sys
import types
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def install(backends_root: Path | None = None, targets_root: Path | None = None) -> None:
    """Make ``load_backend("cuda-sm100")`` and ``load_target("b200")`` resolve to this backend."""
    import tcenv.backends.registry as registry  # the reference's own modules
    import tcenv.target as target

    from . import backend as backend_mod

    pkg_name = "tcenv.backends.cuda_sm100"
    if pkg_name not in sys.modules:
        pkg = types.ModuleType(pkg_name)
        pkg.__path__ = []  # a namespace for the alias below
        sys.modules[pkg_name] = pkg
    sys.modules[pkg_name + ".backend"] = backend_mod
    backends_root = Path(backends_root or ROOT / "backends")
    targets_root = Path(targets_root or ROOT / "targets")
    registry.BACKENDS = backends_root
    target.BACKENDS = backends_root
    target.TARGETS = targets_root
    registry.load_backend.cache_clear()
