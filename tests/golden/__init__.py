"""Golden fixtures (reference-generated) and their loader."""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def available() -> list[str]:
    return sorted(p.stem for p in HERE.glob("*.npz"))


def load(name: str) -> dict:
    """Load ``tests/golden/<name>.npz`` into ``{meta..., records: [{case, seed, inputs, refs, scales}]}``."""
    z = np.load(HERE / f"{name}.npz")
    meta = json.loads(bytes(z["meta"]).decode())
    for i, rec in enumerate(meta["records"]):
        rec["inputs"] = {k: z[f"{i}/in/{k}"] for k in rec["inputs"]}
        rec["refs"] = {k: z[f"{i}/ref/{k}"] for k in rec["refs"]}
        rec["scales"] = {k: z[f"{i}/scale/{k}"] for k in rec["scales"]}
    return meta
