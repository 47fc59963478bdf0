"""Loader for the committed golden vectors (tests/golden/*.npz)."""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np

import scan_cases as sc

GOLDEN = Path(__file__).resolve().parent / "golden"


@dataclass
class GoldenCase:
    name: str
    op: str
    recipe: dict
    shape: tuple
    input_sha256: str
    out_torch32: np.ndarray
    out_cpp: np.ndarray
    rows: np.ndarray | None
    tol: float

    def inputs(self):
        return sc.recipe_inputs(self.recipe)

    def select(self, full):
        """Rows of a full [B, D, L] output that this fixture stores."""
        if self.rows is None:
            return full
        return full.reshape(-1, full.shape[-1])[self.rows]


def manifest():
    return json.loads((GOLDEN / "manifest.json").read_text())


def load(name: str) -> GoldenCase:
    z = np.load(GOLDEN / f"{name}.npz")
    m = manifest()[name]
    return GoldenCase(name=name, op=str(z["op"]), recipe=json.loads(str(z["recipe"])),
                      shape=tuple(int(x) for x in z["shape"]),
                      input_sha256=str(z["input_sha256"]), out_torch32=z["out_torch32"],
                      out_cpp=z["out_cpp"], rows=z["rows"] if "rows" in z.files else None,
                      tol=float(m["tol"]))


def names():
    return sorted(manifest().keys())
