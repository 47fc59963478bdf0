"""Generate the golden vectors under tests/golden/ (run where the reference tree exists).

    python tests/golden/gen_golden.py --reference <path of the reference checkout>

For every case of the reference's own test suite (tests/test_ops.py) this
records the input recipe (rebuilt by tests/scan_cases.py), a sha256 of the
inputs, and two float32 outputs (all rows, or a seeded sample of rows for the
larger cases):

* out_torch32 — the reference's test oracle, reference_selective_scan
                (tests/test_ops.py:17-63), in float32: the comparison the
                reference's tests make;
* out_cpp     — the reference's own C++ plugin (src/native/cpp/
                selective_scan.cc), compiled unmodified (oracle/Makefile) and
                run through its ORT entry points (oracle/ref_host.cc).

manifest.json records, per case, how far each of these and the float64
oracle restatement sit from the same torch function run in float64.

reference_selective_scan is taken from the reference test file by parsing it
(the file itself cannot be imported here: it imports onnx and onnxruntime,
which are not installed), and executed with torch in scope.

It also records the 1x1536x512 benchmark configuration (all four ops, config
distributions, seed 0) for 16 sampled rows.
"""
from __future__ import annotations

import argparse
import ast
import json
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))
sys.path.insert(0, str(REPO / "tests"))

from oracle import oracle  # noqa: E402
import scan_cases as sc  # noqa: E402


def load_reference_fn(reference: Path):
    src = (reference / "tests" / "test_ops.py").read_text()
    tree = ast.parse(src)
    fns = [n for n in tree.body if isinstance(n, ast.FunctionDef)
           and n.name == "reference_selective_scan"]
    ns = {"torch": torch, "F": F}
    exec(compile(ast.Module(body=fns, type_ignores=[]), "test_ops.py", "exec"), ns)
    return ns["reference_selective_scan"]


def run_torch(ref_fn, inputs, fused, exact, dtype):
    u, delta, A, B, C, D, z = [torch.from_numpy(np.asarray(x)).to(dtype) if x is not None else None
                               for x in inputs[:7]]
    with torch.no_grad():
        return ref_fn(u, delta, A, B, C, D, z, fused, exact).numpy()


def save_case(name, op, recipe, inputs, ref_fn, tol, manifest, rows=None):
    """Record one case: recipe + input hash + float32 outputs (all rows or a sample)."""
    fused, exact = sc_flags(op)
    u, delta, A, B, C, D, z = inputs[:7]
    t32 = run_torch(ref_fn, inputs, fused, exact, torch.float32)
    t64 = run_torch(ref_fn, inputs, fused, exact, torch.float64)
    cpp = oracle.ref_run(op, u, delta, A, B, C, D, z, n_threads=4)
    f64 = oracle.scan_f64(op, u, delta, A, B, C, D, z)
    flat = (lambda a: a.reshape(-1, a.shape[-1])[rows]) if rows is not None else (lambda a: a)
    payload = {
        "op": np.array(op), "recipe": np.array(json.dumps(recipe)),
        "shape": np.array(u.shape), "input_sha256": np.array(sc.sha256_arrays(inputs[:7])),
        "out_torch32": flat(t32).astype(np.float32), "out_cpp": flat(cpp).astype(np.float32),
    }
    if rows is not None:
        payload["rows"] = rows
    np.savez_compressed(HERE / f"{name}.npz", **payload)
    scale = max(1.0, float(np.max(np.abs(t64))))
    manifest[name] = {
        "op": op, "shape": list(u.shape), "recipe": recipe, "tol": tol,
        "rows_stored": "all" if rows is None else int(len(rows)),
        "maxabs_cpp_vs_torch64": float(np.max(np.abs(cpp - t64))),
        "maxabs_torch32_vs_torch64": float(np.max(np.abs(t32 - t64))),
        "maxabs_oracle_f64_vs_torch64": float(np.max(np.abs(f64 - t64))),
        "max_abs_output": scale,
        "cpp_allclose_torch32_at_tol": bool(np.allclose(cpp, t32, rtol=tol, atol=tol)),
    }
    print(f"{name:32s} {op:24s} cpp-t64 {manifest[name]['maxabs_cpp_vs_torch64']:.2e} "
          f"f64oracle-t64 {manifest[name]['maxabs_oracle_f64_vs_torch64']:.2e}")


def sc_flags(op):
    return oracle.OPS[op][1], oracle.OPS[op][2]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True,
                    help="root of the acmiyaguchi/mamba-onnx checkout whose tests/test_ops.py "
                         "and compiled plugin (oracle/_ref) produce the vectors")
    args = ap.parse_args()
    ref_fn = load_reference_fn(Path(args.reference))
    manifest = {}
    for old in HERE.glob("*.npz"):
        old.unlink()
    # tests/test_ops.py:156-171 — every op at B=1, D=64, L=32, seed 42, tol 1e-4
    for op, fused, exact in sc.ALL_OPS:
        r = {"kind": "reference_test", "B": 1, "D": 64, "L": 32, "fused": fused, "seed": 42}
        save_case(f"core_{op}", op, r, recipe_inputs(r), ref_fn, 1e-4, manifest)
    # tests/test_ops.py:178-203 — SelectiveScan shapes, seed 42, tol 1e-4
    for (B, D, L), sid in zip(sc.REFERENCE_SHAPES, sc.REFERENCE_SHAPE_IDS):
        r = {"kind": "reference_test", "B": B, "D": D, "L": L, "fused": False, "seed": 42}
        rows = None
        if B * D > 256:
            rows = np.sort(np.random.default_rng(7).choice(B * D, 96, replace=False))
        save_case(f"shape_{sid}", "SelectiveScan", r, recipe_inputs(r), ref_fn, 1e-4, manifest,
                  rows=rows)
    # tests/test_ops.py:210-248 — edge regimes, SelectiveScan, seed 99, tol 1e-3
    for regime in sc.EDGE_REGIMES:
        r = {"kind": "edge", "regime": regime}
        save_case(f"edge_{regime}", "SelectiveScan", r, recipe_inputs(r), ref_fn, 1e-3, manifest)
    # tests/test_ops.py:251-273 — SelectiveScanExact, A=-5, seed 99, tol 1e-3
    r = {"kind": "edge_exact"}
    save_case("edge_exact", "SelectiveScanExact", r, recipe_inputs(r), ref_fn, 1e-3, manifest)
    # tests/test_ops.py:280-294 — cross-backend shape B=2, D=128, L=64, seed 42
    for op, fused, exact in sc.ALL_OPS:
        r = {"kind": "reference_test", "B": 2, "D": 128, "L": 64, "fused": fused, "seed": 42}
        rows = np.sort(np.random.default_rng(8).choice(256, 64, replace=False))
        save_case(f"cross_{op}", op, r, recipe_inputs(r), ref_fn, 1e-4, manifest, rows=rows)
    # 1x1536x512 configuration, seed 0, 16 sampled rows
    rows = np.sort(np.random.default_rng(1234).choice(1536, size=16, replace=False))
    for op, fused, exact in sc.ALL_OPS:
        r = {"kind": "config", "B": 1, "D": 1536, "L": 512, "fused": fused, "seed": 0}
        save_case(f"cfg0_{op}", op, r, recipe_inputs(r), ref_fn, 1e-3, manifest, rows=rows)
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")


def recipe_inputs(r):
    return sc.recipe_inputs(r)


if __name__ == "__main__":
    main()
