"""ORACLE — CPU checker for the selective-scan CUDA path (test infrastructure).

Nothing in the product imports this module. Only tests/, the smoke check in
__graft_entry__.py and bench.py's CPU-baseline / reference legs load it, and
only as the checker (or, for the reference leg, to time the reference's own
CPU implementation).

Three CPU implementations are exposed:

* scan_f64      — float64 ground truth, a C restatement of the reference
                  algorithm (scan_oracle.c; reference tests/test_ops.py:17-63
                  and src/native/cpp/selective_scan.cc:232-305).
* scan_f32ref   — float32 restatement of the reference C++ numerics
                  (fast_exp, fast_softplus, fast_silu, update order,
                  horizontal-sum order; selective_scan.cc:33-148, 244-305).
* ref_run       — the reference's own C++ plugin, compiled unmodified
                  (oracle/_ref/libref_scan.so, see oracle/Makefile) and driven
                  through its ORT custom-op entry points by ref_host.cc.

The restatements are pinned against the committed golden vectors
(tests/golden/), which hold outputs of the reference's torch oracle and of the
compiled reference plugin on the reference test suite's own inputs.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

ORACLE_DIR = Path(__file__).resolve().parent
_LIB_PATH = ORACLE_DIR / "_build" / "liboracle_scan.so"
_REF_PATH = ORACLE_DIR / "_ref" / "libref_scan.so"

# Op name -> (variant id, fused, exact); ids match scan_oracle.c and the C-ABI.
OPS = {
    "SelectiveScan": (0, False, False),
    "SelectiveScanExact": (1, False, True),
    "SelectiveScanFused": (2, True, False),
    "SelectiveScanFusedExact": (3, True, True),
}

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)

_lib = None
_ref = None


def build() -> None:
    """Compile the restatement (and the reference plugin where its source exists)."""
    subprocess.run(["make", "-s", "-C", str(ORACLE_DIR)], check=True)


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        lib.oracle_scan_f64.restype = ctypes.c_int
        lib.oracle_scan_f64.argtypes = [ctypes.c_int] + [_f32p] * 8 + [_f64p, _f64p, _f64p] + \
            [ctypes.c_int64] * 4 + [_i64p, ctypes.c_int64]
        lib.oracle_scan_f32ref.restype = ctypes.c_int
        lib.oracle_scan_f32ref.argtypes = [ctypes.c_int] + [_f32p] * 8 + [ctypes.c_int64] * 4
        lib.oracle_ref_fast_exp.restype = None
        lib.oracle_ref_fast_exp.argtypes = [_f32p, _f32p, ctypes.c_int64]
        _lib = lib
    return _lib


def ref_available() -> bool:
    return _REF_PATH.exists()


def _load_ref():
    global _ref
    if _ref is None:
        if not _REF_PATH.exists():
            raise FileNotFoundError(f"{_REF_PATH} is not built (needs the reference source tree)")
        lib = ctypes.CDLL(str(_REF_PATH))
        lib.ref_scan_run.restype = ctypes.c_int
        lib.ref_scan_run.argtypes = [ctypes.c_char_p] + [_f32p] * 8 + [ctypes.c_int64] * 4 + \
            [ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        lib.ref_scan_op_count.restype = ctypes.c_int
        lib.ref_scan_op_name.restype = ctypes.c_char_p
        lib.ref_scan_op_name.argtypes = [ctypes.c_int]
        _ref = lib
    return _ref


def _f32(a):
    if a is None:
        return None
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a


def _p32(a):
    return a.ctypes.data_as(_f32p) if a is not None else None


def scan_f64(op: str, u, delta, A, B, C, D, z=None, delta_bias=None, h0=None, rows=None,
             return_state: bool = False):
    """Float64 ground truth. Shapes: u/delta/z [B,D,L], A [D,N], B/C [B,L,N], D [D].

    rows: optional 1-D array of row indices b*D+d; the output is then
    [len(rows), L] instead of [B, D, L]. h0: optional [B*D, N] float64 initial
    state. return_state: also return the final state ([rows or B*D, N]).
    """
    variant = OPS[op][0]
    u, delta, A, B, C, D, z, delta_bias = map(_f32, (u, delta, A, B, C, D, z, delta_bias))
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    if rows is not None:
        rows = np.ascontiguousarray(rows, dtype=np.int64)
        n_rows = rows.shape[0]
    else:
        n_rows = batch * dim
    out = np.empty((n_rows, seqlen), dtype=np.float64)
    hl = np.empty((n_rows, dstate), dtype=np.float64) if return_state else None
    h0a = np.ascontiguousarray(h0, dtype=np.float64) if h0 is not None else None
    rc = _load().oracle_scan_f64(
        variant, _p32(u), _p32(delta), _p32(A), _p32(B), _p32(C), _p32(D), _p32(z),
        _p32(delta_bias),
        h0a.ctypes.data_as(_f64p) if h0a is not None else None,
        out.ctypes.data_as(_f64p),
        hl.ctypes.data_as(_f64p) if hl is not None else None,
        batch, dim, seqlen, dstate,
        rows.ctypes.data_as(_i64p) if rows is not None else None, n_rows)
    if rc != 0:
        raise ValueError(f"oracle_scan_f64 failed ({rc})")
    if rows is None:
        out = out.reshape(batch, dim, seqlen)
    return (out, hl) if return_state else out


def scan_f32ref(op: str, u, delta, A, B, C, D, z=None):
    """Float32 restatement of the reference C++ numerics (dstate must be 16)."""
    variant = OPS[op][0]
    u, delta, A, B, C, D, z = map(_f32, (u, delta, A, B, C, D, z))
    batch, dim, seqlen = u.shape
    out = np.empty((batch, dim, seqlen), dtype=np.float32)
    rc = _load().oracle_scan_f32ref(variant, _p32(u), _p32(delta), _p32(A), _p32(B), _p32(C),
                                    _p32(D), _p32(z), _p32(out), batch, dim, seqlen, A.shape[1])
    if rc != 0:
        raise ValueError(f"oracle_scan_f32ref failed ({rc})")
    return out


def ref_fast_exp(x):
    x = _f32(x)
    y = np.empty_like(x)
    _load().oracle_ref_fast_exp(_p32(x), _p32(y), x.size)
    return y


def ref_run(op: str, u, delta, A, B, C, D, z=None, n_threads: int = 0, out=None):
    """Run the reference's own compiled C++ plugin (CPU, OpenMP) on host arrays."""
    lib = _load_ref()
    u, delta, A, B, C, D, z = map(_f32, (u, delta, A, B, C, D, z))
    batch, dim, seqlen = u.shape
    if out is None:
        out = np.empty((batch, dim, seqlen), dtype=np.float32)
    err = ctypes.create_string_buffer(512)
    rc = lib.ref_scan_run(op.encode(), _p32(u), _p32(delta), _p32(A), _p32(B), _p32(C), _p32(D),
                          _p32(z), _p32(out), batch, dim, seqlen, A.shape[1], int(n_threads),
                          err, len(err))
    if rc != 0:
        raise RuntimeError(f"reference plugin failed ({rc}): {err.value.decode()}")
    return out


def ref_op_names():
    lib = _load_ref()
    return [lib.ref_scan_op_name(i).decode() for i in range(lib.ref_scan_op_count())]


def host_threads() -> int:
    """Threads the reference's OpenMP pool may use on this host."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1
