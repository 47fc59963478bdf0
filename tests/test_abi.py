"""CPU: the built library, its C ABI, the ORT op table and the Python loader.

No kernel is launched here (there is no GPU in the build container); every
call below returns before the library touches CUDA.
"""
import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import mamba_onnx
from fake_ort import ort_shim
from mamba_onnx import cuda

ROOT = Path(__file__).resolve().parent.parent
HEADERS = sorted((ROOT / "include").glob("*.h"))


def declared_functions():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"^\s*#.*$", "", text, flags=re.M)
        text = re.sub(r"__attribute__\s*\(\(.*?\)\)", "", text)
        for m in re.finditer(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(([^;{}]*)\)\s*;", text):
            name = m.group(1)
            if name not in {"defined", "__attribute__", "visibility"}:
                names.add(name)
    return names


def test_headers_declare_the_boundary():
    names = declared_functions()
    assert {"RegisterCustomOps", "mamba_scan_launch", "mamba_scan_workspace_size",
            "mamba_scan_last_error", "mamba_scan_status_string",
            "mamba_scan_check_device_error", "mamba_scan_abi_version"} <= names


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(cuda.library_path()))
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_abi_version_and_status_strings():
    lib = cuda.library()
    assert lib.mamba_scan_abi_version() == 2
    assert lib.mamba_scan_status_string(2) == b"unsupported dstate"
    assert lib.mamba_scan_status_string(99) == b"unknown status"


def _args(**kw):
    a = cuda.ScanArgs()
    fake = 0x10000  # never dereferenced: these calls fail validation first
    for f in ("u", "delta", "A", "B", "C", "D", "z", "out"):
        setattr(a, f, fake * (1 + len(f)))
    a.batch, a.dim, a.seqlen, a.dstate = 1, 64, 32, 16
    for k, v in kw.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("kw,variant,status,msg", [
    (dict(dstate=8), 0, 2, "dstate=16"),
    (dict(), 7, 1, "variant"),
    (dict(seqlen=-1), 0, 1, "negative"),
    (dict(u=None), 1, 1, "non-NULL"),
    (dict(z=None), 2, 1, "need z"),
    (dict(), 0 | 0x200, 1, "exact variants only"),   # exp flag on a linear op
    (dict(), 2 | 0x100, 1, "exact variants only"),
    (dict(), 1 | 0x300, 1, "at most one"),            # two exp flags
    (dict(), 1 | 0x400, 1, "variant"),                # unknown flag
])
def test_launch_rejects_bad_arguments_before_any_cuda_call(kw, variant, status, msg):
    lib = cuda.library()
    rc = lib.mamba_scan_launch(variant, ctypes.byref(_args(**kw)), None, 0, None)
    assert rc == status
    assert msg in lib.mamba_scan_last_error().decode()


def test_launch_rejects_aliasing_output():
    lib = cuda.library()
    a = _args()
    a.out = a.u
    assert lib.mamba_scan_launch(0, ctypes.byref(a), None, 0, None) == 4


@pytest.mark.parametrize("field", ["u", "delta", "z", "B", "C", "A", "D", "out"])
def test_launch_rejects_workspace_overlapping_a_tensor(field):
    """The workspace is written while the inputs are read: no overlap allowed."""
    lib = cuda.library()
    a = _args()
    ws = getattr(a, field) + 8
    rc = lib.mamba_scan_launch(2, ctypes.byref(a), ws, 64, None)
    assert rc == 4
    assert "workspace overlaps" in lib.mamba_scan_last_error().decode()


def test_model_kernels_validate_before_launch():
    """include/mamba_model_ops.h entry points reject bad arguments without CUDA."""
    lib = cuda.library()
    fake = 0x10000
    # rmsnorm: cols must be positive; y must not overlap x
    assert lib.mamba_rmsnorm(fake, fake * 2, fake * 3, 4, 0, 1e-5, None) == 1
    assert lib.mamba_rmsnorm(fake, fake * 9, fake + 8, 4, 16, 1e-5, None) == 4
    assert "overlaps" in lib.mamba_scan_last_error().decode()
    assert lib.mamba_rmsnorm(fake, fake * 2, fake * 3, 0, 16, 1e-5, None) == 0  # no rows
    # conv: width 1..8, batch stride >= dim * seqlen, y disjoint from x
    assert lib.mamba_causal_conv1d_silu(fake, 64, fake * 2, None, fake * 3, 1, 4, 16, 9,
                                        None) == 1
    assert "width" in lib.mamba_scan_last_error().decode()
    assert lib.mamba_causal_conv1d_silu(fake, 63, fake * 2, None, fake * 3, 2, 4, 16, 4,
                                        None) == 1
    assert lib.mamba_causal_conv1d_silu(fake, 64, fake * 2, None, fake + 16, 1, 4, 16, 4,
                                        None) == 4
    assert lib.mamba_causal_conv1d_silu(fake, 64, fake * 2, None, fake * 3, 1, 0, 16, 4,
                                        None) == 0  # empty


def test_gemm_and_split_validate_before_launch():
    """mamba_split_tf32 / mamba_gemm_tf32x3 reject bad arguments without CUDA."""
    lib = cuda.library()
    f = 0x100000  # 16-byte aligned fake device addresses, 1 MiB apart
    # split: ld >= cols, ldx >= cols (rows when transposing), no NULLs; empty is a no-op
    assert lib.mamba_split_tf32(f, 4, 8, 8, 0, 2 * f, 3 * f, 7, None) == 1
    assert lib.mamba_split_tf32(f, 4, 8, 7, 0, 2 * f, 3 * f, 8, None) == 1
    assert lib.mamba_split_tf32(f, 4, 8, 3, 1, 2 * f, 3 * f, 8, None) == 1
    assert lib.mamba_split_tf32(None, 4, 8, 8, 0, 2 * f, 3 * f, 8, None) == 1
    assert lib.mamba_split_tf32(f, 0, 8, 8, 0, 2 * f, 3 * f, 8, None) == 0

    def gemm(a_hi=f, a_lo=2 * f, lda=16, b_hi=3 * f, b_lo=4 * f, ldb=16, c_in=None, c=5 * f,
             ldc_m=8, ldc_n=1, M=4, N=8, K=16):
        return lib.mamba_gemm_tf32x3(a_hi, a_lo, lda, b_hi, b_lo, ldb, c_in, c, ldc_m, ldc_n,
                                     M, N, K, None)

    assert gemm(K=0) == 1
    assert gemm(M=0) == 0 and gemm(N=0) == 0  # empty product
    assert gemm(lda=12) == 1 and gemm(ldb=18) == 1  # < K / not a multiple of 4
    assert gemm(b_lo=4 * f + 8) == 1 and b"aligned" in lib.mamba_scan_last_error()
    assert gemm(c=f + 64) == 4 and b"overlaps" in lib.mamba_scan_last_error()
    assert gemm(c_in=5 * f + 16) == 4  # partly overlapping C
    assert gemm(ldc_m=0) == 1


def test_rmsnorm_split_validates_before_launch():
    lib = cuda.library()
    f = 0x100000

    def call(x=f, w=2 * f, rows=4, cols=8, hi=3 * f, lo=4 * f, ld=8):
        return lib.mamba_rmsnorm_split_tf32(x, w, rows, cols, 1e-5, hi, lo, ld, None)

    assert call(rows=0) == 0
    assert call(cols=6, ld=8) == 1 and call(ld=4) == 1 and call(ld=10) == 1
    assert call(hi=3 * f + 4) == 1 and b"aligned" in lib.mamba_scan_last_error()
    assert call(lo=None) == 1
    assert call(hi=f + 64) == 4 and call(lo=3 * f + 16) == 4


def test_gemm_split_workspace_validates_before_launch():
    """mamba_gemm_tf32x3_ws: the split of K is planned on the host; a short,
    misaligned or overlapping workspace is rejected before any launch."""
    lib = cuda.library()
    f = 0x1000000  # 16 MiB apart
    # the out_proj product of a 1024-token Mamba-130m forward splits K; the
    # in_proj and LM-head products (enough output tiles) do not
    need = cuda.gemm_workspace_size(768, 1024, 1536)
    assert need > 0 and need % (768 * 1024 * 4) == 0
    assert cuda.gemm_workspace_size(3072, 1024, 768) == 0
    assert cuda.gemm_workspace_size(1024, 50280, 768) == 0
    assert cuda.gemm_workspace_size(0, 1024, 1536) == 0

    def gemm_ws(ws, ws_bytes, c=40 * f, c_in=None):
        return lib.mamba_gemm_tf32x3_ws(f, 2 * f, 1536, 3 * f, 4 * f, 1536, c_in, c, 1, 768,
                                        768, 1024, 1536, ws, ws_bytes, None)

    assert gemm_ws(60 * f, need - 1) == 3 and b"workspace" in lib.mamba_scan_last_error()
    assert gemm_ws(60 * f + 8, need) == 1 and b"aligned" in lib.mamba_scan_last_error()
    assert gemm_ws(40 * f, need) == 4 and b"overlaps C" in lib.mamba_scan_last_error()
    assert gemm_ws(60 * f, need, c_in=60 * f + 4096) == 4
    assert gemm_ws(2 * f, need) == 4 and b"operand" in lib.mamba_scan_last_error()


def test_conv1d_step_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    assert lib.mamba_causal_conv1d_step(f, 2 * f, 64, 3 * f, None, 4 * f, 1, 64, 9, None) == 1
    assert lib.mamba_causal_conv1d_step(f, 2 * f, 63, 3 * f, None, 4 * f, 2, 64, 4, None) == 1
    assert lib.mamba_causal_conv1d_step(f, 2 * f, 64, 3 * f, None, f + 16, 1, 64, 4, None) == 4
    assert lib.mamba_causal_conv1d_step(f, 2 * f, 64, 3 * f, None, 4 * f, 0, 64, 4, None) == 0


def test_ssm_decode_step_validates_before_launch():
    lib = cuda.library()
    f = 0x100000

    def call(dstate=16, rank=8, state=10 * f, y=11 * f, zs=64, batch=1):
        return lib.mamba_ssm_decode_step(f, 2 * f, zs, 3 * f, 4 * f, 5 * f, 6 * f, 7 * f, 8 * f,
                                         9 * f, state, y, batch, 64, rank, dstate, None)

    assert call(dstate=8) == 2
    assert call(rank=0) == 1 and call(rank=300) == 1
    assert call(zs=63, batch=2) == 1
    assert call(y=f + 16) == 4 and call(state=8 * f) == 4
    assert call(batch=0) == 0


def test_rmsnorm_gemv_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    assert lib.mamba_rmsnorm_gemv(f, 2 * f, 1e-5, 3 * f, 4 * f, 1, 66, 8, None) == 1  # cols % 4
    assert lib.mamba_rmsnorm_gemv(f, 2 * f, 1e-5, 3 * f, 4 * f, 1, 8192, 8, None) == 1
    assert lib.mamba_rmsnorm_gemv(f, 2 * f, 1e-5, 3 * f + 4, 4 * f, 1, 64, 8, None) == 1
    assert lib.mamba_rmsnorm_gemv(f, 2 * f, 1e-5, 3 * f, f + 8, 1, 64, 8, None) == 4
    assert lib.mamba_rmsnorm_gemv(f, 2 * f, 1e-5, 3 * f, 4 * f, 0, 64, 8, None) == 0


def test_gemv_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    assert lib.mamba_gemv(f, 2 * f, None, 3 * f, 1, 66, 8, None) == 1
    assert lib.mamba_gemv(f, 2 * f + 4, None, 3 * f, 1, 64, 8, None) == 1
    assert lib.mamba_gemv(f, 2 * f, None, f + 8, 1, 64, 8, None) == 4
    assert lib.mamba_gemv(f, 2 * f, 3 * f + 4, 3 * f, 1, 64, 8, None) == 4  # partial overlap
    assert lib.mamba_gemv(f, 2 * f, None, 3 * f, 0, 64, 8, None) == 0


def test_x_proj_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    # x_proj: rank + 2 dstate <= 128, outputs disjoint from inputs and each other
    assert lib.mamba_x_proj(f, 2 * f, 3 * f, 4 * f, 5 * f, 1, 64, 16, 100, 16, None) == 1
    assert lib.mamba_x_proj(f, 2 * f, 3 * f, 4 * f, 5 * f, 1, 64, 16, 0, 16, None) == 1
    assert lib.mamba_x_proj(f, 2 * f, f + 64, 4 * f, 5 * f, 1, 64, 16, 8, 16, None) == 4
    assert lib.mamba_x_proj(f, 2 * f, 3 * f, 3 * f + 64, 5 * f, 1, 64, 16, 8, 16, None) == 4
    assert lib.mamba_x_proj(f, 2 * f, 3 * f, 4 * f, 5 * f, 0, 64, 16, 8, 16, None) == 0


def test_dt_proj_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    assert lib.mamba_dt_proj(f, 2 * f, 3 * f, 1, 64, 16, 0, None) == 1  # rank 0
    assert lib.mamba_dt_proj(f, 2 * f, 3 * f, -1, 64, 16, 8, None) == 1
    assert lib.mamba_dt_proj(None, 2 * f, 3 * f, 1, 64, 16, 8, None) == 1
    assert lib.mamba_dt_proj(f, 2 * f, f + 64, 1, 64, 16, 8, None) == 4  # delta over dt
    assert lib.mamba_dt_proj(f, 2 * f, 2 * f + 4, 1, 64, 16, 8, None) == 4  # delta over weight
    assert lib.mamba_dt_proj(f, 2 * f, 3 * f, 0, 64, 16, 8, None) == 0  # empty: nothing to do
    assert lib.mamba_dt_proj(f, 2 * f, 3 * f, 1, 64, 0, 8, None) == 0


def test_x_proj_delta_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    args = lambda **k: [k.get(n, v) for n, v in [  # noqa: E731
        ("x", f), ("w", 2 * f), ("wdt", 3 * f), ("delta", 4 * f), ("B", 5 * f), ("C", 6 * f),
        ("batch", 1), ("dim", 64), ("seqlen", 16), ("rank", 8), ("dstate", 16)]] + [None]
    assert lib.mamba_x_proj_delta(*args(rank=97)) == 1  # dt_rank above 96
    assert lib.mamba_x_proj_delta(*args(rank=80, dstate=40)) == 1  # rank + 2 dstate > 128
    assert lib.mamba_x_proj_delta(*args(wdt=None)) == 1
    assert lib.mamba_x_proj_delta(*args(delta=f + 64)) == 4  # delta over x
    assert lib.mamba_x_proj_delta(*args(B=3 * f + 8)) == 4  # B over dt_weight
    assert lib.mamba_x_proj_delta(*args(C=5 * f + 4)) == 4  # C over B
    assert lib.mamba_x_proj_delta(*args(batch=0)) == 0


def test_decode_step_validates_before_launch():
    lib = cuda.library()
    f = 0x100000
    need = lib.mamba_decode_scratch_size(1, 1536, 48, 16)
    assert need > 16 and lib.mamba_decode_scratch_size(0, 1536, 48, 16) == 0

    def call(**k):
        a = dict(layers=f, n=24, h=2 * f, nf=3 * f, lm=1 << 36, logits=5 * f, scratch=6 * f,
                 sbytes=need, batch=1, dm=768, di=1536, conv=4, rank=48, dstate=16,
                 vocab=50280)
        a.update(k)
        return lib.mamba_decode_step(*a.values(), 1e-5, None)

    assert call(batch=5) == 1          # at most 4 tokens
    assert call(dstate=8) == 1
    assert call(conv=9) == 1
    assert call(dm=770) == 1           # d_model a multiple of 4
    assert call(h=None) == 1
    assert call(sbytes=need - 4) == 3  # scratch too small
    assert call(scratch=6 * f + 8) == 3  # scratch misaligned
    assert call(lm=(1 << 36) + 4) == 1  # LM head misaligned
    assert call(batch=4, dm=16384, sbytes=1 << 20) == 1  # beyond the kernel's widths
    assert call(logits=2 * f + 512) == 4  # logits inside h
    assert call(scratch=5 * f + 64) == 4  # scratch inside logits
    assert call(h=(1 << 36) + 4096) == 4  # h inside the LM head


def test_decode_layer_table_checks_its_tensors():
    import torch

    good = {f: torch.zeros(4) for f in cuda.DECODE_LAYER_FIELDS}
    with pytest.raises(TypeError, match="contiguous CUDA float32"):
        cuda.decode_layer_table([good], "cpu")  # host tensors are refused
    missing = dict(good)
    del missing["A"]
    with pytest.raises(ValueError, match="needs A"):
        cuda.decode_layer_table([missing], "cpu")


def test_empty_batch_is_a_no_op():
    lib = cuda.library()
    assert lib.mamba_scan_launch(0, ctypes.byref(_args(batch=0)), None, 0, None) == 0


# ---- Python loader (mirror of the reference's src/mamba_onnx/__init__.py) ----

def test_loader_lists_cuda_backend():
    assert "cuda" in mamba_onnx.available_backends()
    assert mamba_onnx.get_library_path("cuda").endswith("libmamba_ops_cuda.so")
    assert mamba_onnx.get_library_path("auto") == mamba_onnx.get_library_path("cuda")


def test_loader_has_no_cpu_fallback():
    with pytest.raises(FileNotFoundError):
        mamba_onnx.get_library_path("cpp")
    with pytest.raises(ValueError):
        mamba_onnx.get_library_path("metal")


def test_register_custom_ops_passes_the_library_to_the_session_options():
    class Opts:
        def __init__(self):
            self.paths = []

        def register_custom_ops_library(self, path):
            self.paths.append(path)

    opts = Opts()
    path = mamba_onnx.register_custom_ops(opts, backend="cuda")
    assert opts.paths == [path] and path.endswith("libmamba_ops_cuda.so")


# ---- ORT op table through the fake CUDA-EP host ----

def test_op_table_matches_reference_ops():
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    infos = {i.name: i for i in ort_shim.op_infos(opts.libraries[0])}
    # selective_scan.cc:332-371: names, input counts, one float output, opset 1..INT_MAX
    assert list(infos) == ["SelectiveScan", "SelectiveScanExact", "SelectiveScanFused",
                           "SelectiveScanFusedExact"]
    for name, info in infos.items():
        assert info.ep == "CUDAExecutionProvider"
        assert info.n_outputs == 1 and info.version_range == (1, 2147483647)
        assert info.has_v2
    assert infos["SelectiveScan"].input_characteristics == "R" * 6
    assert infos["SelectiveScanExact"].input_characteristics == "R" * 6
    assert infos["SelectiveScanFused"].input_characteristics == "R" * 7 + "O"
    assert infos["SelectiveScanFusedExact"].input_characteristics == "R" * 7 + "O"


def test_register_failure_is_reported_not_swallowed():
    ort_shim.fail_next("CustomOpDomain_Add")
    with pytest.raises(ort_shim.OrtError, match="injected failure in CustomOpDomain_Add"):
        ort_shim.load_library(mamba_onnx.get_library_path("cuda"))


def _session(op):
    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    fused = "Fused" in op
    return ort_shim.InferenceSession(ort_shim.make_model(op, fused), opts,
                                     providers=["CUDAExecutionProvider"])


def _fake_run(sess, shapes, types=None, out_shape=(1, 64, 32)):
    """Drive the op with fake device pointers; validation must fail first."""
    h = ort_shim.host()
    n = len(shapes)
    ptrs = (ctypes.c_void_p * n)(*[0x100000 * (i + 1) for i in range(n)])
    dims = [d for s in shapes for d in s]
    ranks = (ctypes.c_int * n)(*[len(s) for s in shapes])
    tys = (ctypes.c_int * n)(*(types or [1] * n))
    err = ctypes.create_string_buffer(1024)
    rc = h.fake_ort_run(sess.lib, sess.model.op_type.encode(), n, ptrs,
                        (ctypes.c_int64 * len(dims))(*dims), ranks, tys, 0x900000,
                        (ctypes.c_int64 * 3)(*out_shape), 3, None, 1, err, len(err))
    return rc, err.value.decode()


GOOD = [(1, 64, 32), (1, 64, 32), (64, 16), (1, 32, 16), (1, 32, 16), (64,)]


@pytest.mark.parametrize("shapes,types,msg", [
    ([(64, 32)] + GOOD[1:], None, "u must be"),
    (GOOD[:2] + [(64, 8)] + [(1, 32, 8), (1, 32, 8), (64,)], None, "Only dstate=16"),
    (GOOD[:3] + [(1, 31, 16)] + GOOD[4:], None, "B and C"),
    (GOOD[:5] + [(63,)], None, "D must be"),
    (GOOD, [1, 11, 1, 1, 1, 1], "float32"),
    (GOOD[:5], None, "expected 6 inputs"),
])
def test_ort_layer_validates_before_launch(shapes, types, msg):
    rc, err = _fake_run(_session("SelectiveScan"), shapes, types)
    assert rc == 2, err  # ORT_INVALID_ARGUMENT
    assert msg in err


def test_ort_layer_propagates_host_failures():
    sess = _session("SelectiveScan")
    for api in ["KernelContext_GetInput", "KernelContext_GetOutput", "GetTensorTypeAndShape",
                "KernelContext_GetGPUComputeStream"]:
        ort_shim.fail_next(api)
        rc, err = _fake_run(sess, GOOD)
        assert rc == 1 and f"injected failure in {api}" in err


def test_ort_layer_fused_delta_bias_shape_checked():
    sess = _session("SelectiveScanFused")
    sess.model.inputs.append("delta_bias")
    rc, err = _fake_run(sess, GOOD + [(1, 64, 32), (63,)])
    assert rc == 2 and "delta_bias" in err


def test_workspace_plan():
    """Workspace is needed exactly when some row tiles are split into chunks.

    Off the GPU the planner assumes 148 SMs and 8 resident CTAs per SM, i.e.
    waves of 1184 row tiles.
    """
    # 37 x 1024 rows = 1184 row tiles = one full wave: one pass, no workspace
    assert cuda.workspace_size("SelectiveScanFused", 37, 1024, 2048) == 0
    # short sequences never split
    assert cuda.workspace_size("SelectiveScan", 1, 64, 32) == 0
    # 8 x 5120 rows = 1280 row tiles: the 96 past one wave are split into
    # 6 chunks of 352 steps: 96 * 32 rows * 5 aggregates * 32 floats
    assert cuda.workspace_size("SelectiveScanFused", 8, 5120, 2048) == 96 * 32 * 5 * 32 * 4
    # few row tiles, long sequence: everything is split
    assert cuda.workspace_size("SelectiveScanExact", 1, 2048, 16384) > 0


def test_python_binding_checks_exp_modes():
    assert cuda._variant("SelectiveScanExact", "reference") == 1 | 0x200
    assert cuda._variant("SelectiveScanFusedExact", "ieee") == 3 | 0x100
    with pytest.raises(ValueError, match="Exact ops only"):
        cuda._variant("SelectiveScanFused", "ieee")
    with pytest.raises(ValueError, match="exp must be"):
        cuda._variant("SelectiveScanExact", "fast")
