"""Direct access to the CUDA selective-scan kernels through their C ABI.

A thin ctypes binding of include/mamba_scan.h. Tensors are torch CUDA
tensors (torch provides device memory and the current stream); the work runs
in libmamba_ops_cuda.so. Importing this module on a machine without the
library raises: there is no CPU implementation behind it.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

from . import get_library_path

OPS = {
    "SelectiveScan": 0,
    "SelectiveScanExact": 1,
    "SelectiveScanFused": 2,
    "SelectiveScanFusedExact": 3,
}
FUSED = {"SelectiveScanFused", "SelectiveScanFusedExact"}
EXACT = {"SelectiveScanExact", "SelectiveScanFusedExact"}
# How the Exact ops form exp (include/mamba_scan.h, MAMBA_SCAN_EXP_*): None =
# the SFU's ex2.approx; "ieee" = CUDA's expf; "reference" = the reference C++
# backend's own polynomial exp, to follow that backend's numbers.
EXP_FLAGS = {None: 0, "ieee": 0x100, "reference": 0x200}

STATUS_OK = 0


class ScanArgs(ctypes.Structure):
    """struct mamba_scan_args (include/mamba_scan.h)."""

    _fields_ = [
        ("u", ctypes.c_void_p),
        ("delta", ctypes.c_void_p),
        ("A", ctypes.c_void_p),
        ("B", ctypes.c_void_p),
        ("C", ctypes.c_void_p),
        ("D", ctypes.c_void_p),
        ("z", ctypes.c_void_p),
        ("delta_bias", ctypes.c_void_p),
        ("h0", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("h_last", ctypes.c_void_p),
        ("batch", ctypes.c_int64),
        ("dim", ctypes.c_int64),
        ("seqlen", ctypes.c_int64),
        ("dstate", ctypes.c_int64),
    ]


class ScanError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


_lib = None


def library() -> ctypes.CDLL:
    """Load libmamba_ops_cuda.so (once) and declare the C ABI."""
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(get_library_path("cuda"))
        lib.mamba_scan_launch.restype = ctypes.c_int
        lib.mamba_scan_launch.argtypes = [ctypes.c_int, ctypes.POINTER(ScanArgs), ctypes.c_void_p,
                                          ctypes.c_size_t, ctypes.c_void_p]
        lib.mamba_scan_workspace_size.restype = ctypes.c_size_t
        lib.mamba_scan_workspace_size.argtypes = [ctypes.c_int] + [ctypes.c_int64] * 4
        lib.mamba_scan_last_error.restype = ctypes.c_char_p
        lib.mamba_scan_status_string.restype = ctypes.c_char_p
        lib.mamba_scan_status_string.argtypes = [ctypes.c_int]
        lib.mamba_scan_check_device_error.restype = ctypes.c_int
        lib.mamba_scan_abi_version.restype = ctypes.c_int
        lib.mamba_scan_launch_static_workspace.restype = ctypes.c_int
        lib.mamba_scan_launch_static_workspace.argtypes = [ctypes.c_int, ctypes.POINTER(ScanArgs),
                                                           ctypes.c_void_p]
        lib.mamba_scan_selftest_wait_timeout.restype = ctypes.c_int
        lib.mamba_scan_selftest_wait_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p]
        lib.mamba_rmsnorm.restype = ctypes.c_int
        lib.mamba_rmsnorm.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 2 + \
            [ctypes.c_float, ctypes.c_void_p]
        lib.mamba_causal_conv1d_silu.restype = ctypes.c_int
        lib.mamba_causal_conv1d_silu.argtypes = [ctypes.c_void_p, ctypes.c_int64] + \
            [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_void_p]
        lib.mamba_causal_conv1d_step.restype = ctypes.c_int
        lib.mamba_causal_conv1d_step.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int64] + \
            [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
        lib.mamba_rmsnorm_gemv.restype = ctypes.c_int
        lib.mamba_rmsnorm_gemv.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_float] + \
            [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
        lib.mamba_gemv.restype = ctypes.c_int
        lib.mamba_gemv.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 3 + [ctypes.c_void_p]
        lib.mamba_ssm_decode_step.restype = ctypes.c_int
        lib.mamba_ssm_decode_step.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int64] + \
            [ctypes.c_void_p] * 9 + [ctypes.c_int64] * 4 + [ctypes.c_void_p]
        lib.mamba_x_proj.restype = ctypes.c_int
        lib.mamba_x_proj.argtypes = [ctypes.c_void_p] * 5 + [ctypes.c_int64] * 5 + [ctypes.c_void_p]
        lib.mamba_decode_scratch_size.restype = ctypes.c_size_t
        lib.mamba_decode_scratch_size.argtypes = [ctypes.c_int64] * 4
        lib.mamba_decode_step.restype = ctypes.c_int
        lib.mamba_decode_step.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                          ctypes.c_void_p, ctypes.c_size_t] + \
            [ctypes.c_int64] * 7 + [ctypes.c_float, ctypes.c_void_p]
        lib.mamba_decode_selftest_barrier_timeout.restype = ctypes.c_int
        lib.mamba_decode_selftest_barrier_timeout.argtypes = [ctypes.c_int64, ctypes.c_void_p,
                                                              ctypes.c_size_t, ctypes.c_void_p]
        lib.mamba_x_proj_delta.restype = ctypes.c_int
        lib.mamba_x_proj_delta.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int64] * 5 + \
            [ctypes.c_void_p]
        lib.mamba_dt_proj.restype = ctypes.c_int
        lib.mamba_dt_proj.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int64] * 4 + [ctypes.c_void_p]
        lib.mamba_split_tf32.restype = ctypes.c_int
        lib.mamba_split_tf32.argtypes = [ctypes.c_void_p] + [ctypes.c_int64] * 3 + \
            [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.mamba_gemm_tf32x3.restype = ctypes.c_int
        lib.mamba_gemm_tf32x3.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] * 2 + \
            [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 5 + [ctypes.c_void_p]
        lib.mamba_gemm_tf32x3_ws.restype = ctypes.c_int
        lib.mamba_gemm_tf32x3_ws.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] * 2 + \
            [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 5 + \
            [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        lib.mamba_gemm_tf32x3_workspace_size.restype = ctypes.c_size_t
        lib.mamba_rmsnorm_split_tf32.restype = ctypes.c_int
        lib.mamba_rmsnorm_split_tf32.argtypes = [ctypes.c_void_p] * 2 + [ctypes.c_int64] * 2 + \
            [ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        lib.mamba_gemm_tf32x3_workspace_size.argtypes = [ctypes.c_int64] * 3
        _lib = lib
    return _lib


def library_path() -> Path:
    return Path(get_library_path("cuda"))


def _ptr(t):
    return None if t is None else t.data_ptr()


def _check(name, t, shape):
    import torch

    if t is None:
        return
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor")
    if t.dtype != torch.float32:
        raise TypeError(f"{name} must be float32, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")


def _variant(op: str, exp) -> int:
    if op not in OPS:
        raise ValueError(f"unknown op {op!r}")
    if exp not in EXP_FLAGS:
        raise ValueError(f"exp must be one of {list(EXP_FLAGS)}, got {exp!r}")
    if exp is not None and op not in EXACT:
        raise ValueError(f"exp={exp!r} applies to the Exact ops only, not {op}")
    return OPS[op] | EXP_FLAGS[exp]


def workspace_size(op: str, batch: int, dim: int, seqlen: int, dstate: int = 16,
                   exp=None) -> int:
    return int(library().mamba_scan_workspace_size(_variant(op, exp), batch, dim, seqlen,
                                                   dstate))


def selective_scan(op: str, u, delta, A, B, C, D, z=None, *, delta_bias=None, h0=None,
                   out=None, h_last=None, workspace=None, chunked=True, stream=None, exp=None):
    """Run one selective-scan op on CUDA tensors; returns ``out`` ([batch, dim, seqlen]).

    op: one of the four reference op names. Layouts: u/delta/z [B,D,L], A [D,N],
    B/C [B,L,N], D [D]; optional delta_bias [D] (fused ops), h0 / h_last [B,D,N].
    workspace: optional uint8 CUDA tensor; by default one of
    workspace_size(...) bytes is taken from torch's allocator.
    chunked: False passes no workspace, so the sequence runs as one pass.
    stream: a torch.cuda.Stream (default: the current stream).
    exp: Exact ops only: None (SFU exp), "ieee" (CUDA's expf) or "reference"
    (the reference C++ backend's polynomial exp; see EXP_FLAGS).
    """
    import torch

    code = _variant(op, exp)
    if u.dim() != 3 or A.dim() != 2:
        raise ValueError("u must be [batch, dim, seqlen] and A [dim, dstate]")
    batch, dim, seqlen = u.shape
    dstate = A.shape[1]
    for name, t, shape in [("u", u, (batch, dim, seqlen)), ("delta", delta, (batch, dim, seqlen)),
                           ("A", A, (dim, dstate)), ("B", B, (batch, seqlen, dstate)),
                           ("C", C, (batch, seqlen, dstate)), ("D", D, (dim,)),
                           ("z", z, (batch, dim, seqlen)), ("delta_bias", delta_bias, (dim,)),
                           ("h0", h0, (batch, dim, dstate)), ("h_last", h_last, (batch, dim, dstate))]:
        _check(name, t, shape)
    if op in FUSED and z is None:
        raise ValueError(f"{op} needs z")
    if out is None:
        out = torch.empty((batch, dim, seqlen), dtype=torch.float32, device=u.device)
    else:
        _check("out", out, (batch, dim, seqlen))
    lib = library()
    ws_bytes = int(lib.mamba_scan_workspace_size(code, batch, dim, seqlen, dstate))
    if not chunked:
        workspace = None
    elif workspace is None and ws_bytes > 0:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=u.device)
    args = ScanArgs(_ptr(u), _ptr(delta), _ptr(A), _ptr(B), _ptr(C), _ptr(D),
                    _ptr(z) if op in FUSED else None, _ptr(delta_bias), _ptr(h0), _ptr(out),
                    _ptr(h_last), batch, dim, seqlen, dstate)
    st = stream if stream is not None else torch.cuda.current_stream(u.device)
    rc = lib.mamba_scan_launch(code, ctypes.byref(args), _ptr(workspace),
                               0 if workspace is None else workspace.numel(), st.cuda_stream)
    if rc != STATUS_OK:
        raise ScanError(rc, f"{op}: {lib.mamba_scan_status_string(rc).decode()}: "
                            f"{lib.mamba_scan_last_error().decode()}")
    return out


def launch_raw(op_id: int, args: ScanArgs, workspace_ptr, workspace_bytes: int,
               stream_handle) -> int:
    """Call mamba_scan_launch with a prepared argument struct; returns the status."""
    return int(library().mamba_scan_launch(op_id, ctypes.byref(args), workspace_ptr,
                                           workspace_bytes, stream_handle))


def launch_static_workspace(op_id: int, args: ScanArgs, stream_handle) -> int:
    """Call mamba_scan_launch_static_workspace: the scan with no device allocation.

    For callers that cannot allocate device memory; the scratch of long-sequence
    shapes comes from a fixed array inside the library (include/mamba_scan.h
    states its size and its rules). Returns the status.
    """
    return int(library().mamba_scan_launch_static_workspace(op_id, ctypes.byref(args),
                                                            stream_handle))


def check_device_error() -> int:
    """Synchronise and return/clear the kernels' device error word (0 = none)."""
    return int(library().mamba_scan_check_device_error())


def selftest_wait_timeout(limit_ns: int, stream=None) -> int:
    """Enqueue the bounded-wait self-test (a wait that must give up after
    limit_ns); check_device_error() then returns MAMBA_SCAN_ERR_DEVICE_TIMEOUT."""
    import torch

    st = stream if stream is not None else torch.cuda.current_stream()
    return int(library().mamba_scan_selftest_wait_timeout(int(limit_ns), st.cuda_stream))


# ---- kernels of the Mamba block around the scan (include/mamba_model_ops.h) ----

def _raise(rc, what):
    lib = library()
    raise ScanError(rc, f"{what}: {lib.mamba_scan_status_string(rc).decode()}: "
                        f"{lib.mamba_scan_last_error().decode()}")


def rmsnorm(x, weight, eps: float, out=None, stream=None):
    """RMSNorm over the last dimension of a contiguous CUDA float32 tensor:
    x * rsqrt(mean(x^2, -1) + eps) * weight. Returns ``out`` (new if None)."""
    import torch

    cols = x.shape[-1]
    _check("x", x, tuple(x.shape))
    _check("weight", weight, (cols,))
    if out is None:
        out = torch.empty_like(x)
    else:
        _check("out", out, tuple(x.shape))
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_rmsnorm(_ptr(x), _ptr(weight), _ptr(out), x.numel() // cols, cols,
                                 float(eps), st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "rmsnorm")
    return out


def causal_conv1d_silu(x, weight, bias=None, out=None, stream=None):
    """silu(causal depthwise conv1d over the sequence): x [B, D, L] CUDA float32
    whose rows are contiguous and D-stride is L (e.g. the first half of the
    in_proj output [B, 2D, L]); weight [D, 1, K] or [D, K]; bias [D] or None.
    Equals F.silu(F.conv1d(x, weight, bias, padding=K-1, groups=D)[..., :L]).
    Returns ``out`` ([B, D, L], new if None)."""
    import torch

    if x.dim() != 3 or not x.is_cuda or x.dtype != torch.float32:
        raise TypeError("x must be a [batch, dim, seqlen] CUDA float32 tensor")
    batch, dim, seqlen = x.shape
    if (seqlen > 1 and x.stride(2) != 1) or (dim > 1 and x.stride(1) != seqlen):
        raise ValueError("x rows must be contiguous with dim stride seqlen")
    w = weight.reshape(dim, -1)
    _check("weight", w, (dim, w.shape[1]))
    _check("bias", bias, (dim,))
    if out is None:
        out = torch.empty((batch, dim, seqlen), dtype=torch.float32, device=x.device)
    else:
        _check("out", out, (batch, dim, seqlen))
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    bstride = x.stride(0) if batch > 1 else dim * seqlen
    rc = library().mamba_causal_conv1d_silu(_ptr(x), bstride, _ptr(w), _ptr(bias), _ptr(out),
                                            batch, dim, seqlen, w.shape[1], st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "causal_conv1d_silu")
    return out


def causal_conv1d_step(state, x, weight, bias=None, stream=None):
    """One decoding step of silu(causal depthwise conv1d): state [B, D, K]
    (contiguous, oldest input first) shifts in x [B, D] (rows contiguous, any
    batch stride) in place; returns y [B, D]."""
    import torch

    batch, dim, width = state.shape
    _check("state", state, (batch, dim, width))
    if x.dim() != 2 or tuple(x.shape) != (batch, dim) or not x.is_cuda or \
            x.dtype != torch.float32 or (dim > 1 and x.stride(1) != 1):
        raise ValueError("x must be a [batch, dim] CUDA float32 tensor with contiguous rows")
    w = weight.reshape(dim, -1)
    _check("weight", w, (dim, width))
    _check("bias", bias, (dim,))
    y = torch.empty(batch, dim, dtype=torch.float32, device=state.device)
    st = stream if stream is not None else torch.cuda.current_stream(state.device)
    bstride = x.stride(0) if batch > 1 else dim
    rc = library().mamba_causal_conv1d_step(_ptr(state), _ptr(x), bstride, _ptr(w), _ptr(bias),
                                            _ptr(y), batch, dim, width, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "causal_conv1d_step")
    return y


def rmsnorm_gemv(x, norm_weight, eps: float, weight, stream=None):
    """weight @ rmsnorm(x) for a few tokens: x [batch, cols], norm_weight
    [cols], weight [rows_out, cols] -> [batch, rows_out]."""
    import torch

    batch, cols = x.shape
    rows_out = weight.shape[0]
    _check("x", x, (batch, cols))
    _check("norm_weight", norm_weight, (cols,))
    _check("weight", weight, (rows_out, cols))
    out = torch.empty(batch, rows_out, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_rmsnorm_gemv(_ptr(x), _ptr(norm_weight), float(eps), _ptr(weight),
                                      _ptr(out), batch, cols, rows_out, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "rmsnorm_gemv")
    return out


def gemv(x, weight, residual=None, stream=None):
    """(residual +) x @ weight.T for a few tokens: x [batch, cols], weight
    [rows_out, cols], residual [batch, rows_out] or None -> [batch, rows_out]."""
    import torch

    batch, cols = x.shape
    rows_out = weight.shape[0]
    _check("x", x, (batch, cols))
    _check("weight", weight, (rows_out, cols))
    _check("residual", residual, (batch, rows_out))
    out = torch.empty(batch, rows_out, dtype=torch.float32, device=x.device)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_gemv(_ptr(x), _ptr(weight), _ptr(residual), _ptr(out), batch, cols,
                              rows_out, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "gemv")
    return out


def ssm_decode_step(u, z, dt, B, C, dt_weight, dt_bias, A, D, state, stream=None):
    """One decoding step of a SelectiveScanFusedExact block with dt_proj fused
    in front: u [batch, dim], z [batch, dim] (rows contiguous, any batch
    stride), dt [batch, rank], B/C [batch, 16], dt_weight [dim, rank],
    dt_bias [dim] or None, A [dim, 16], D [dim]; state [batch, dim, 16] is
    updated in place. Returns y [batch, dim]."""
    import torch

    batch, dim = u.shape
    rank, dstate = dt.shape[1], A.shape[1]
    for name, t, shape in [("u", u, (batch, dim)), ("dt", dt, (batch, rank)),
                           ("B", B, (batch, dstate)), ("C", C, (batch, dstate)),
                           ("dt_weight", dt_weight, (dim, rank)), ("dt_bias", dt_bias, (dim,)),
                           ("A", A, (dim, dstate)), ("D", D, (dim,)),
                           ("state", state, (batch, dim, dstate))]:
        _check(name, t, shape)
    if tuple(z.shape) != (batch, dim) or not z.is_cuda or z.dtype != torch.float32 or \
            (dim > 1 and z.stride(1) != 1):
        raise ValueError("z must be a [batch, dim] CUDA float32 tensor with contiguous rows")
    y = torch.empty(batch, dim, dtype=torch.float32, device=u.device)
    st = stream if stream is not None else torch.cuda.current_stream(u.device)
    zstride = z.stride(0) if batch > 1 else dim
    rc = library().mamba_ssm_decode_step(_ptr(u), _ptr(z), zstride, _ptr(dt), _ptr(B), _ptr(C),
                                         _ptr(dt_weight), _ptr(dt_bias), _ptr(A), _ptr(D),
                                         _ptr(state), _ptr(y), batch, dim, rank, dstate,
                                         st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "ssm_decode_step")
    return y


def x_proj(x, weight, rank: int, dstate: int, stream=None):
    """Mamba's x_proj split into the scan's inputs: x [B, D, L] (contiguous
    CUDA float32), weight [rank + 2*dstate, D]. Returns (dt [B, L, rank],
    B [B, L, dstate], C [B, L, dstate]), all contiguous."""
    import torch

    if x.dim() != 3:
        raise ValueError("x must be [batch, dim, seqlen]")
    batch, dim, seqlen = x.shape
    _check("x", x, (batch, dim, seqlen))
    _check("weight", weight, (rank + 2 * dstate, dim))
    kw = dict(dtype=torch.float32, device=x.device)
    dt = torch.empty(batch, seqlen, rank, **kw)
    Bm = torch.empty(batch, seqlen, dstate, **kw)
    Cm = torch.empty(batch, seqlen, dstate, **kw)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_x_proj(_ptr(x), _ptr(weight), _ptr(dt), _ptr(Bm), _ptr(Cm), batch, dim,
                                seqlen, rank, dstate, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "x_proj")
    return dt, Bm, Cm


DECODE_LAYER_FIELDS = ("norm_weight", "in_proj_weight", "conv_weight", "conv_bias",
                       "x_proj_weight", "dt_proj_weight", "dt_proj_bias", "A", "D",
                       "out_proj_weight", "conv_state", "ssm_state")


def decode_layer_table(layers, device):
    """The DEVICE array of struct mamba_decode_layer (include/mamba_model_ops.h)
    for mamba_decode_step: ``layers`` is a list of dicts mapping each name of
    DECODE_LAYER_FIELDS to a contiguous CUDA float32 tensor (conv_bias and
    dt_proj_bias may be None). Returns an int64 tensor of the pointers; the
    tensors must outlive it."""
    import torch

    rows = []
    for lay in layers:
        for f in DECODE_LAYER_FIELDS:
            if lay.get(f) is None and f not in ("conv_bias", "dt_proj_bias"):
                raise ValueError(f"decode layer needs {f}")
        row = []
        for f in DECODE_LAYER_FIELDS:
            t = lay.get(f)
            if t is not None and (not t.is_cuda or t.dtype != torch.float32
                                  or not t.is_contiguous()):
                raise TypeError(f"{f} must be a contiguous CUDA float32 tensor")
            if f in ("in_proj_weight", "out_proj_weight") and t.data_ptr() % 16:
                raise ValueError(f"{f} must be 16-byte aligned")
            row.append(0 if t is None else t.data_ptr())
        rows.append(row)
    return torch.tensor(rows, dtype=torch.int64).to(device)


def decode_scratch_size(batch: int, d_inner: int, rank: int, dstate: int = 16) -> int:
    return int(library().mamba_decode_scratch_size(batch, d_inner, rank, dstate))


def decode_step(table, n_layer: int, h, norm_f_weight, lm_head, logits, scratch, *, d_inner: int,
                d_conv: int, rank: int, dstate: int, eps: float, stream=None):
    """One decoding step of the whole model in one persistent kernel
    (mamba_decode_step): h [B, d_model] (the embedded tokens; becomes the
    final residual stream), logits [B, vocab] written; the layers' states in
    ``table`` (decode_layer_table) advance by one token. scratch: a uint8
    CUDA tensor of decode_scratch_size(...) bytes, used by one call at a time."""
    batch, d_model = h.shape
    vocab = lm_head.shape[0]
    _check("h", h, (batch, d_model))
    _check("norm_f_weight", norm_f_weight, (d_model,))
    _check("lm_head", lm_head, (vocab, d_model))
    _check("logits", logits, (batch, vocab))
    import torch

    st = stream if stream is not None else torch.cuda.current_stream(h.device)
    rc = library().mamba_decode_step(_ptr(table), n_layer, _ptr(h), _ptr(norm_f_weight),
                                     _ptr(lm_head), _ptr(logits), _ptr(scratch), scratch.numel(),
                                     batch, d_model, d_inner, d_conv, rank, dstate, vocab,
                                     float(eps), st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "decode_step")
    return logits


def decode_selftest_barrier_timeout(limit_ns: int, scratch, stream=None) -> int:
    """Enqueue the decoding kernel's barrier self-test (a grid barrier that
    no other CTA joins, giving up after limit_ns); check_device_error() then
    returns MAMBA_SCAN_ERR_DEVICE_TIMEOUT. scratch: a uint8 CUDA tensor of
    at least 128 bytes. Returns the status."""
    import torch

    st = stream if stream is not None else torch.cuda.current_stream()
    return int(library().mamba_decode_selftest_barrier_timeout(
        int(limit_ns), _ptr(scratch), 0 if scratch is None else scratch.numel(), st.cuda_stream))


X_PROJ_DELTA_MAX_RANK = 96


def x_proj_delta(x, weight, dt_weight, rank: int, dstate: int, stream=None):
    """x_proj with dt_proj fused behind it: x [B, D, L] (contiguous CUDA
    float32), weight [rank + 2*dstate, D], dt_weight [D, rank] (rank <= 96).
    Returns (delta [B, D, L], B [B, L, dstate], C [B, L, dstate]) with
    delta[b, d, t] = sum_k dt_weight[d, k] * dt[b, t, k], dt being x_proj's
    first rank outputs (dt_proj's bias is not added)."""
    import torch

    if x.dim() != 3:
        raise ValueError("x must be [batch, dim, seqlen]")
    batch, dim, seqlen = x.shape
    _check("x", x, (batch, dim, seqlen))
    _check("weight", weight, (rank + 2 * dstate, dim))
    _check("dt_weight", dt_weight, (dim, rank))
    kw = dict(dtype=torch.float32, device=x.device)
    delta = torch.empty(batch, dim, seqlen, **kw)
    Bm = torch.empty(batch, seqlen, dstate, **kw)
    Cm = torch.empty(batch, seqlen, dstate, **kw)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_x_proj_delta(_ptr(x), _ptr(weight), _ptr(dt_weight), _ptr(delta),
                                      _ptr(Bm), _ptr(Cm), batch, dim, seqlen, rank, dstate,
                                      st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "x_proj_delta")
    return delta, Bm, Cm


def dt_proj(dt, weight, out=None, stream=None):
    """Mamba's dt_proj without its bias: dt [B, L, rank] (x_proj's output,
    contiguous CUDA float32), weight [D, rank] -> delta [B, D, L] with
    delta[b, d, t] = sum_k weight[d, k] * dt[b, t, k] (the scan op's layout)."""
    import torch

    if dt.dim() != 3 or weight.dim() != 2:
        raise ValueError("dt must be [batch, seqlen, rank] and weight [dim, rank]")
    batch, seqlen, rank = dt.shape
    dim = weight.shape[0]
    _check("dt", dt, (batch, seqlen, rank))
    _check("weight", weight, (dim, rank))
    if out is None:
        out = torch.empty(batch, dim, seqlen, dtype=torch.float32, device=dt.device)
    else:
        _check("out", out, (batch, dim, seqlen))
    st = stream if stream is not None else torch.cuda.current_stream(dt.device)
    rc = library().mamba_dt_proj(_ptr(dt), _ptr(weight), _ptr(out), batch, dim, seqlen, rank,
                                 st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "dt_proj")
    return out


class SplitTF32:
    """An fp32 matrix [rows][cols] as two tf32 parts (hi = tf32(x), lo =
    tf32(x - hi)), rows padded to a multiple of 4 floats: the operand form of
    gemm_tf32x3. Built by split_tf32."""

    def __init__(self, hi, lo, rows: int, cols: int):
        self.hi, self.lo, self.rows, self.cols = hi, lo, rows, cols

    @property
    def ld(self) -> int:
        return self.hi.shape[1]

    def row_block(self, start: int, count: int) -> "SplitTF32":
        """Rows [start, start + count) as a SplitTF32 (views, no copy)."""
        return SplitTF32(self.hi[start:start + count], self.lo[start:start + count], count,
                         self.cols)


def split_tf32(x, transpose: bool = False, out: SplitTF32 | None = None,
               stream=None) -> SplitTF32:
    """Split a 2-D CUDA float32 matrix (rows contiguous, any row stride) into
    its tf32 parts; ``transpose`` splits x.t() instead (x [cols][rows])."""
    import torch

    if x.dim() != 2 or not x.is_cuda or x.dtype != torch.float32:
        raise TypeError("x must be a 2-D CUDA float32 tensor")
    if x.shape[1] > 1 and x.stride(1) != 1:
        raise ValueError("x rows must be contiguous")
    rows, cols = (x.shape[1], x.shape[0]) if transpose else (x.shape[0], x.shape[1])
    ldx = x.stride(0) if x.shape[0] > 1 else x.shape[1]
    ld = (cols + 3) // 4 * 4
    if out is None:
        out = SplitTF32(torch.empty((rows, ld), dtype=torch.float32, device=x.device),
                        torch.empty((rows, ld), dtype=torch.float32, device=x.device), rows, cols)
    elif (out.rows, out.cols) != (rows, cols):
        raise ValueError("out has the wrong shape")
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_split_tf32(_ptr(x), rows, cols, ldx, int(transpose), _ptr(out.hi),
                                    _ptr(out.lo), out.ld, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "split_tf32")
    return out


def rmsnorm_split_tf32(x, weight, eps: float, stream=None) -> SplitTF32:
    """rmsnorm(x, weight, eps) over the last dimension of a contiguous CUDA
    float32 tensor, delivered as the GEMM operand split_tf32 would make of it
    ([rows][cols], rows = all leading dimensions; mamba_rmsnorm_split_tf32).
    cols must be a multiple of 4."""
    import torch

    cols = x.shape[-1]
    _check("x", x, tuple(x.shape))
    _check("weight", weight, (cols,))
    rows = x.numel() // cols
    out = SplitTF32(torch.empty((rows, cols), dtype=torch.float32, device=x.device),
                    torch.empty((rows, cols), dtype=torch.float32, device=x.device), rows, cols)
    st = stream if stream is not None else torch.cuda.current_stream(x.device)
    rc = library().mamba_rmsnorm_split_tf32(_ptr(x), _ptr(weight), rows, cols, float(eps),
                                            _ptr(out.hi), _ptr(out.lo), cols, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "rmsnorm_split_tf32")
    return out


def gemm_workspace_size(M: int, N: int, K: int) -> int:
    """Workspace bytes with which gemm_tf32x3 splits K for an M x N x K
    product (0: it runs unsplit; mamba_gemm_tf32x3_workspace_size)."""
    return int(library().mamba_gemm_tf32x3_workspace_size(M, N, K))


def gemm_tf32x3(a: SplitTF32, b: SplitTF32, c, *, transpose_c: bool = False,
                c_in=None, stream=None, workspace=None):
    """c = (c_in +) a @ b.T on the tensor cores, fp32-accurate (3xTF32): a
    [M][K], b [N][K] split operands; c a CUDA float32 tensor viewed as [M, N]
    (or, with ``transpose_c``, as [N, M]: c[n][m] receives element (m, n));
    c_in None or a tensor with c's shape and strides (c itself allowed).
    ``workspace``: None, or a CUDA tensor of at least
    gemm_workspace_size(M, N, K) bytes (mamba_gemm_tf32x3_ws), with which a
    product of few output tiles splits K across the SMs. Returns c."""
    import torch

    if a.cols != b.cols:
        raise ValueError(f"inner sizes differ: {a.cols} vs {b.cols}")
    M, N, K = a.rows, b.rows, a.cols
    if c.dim() != 2 or not c.is_cuda or c.dtype != torch.float32:
        raise TypeError("c must be a 2-D CUDA float32 tensor")
    if tuple(c.shape) != ((N, M) if transpose_c else (M, N)):
        raise ValueError(f"c must be {(N, M) if transpose_c else (M, N)}, got {tuple(c.shape)}")
    s0, s1 = c.stride()
    ldc_m, ldc_n = (s1, s0) if transpose_c else (s0, s1)
    if c_in is not None and (c_in.shape != c.shape or c_in.stride() != c.stride()
                             or not c_in.is_cuda or c_in.dtype != torch.float32):
        raise ValueError("c_in must be a CUDA float32 tensor with c's shape and strides")
    st = stream if stream is not None else torch.cuda.current_stream(c.device)
    if workspace is not None and (not workspace.is_cuda or not workspace.is_contiguous()):
        raise ValueError("workspace must be a contiguous CUDA tensor")
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = library().mamba_gemm_tf32x3_ws(_ptr(a.hi), _ptr(a.lo), a.ld, _ptr(b.hi), _ptr(b.lo),
                                        b.ld, _ptr(c_in), _ptr(c), ldc_m, ldc_n, M, N, K,
                                        _ptr(workspace), ws_bytes, st.cuda_stream)
    if rc != STATUS_OK:
        _raise(rc, "gemm_tf32x3")
    return c
