"""A small stand-in for the parts of onnxruntime's Python API the tests use.

onnxruntime and onnx are not installed here, so the tests drive the custom-op
library through fake_ort_host.cu, which plays ONNX Runtime's CUDA execution
provider. This module wraps it in the shapes of the real API, so the parity
tests read like the reference's tests/test_ops.py:

    opts = ort_shim.SessionOptions()
    mamba_onnx.register_custom_ops(opts, backend="cuda")
    sess = ort_shim.InferenceSession(model, opts, providers=["CUDAExecutionProvider"])
    out = sess.run(None, feed)[0]

`model` is a single-node description built by make_model() in place of the
ONNX file that tests/test_ops.py:66-92 writes (same op name, input names and
domain).
"""
from __future__ import annotations

import ctypes
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_HOST_PATH = HERE / "_build" / "libfake_ort_host.so"
FLOAT = 1  # ONNX_TENSOR_ELEMENT_DATA_TYPE_FLOAT
DOUBLE = 11
_host = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def host():
    global _host
    if _host is None:
        if not _HOST_PATH.exists():
            build()
        h = ctypes.CDLL(str(_HOST_PATH))
        h.fake_ort_load.restype = ctypes.c_int
        h.fake_ort_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]
        h.fake_ort_op_count.restype = ctypes.c_int
        h.fake_ort_op_info.restype = ctypes.c_int
        h.fake_ort_op_info.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t,
                                       ctypes.c_char_p, ctypes.c_size_t] + \
            [ctypes.POINTER(ctypes.c_int)] * 5 + [ctypes.c_char_p, ctypes.c_size_t]
        h.fake_ort_fail_next.argtypes = [ctypes.c_char_p]
        h.fake_ort_live_allocations.restype = ctypes.c_int
        h.fake_ort_kernel_create.restype = ctypes.c_int
        h.fake_ort_kernel_create.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                             ctypes.c_char_p, ctypes.c_size_t]
        h.fake_ort_kernel_run.restype = ctypes.c_int
        h.fake_ort_kernel_run.argtypes = [ctypes.c_int, ctypes.c_int,
                                          ctypes.POINTER(ctypes.c_void_p),
                                          ctypes.POINTER(ctypes.c_int64),
                                          ctypes.POINTER(ctypes.c_int),
                                          ctypes.POINTER(ctypes.c_int), ctypes.c_void_p,
                                          ctypes.POINTER(ctypes.c_int64), ctypes.c_int,
                                          ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t]
        h.fake_ort_kernel_destroy.argtypes = [ctypes.c_int]
        h.fake_ort_run.restype = ctypes.c_int
        h.fake_ort_run.argtypes = [ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                   ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int64),
                                   ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                   ctypes.c_void_p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int,
                                   ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_size_t]
        _host = h
    return _host


class OrtError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(msg)
        self.code = code


@dataclass
class OpInfo:
    name: str
    ep: str
    n_inputs: int
    n_outputs: int
    version_range: tuple
    has_v2: bool
    input_characteristics: str


def load_library(path: str) -> int:
    err = ctypes.create_string_buffer(1024)
    lib = host().fake_ort_load(str(path).encode(), err, len(err))
    if lib < 0:
        raise OrtError(1, f"register_custom_ops_library({path}) failed: {err.value.decode()}")
    return lib


def op_infos(lib: int) -> list[OpInfo]:
    h = host()
    infos = []
    for i in range(h.fake_ort_op_count(lib)):
        name, ep, chars = (ctypes.create_string_buffer(128) for _ in range(3))
        ints = [ctypes.c_int() for _ in range(5)]
        rc = h.fake_ort_op_info(lib, i, name, 128, ep, 128, *[ctypes.byref(x) for x in ints],
                                chars, 128)
        assert rc == 0
        infos.append(OpInfo(name.value.decode(), ep.value.decode(), ints[0].value, ints[1].value,
                            (ints[2].value, ints[3].value), bool(ints[4].value),
                            chars.value.decode()))
    return infos


def fail_next(api_name: str) -> None:
    host().fake_ort_fail_next(api_name.encode())


def live_allocations() -> int:
    return host().fake_ort_live_allocations()


class SessionOptions:
    """onnxruntime.SessionOptions: only register_custom_ops_library."""

    def __init__(self):
        self.libraries: list[int] = []
        self.paths: list[str] = []

    def register_custom_ops_library(self, path: str) -> None:
        self.libraries.append(load_library(path))
        self.paths.append(str(path))


@dataclass
class SingleOpModel:
    op_type: str
    inputs: list
    domain: str = "mamba"
    outputs: list = field(default_factory=lambda: ["out"])


def make_model(op_name: str, use_fused: bool, with_delta_bias: bool = False) -> SingleOpModel:
    """Input names of tests/test_ops.py:66-92 (plus delta_bias if asked)."""
    names = ["u", "delta", "A", "B", "C", "D"]
    if use_fused:
        names.append("z")
        if with_delta_bias:
            names.append("delta_bias")
    return SingleOpModel(op_name, names)


class InferenceSession:
    """Runs a SingleOpModel through the registered library on one CUDA device.

    Like ONNX Runtime, a session creates the node's kernel once (through the
    op's CreateKernelV2, or CreateKernel with use_v2=False) and runs that same
    kernel on every run() until close(), which calls KernelDestroy."""

    def __init__(self, model: SingleOpModel, sess_options: SessionOptions, providers=None,
                 use_v2: bool = True):
        if model.domain != "mamba":
            raise OrtError(9, f"no kernel for domain {model.domain}")
        providers = list(providers or ["CUDAExecutionProvider"])
        self.model = model
        self.lib = None
        self.kernel = -1
        for lib in sess_options.libraries:
            for info in op_infos(lib):
                if info.name == model.op_type and info.ep in providers:
                    self.lib, self.info = lib, info
        if self.lib is None:
            raise OrtError(9, f"no kernel registered for {model.op_type} on {providers}")
        self.use_v2 = use_v2
        err = ctypes.create_string_buffer(1024)
        self.kernel = host().fake_ort_kernel_create(self.lib, model.op_type.encode(),
                                                    1 if use_v2 else 0, err, len(err))
        if self.kernel < 0:
            raise OrtError(1, err.value.decode())

    def close(self):
        if self.kernel >= 0:
            host().fake_ort_kernel_destroy(self.kernel)
            self.kernel = -1

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def run_device(self, inputs, out, stream=None):
        """Enqueue one run on device tensors (torch, in the model's input order;
        None = an omitted optional input) writing `out`, on `stream` (default:
        torch's current stream). Nothing is synchronised."""
        import torch

        ptrs, dims, ranks, types = [], [], [], []
        for t in inputs:
            if t is None:
                ptrs.append(None)
                ranks.append(0)
                types.append(FLOAT)
                continue
            ptrs.append(t.data_ptr())
            dims.extend(t.shape)
            ranks.append(t.dim())
            types.append(DOUBLE if t.dtype == torch.float64 else FLOAT)
        st = stream or torch.cuda.current_stream()
        err = ctypes.create_string_buffer(2048)
        out_dims = (ctypes.c_int64 * out.dim())(*out.shape)
        n = len(ptrs)
        rc = host().fake_ort_kernel_run(
            self.kernel, n, (ctypes.c_void_p * n)(*ptrs),
            (ctypes.c_int64 * max(1, len(dims)))(*dims), (ctypes.c_int * n)(*ranks),
            (ctypes.c_int * n)(*types), out.data_ptr(), out_dims, out.dim(), st.cuda_stream,
            err, len(err))
        if rc != 0:
            raise OrtError(rc, err.value.decode())
        return out

    def run(self, output_names, feed: dict, stream=None):
        import torch

        dev = [None if feed.get(name) is None else
               torch.from_numpy(np.ascontiguousarray(feed[name])).cuda()
               for name in self.model.inputs]
        u = feed["u"]
        out = torch.empty(tuple(u.shape), dtype=torch.float32, device="cuda")
        out.fill_(float("nan"))
        st = stream or torch.cuda.current_stream()
        self.run_device(dev, out, st)
        st.synchronize()
        return [out.cpu().numpy()]


class OrtScan:
    """A drop-in for mamba_onnx.cuda.selective_scan that runs every call
    through the library's ONNX Runtime custom-op entry (one session per op
    name: RegisterCustomOps, CreateKernelV2 once, KernelComputeV2 per call)
    on the caller's stream, as ORT's CUDA EP would run a graph's scan nodes.

    Pass it as ``scan=`` to mamba_onnx.model (MambaLM.forward). The op has
    the reference's inputs plus the optional delta_bias; it has no state
    input or output, so h0 / h_last must be None.
    """

    def __init__(self, library_path=None):
        import mamba_onnx

        self.opts = SessionOptions()
        if library_path is None:
            mamba_onnx.register_custom_ops(self.opts, backend="cuda")
        else:
            self.opts.register_custom_ops_library(str(library_path))
        self.sessions = {}

    def session(self, op, with_bias):
        key = (op, with_bias)
        if key not in self.sessions:
            fused = "Fused" in op
            self.sessions[key] = InferenceSession(make_model(op, fused, with_delta_bias=with_bias),
                                                  self.opts, providers=["CUDAExecutionProvider"])
        return self.sessions[key]

    def __call__(self, op, u, delta, A, B, C, D, z=None, *, delta_bias=None, h0=None,
                 out=None, h_last=None, stream=None, **_):
        import torch

        if h0 is not None or h_last is not None:
            raise ValueError("the ONNX Runtime op has no state input or output")
        fused = "Fused" in op
        with_bias = fused and delta_bias is not None
        inputs = [u, delta, A, B, C, D] + ([z] if fused else []) + ([delta_bias] if with_bias else [])
        if out is None:
            out = torch.empty(u.shape, dtype=torch.float32, device=u.device)
        return self.session(op, with_bias).run_device(
            [t.contiguous() for t in inputs], out, stream)

    def close(self):
        for s in self.sessions.values():
            s.close()
        self.sessions.clear()
