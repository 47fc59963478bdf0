"""CPU: mamba-onnx_b200 builds as a wheel that carries the CUDA library, and an
install of that wheel resolves the ``cuda`` backend inside itself.

The reference's wheel carries only its cpp/zig libraries (build_backend.py:83-89)
and its loader looks in a development path (src/mamba_onnx/__init__.py:19-22).
"""
import os
import shutil
import subprocess
import sys
import zipfile
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "mamba-onnx_b200"
OUT = PKG / "_build" / "wheel_test"  # inside the package's git-ignored build folder


def _run(*cmd, **kw):
    return subprocess.run(list(cmd), capture_output=True, text=True, timeout=1200, **kw)


def test_wheel_carries_the_library_and_installs():
    shutil.rmtree(OUT, ignore_errors=True)
    (OUT / "dist").mkdir(parents=True)
    r = _run(sys.executable, "-m", "pip", "wheel", "--no-deps", "--no-build-isolation",
             "--no-index", "--wheel-dir", str(OUT / "dist"), str(PKG))
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    wheels = list((OUT / "dist").glob("mamba_onnx_cuda-*.whl"))
    assert len(wheels) == 1, wheels
    assert "linux" in wheels[0].name and "none-any" not in wheels[0].name
    names = set(zipfile.ZipFile(wheels[0]).namelist())
    for f in ("libmamba_ops_cuda.so", "__init__.py", "cuda.py", "model.py", "distributed.py"):
        assert f"mamba_onnx/{f}" in names, f

    site = OUT / "site"
    r = _run(sys.executable, "-m", "pip", "install", "--no-deps", "--no-index", "--target",
             str(site), str(wheels[0]))
    assert r.returncode == 0, r.stderr[-2000:]
    code = ("import ctypes, pathlib, mamba_onnx\n"
            "p = pathlib.Path(mamba_onnx.get_library_path('cuda'))\n"
            "assert p.parent == pathlib.Path(mamba_onnx.__file__).parent, p\n"
            "assert 'cuda' in mamba_onnx.available_backends()\n"
            "print(ctypes.CDLL(str(p)).mamba_scan_abi_version())\n")
    env = {k: v for k, v in os.environ.items() if k != "PYTHONPATH"}
    env["PYTHONPATH"] = str(site)
    r = _run(sys.executable, "-c", code, env=env, cwd=str(OUT))
    assert r.returncode == 0, r.stderr[-2000:]
    assert r.stdout.strip() == "2"
    assert str(site) in _run(sys.executable, "-c", "import mamba_onnx; print(mamba_onnx.__file__)",
                             env=env, cwd=str(OUT)).stdout
