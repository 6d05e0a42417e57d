"""Build the sm_100a library and its PyTorch glue in-tree.

    python llm-inference-kernels_b200/build.py

Produces, next to the `llmik_cuda` package sources:

* ``llmik_cuda/libllmik_b200.so`` - the CUDA kernels behind the C ABI of
  ``include/llmik.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``);
* ``llmik_cuda/_C<ext-suffix>`` - the PyTorch extension exporting the
  reference's ``llmik_cuda`` op surface, linked to the library above.

Both are built from this checkout only (no JIT cache under the home directory),
so the built files travel with the tree. Rebuilds are skipped when the outputs
are newer than every source.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
OUT = PKG_ROOT / "llmik_cuda"
BUILD = PKG_ROOT / "_build"
INCLUDE = REPO / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = {
    "decode.cu": [],
    "quantize.cu": ["-fmad=false"],   # bit-exact quantization: no contraction
    "cabi.cu": [],
    "noalloc.cu": [],
    "selftest.cu": [],
}
HEADERS = ["lik_device.cuh", "lik_internal.h"]


def _nvcc() -> str:
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda) / "bin" / "nvcc"
    return str(cand) if cand.exists() else (shutil.which("nvcc") or "nvcc")


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def lib_path() -> Path:
    return OUT / "libllmik_b200.so"


def ext_path() -> Path:
    return OUT / ("_C" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_library(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdrs = [CSRC / h for h in HEADERS] + [INCLUDE / "llmik.h"]
    objs = []
    for src, extra in CU_SOURCES.items():
        obj = BUILD / (Path(src).stem + ".o")
        if _stale(obj, [CSRC / src, *hdrs, Path(__file__)]):
            _run([_nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                  *extra, f"-I{INCLUDE}", "-c", CSRC / src, "-o", obj], verbose)
        objs.append(obj)
    lib = lib_path()
    if _stale(lib, objs):
        _run([_nvcc(), *ARCH, "-shared", "-o", lib, *objs], verbose)
    return lib


def build_extension(verbose: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    lib = build_library(verbose)
    ext = ext_path()
    src = CSRC / "torch_ext.cpp"
    if not _stale(ext, [src, lib, INCLUDE / "llmik.h", Path(__file__)]):
        return ext
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    incs = [*ce.include_paths(device_type="cuda"), sysconfig.get_paths()["include"], str(INCLUDE)]
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    incs.append(os.path.join(cuda_home, "include"))
    torch_lib = os.path.join(os.path.dirname(torch.__file__), "lib")
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_C",
           "-DTORCH_API_INCLUDE_EXTENSION_H",
           *[f"-I{i}" for i in incs], str(src), "-o", str(ext),
           f"-L{torch_lib}", "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python",
           "-lc10_cuda", "-ltorch_cuda",
           f"-L{OUT}", "-lllmik_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    _run(cmd, verbose)
    return ext


def build(verbose: bool = False) -> None:
    build_extension(verbose)


if __name__ == "__main__":
    build(verbose="-q" not in sys.argv)
