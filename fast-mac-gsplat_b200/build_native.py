"""Builds the sm_100a shared library libgsplat_b200.so in-tree with nvcc.

The library is plain CUDA C++ behind the C ABI in include/gsplat_b200.h (no
torch headers), so it builds in seconds on a CPU-only machine.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
REPO_ROOT = PKG_ROOT.parent
CSRC = PKG_ROOT / "csrc"
BUILD_DIR = PKG_ROOT / "_build"
LIB_PATH = PKG_ROOT / "torch_gsplat_bridge_fast" / "libgsplat_b200.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    return str(cand) if cand.exists() else "nvcc"


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    deps = [src] + sorted(CSRC.glob("*.cuh")) + [REPO_ROOT / "include" / "gsplat_b200.h"]
    if obj.exists() and all(obj.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return obj
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(REPO_ROOT / "include"), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    log = BUILD_DIR / (src.stem + ".ptxas.txt")
    log.write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    if verbose:
        print(res.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    BUILD_DIR.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(sources))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), sources))
    if LIB_PATH.exists() and all(LIB_PATH.stat().st_mtime >= o.stat().st_mtime for o in objs):
        return LIB_PATH
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
    return LIB_PATH


HOST_SRC = CSRC / "host_ops.cpp"


def _host_ext_path() -> Path:
    import sysconfig

    return PKG_ROOT / "torch_gsplat_bridge_fast" / ("_gsb_host" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_host(verbose: bool = False) -> Path:
    """Builds the native host runtime (_gsb_host, a torch C++ extension module)
    in-tree with g++, linked to libgsplat_b200.so through an $ORIGIN rpath."""
    import sysconfig

    import torch
    from torch.utils import cpp_extension as ce

    lib = build(verbose)
    out = _host_ext_path()
    deps = [HOST_SRC, lib, REPO_ROOT / "include" / "gsplat_b200.h"]
    if out.exists() and all(out.stat().st_mtime >= d.stat().st_mtime for d in deps):
        return out
    torch_inc = ce.include_paths()
    torch_lib = str(Path(torch.__file__).resolve().parent / "lib")
    cuda_home = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    abi = int(torch.compiled_with_cxx11_abi())
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", "-w", str(HOST_SRC), "-o", str(out),
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_gsb_host", "-DTORCH_API_INCLUDE_EXTENSION_H",
           "-I", str(REPO_ROOT / "include"), "-I", sysconfig.get_paths()["include"], "-I", str(cuda_home / "include")]
    for inc in torch_inc:
        cmd += ["-I", inc]
    cmd += ["-L", torch_lib, "-lc10", "-ltorch", "-ltorch_cpu", "-ltorch_python", "-lc10_cuda", "-ltorch_cuda",
            "-L", str(lib.parent), "-lgsplat_b200", "-Wl,-rpath,$ORIGIN", f"-Wl,-rpath,{torch_lib}"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"g++ failed for {HOST_SRC.name}:\n{res.stderr[-4000:]}")
    return out


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
    print(build_host(verbose="-v" in sys.argv))
