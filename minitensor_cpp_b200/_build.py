"""Build recipes for the native libraries of minitensor_cpp_b200.

libmtcuda.so        CUDA kernels for sm_100a behind the C ABI of include/mtcuda.h.
libminitensor_b200.so
                    MiniTensor's own C++20 front-end (Tensor / graph evaluator /
                    autograd / nn / optimizers), compiled from the reference source
                    tree with the two edits a new device needs, plus this package's
                    CUDA device runtime, kernel adapters and fusing evaluator
                    (minitensor_cpp_b200/host/).  The reference sources are only
                    read at build time; nothing of them is copied into the package.

Outputs go to minitensor_cpp_b200/lib/ (git-ignored, shipped with the tree);
objects go to _build/.  Everything is incremental on file modification times.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
HOST = PKG / "host"
LIB = PKG / "lib"
BUILD = ROOT / "_build"
INCLUDE = ROOT / "include"

CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]

CU_SOURCES = ["runtime.cu", "graph.cu", "elementwise.cu", "fused.cu", "copy.cu", "random.cu", "reduce.cu", "gemm.cu",
              "gemm_tc.cu", "comm.cu"]


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd, cwd=None):
    proc = subprocess.run(cmd, cwd=cwd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(map(str, cmd)) + "\n" + proc.stdout + proc.stderr)
    return proc


def _gen_template_include() -> Path:
    """Embeds ew_kernels.cuh as a C++ raw string for the NVRTC-compiled fused kernels."""
    gen = BUILD / "gen"
    gen.mkdir(parents=True, exist_ok=True)
    src = CSRC / "ew_kernels.cuh"
    out = gen / "ew_kernels_src.inc"
    if _newer(out, [src]):
        text = src.read_text()
        assert ")MTCSRC\"" not in text
        out.write_text('R"MTCSRC(' + text + ')MTCSRC"\n')
    return gen


def build_mtcuda(verbose: bool = False) -> Path:
    gen = _gen_template_include()
    obj_dir = BUILD / "mtcuda"
    obj_dir.mkdir(parents=True, exist_ok=True)
    LIB.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + [INCLUDE / "mtcuda.h", gen / "ew_kernels_src.inc"]
    jobs = []
    objs = []
    for name in CU_SOURCES:
        src = CSRC / name
        obj = obj_dir / (name + ".o")
        objs.append(obj)
        if _newer(obj, [src, *headers, Path(__file__)]):
            cmd = [NVCC, *ARCH, *NVCC_FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", f"-I{gen}", "-c", str(src), "-o", str(obj)]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for proc in ex.map(_run, jobs):
            if verbose and proc.stderr:
                print(proc.stderr)
    lib = LIB / "libmtcuda.so"
    if _newer(lib, objs):
        cuda_lib = CUDA_HOME / "lib64"
        cmd = [NVCC, *ARCH, "-shared", "-o", str(lib), *map(str, objs), f"-L{cuda_lib}", "-lnvrtc", "-ldl",
               "-lcudart", f"-Xlinker=-rpath={cuda_lib}"]
        _run(cmd)
    return lib


def build_all(verbose: bool = False) -> None:
    build_mtcuda(verbose)
    try:
        from . import _build_host
    except ImportError:  # host layer not present
        return
    _build_host.build(verbose)


if __name__ == "__main__":
    build_all(verbose=True)
