"""Builds libminitensor_b200.so: MiniTensor's front-end with the CUDA backend.

The MiniTensor sources are compiled from the reference tree (read-only) with the
two edits a new device type needs, which no plugin can avoid, one that lets
the backend's new operations carry gradients, and one that lets a checkpoint
hold the optimizer state:

1. include/minitensor/types.hpp: `DeviceType::Cuda` and the `Device::cuda(i)`
   factory (the enum has only `Cpu` and Device's constructor is private,
   types.hpp:103-136);
2. src/tensor/execution/environment.cpp: the constructor calls
   `register_backend_extensions(runtimes_, kernels_)` after registering the CPU
   runtime and kernels (environment.cpp:16-20), and `evaluate` first offers the
   roots to `evaluate_with_backend_extensions` (environment.cpp:22-26).  Both
   hooks are weak symbols, so the edited file still links without a backend.
3. src/tensor/autograd/vjp_registry.cpp: the registry, built once from the
   reference's own rule sets, also calls `register_backend_vjps(registry)`
   (weak) after them, so relu (an operation this backend adds) has a VJP rule.
   The registry is a sealed function-local static (vjp_registry.cpp:36-48).
4. include/minitensor/nn/optimizers/adamw.hpp: `AdamW::State` befriends
   `minitensor::nn::AdamWStateAccess`, so a checkpoint can hold the step count
   and the moments, which the class keeps private (adamw.hpp:30-53) and the
   reference cannot persist yet (`persistence::Record` is only declared,
   random.hpp:13-16).

The edits are applied to a private working copy under the system temp
directory (never inside this repository); the objects and the library land in
_build/host/ and minitensor_cpp_b200/lib/.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import tempfile
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
HOST = PKG / "host"
LIB = PKG / "lib"
BUILD = ROOT / "_build" / "host"
INCLUDE = ROOT / "include"
# the MiniTensor sources: $MINITENSOR_REFERENCE, else the checkout "reference" beside this repository
REFERENCE = Path(os.environ.get("MINITENSOR_REFERENCE", ROOT.parent / "reference"))

CXX = os.environ.get("CXX", "g++")
# -fno-semantic-interposition: the library binds its own symbols (-Bsymbolic),
# so the compiler may inline calls between functions of one translation unit
# that -fPIC would otherwise treat as interposable (building a lazy graph makes
# many such small calls).
CXXFLAGS = ["-std=c++20", "-O3", "-DNDEBUG", "-fPIC", "-Wall", "-Wno-unused-parameter", "-fno-semantic-interposition"]
LDFLAGS: list[str] = []

# (file, anchor, replacement) edits; each anchor must occur exactly once.
EDITS = [
    ("include/minitensor/types.hpp",
     "enum class DeviceType : std::uint8_t\n{\n    Cpu,\n};",
     "enum class DeviceType : std::uint8_t\n{\n    Cpu,\n    Cuda,\n};"),
    ("include/minitensor/types.hpp",
     "        return Device{DeviceType::Cpu, index};\n    }\n",
     "        return Device{DeviceType::Cpu, index};\n    }\n"
     "    [[nodiscard]] static constexpr Device cuda(std::uint32_t index = 0) noexcept\n    {\n"
     "        return Device{DeviceType::Cuda, index};\n    }\n"),
    ("src/tensor/execution/environment.cpp",
     "namespace minitensor::detail\n{\nExecutionEnvironment::ExecutionEnvironment()",
     "namespace minitensor::detail\n{\n"
     "// Optional device backends (weak: absent unless a backend library defines them).\n"
     "[[gnu::weak]] void register_backend_extensions(RuntimeRegistry &runtimes, KernelRegistry &kernels);\n"
     "[[gnu::weak]] bool evaluate_with_backend_extensions(const RuntimeRegistry &runtimes, "
     "const KernelRegistry &kernels, std::span<const ValueRef> roots);\n\n"
     "ExecutionEnvironment::ExecutionEnvironment()"),
    ("src/tensor/execution/environment.cpp",
     "    cpu::register_kernels(kernels_);\n}",
     "    cpu::register_kernels(kernels_);\n"
     "    if (register_backend_extensions != nullptr)\n    {\n"
     "        register_backend_extensions(runtimes_, kernels_);\n    }\n}"),
    ("src/tensor/execution/environment.cpp",
     "void ExecutionEnvironment::evaluate(std::span<const ValueRef> roots)\n{\n",
     "void ExecutionEnvironment::evaluate(std::span<const ValueRef> roots)\n{\n"
     "    if (evaluate_with_backend_extensions != nullptr && "
     "evaluate_with_backend_extensions(runtimes_, kernels_, roots))\n    {\n        return;\n    }\n"),
    ("src/tensor/autograd/vjp_registry.cpp",
     "namespace minitensor::detail\n{\nvoid VjpRegistry::register_erased",
     "namespace minitensor::detail\n{\n"
     "// Optional rules of a device backend's own operations (weak: absent without one).\n"
     "[[gnu::weak]] void register_backend_vjps(VjpRegistry &registry);\n\n"
     "void VjpRegistry::register_erased"),
    ("include/minitensor/nn/optimizers/adamw.hpp",
     "        friend class AdamW;\n        friend State leafify_optimizer_state(State state);",
     "        friend class AdamW;\n        friend State leafify_optimizer_state(State state);\n"
     "        friend struct AdamWStateAccess;  // checkpoints of the backend build"),
    ("src/tensor/autograd/vjp_registry.cpp",
     "        register_reduction_vjps(result);\n        return result;",
     "        register_reduction_vjps(result);\n"
     "        if (register_backend_vjps != nullptr)\n        {\n            register_backend_vjps(result);\n        }\n"
     "        return result;"),
]

HOST_SOURCES = ["cuda_runtime.cpp", "cuda_kernels.cpp", "cuda_evaluator.cpp", "extensions.cpp", "ops_ext.cpp",
                "workloads.cpp"]


def _run(cmd):
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError("command failed:\n" + " ".join(map(str, cmd)) + "\n" + proc.stdout + proc.stderr)
    return proc


def _working_copy() -> Path:
    """Copies the reference include/ and src/ trees to a temp dir and applies EDITS."""
    digest = hashlib.sha1()
    files = sorted(p for p in (list((REFERENCE / "include").rglob("*")) + list((REFERENCE / "src").rglob("*")))
                   if p.is_file())
    for p in files:
        digest.update(str(p.relative_to(REFERENCE)).encode())
        digest.update(str(p.stat().st_mtime_ns).encode())
    digest.update(repr(EDITS).encode())
    work = Path(tempfile.gettempdir()) / f"mtb_reference_{digest.hexdigest()[:12]}"
    stamp = work / ".complete"
    if stamp.exists():
        return work
    if work.exists():
        shutil.rmtree(work)
    for sub in ("include", "src"):
        shutil.copytree(REFERENCE / sub, work / sub)
    for rel, anchor, replacement in EDITS:
        path = work / rel
        text = path.read_text()
        if text.count(anchor) != 1:
            raise RuntimeError(f"edit anchor not found exactly once in {rel}: {anchor!r}")
        path.write_text(text.replace(anchor, replacement))
    stamp.write_text("ok")
    return work


def _newer(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(verbose: bool = False) -> Path | None:
    lib = LIB / "libminitensor_b200.so"
    if not REFERENCE.exists():
        if lib.exists():
            return lib  # prebuilt (the reference tree is only needed to build)
        raise RuntimeError(f"MiniTensor sources not found at {REFERENCE}; set MINITENSOR_REFERENCE")
    work = _working_copy()
    BUILD.mkdir(parents=True, exist_ok=True)
    includes = [f"-I{work / 'include'}", f"-I{work / 'src'}", f"-I{INCLUDE}", f"-I{HOST}"]
    ref_sources = sorted((work / "src").rglob("*.cpp"))
    host_headers = list(HOST.glob("*.hpp")) + [INCLUDE / "mtcuda.h"]
    jobs, objs = [], []
    for src in ref_sources:
        obj = BUILD / "ref" / (str(src.relative_to(work / "src")).replace("/", "__") + ".o")
        objs.append(obj)
        if _newer(obj, [src, Path(__file__)]):
            obj.parent.mkdir(parents=True, exist_ok=True)
            jobs.append([CXX, *CXXFLAGS, *includes, "-c", str(src), "-o", str(obj)])
    for name in HOST_SOURCES:
        src = HOST / name
        obj = BUILD / (name + ".o")
        objs.append(obj)
        if _newer(obj, [src, *host_headers, Path(__file__)]):
            jobs.append([CXX, *CXXFLAGS, *includes, "-c", str(src), "-o", str(obj)])
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        for proc in ex.map(_run, jobs):
            if verbose and proc.stderr:
                print(proc.stderr)
    mtcuda = LIB / "libmtcuda.so"
    if _newer(lib, objs + [mtcuda]):
        _run([CXX, "-shared", *LDFLAGS, "-Wl,-Bsymbolic", "-o", str(lib), *map(str, objs), f"-L{LIB}", "-lmtcuda",
              "-Wl,-rpath,$ORIGIN"])
    return lib


if __name__ == "__main__":
    print(build(verbose=True))
