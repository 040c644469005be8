"""Build the native extensions in-tree (no pip install): ``python -m minisgl._build``.

* ``minisgl/_host*.so``     - host C++ runtime (radix tree), pybind11 only.
* ``minisgl/_cuda*.so``     - sm_100a CUDA kernels + torch bindings.
* ``minisgl/_cuda_bc*.so``  - the same kernels compiled with ``-DMINISGL_BOUNDS_CHECK=1``: every
  data-dependent index (token ids, KV slots, positions, page-table rows and entries, MoE rows) is
  checked, a violation is recorded in the device error word and the access is skipped. Loaded
  instead of ``_cuda`` when ``MINISGL_BOUNDS_CHECK=1``.

CUDA sources are compiled with ``-gencode arch=compute_100a,code=sm_100a`` only. Kernel .cu files
do not include torch headers (fast to compile); ``csrc/bindings.cpp`` adapts tensors to them.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys
import sysconfig

ROOT = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(ROOT, "csrc")
BUILD = os.path.join(os.path.dirname(ROOT), "_build")
EXT_SUFFIX = sysconfig.get_config_var("EXT_SUFFIX")
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _py_includes():
    import pybind11

    return [sysconfig.get_paths()["include"], pybind11.get_include()]


def _torch_paths():
    import torch.utils.cpp_extension as ce

    return ce.include_paths(), ce.library_paths()


def _cuda_home() -> str:
    return os.environ.get("CUDA_HOME", "/usr/local/cuda")


def _abi_flag() -> str:
    import torch

    return f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"


def _write_ninja(path: str, text: str) -> None:
    old = open(path).read() if os.path.exists(path) else None
    if old != text:
        with open(path, "w") as f:
            f.write(text)


def host_target() -> str:
    return os.path.join(ROOT, "_host" + EXT_SUFFIX)


def cuda_target(bounds_check: bool = False) -> str:
    return os.path.join(ROOT, ("_cuda_bc" if bounds_check else "_cuda") + EXT_SUFFIX)


def ninja_file() -> str:
    os.makedirs(BUILD, exist_ok=True)
    cuda = _cuda_home()
    pyinc = _py_includes()
    tinc, tlib = _torch_paths()
    inc = " ".join(f"-I{p}" for p in [CSRC] + pyinc)
    tinc_s = " ".join(f"-isystem {p}" for p in tinc)
    lines = [
        "ninja_required_version = 1.3",
        f"cxx = g++",
        f"nvcc = {cuda}/bin/nvcc",
        f"cxxflags = -O3 -std=c++17 -fPIC -fvisibility=hidden {inc} {_abi_flag()}",
        f"torchflags = {tinc_s} -DTORCH_API_INCLUDE_EXTENSION_H",
        f"nvccflags = -O3 -std=c++17 {' '.join(GENCODE)} -lineinfo --expt-relaxed-constexpr "
        f"-Xcompiler -fPIC -Xcompiler -fvisibility=hidden {inc} -I{cuda}/include "
        f"-DNDEBUG -Xptxas -warn-spills",
        "rule cxx",
        "  command = $cxx -MMD -MF $out.d $cxxflags $extra -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "rule nvcc",
        "  command = $nvcc -MD -MF $out.d $nvccflags $extra -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "rule link",
        "  command = $cxx -shared $in -o $out $ldflags",
        "",
    ]
    # host runtime
    host_srcs = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    host_objs = []
    for s in host_srcs:
        o = os.path.join(BUILD, "host_" + os.path.basename(s) + ".o")
        host_objs.append(o)
        lines.append(f"build {o}: cxx {s}")
    lines.append(f"build {host_target()}: link {' '.join(host_objs)}")
    lines.append("  ldflags = ")
    # cuda kernels: release and bounds-check variants of the same sources
    cu_srcs = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    bind = os.path.join(CSRC, "bindings.cpp")
    libdirs = " ".join(f"-L{p} -Wl,-rpath,{p}" for p in tlib)
    for bc in (False, True):
        tag = "bc_" if bc else ""
        name = "_cuda_bc" if bc else "_cuda"
        cu_objs = []
        for s in cu_srcs:
            o = os.path.join(BUILD, f"cu_{tag}" + os.path.basename(s) + ".o")
            cu_objs.append(o)
            lines.append(f"build {o}: nvcc {s}")
            if bc:
                lines.append("  extra = -DMINISGL_BOUNDS_CHECK=1")
        bind_o = os.path.join(BUILD, f"bindings_{tag}.o" if bc else "bindings.o")
        lines.append(f"build {bind_o}: cxx {bind}")
        lines.append(f"  extra = $torchflags -DTORCH_EXTENSION_NAME={name} -I{cuda}/include")
        lines.append(f"build {cuda_target(bc)}: link {' '.join(cu_objs + [bind_o])}")
        lines.append(
            f"  ldflags = {libdirs} -L{cuda}/lib64 -lc10 -ltorch -ltorch_cpu -ltorch_python "
            f"-lc10_cuda -ltorch_cuda -lcudart"
        )
    path = os.path.join(BUILD, "build.ninja")
    _write_ninja(path, "\n".join(lines) + "\n")
    return path


def build(targets: list[str] | None = None, jobs: int | None = None, verbose: bool = False) -> None:
    path = ninja_file()
    cmd = ["ninja", "-f", path]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd += ["-v"]
    cmd += targets or []
    r = subprocess.run(cmd, cwd=BUILD, capture_output=not verbose, text=True)
    if r.returncode != 0:
        sys.stderr.write((r.stdout or "") + (r.stderr or ""))
        raise RuntimeError("native build failed")


def build_host() -> None:
    build([host_target()])


if __name__ == "__main__":
    names = {"host": host_target(), "cuda": cuda_target(), "bounds": cuda_target(True)}
    which = [w for w in sys.argv[1:] if w in names]
    build([names[w] for w in which] or None, verbose="-v" in sys.argv)
