"""Native build of the dlvk_b200 extension (`dlvk_b200/_C*.so`).

Every CUDA source is compiled by nvcc for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a -lineinfo`); host C++ sources are
compiled by g++.  The build is driven by a generated `build.ninja` under
`dlvk_b200/_build/` so rebuilds are incremental and parallel.  The finished
shared object is written next to this file (in-tree), so it travels with the
source tree and is imported directly by :mod:`dlvk_b200._ext` without any JIT
step at import time.

Kernel sources (`csrc/kernels/*.cu`) include no PyTorch headers, which keeps
their compile time to seconds; only `csrc/bindings/*.cpp` see torch.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
EXT_NAME = "_C"
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


LIB_NAME = "libdlvk_b200.so"  # kernels + runtime + ATen op layer + C++ API
BIN_DIR = PKG_DIR / "_bin"     # C++ programs built against the library (tests, examples)


def ext_path() -> Path:
    return PKG_DIR / (EXT_NAME + sysconfig.get_config_var("EXT_SUFFIX"))


def lib_path() -> Path:
    return PKG_DIR / LIB_NAME


def _torch_paths():
    import torch.utils.cpp_extension as ce  # noqa: WPS433

    inc = ce.include_paths(device_type="cuda")
    lib = ce.library_paths(device_type="cuda")
    return inc, lib


def _sources():
    cu = sorted(str(p) for p in (CSRC / "kernels").glob("*.cu"))
    cu += sorted(str(p) for p in (CSRC / "runtime").glob("*.cu"))
    cpp = sorted(str(p) for p in (CSRC / "runtime").glob("*.cpp"))
    cpp += sorted(str(p) for p in (CSRC / "ref").glob("*.cpp"))
    # ATen-level op wrappers and the C++ API: torch headers, no Python
    aten = sorted(str(p) for p in (CSRC / "aten").glob("*.cpp"))
    aten += sorted(str(p) for p in (CSRC / "api").glob("*.cpp"))
    bind = sorted(str(p) for p in (CSRC / "bindings").glob("*.cpp"))
    # C++ programs over the C++ API (built into _bin/)
    progs = sorted(str(p) for p in (CSRC / "tests").glob("cpp_api_*.cpp"))
    return cu, cpp, aten, bind, progs


def _q(s: str) -> str:
    return s.replace(" ", "$ ").replace(":", "$:")


def write_ninja(debug_bounds: bool = False) -> Path:
    import torch

    inc, lib = _torch_paths()
    py_inc = sysconfig.get_paths()["include"]
    own_inc = str(CSRC / "include")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = []
    if debug_bounds:
        defs.append("-DDLVK_DEBUG_BOUNDS=1")
    nvcc_flags = ARCH_FLAGS + [
        "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-Xptxas", "-v", f"-I{own_inc}",
        f"-I{CUDA_HOME}/include", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
    ] + defs
    cxx_flags = [
        "-O2", "-std=c++17", "-fPIC", "-Wall", "-Wno-unused-function",
        f"-I{own_inc}", f"-I{CUDA_HOME}/include", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
    ] + defs
    aten_flags = cxx_flags + [f"-I{p}" for p in inc] + ["-Wno-sign-compare"]
    bind_flags = aten_flags + [
        f"-I{py_inc}", f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
    ]
    # --no-as-needed: nothing references libtorch_cuda directly, but it must
    # be loaded for ATen's CUDA kernels to be registered in a C++ program.
    torch_libs = [f"-L{p}" for p in lib] + [f"-Wl,-rpath,{p}" for p in lib] + [
        "-Wl,--no-as-needed", "-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda", "-Wl,--as-needed",
        "-lcudart", "-lpthread"]
    lib_ldflags = ["-shared", f"-Wl,-soname,{LIB_NAME}"] + torch_libs
    # the module and the programs find the library next to them / one level up
    ldflags = ["-shared", f"-L{PKG_DIR}", f"-l:{LIB_NAME}", "-Wl,-rpath,'$$ORIGIN'"] + torch_libs + [
        "-ltorch_python"]
    prog_ldflags = [f"-L{PKG_DIR}", f"-l:{LIB_NAME}", "-Wl,-rpath,'$$ORIGIN/..'"] + torch_libs

    cu, cpp, aten, bind, progs = _sources()
    BUILD_DIR.mkdir(exist_ok=True)
    BIN_DIR.mkdir(exist_ok=True)
    lines = [
        "ninja_required_version = 1.3",
        f"nvcc = {CUDA_HOME}/bin/nvcc",
        "cxx = g++",
        "nvcc_flags = " + " ".join(nvcc_flags),
        "cxx_flags = " + " ".join(cxx_flags),
        "aten_flags = " + " ".join(aten_flags),
        "bind_flags = " + " ".join(bind_flags),
        "ldflags = " + " ".join(ldflags),
        "lib_ldflags = " + " ".join(lib_ldflags),
        "prog_ldflags = " + " ".join(prog_ldflags),
        "rule nvcc",
        "  command = $nvcc $nvcc_flags -MD -MF $out.d -c $in -o $out > $out.ptxas.log 2>&1 || (cat $out.ptxas.log; exit 1)",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = NVCC $in",
        "rule cxx",
        "  command = $cxx $cxx_flags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = CXX $in",
        "rule aten",
        "  command = $cxx $aten_flags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = ATEN $in",
        "rule bind",
        "  command = $cxx $bind_flags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  deps = gcc",
        "  description = BIND $in",
        "rule link_lib",
        "  command = $cxx $in $lib_ldflags -o $out",
        "  description = LINK $out",
        "rule link",
        "  command = $cxx $in $ldflags -o $out",
        "  description = LINK $out",
        "rule link_prog",
        "  command = $cxx $in $prog_ldflags -o $out",
        "  description = LINK $out",
    ]
    objs = []
    for src in cu:
        o = str(BUILD_DIR / (Path(src).stem + ".cu.o"))
        lines.append(f"build {_q(o)}: nvcc {_q(src)}")
        objs.append(o)
    for src in cpp:
        o = str(BUILD_DIR / (Path(src).parent.name + "_" + Path(src).stem + ".o"))
        lines.append(f"build {_q(o)}: cxx {_q(src)}")
        objs.append(o)
    for src in aten:
        o = str(BUILD_DIR / (Path(src).parent.name + "_" + Path(src).stem + ".o"))
        lines.append(f"build {_q(o)}: aten {_q(src)}")
        objs.append(o)
    libo = str(lib_path())
    lines.append(f"build {_q(libo)}: link_lib " + " ".join(_q(o) for o in objs))
    bobjs = []
    for src in bind:
        o = str(BUILD_DIR / ("bind_" + Path(src).stem + ".o"))
        lines.append(f"build {_q(o)}: bind {_q(src)}")
        bobjs.append(o)
    out = str(ext_path())
    lines.append(f"build {_q(out)}: link " + " ".join(_q(o) for o in bobjs) + f" | {_q(libo)}")
    targets = [out]
    for src in progs:
        o = str(BUILD_DIR / ("prog_" + Path(src).stem + ".o"))
        lines.append(f"build {_q(o)}: aten {_q(src)}")
        exe = str(BIN_DIR / Path(src).stem)
        lines.append(f"build {_q(exe)}: link_prog {_q(o)} | {_q(libo)}")
        targets.append(exe)
    lines.append("default " + " ".join(_q(t) for t in targets))
    path = BUILD_DIR / "build.ninja"
    path.write_text("\n".join(lines) + "\n")
    return path


def build(verbose: bool = False, debug_bounds: bool = False) -> Path:
    """Compile (incrementally) every native source and return the .so path."""
    ninja_file = write_ninja(debug_bounds=debug_bounds)
    ninja = shutil.which("ninja")
    if ninja is None:
        try:
            import ninja as _nj  # noqa: WPS433

            ninja = os.path.join(_nj.BIN_DIR, "ninja")
        except ImportError as exc:  # pragma: no cover
            raise RuntimeError("ninja is required to build dlvk_b200") from exc
    jobs = str(max(1, (os.cpu_count() or 2)))
    cmd = [ninja, "-f", str(ninja_file), "-j", jobs]
    if verbose:
        cmd.append("-v")
    res = subprocess.run(cmd, cwd=str(BUILD_DIR), capture_output=not verbose, text=True)
    if res.returncode != 0:
        msg = (res.stdout or "") + (res.stderr or "")
        raise RuntimeError("dlvk_b200 native build failed:\n" + msg[-20000:])
    return ext_path()


def ptxas_report() -> str:
    """Concatenated `-Xptxas -v` output (registers / spills / smem) of the last build."""
    out = []
    for log in sorted(BUILD_DIR.glob("*.ptxas.log")):
        out.append(f"== {log.name}\n" + log.read_text())
    return "\n".join(out)


if __name__ == "__main__":
    p = build(verbose="-v" in sys.argv, debug_bounds="--debug-bounds" in sys.argv)
    print(p)
