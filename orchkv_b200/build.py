"""Build the orchkv B200 native library and the `orchkv_core` Python module.

    python -m orchkv_b200.build          # incremental
    python -m orchkv_b200.build --clean  # rebuild everything
    python -m orchkv_b200.build --checked  # also the bounds-checked build

Outputs (in-tree, git-ignored, shipped with the working tree):
    orchkv_b200/liborchkv_b200.so               C ABI: orchkv_* and tm_*
    orchkv_b200/orchkv_core<ext-suffix>.so      pybind11 module (same names as
                                                the reference binding)
    orchkv_b200/_checked/...                    the same two, built with
                                                -DOKV_CHECKED (--checked;
                                                selected by ORCHKV_CHECKED=1)
Every CUDA source is compiled for sm_100a only.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
INCLUDE = os.path.join(ROOT, "include")
LIB = os.path.join(PKG, "liborchkv_b200.so")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                  "-Xcompiler", "-Wall", "-I" + INCLUDE, "-I" + CSRC]

CU_SOURCES = ["sched_kernels.cu", "select_kernels.cu", "pool_kernels.cu", "tm.cu",
              "api.cu", "comm.cu", "static_select.cu", "manager_kernels.cu",
              "integrity_kernels.cu"]


CHECKED = os.path.join(PKG, "_checked")        # the checked build's library and module


def core_module_path(directory: str = PKG) -> str:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    return os.path.join(directory, "orchkv_core" + suffix)


def _headers():
    hs = []
    for d in (CSRC, os.path.join(INCLUDE, "orchkv")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh")):
                hs.append(os.path.join(d, f))
    return hs


def _newer(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def _run(cmd):
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("build step failed:\n" + " ".join(cmd) + "\n" + r.stdout)
    return r.stdout


def build(clean: bool = False, verbose: bool = False, checked: bool = False) -> None:
    """The regular build into orchkv_b200/, or with checked=True the
    bounds-checked build (-DOKV_CHECKED) into orchkv_b200/_checked/."""
    out_dir = CHECKED if checked else PKG
    obj_dir = BUILD + "_checked" if checked else BUILD
    lib = os.path.join(out_dir, "liborchkv_b200.so")
    flags = NVFLAGS + (["-DOKV_CHECKED"] if checked else [])
    os.makedirs(obj_dir, exist_ok=True)
    os.makedirs(out_dir, exist_ok=True)
    hdrs = _headers()
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(obj_dir, src.replace(".cu", ".o"))
        objs.append(o)
        if clean or _newer(o, [s] + hdrs):
            jobs.append([NVCC] + flags + ["-c", s, "-o", o])
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        for out in ex.map(_run, jobs):
            if verbose and out.strip():
                print(out)
    if clean or _newer(lib, objs):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", lib] + objs +
             ["-Xlinker", "-soname=liborchkv_b200.so", "-Xlinker", "-Bsymbolic",
              "-lpthread", "-ldl"])

    # pybind11 module linking the library above (rpath $ORIGIN)
    import pybind11
    mod = core_module_path(out_dir)
    src = os.path.join(CSRC, "pybind_module.cpp")
    if clean or _newer(mod, [src, lib] + hdrs):
        py_inc = sysconfig.get_paths()["include"]
        _run(["g++", "-O2", "-std=c++17", "-shared", "-fPIC", "-fvisibility=hidden",
              "-I" + py_inc, "-I" + pybind11.get_include(), "-I" + INCLUDE,
              "-I/usr/local/cuda/include", src, "-o", mod, "-L" + out_dir,
              "-l:liborchkv_b200.so", "-Wl,-rpath,$ORIGIN"])


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("--checked", action="store_true", help="also the bounds-checked build")
    a = ap.parse_args(argv)
    build(clean=a.clean, verbose=a.verbose)
    print("built", LIB, core_module_path())
    if a.checked:
        build(clean=a.clean, verbose=a.verbose, checked=True)
        print("built", os.path.join(CHECKED, "liborchkv_b200.so"), core_module_path(CHECKED))


if __name__ == "__main__":
    sys.exit(main())
