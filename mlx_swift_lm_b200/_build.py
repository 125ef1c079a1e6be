"""In-tree build of the native parts of the framework.

Two shared objects are produced under ``mlx_swift_lm_b200/_lib/``:

* ``libb200kernels.so`` - every CUDA kernel in ``csrc/kernels/*.cu``, compiled
  for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``) and exposed
  through a plain C ABI (loaded with ctypes). nvcc cross-compiles without a GPU.
  ``libb200kernels_checked.so`` is the same library built with
  ``-DB200_CHECKED=1`` (extra bounds checks that record a status code
  instead of trapping); ``B200LM_CHECKED=1`` loads it instead.
* ``_b200host*.so`` - the host runtime in ``csrc/host/*.cpp`` (page pool, block
  hasher, grammar engine, safetensors reader) as a pybind11
  module.

Sources are rebuilt only when they (or a header) are newer than the output.
Run it as a script (``python mlx_swift_lm_b200/_build.py``): importing the
package needs the host module that this build produces.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys
import sysconfig

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
LIBDIR = os.path.join(PKG, "_lib")
OBJDIR = os.path.join(LIBDIR, "obj")
KERNEL_SO = os.path.join(LIBDIR, "libb200kernels.so")
# bounds-checked variant (-DB200_CHECKED=1), loaded with B200LM_CHECKED=1
KERNEL_SO_CHECKED = os.path.join(LIBDIR, "libb200kernels_checked.so")
OBJDIR_CHECKED = os.path.join(LIBDIR, "obj_checked")
HOST_SO = os.path.join(LIBDIR, "_b200host" + sysconfig.get_config_var("EXT_SUFFIX"))

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I" + os.path.join(CSRC, "include")]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC", "-shared", "-Wall", "-Wno-unused-function"]


def _newer(src_files, out):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(s) > t for s in src_files)


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("build failed: " + " ".join(cmd) + "\n" + r.stdout + r.stderr)
    return r


def build_kernels(verbose: bool = False, jobs: int | None = None, checked: bool = False) -> str:
    objdir, out = (OBJDIR_CHECKED, KERNEL_SO_CHECKED) if checked else (OBJDIR, KERNEL_SO)
    flags = NVCC_FLAGS + (["-DB200_CHECKED=1"] if checked else [])
    os.makedirs(objdir, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "include", "*.cuh")) + glob.glob(os.path.join(CSRC, "include", "*.h"))
    sources = sorted(glob.glob(os.path.join(CSRC, "kernels", "*.cu")))
    objs = []
    todo = []
    for s in sources:
        o = os.path.join(objdir, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if _newer([s] + headers, o):
            todo.append((s, o))

    def compile_one(so):
        s, o = so
        cmd = [NVCC] + ARCH + flags + ["-c", s, "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        _run(cmd)
        return o

    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(compile_one, todo))
    if todo or _newer(objs, out):
        _run([NVCC] + ARCH + ["-shared", "-cudart", "static", "-o", out] + objs)
    return out


def build_host(verbose: bool = False) -> str:
    sources = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    headers = glob.glob(os.path.join(CSRC, "host", "*.h"))
    if not sources:
        return ""
    if not _newer(sources + headers, HOST_SO):
        return HOST_SO
    import pybind11

    inc = ["-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"], "-I" + os.path.join(CSRC, "host")]
    os.makedirs(LIBDIR, exist_ok=True)
    cmd = ["g++"] + CXX_FLAGS + inc + sources + ["-o", HOST_SO, "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    _run(cmd)
    return HOST_SO


def build_host_sanitized(outdir: str, sanitizer: str = "address,undefined") -> str:
    """The host module built with ``-fsanitize=<sanitizer>`` into `outdir`
    (same module name, so a process that puts `outdir` first on sys.path and
    preloads the sanitizer runtime imports the instrumented code)."""
    import pybind11

    sources = sorted(glob.glob(os.path.join(CSRC, "host", "*.cpp")))
    inc = ["-I" + pybind11.get_include(), "-I" + sysconfig.get_paths()["include"], "-I" + os.path.join(CSRC, "host")]
    os.makedirs(outdir, exist_ok=True)
    out = os.path.join(outdir, os.path.basename(HOST_SO))
    flags = [f for f in CXX_FLAGS if f != "-O3"] + ["-O1", "-g", "-fno-omit-frame-pointer", "-fsanitize=" + sanitizer,
                                                     "-fno-sanitize-recover=all"]
    _run(["g++"] + flags + inc + sources + ["-o", out, "-lpthread"])
    return out


def build_all(verbose: bool = False, checked: bool = True) -> None:
    """Release kernels, the host module, and (unless `checked` is False) the
    bounds-checked kernel variant."""
    with cf.ThreadPoolExecutor(max_workers=3) as ex:
        fk = ex.submit(build_kernels, verbose)
        fh = ex.submit(build_host, verbose)
        fc = ex.submit(build_kernels, verbose, None, True) if checked else None
        fk.result()
        fh.result()
        if fc is not None:
            fc.result()


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print(KERNEL_SO)
    print(HOST_SO)
