"""Build libpm_sample.so (the C ABI of include/pm_sample.h) for sm_100a.

nvcc cross-compiles without a GPU.  The library is written next to this file
(git-ignored, but it travels with the repository snapshot to the GPU box).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
SO = os.path.join(HERE, "libpm_sample.so")
SOURCES = ["pm_sample.cu", "pm_masked.cu", "pm_lmhead.cu"]
OBJDIR = os.path.join(HERE, "_build")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


class CompilerMissing(RuntimeError):
    """No compiler on this machine: a prebuilt library is used as it is.
    Any other build failure is an error (never a silent fall back to a stale
    library)."""


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise CompilerMissing("nvcc not found")


def sources() -> list:
    return [os.path.join(CSRC, s) for s in SOURCES if os.path.exists(os.path.join(CSRC, s))]


def _headers() -> list:
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    return hs + [os.path.join(ROOT, "include", "pm_sample.h")]


def _stale() -> bool:
    if not os.path.exists(SO):
        return True
    t = os.path.getmtime(SO)
    return any(os.path.getmtime(d) > t for d in sources() + _headers() if os.path.exists(d))


class _BuildLock:
    """An exclusive lock on a file beside the library while a build runs:
    processes that start together (ranks of one job, test workers) build
    once, the others wait and then find the outputs fresh."""

    def __enter__(self):
        import fcntl
        self.f = open(os.path.join(HERE, ".build.lock"), "a+")
        fcntl.flock(self.f, fcntl.LOCK_EX)
        return self

    def __exit__(self, *exc):
        import fcntl
        fcntl.flock(self.f, fcntl.LOCK_UN)
        self.f.close()


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every translation unit (in parallel) and link the library."""
    if not force and not _stale():
        return SO
    with _BuildLock():
        if not force and not _stale():
            return SO
        return _build_locked(verbose)


def _build_locked(verbose: bool) -> str:
    os.makedirs(OBJDIR, exist_ok=True)
    cc = nvcc()
    procs = []
    objs = []
    for src in sources():
        obj = os.path.join(OBJDIR, os.path.basename(src) + ".o")
        objs.append(obj)
        cmd = [cc, *NVCC_FLAGS, "-c", "-o", obj + f".{os.getpid()}.tmp", src]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    failed = False
    for obj, pr in procs:
        out, _ = pr.communicate()
        if pr.returncode != 0:
            sys.stderr.write(out)
            failed = True
        else:
            if verbose and out:
                sys.stderr.write(out)
            os.replace(obj + f".{os.getpid()}.tmp", obj)
    if failed:
        raise RuntimeError("nvcc failed building libpm_sample.so")
    tmp = SO + f".{os.getpid()}.tmp"
    cmd = [cc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", tmp, *objs, "-lcudart"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("linking libpm_sample.so failed")
    os.replace(tmp, SO)
    return SO


EXT_SRC = os.path.join(CSRC, "pm_torch.cpp")


def ext_path() -> str:
    import sysconfig
    return os.path.join(HERE, "_pm_torch" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_ext(force: bool = False, verbose: bool = False) -> str:
    """Compile the PyTorch extension module _pm_torch (pm_torch.cpp) against
    torch's headers, linked to libpm_sample.so beside it (rpath $ORIGIN)."""
    out = ext_path()
    # the module links libpm_sample.so dynamically: only its own source and
    # the C ABI's header make it stale
    deps = [EXT_SRC, os.path.join(ROOT, "include", "pm_sample.h")]

    def fresh():
        return os.path.exists(out) and all(os.path.getmtime(d) <= os.path.getmtime(out) for d in deps)

    if not force and fresh():
        return out
    with _BuildLock():
        if not force and fresh():
            return out
        return _build_ext_locked(out, verbose)


def _build_ext_locked(out: str, verbose: bool) -> str:
    import sysconfig
    cxx = os.environ.get("CXX", "g++")
    if not shutil.which(cxx):
        raise CompilerMissing(f"{cxx} not found")
    import torch
    from torch.utils import cpp_extension as ce
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={abi}", "-DTORCH_EXTENSION_NAME=_pm_torch", "-DTORCH_API_INCLUDE_EXTENSION_H",
           f"-I{sysconfig.get_paths()['include']}", f"-I{os.path.join(cuda_home, 'include')}"]
    cmd += [f"-I{p}" for p in ce.include_paths()]
    tmp = out + f".{os.getpid()}.tmp"
    cmd += ["-o", tmp, EXT_SRC]
    cmd += [f"-L{p}" for p in ce.library_paths()]
    cmd += [f"-L{HERE}", "-lpm_sample", "-Wl,-rpath,$ORIGIN",
            "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
            f"-L{os.path.join(cuda_home, 'lib64')}", "-lcudart"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError("building the _pm_torch extension failed")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(SO)
    print(build_ext(force="--force" in sys.argv, verbose=True))
