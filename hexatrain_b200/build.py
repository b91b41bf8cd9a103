"""Builds libhexatrain_b200.so in-tree with nvcc for sm_100a.

Every ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in
parallel, skipped when up to date) and linked into
``hexatrain_b200/libhexatrain_b200.so`` with the CUDA runtime linked
statically, so the library has no dependency on PyTorch.
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libhexatrain_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                 "-Xptxas", "-warn-spills", f"-I{os.path.join(ROOT, 'include')}"]


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, extra) -> str:
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if _stale(obj, [src] + _headers()):
        cmd = [NVCC] + CFLAGS + list(extra) + ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip():
            sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False, extra=()) -> str:
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, extra), sources))
    if _stale(LIB, objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB, "-Xlinker", "-soname=libhexatrain_b200.so"] + objs + \
            ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    build_jni(verbose)
    if verbose:
        print(LIB)
    return LIB


JNI_SRC = os.path.join(HERE, "jni", "native_bridge_b200.cpp")
JNI_LIB = os.path.join(HERE, "libhexatrain_b200_jni.so")


def jni_include_dirs():
    """Directories holding a JDK's jni.h (and its platform jni_md.h), from
    HX_JNI_INCLUDE or JAVA_HOME; None when no JDK is present."""
    base = os.environ.get("HX_JNI_INCLUDE") or (
        os.path.join(os.environ["JAVA_HOME"], "include") if os.environ.get("JAVA_HOME") else None)
    if not base or not os.path.exists(os.path.join(base, "jni.h")):
        return None
    return [base] + [os.path.join(base, d) for d in ("linux",) if os.path.isdir(os.path.join(base, d))]


def build_jni(verbose: bool = False, include_dirs=None, out: str = JNI_LIB):
    """The JNI wrapper library (NativeBridge symbols over the bridge core).
    Skipped, returning None, when no jni.h is available."""
    inc = include_dirs or jni_include_dirs()
    if not inc:
        if verbose:
            print("no jni.h (set JAVA_HOME or HX_JNI_INCLUDE): JNI bridge not built")
        return None
    if not _stale(out, [JNI_SRC, LIB, os.path.join(ROOT, "include", "hexatrain_bridge.h")]):
        return out
    cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-o", out, JNI_SRC, f"-I{os.path.join(ROOT, 'include')}"]
    cmd += [f"-I{d}" for d in inc] + [f"-L{HERE}", "-lhexatrain_b200", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"JNI bridge build failed:\n{r.stdout}\n{r.stderr}")
    return out


if __name__ == "__main__":
    build(verbose=True, extra=sys.argv[1:])
