"""Build the in-tree CUDA library ``libtssm_b200.so`` for sm_100a with nvcc.

    python -m triton_ssm_b200.build [--force] [-j N]

Objects go to ``triton_ssm_b200/_build/`` and the shared library next to this
file, so it travels with the source tree.  Only files whose sources (or the
shared headers) changed are recompiled.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libtssm_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
                     "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))


def _stale(src, obj, hdr_mtime):
    if not os.path.exists(obj):
        return True
    om = os.path.getmtime(obj)
    return os.path.getmtime(src) > om or hdr_mtime > om


def _compile(nvcc, src, obj, extra):
    cmd = [nvcc] + NVCC_FLAGS + extra + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, " ".join(cmd), r.stderr[-6000:]))
    return obj


def build(force=False, jobs=None, verbose=False, extra_flags=()):
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdr = max([os.path.getmtime(h) for h in _headers()] + [0.0])
    objs, todo = [], []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(s, o, hdr):
            todo.append((s, o))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, list(extra_flags)) for s, o in todo]
            for f in futs:
                o = f.result()
                if verbose:
                    print("compiled", os.path.relpath(o, ROOT))
    if todo or force or not os.path.exists(LIB) or \
            any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [nvcc] + ARCH + ["-shared", "--cudart", "static", "-o", LIB + ".tmp"] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s\n%s" % (" ".join(cmd), r.stderr[-4000:]))
        os.replace(LIB + ".tmp", LIB)
        if verbose:
            print("linked", os.path.relpath(LIB, ROOT))
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    a = ap.parse_args(argv)
    build(force=a.force, jobs=a.j, verbose=True)


if __name__ == "__main__":
    sys.exit(main())
