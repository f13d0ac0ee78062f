"""Build the B200 library: pathpack.jl_b200/lib/libpathpack_b200.so (sm_100a).

    python pathpack.jl_b200/build.py [-j N] [--force]

Each CUDA/C++ source compiles to an object under pathpack.jl_b200/_build/ (rebuilt when it or a header is
newer), then one shared library is linked with the CUDA runtime linked statically, so the library needs
only the driver on the GPU box.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libpathpack_b200.so")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUFLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3",
                  "-I" + os.path.join(REPO, "include"), "-I" + CSRC]
CXXFLAGS = ["-O3", "-std=c++17", "-fPIC", "-Wall", "-I" + os.path.join(REPO, "include"), "-I" + CSRC,
            "-march=x86-64-v2"]


def _headers():
    hs = glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh"))
    hs.append(os.path.join(REPO, "include", "pathpack_b200.h"))
    return hs


def _compile(src, force, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in _headers()])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, None
    if src.endswith(".cu"):
        cmd = [NVCC] + CUFLAGS + ["-c", src, "-o", obj]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
    else:
        cmd = ["g++"] + CXXFLAGS + ["-I/usr/local/cuda/include", "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, "compile failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr)
    return obj, (r.stderr if verbose else None)


def build(jobs=None, force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    jobs = jobs or min(len(srcs), os.cpu_count() or 4)
    objs, errs = [], []
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        for obj, msg in ex.map(lambda s: _compile(s, force, verbose), srcs):
            objs.append(obj)
            if msg and msg.startswith("compile failed"):
                errs.append(msg)
            elif msg:
                print(msg)
    if errs:
        raise RuntimeError("\n".join(errs))
    newest = max(os.path.getmtime(o) for o in objs)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-Xcompiler", "-fPIC", "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed: %s\n%s\n%s" % (" ".join(cmd), r.stdout, r.stderr))
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", action="store_true", help="print ptxas register/spill info")
    a = ap.parse_args()
    try:
        print(build(a.j, a.force, a.v))
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
