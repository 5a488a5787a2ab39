"""Build libmoe_b200.so in-tree from mvcc_b200/csrc with nvcc for sm_100a.

    python mvcc_b200/build.py [--verbose] [--force]

Each .cu and .cpp file compiles to an object in mvcc_b200/_build/ (in parallel), then one shared library is linked next to
this file, where mvcc_b200/__init__.py loads it. Rebuilds only what changed (source or header newer than object).
"""
import concurrent.futures
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmoe_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

NVCC = os.environ.get("NVCC", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr", "-I" + INCLUDE]


def _sources():
    return sorted(f for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def _headers_mtime():
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    paths += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def _compile(src, verbose):
    obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", os.path.join(CSRC, src), "-o", obj]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False, force=False):
    os.makedirs(BUILD, exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    objs = []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.splitext(src)[0] + ".o")
        objs.append(obj)
        s_m = max(os.path.getmtime(os.path.join(CSRC, src)), hdr)
        if force or verbose or not os.path.exists(obj) or os.path.getmtime(obj) < s_m:
            todo.append(src)
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, max(1, len(todo)))) as ex:
        for obj, log in ex.map(lambda s: _compile(s, verbose), todo):
            if verbose and log:
                sys.stderr.write(log)
    if todo or not os.path.exists(LIB):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="--verbose" in sys.argv, force="--force" in sys.argv))
