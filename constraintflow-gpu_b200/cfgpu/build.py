"""Build libcfgpu.so in-tree for sm_100a with nvcc (no JIT cache, no torch extension).

    python -m cfgpu.build        (from constraintflow-gpu_b200/)

Every csrc/*.cu file is compiled with
``-gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` into an object under
cfgpu/_objs/, then linked into cfgpu/libcfgpu.so.  Objects are rebuilt when their
source, any header, or the flags change.
"""
import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                       # constraintflow-gpu_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
OBJ_DIR = os.path.join(PKG_DIR, "_objs")
LIB = os.path.join(PKG_DIR, "libcfgpu.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: libcfgpu.so cannot be built")


def _headers_digest():
    h = hashlib.sha1()
    for d in (CSRC, INCLUDE):
        for f in sorted(os.listdir(d)):
            if f.endswith((".h", ".cuh")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    h.update(" ".join(FLAGS).encode())
    return h.hexdigest()


def _compile(src, obj, verbose):
    cmd = [nvcc()] + FLAGS + ["-c", src, "-o", obj]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(verbose=False, force=False, extra_flags=()):
    """Compile csrc/*.cu and link libcfgpu.so; returns the library path."""
    os.makedirs(OBJ_DIR, exist_ok=True)
    digest = _headers_digest() + hashlib.sha1(" ".join(extra_flags).encode()).hexdigest()
    stamp = os.path.join(OBJ_DIR, "stamp")
    old = open(stamp).read() if os.path.exists(stamp) else ""
    force = force or old != digest
    sources = sorted(f for f in os.listdir(CSRC) if f.endswith(".cu"))
    jobs = []
    objs = []
    for f in sources:
        src = os.path.join(CSRC, f)
        obj = os.path.join(OBJ_DIR, f[:-3] + ".o")
        objs.append(obj)
        if force or not os.path.exists(obj) or os.path.getmtime(obj) < os.path.getmtime(src):
            jobs.append((src, obj))
    if jobs:
        global FLAGS
        saved = FLAGS
        FLAGS = FLAGS + list(extra_flags)
        try:
            with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
                for msg in ex.map(lambda j: _compile(j[0], j[1], verbose), jobs):
                    if msg and verbose:
                        print(msg, end="")
        finally:
            FLAGS = saved
    if jobs or not os.path.exists(LIB):
        cmd = [nvcc()] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcuda"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    with open(stamp, "w") as fh:
        fh.write(digest)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
