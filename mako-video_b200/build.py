"""Builds libh3b200.so in-tree for sm_100a: every csrc/*.cu and csrc/*.cpp through nvcc (relocatable device code,
one device link), linked against the NCCL that ships with the image's PyTorch. Objects are cached under _build/ and
rebuilt when a source or header is newer.

    python mako-video_b200/build.py [--jobs N] [--force]
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIBDIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIBDIR, "libh3b200.so")
REPO = os.path.dirname(HERE)
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs():
    """The NCCL headers and library of the installed PyTorch (nvidia-nccl wheel), else the system's."""
    for base in (sysconfig.get_paths()["purelib"], sysconfig.get_paths()["platlib"]):
        inc = os.path.join(base, "nvidia", "nccl", "include")
        lib = os.path.join(base, "nvidia", "nccl", "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")) and os.path.exists(os.path.join(lib, "libnccl.so.2")):
            return inc, lib
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def nvcc():
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", "nvcc"):
        if c and (os.path.exists(c) or c == "nvcc"):
            return c
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cu", ".cpp")))


def headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".hpp", ".h"))]
    hs.append(os.path.join(REPO, "include", "h3_c.h"))
    return hs


def compile_one(src, flags, force):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    newest = max([os.path.getmtime(src)] + [os.path.getmtime(h) for h in headers()] + [os.path.getmtime(__file__)])
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, None
    cmd = [nvcc()] + ARCH + flags + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, f"{' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, None


def build(jobs=8, force=False, verbose=False):
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    nccl_inc, nccl_lib = nccl_dirs()
    flags = ["-O3", "-std=c++17", "-rdc=true", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
             "-I", CSRC, "-I", os.path.join(REPO, "include"), "-I", nccl_inc, "--expt-relaxed-constexpr"]
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        results = list(ex.map(lambda s: compile_one(s, flags, force), srcs))
    errors = [e for _, e in results if e]
    if errors:
        raise RuntimeError("build failed:\n" + "\n".join(errors))
    objs = [o for o, _ in results]
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cmd = [nvcc()] + ARCH + ["-shared", "-rdc=true", "-o", LIB] + objs + [
            "-L", nccl_lib, "-l:libnccl.so.2", "-Xlinker", "-rpath", "-Xlinker", nccl_lib]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--jobs", type=int, default=os.cpu_count() or 8)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    try:
        build(a.jobs, a.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
