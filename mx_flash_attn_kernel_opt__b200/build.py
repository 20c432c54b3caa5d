"""Builds libpgqa.so in-tree with nvcc for sm_100a (no JIT cache: the .so travels with
the source tree)."""
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
SOURCES = [os.path.join(CSRC, "pgqa_decode.cu"), os.path.join(CSRC, "pgqa_append.cu"),
           os.path.join(CSRC, "pgqa_tc.cu")]
DEPS = SOURCES + [
    os.path.join(CSRC, "pgqa_append.h"),
    os.path.join(CSRC, "pgqa_partition.h"),
    os.path.join(CSRC, "pgqa_ptx.cuh"),
    os.path.join(CSRC, "pgqa_tc.h"),
    os.path.join(REPO_DIR, "include", "pgqa.h"),
]
LIB_NAME = "libpgqa.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found (set NVCC=...)")


def needs_build(lib=LIB_PATH):
    if not os.path.exists(lib):
        return True
    t = os.path.getmtime(lib)
    return any(os.path.getmtime(d) > t for d in DEPS)


def build(force=False, verbose=False, ptxas_verbose=False):
    """Compile csrc/*.cu (one nvcc per file, in parallel) and link libpgqa.so next to this
    file; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    from concurrent.futures import ThreadPoolExecutor
    nvcc = nvcc_path()
    objdir = os.path.join(PKG_DIR, "_build")
    os.makedirs(objdir, exist_ok=True)
    common = [*ARCH_FLAGS, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
              "--expt-relaxed-constexpr"]
    if ptxas_verbose:
        common.insert(0, "-Xptxas=-v")

    def compile_one(src):
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc, *common, "-c", "-o", obj, src]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src} ({res.returncode}):\n{res.stdout}\n{res.stderr}")
        if verbose or ptxas_verbose:
            print(res.stdout + res.stderr, file=sys.stderr)
        return obj

    with ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", "-o", tmp, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_verbose="-v" in sys.argv)
    print(LIB_PATH)
