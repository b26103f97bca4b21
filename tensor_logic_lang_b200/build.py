"""Build libtl_cuda.so in-tree for sm_100a (python -m tensor_logic_lang_b200.build).

Every source in csrc/ is compiled by nvcc with
`-gencode arch=compute_100a,code=sm_100a -lineinfo -O3` and linked into one
shared library next to this file, so the built library travels with the
source tree.  NCCL headers and library come from the nvidia-nccl wheel that
PyTorch uses (one NCCL in the process), with the system NCCL as fallback.
"""
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
OUT = os.path.join(PKG, "libtl_cuda.so")
BUILD_DIR = os.path.join(PKG, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_paths():
    try:
        import nvidia.nccl
        # a namespace package: no __file__, one directory in __path__
        base = list(nvidia.nccl.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return inc, lib
    except Exception:
        pass
    return "/usr/include", "/usr/lib/x86_64-linux-gnu"


def _compile(src, inc, verbose):
    obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(
            os.path.getmtime(src), *[os.path.getmtime(h) for h in glob.glob(os.path.join(CSRC, "*.h"))],
            os.path.getmtime(os.path.join(PKG, "..", "include", "tl_cuda.h"))):
        return obj, ""
    cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC,-O3", "-I", inc,
           "--expt-relaxed-constexpr", "-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd[1:1] = ["-x", "cu"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stderr}")
    return obj, r.stderr


def build(verbose=False, force=False):
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD_DIR, "*.o")):
            os.remove(o)
    inc, lib = nccl_paths()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        results = list(ex.map(lambda s: _compile(s, inc, verbose), srcs))
    if verbose:
        for _, log in results:
            if log:
                sys.stderr.write(log)
    objs = [o for o, _ in results]
    newest = max(os.path.getmtime(o) for o in objs)
    if not force and os.path.exists(OUT) and os.path.getmtime(OUT) >= newest:
        return OUT
    cmd = [NVCC, *ARCH, "-shared", "-o", OUT, *objs, "-L", lib, "-lnccl", f"-Xlinker=-rpath={lib}", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stderr}")
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
