"""Build libqdec.so in-tree (next to this file) for sm_100a.

    python qwen-3.8-in-rust_b200/build.py [--verbose-ptxas]

Every .cu / .cpp under csrc/ is compiled by nvcc into _build/*.o (rebuilt when the source or a header is
newer) and linked into libqdec.so with the CUDA runtime.  --fmad=false keeps every float multiply and add
separately rounded, the order the reference engine computes in.
"""
import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libqdec.so")
CLI = os.path.join(HERE, "qdec")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC,-O2,-ffp-contract=off",
         "-I" + os.path.join(HERE, "..", "include")]


def _newest_header():
    hs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
    hs.append(os.path.join(HERE, "..", "include", "qdec.h"))
    return max((os.path.getmtime(h) for h in hs if os.path.exists(h)), default=0)


def _compile(src, ptxas_v):
    obj = os.path.join(OBJ, os.path.basename(src) + ".o")
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), _newest_header()):
        return obj, None
    cmd = [NVCC] + ARCH + FLAGS + ["-c", src, "-o", obj]
    if ptxas_v and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stderr if ptxas_v else None)


def build(ptxas_v=False, quiet=True):
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp")))
    lib_srcs = [s for s in srcs if not os.path.basename(s).startswith("cli_")]
    cli_srcs = [s for s in srcs if os.path.basename(s).startswith("cli_")]
    with cf.ThreadPoolExecutor(max_workers=os.cpu_count() or 4) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_v), srcs))
    objs = {s: o for s, (o, _) in zip(srcs, results)}
    for s, (_, log) in zip(srcs, results):
        if log:
            print(f"== {os.path.basename(s)}\n{log}")
    lib_objs = [objs[s] for s in lib_srcs]
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in lib_objs):
        cmd = [NVCC] + ARCH + ["-shared", "-o", LIB] + lib_objs + ["-lcudart", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if cli_srcs:
        cli_objs = [objs[s] for s in cli_srcs]
        if not os.path.exists(CLI) or os.path.getmtime(CLI) < max(os.path.getmtime(o) for o in cli_objs + [LIB]):
            cmd = [NVCC] + ARCH + ["-o", CLI] + cli_objs + ["-L" + HERE, "-lqdec", "-Xlinker", "-rpath=$ORIGIN",
                                                          "-lcudart", "-lpthread"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"CLI link failed:\n{r.stdout}\n{r.stderr}")
    if not quiet:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    try:
        build(ptxas_v=a.verbose_ptxas, quiet=False)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
