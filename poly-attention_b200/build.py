"""Build libpolyattn.so (sm_100a) in-tree with nvcc.

    python poly-attention_b200/build.py [--debug]

Compiles every csrc/*.cu for arch sm_100a and links one shared library into
poly_attention_b200/libpolyattn.so. Objects are rebuilt only when a source
or header is newer than the library.
"""
from __future__ import annotations

import argparse
import glob
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "poly_attention_b200", "libpolyattn.so")
BUILD = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
         f"-I{os.path.join(ROOT, 'include')}", f"-I{CSRC}"]


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose=False, debug=False, ptxas_v=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    headers = sorted(glob.glob(os.path.join(CSRC, "*.cuh"))) + [os.path.join(ROOT, "include", "poly_attention.h")]
    flags = FLAGS + (["-DPOLY_DEBUG=1"] if debug else []) + (["-Xptxas", "-v"] if ptxas_v else [])
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s) + ".o")
        objs.append(o)
        if _stale(o, [s] + headers) or ptxas_v:
            jobs.append([NVCC, *flags, "-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0 or ptxas_v or "warning" in r.stderr:
            sys.stderr.write(r.stdout + r.stderr)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {cmd[-3]}")

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        list(ex.map(run, jobs))
    if jobs or _stale(OUT, objs):
        cmd = [NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", OUT, *objs, "-lcudart_static",
               "-ldl", "-lrt", "-lpthread"]
        run(cmd)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true")
    ap.add_argument("-v", action="store_true")
    args = ap.parse_args()
    print(build(verbose=args.v, debug=args.debug, ptxas_v=args.ptxas_v))
