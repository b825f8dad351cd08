"""Build libtcb.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m tcb_b200.build          # or tcb_b200.build.build()

The library lands next to this file (tcb_b200/libtcb.so) so it travels
with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtcb.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
SOURCES = ["tcb_capi.cu", "tcb_dequant.cu", "tcb_gemv_simt.cu", "tcb_matvec.cu", "tcb_mv_q4k.cu", "tcb_mv_q6k.cu", "tcb_gemm_tc.cu", "tcb_gemm_i8.cu", "tcb_mv_rows.cu", "tcb_llama.cu", "tcb_static.cu", "tcb_attn_prefill.cu"]


def _stale(objs, deps) -> bool:
    if not all(os.path.exists(o) for o in objs):
        return True
    newest = max(os.path.getmtime(d) for d in deps)
    return any(os.path.getmtime(o) < newest for o in objs)


def build(verbose: bool = False, force: bool = False) -> str:
    bdir = os.path.join(HERE, "_build")
    os.makedirs(bdir, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    headers.append(os.path.join(os.path.dirname(HERE), "include", "tcb.h"))
    objs, cmds = [], []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(bdir, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale([o], [s] + headers):
            cmds.append([NVCC, *ARCH, *FLAGS, "-c", s, "-o", o])

    def compile_one(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)

    # the translation units are independent: compile them side by side
    with ThreadPoolExecutor(max_workers=max(1, min(len(cmds), os.cpu_count() or 1))) as ex:
        for f in [ex.submit(compile_one, c) for c in cmds]:
            f.result()
    if force or _stale([LIB], objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
