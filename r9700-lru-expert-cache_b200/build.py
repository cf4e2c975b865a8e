"""Build the two C-ABI shared libraries of this package, in-tree, for sm_100a.

* ``librlu.so``       -- csrc/lru.cu: r4d_lru_manage / r4d_lru_fused / r4d_lru_gather.
* ``libb200lmhead.so`` -- csrc/quant.cu + csrc/lmhead.cu + csrc/gate.cu + csrc/moe_sum.cu +
  csrc/moe_gemm.cu: SiLU-mul FP8 quant, per-token (group) FP8 quant, FP8 and W4 lm_head
  GEMVs, the stream control, the shared-expert gate, the routed experts' sum and the grouped
  MXFP4 x FP8 MoE GEMM.

No fast math: the SiLU-quant parity needs IEEE division and the accurate expf.
Usage: ``python build.py [--force]`` (also called by ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared",
         "--expt-relaxed-constexpr"]

LIBS = {
    "librlu.so": ["lru.cu"],
    "libb200lmhead.so": ["quant.cu", "lmhead.cu", "gate.cu", "moe_sum.cu", "moe_gemm.cu"],
}


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _stale(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    deps = srcs + [os.path.join(CSRC, "common.cuh"), os.path.abspath(__file__)]
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> list[str]:
    nvcc = _nvcc()
    built = []
    for lib, files in LIBS.items():
        out = os.path.join(HERE, lib)
        srcs = [os.path.join(CSRC, f) for f in files]
        if not force and not _stale(out, srcs):
            continue
        cmd = [nvcc, *ARCH, *FLAGS, "-I", CSRC, *srcs, "-o", out + ".tmp"]
        if verbose:
            print(" ".join(cmd))
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {lib}:\n{r.stdout}\n{r.stderr}")
        os.replace(out + ".tmp", out)
        built.append(out)
    return built


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose=True):
        print("built", p)
