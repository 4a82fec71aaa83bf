"""Build libytm.so in-tree for sm_100a (B200).

    python -m ytm_b200.build          # or ytm_b200.build.build()

nvcc cross-compiles without a GPU.  The library lands next to this file so it
travels with the source tree; nothing is installed into site-packages.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libytm.so")
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-shared",
    "--expt-relaxed-constexpr",
]


def nccl_flags() -> list[str]:
    """Include/link flags for NCCL: the headers of the NCCL wheel that torch
    loads (same version at run time), else the system's."""
    try:
        import nvidia.nccl as n  # the wheel torch depends on
        base = os.path.dirname(n.__file__) if getattr(n, "__file__", None) else list(n.__path__)[0]
        inc, lib = os.path.join(base, "include"), os.path.join(base, "lib")
        if os.path.exists(os.path.join(inc, "nccl.h")):
            return ["-I" + inc, "-L" + lib, "-l:libnccl.so.2"]
    except ImportError:
        pass
    return ["-lnccl"]


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(HERE, "..", "include", "ytm.h"), __file__]
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not _stale():
        return LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    tmp = LIB + ".tmp"
    cmd = [nvcc, *NVCC_FLAGS, *(extra or []), *sources(), *nccl_flags(), "-o", tmp]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


PROBE_SRC = os.path.join(HERE, "..", "bench_probe.cu")
PROBE_LIB = os.path.join(HERE, "..", "bench_probe.so")


def build_probe(force: bool = False) -> str | None:
    """bench.py's LOP3 throughput probe (not part of libytm), beside bench.py."""
    if not os.path.exists(PROBE_SRC):
        return None
    if not force and os.path.exists(PROBE_LIB) and os.path.getmtime(PROBE_LIB) >= os.path.getmtime(PROBE_SRC):
        return PROBE_LIB
    nvcc = os.environ.get("NVCC", "nvcc")
    subprocess.run([nvcc, *NVCC_FLAGS, PROBE_SRC, "-o", PROBE_LIB + ".tmp"], check=True)
    os.replace(PROBE_LIB + ".tmp", PROBE_LIB)
    return PROBE_LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True,
                extra=["-Xptxas", "-v"] if "--ptxas" in sys.argv else None))
