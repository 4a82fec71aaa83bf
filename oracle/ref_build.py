"""Compile the reference's own kernels into oracle/_ref/ (test infrastructure).

For each shape below this writes the macro preamble that Mayur1009/YTM
src/cutm/base.py:129-152 builds for that model, and runs nvcc on
oracle/ref_launcher.cu, which #includes the reference's
src/cutm/cuda/kernel.cu from the reference checkout (nothing is copied into
this repository).  Flags follow base.py:155-159 (-O3 --use_fast_math), with
the B200 architecture made explicit.  Outputs: oracle/_ref/ref_<shape>.so.

The reference checkout is only present on the build machine; the GPU box runs
the prebuilt .so files.  Usage:  python oracle/ref_build.py [--ref PATH]
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
# the reference checkout: $YTM_REFERENCE, else a `reference` directory beside
# this repository's root
DEFAULT_REF = os.environ.get("YTM_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
KERNEL_REL = os.path.join("src", "cutm", "cuda", "kernel.cu")

# name -> reference constructor kwargs (BaseTM.__init__, base.py:42-74).
# Every shape has LITERALS % 4 == 0: the reference's uint4 loads of TA states
# (kernel.cu:176, 412, 455, 483) are misaligned otherwise and fault.
SHAPES = {
    # inference shapes (any hyper-parameters)
    "inf_p1": dict(number_of_clauses_per_class=8, T=50, s=10.0, dim=(28, 28, 1), n_classes=10, coalesced=False),
    "inf_conv": dict(number_of_clauses_per_class=64, T=100, s=5.0, dim=(28, 28, 1), n_classes=10,
                     patch_dim=(10, 10)),
    "inf_rgb": dict(number_of_clauses_per_class=32, T=100, s=10.0, dim=(12, 12, 6), n_classes=4,
                    patch_dim=(5, 5)),
    "inf_nonsq": dict(number_of_clauses_per_class=24, T=10, s=3.0, dim=(9, 7, 2), n_classes=3,
                      patch_dim=(4, 4)),
    "inf_noloc": dict(number_of_clauses_per_class=16, T=10, s=3.0, dim=(8, 8, 1), n_classes=2,
                      patch_dim=(4, 4), encode_loc=False),
    "inf_noneg": dict(number_of_clauses_per_class=16, T=10, s=3.0, dim=(16, 1, 1), n_classes=2,
                      append_negated=False),
    "inf_4096": dict(number_of_clauses_per_class=40, T=100, s=20.0, dim=(64, 1, 1), n_classes=5,
                     number_of_ta_states=4096),
    # training shapes with every random decision forced: s = 1, q = K - 1, T = 1
    "tr_vanilla": dict(number_of_clauses_per_class=6, T=1, s=1.0, dim=(40, 1, 1), n_classes=3, q=2.0,
                       coalesced=False),
    "tr_coal": dict(number_of_clauses_per_class=24, T=1, s=1.0, dim=(40, 1, 1), n_classes=4, q=3.0),
    "tr_conv": dict(number_of_clauses_per_class=16, T=1, s=1.0, dim=(6, 6, 1), n_classes=3, q=2.0,
                    patch_dim=(4, 4)),
    # accuracy-parity shapes (configuration 1 / 2 rules, fewer clauses)
    "acc_vanilla": dict(number_of_clauses_per_class=50, T=15, s=3.9, dim=(28, 28, 1), n_classes=10, coalesced=False),
    "acc_coal": dict(number_of_clauses_per_class=400, T=100, s=5.0, dim=(28, 28, 1), n_classes=10),
    # configuration 2's model (10k shared clauses, T=1000, s=15), batch 1 as the reference trains
    "acc_c2": dict(number_of_clauses_per_class=10000, T=1000, s=15.0, dim=(28, 28, 1), n_classes=10),
    "tr_maxinc": dict(number_of_clauses_per_class=24, T=1, s=1.0, dim=(40, 1, 1), n_classes=4, q=3.0,
                      max_included_literals=3, negative_polarity=False),
}


def derived(kw):
    """Sizes per base.py:76-121."""
    dim = kw["dim"]
    K = kw["n_classes"]
    pd = kw.get("patch_dim", (dim[0], dim[1]))
    coalesced = kw.get("coalesced", True)
    banks = 1 if coalesced else K
    C = banks * kw["number_of_clauses_per_class"]
    if kw.get("encode_loc", True):
        L = pd[0] * pd[1] * dim[2] + (dim[0] - pd[0]) + (dim[1] - pd[1])
    else:
        L = pd[0] * pd[1] * dim[2]
    if kw.get("append_negated", True):
        L *= 2
    W = (L - 1) // 32 + 1
    P = (dim[0] - pd[0] + 1) * (dim[1] - pd[1] + 1)
    return dict(C=C, K=K, L=L, W=W, P=P, banks=banks, patch_dim=pd)


def preamble(kw) -> str:
    """The #define block of base.py:129-152 for these kwargs."""
    d = derived(kw)
    K = kw["n_classes"]
    q = min(float(kw.get("q", 1.0)), float(K))
    mil = kw.get("max_included_literals", None)
    h = [float(kw.get("h", 1.0))] * K
    lines = [
        f"#define CLAUSES {d['C']}",
        f"#define THRESH {kw['T']}",
        f"#define S {float(kw['s'])}",
        f"#define Q {q}",
        f"#define DIM0 {kw['dim'][0]}",
        f"#define DIM1 {kw['dim'][1]}",
        f"#define DIM2 {kw['dim'][2]}",
        f"#define PATCH_DIM0 {d['patch_dim'][0]}",
        f"#define PATCH_DIM1 {d['patch_dim'][1]}",
        f"#define PATCHES {d['P']}",
        f"#define LITERALS {d['L']}",
        f"#define MAX_INCLUDED_LITERALS {d['L'] if mil is None else mil}",
        f"#define APPEND_NEGATED {1 if kw.get('append_negated', True) else 0}",
        f"#define INIT_NEG_WEIGHTS {1 if kw.get('init_neg_weights', True) else 0}",
        f"#define NEGATIVE_CLAUSES {1 if kw.get('negative_polarity', True) else 0}",
        f"#define CLASSES {K}",
        f"#define MAX_TA_STATE {kw.get('number_of_ta_states', 256)}",
        f"#define ENCODE_LOC {1 if kw.get('encode_loc', True) else 0}",
        f"#define COALESCED {1 if kw.get('coalesced', True) else 0}",
        f"#define CLAUSE_BANKS {d['banks']}",
        "__constant__ const double H[%d] = {%s};" % (K, ",".join(map(str, h))),
        f"#define BIAS {1 if kw.get('bias', False) else 0}",
    ]
    return "\n".join(lines) + "\n"


def build(ref_root=DEFAULT_REF, names=None, quiet=False) -> list[str]:
    kernel = os.path.join(ref_root, KERNEL_REL)
    if not os.path.exists(kernel):
        raise FileNotFoundError(f"reference kernel not found: {kernel}")
    os.makedirs(OUT, exist_ok=True)
    built = []
    for name, kw in SHAPES.items():
        if names and name not in names:
            continue
        pre = os.path.join(OUT, f"pre_{name}.h")
        with open(pre, "w") as f:
            f.write(preamble(kw))
        so = os.path.join(OUT, f"ref_{name}.so")
        if os.path.exists(so) and os.path.getmtime(so) > max(
                os.path.getmtime(kernel), os.path.getmtime(os.path.join(HERE, "ref_launcher.cu")),
                os.path.getmtime(__file__)):
            built.append(so)
            continue
        cmd = ["nvcc", "-O3", "--use_fast_math", "-gencode", "arch=compute_100a,code=sm_100a",
               "-shared", "-Xcompiler", "-fPIC", "-w", "-include", pre, f'-DREF_KERNEL="{kernel}"',
               os.path.join(HERE, "ref_launcher.cu"), "-o", so]
        if not quiet:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        built.append(so)
    return built


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=DEFAULT_REF)
    ap.add_argument("names", nargs="*")
    a = ap.parse_args()
    for p in build(a.ref, a.names or None):
        print(p)
