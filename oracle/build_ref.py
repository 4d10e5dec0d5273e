"""Build the reference plugin's own CUDA extension (vllm_espalier/csrc of the reference checkout) into oracle/_ref/.

Test infrastructure only: the built module is the *checker* used to pin the CPU oracle and to produce the golden
fixtures under tests/golden/ (tests/golden/make_golden.py). Nothing on the product path loads it.

The sources are compiled where they lie in the reference checkout (nothing is copied into this repository); only the
build products land in oracle/_ref/ (git-ignored). The recipe is ours: torch.utils.cpp_extension with explicit sm_100a
flags, the four translation units the reference's extension is made of (experts.cpp, experts.cu, dense.cu, route.cu).

usage: python oracle/build_ref.py --reference PATH   (or ESPALIER_REFERENCE=PATH)     (about 3 minutes on 8 cores)
"""
from __future__ import annotations

import argparse
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
SOURCES = ("experts.cpp", "experts.cu", "dense.cu", "route.cu")


def build(reference: Path, verbose: bool = False) -> Path | None:
    csrc = reference / "vllm_espalier" / "csrc"
    if not all((csrc / s).exists() for s in SOURCES):
        print(f"reference sources not found under {csrc}; oracle/_ref not built", file=sys.stderr)
        return None
    OUT.mkdir(exist_ok=True)
    from torch.utils.cpp_extension import load
    os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))
    mod = load(name="espalier_ref_ext", sources=[str(csrc / s) for s in SOURCES], build_directory=str(OUT),
               extra_cuda_cflags=["-O3", "-lineinfo", "-gencode", "arch=compute_100a,code=sm_100a"],
               extra_cflags=["-O3"], verbose=verbose)
    so = Path(mod.__file__)
    print(f"built {so}")
    return so


def main():
    ap = argparse.ArgumentParser()
    env = os.environ.get("ESPALIER_REFERENCE")
    ap.add_argument("--reference", type=Path, default=Path(env) if env else None, required=not env,
                    help="the reference checkout (default: $ESPALIER_REFERENCE)")
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", action="store_true")
    a = ap.parse_args()
    if a.clean and OUT.exists():
        shutil.rmtree(OUT)
    build(a.reference, a.v)


if __name__ == "__main__":
    main()
