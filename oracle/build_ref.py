"""Compile the reference's own append / exact-tail extension
(tests/page_gauge_append_extension.cu of ahmed123hds/PageGauge, one source
file) for sm_100a into oracle/_ref/, as a checker for the GPU parity tests.

Test infrastructure only: the product never loads it.  The recipe is this
script's own (torch.utils.cpp_extension with the flags the reference's
loader passes, scripts/page_gauge_runtime.py:16-29: -O3, no fast-math);
the source is compiled where it lies and is not copied.  Without the
reference checkout (e.g. on a GPU box) it does nothing; the built module
travels with the tree.

    python oracle/build_ref.py [--reference /path/to/PageGauge]
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
NAME = "page_gauge_append_ext_ref"
SOURCE = Path("tests") / "page_gauge_append_extension.cu"


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    # Default: $PAGEGAUGE_REFERENCE, else a "reference" checkout beside this
    # repository.
    default = os.environ.get("PAGEGAUGE_REFERENCE") or str(HERE.parent.parent / "reference")
    parser.add_argument("--reference", type=Path, default=Path(default))
    args = parser.parse_args()
    src = args.reference / SOURCE
    if not src.is_file():
        print(f"reference source not found ({src}); nothing to build")
        return 0
    OUT.mkdir(exist_ok=True)
    built = OUT / (NAME + ".so")
    if built.is_file() and built.stat().st_mtime >= src.stat().st_mtime:
        print(f"{built} is up to date")
        return 0
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0a"
    os.environ.setdefault("MAX_JOBS", "4")
    from torch.utils.cpp_extension import load

    load(name=NAME, sources=[str(src)], build_directory=str(OUT), extra_cflags=["-O3"],
         extra_cuda_cflags=["-O3"], verbose=False)
    print(f"built {OUT / (NAME + '.so')}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
