"""Build libpagegauge_b200.so in-tree with nvcc for sm_100a.

    python -m pagegauge_b200.build [--force]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parent
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
OUTPUT = ROOT / "libpagegauge_b200.so"
SOURCES = [CSRC / "pg_capi.cu"]
DEPENDS = SOURCES + sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    return str(Path(cuda) / "bin" / "nvcc")


def command(output: Path = OUTPUT) -> list[str]:
    return [
        nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-shared", "-Xptxas", "-v",
        "-I", str(INCLUDE),
        "-o", str(output), *map(str, SOURCES),
    ]


def up_to_date() -> bool:
    if not OUTPUT.is_file():
        return False
    built = OUTPUT.stat().st_mtime
    return all(path.stat().st_mtime <= built for path in DEPENDS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    proc = subprocess.run(command(tmp), capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{proc.stdout}\n{proc.stderr}")
    if verbose:
        print(proc.stderr)
    tmp.replace(OUTPUT)
    return OUTPUT


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=True))


if __name__ == "__main__":
    main()
