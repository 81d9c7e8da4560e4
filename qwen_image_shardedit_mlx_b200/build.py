"""Build libq6b200.so (the C-ABI library) in-tree with nvcc for sm_100a.

    python -m qwen_image_shardedit_mlx_b200.build [--force] [--verbose]

Each .cu under csrc/ is compiled to an object under csrc/_build/ (skipped when
up to date) and the objects are linked into qwen_image_shardedit_mlx_b200/libq6b200.so
with a static CUDA runtime, so the library carries no dependency on a
particular libcudart next to it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = CSRC / "_build"
LIB = PKG / "libq6b200.so"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path("/usr/local/cuda/bin/nvcc")
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def _needs(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    headers = _headers()
    flags = NVCC_FLAGS + (extra_flags or [])
    cmds: list[list[str]] = []
    objs: list[Path] = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or _needs(obj, [src, *headers]):
            cmds.append([nvcc(), *ARCH, *flags, "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)])

    def run(cmd: list[str]) -> None:
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if verbose or res.returncode != 0:
            sys.stdout.write(res.stdout)
            sys.stderr.write(res.stderr)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}")

    if cmds:
        with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 4)) as pool:
            list(pool.map(run, cmds))
    if force or cmds or _needs(LIB, objs):
        link = [nvcc(), *ARCH, "-shared", "-cudart", "static", *[str(o) for o in objs], "-o", str(LIB)]
        run(link)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", "-v", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print register / smem use per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else None
    print(build(force=args.force or args.ptxas_info, verbose=args.verbose or args.ptxas_info, extra_flags=extra))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
