"""Build the sm_100a shared library behind muzo_clip_b200.

Compiles every ``csrc/*.cu`` and ``csrc/*.cpp`` with nvcc for ``sm_100a`` (nvcc cross-compiles,
no GPU is needed) and links them into ``muzo_clip_b200/libmuzo_b200.so`` next to the Python
package, where ``muzo_clip_b200._lib`` loads it. Objects go to ``_build/`` and are rebuilt only
when a source or header is newer.

Usage: ``python build.py [--force] [--jobs N]``
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
BUILD = HERE / "_build"
OUT = HERE / "muzo_clip_b200" / "libmuzo_b200.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", f"-I{INCLUDE}", f"-I{CSRC}"]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers() -> list[Path]:
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def _compile(src: Path, force: bool) -> Path:
    obj = BUILD / (src.name + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cpp":
        cmd = [NVCC, *COMMON, "-x", "c++", "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not OUT.exists() or OUT.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(OUT), *map(str, objs)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    return OUT


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    args = ap.parse_args()
    out = build(force=args.force, jobs=args.jobs)
    print(out)
    return 0


if __name__ == "__main__":
    sys.exit(main())
