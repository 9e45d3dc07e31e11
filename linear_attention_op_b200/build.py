"""Build recipe for libgdn_b200.so: every CUDA source compiled for sm_100a with nvcc, linked in-tree.

    python -m linear_attention_op_b200.build [--force] [--jobs N]

The library is placed next to this file (``linear_attention_op_b200/libgdn_b200.so``) so that it travels with
the source tree; object files go to ``linear_attention_op_b200/_build/``.
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
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libgdn_b200.so"
SOURCES = ["gemm.cu", "recurrence.cu", "conv.cu", "chunk_tc.cu", "allreduce.cu", "decoder.cu", "gdn_api.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def nccl_include() -> list[str]:
    """Header of the NCCL that torch ships (the library itself is dlopen'ed at run time)."""
    try:
        import nvidia.nccl  # type: ignore

        for base in list(getattr(nvidia.nccl, "__path__", [])):
            inc = Path(base) / "include"
            if (inc / "nccl.h").exists():
                return ["-I", str(inc)]
    except Exception:
        pass
    for inc in (Path("/usr/include"), Path("/usr/local/cuda/include")):
        if (inc / "nccl.h").exists():
            return ["-I", str(inc)]
    raise RuntimeError("nccl.h not found")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    inc = nccl_include()
    headers = _headers()
    objs = []
    cmds = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (s.stem + ".o")
        objs.append(o)
        if force or _stale(o, [s] + headers):
            cmds.append([cc, *ARCH, *FLAGS, *inc, "-I", str(INCLUDE), "-c", str(s), "-o", str(o)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr)

    if cmds:
        with ThreadPoolExecutor(max_workers=jobs or min(len(cmds), os.cpu_count() or 4)) as ex:
            list(ex.map(run, cmds))
    if force or cmds or _stale(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        run([cc, "-shared", "-rdc=true", *ARCH, *[str(o) for o in objs], "-o", str(tmp), "-ldl"])
        os.replace(tmp, LIB)
    return LIB


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(force=a.force, jobs=a.jobs, verbose=a.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
