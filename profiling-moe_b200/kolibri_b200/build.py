"""Build libkolibri_b200.so (sm_100a) in-tree with nvcc.

The library is a plain C-ABI shared object; nothing here depends on torch.  Objects are
compiled in parallel and relinked only when a source or header is newer than the library.

    python -m kolibri_b200.build          # from the package root (profiling-moe_b200/)
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
ROOT = PKG_DIR.parent                     # profiling-moe_b200/
CSRC = ROOT / "csrc"
INCLUDE = ROOT.parent / "include"
LIB_DIR = PKG_DIR / "lib"
LIB_PATH = LIB_DIR / "libkolibri_b200.so"
BUILD_DIR = ROOT / "_build"

SOURCES = ["capi.cu", "routing.cu", "norms.cu", "qk_norm_rope.cu", "expand.cu", "chain.cu", "finalize.cu", "ep_peer.cu", "router_gemm.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    # No --use_fast_math: expf, sqrtf and division stay IEEE-accurate.
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put /usr/local/cuda/bin on PATH")


def _deps() -> list[Path]:
    return [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    t = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > t for p in _deps())


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose:
        sys.stderr.write(res.stderr)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every source for sm_100a and link libkolibri_b200.so.  Returns its path."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    objs = [BUILD_DIR / (Path(s).stem + ".o") for s in SOURCES]
    with cf.ThreadPoolExecutor(max_workers=min(len(SOURCES), os.cpu_count() or 1)) as ex:
        futs = [ex.submit(_compile, nvcc, CSRC / s, o, verbose) for s, o in zip(SOURCES, objs)]
        for f in futs:
            f.result()
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
           *map(str, objs), "-lcudart_static", "-lrt", "-ldl", "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    p = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(p)
