"""In-tree build of the sm_100a library and its compiled-kernel shims.

    python -m kernelcode_generate_b200._build        # build (incremental)
    python -m kernelcode_generate_b200._build clean

Outputs (git-ignored, shipped with the working tree):
    kernelcode_generate_b200/lib/libkg_sm100.so                 all kernels + the C ABI
    kernelcode_generate_b200/lib/libkg_sm100_<kernel>.so        `kg_execute_entry` (+ `_capture`) shims

The CUDA runtime is linked statically so the library depends only on the driver (libcuda).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "lib"
OBJ_DIR = PKG_DIR / "_build"
INCLUDE_DIR = REPO_DIR / "include"

LIB_NAME = "libkg_sm100.so"
SHIMS = {
    "matmul": "kg_sm100_matmul_entry",
    "conv2d": "kg_sm100_conv2d_entry",
    "flash_attention": "kg_sm100_flash_attention_entry",
}
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                           "--expt-relaxed-constexpr", "-I", str(CSRC), "-I", str(INCLUDE_DIR)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE_DIR.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def build(verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ for sm_100a and link the library and shims. Incremental."""
    OBJ_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    headers = _headers()
    compiler = nvcc()
    jobs = []
    objs = []
    for src in _sources():
        obj = OBJ_DIR / (src.stem + ".o")
        objs.append(obj)
        if _stale(obj, [src] + headers):
            jobs.append([compiler, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            list(ex.map(_run, jobs))
    lib = LIB_DIR / LIB_NAME
    if _stale(lib, objs):
        _run([compiler, *ARCH_FLAGS, "-shared", "-cudart", "static", *map(str, objs), "-o", str(lib), "-ldl", "-lpthread", "-lrt"])
    shim_src = CSRC / "kg_entry_shim.cpp"
    for name, target in SHIMS.items():
        shim = LIB_DIR / f"libkg_sm100_{name}.so"
        if _stale(shim, [shim_src, lib, INCLUDE_DIR / "kg_sm100.h"]):
            capture = target.replace("_entry", "_capture")
            _run(["g++", "-std=c++17", "-O2", "-fPIC", "-shared", f"-DKG_SHIM_TARGET={target}", f"-DKG_SHIM_CAPTURE={capture}", str(shim_src),
                  "-L", str(LIB_DIR), "-l:" + LIB_NAME, "-Wl,-rpath,$ORIGIN", "-o", str(shim)])
    if verbose:
        print(f"built {lib}")
    return lib


API_CHECKS_SRC = REPO_DIR / "tests" / "cuda_api" / "api_checks.cu"
API_CHECKS_LIB = REPO_DIR / "tests" / "_build" / "libkg_api_checks.so"


def build_api_checks() -> Path:
    """Compile the device checks of the include/cuda_sm100 operator surface (tests only)."""
    deps = [API_CHECKS_SRC] + sorted((INCLUDE_DIR / "cuda_sm100").glob("*.h"))
    if _stale(API_CHECKS_LIB, deps):
        API_CHECKS_LIB.parent.mkdir(exist_ok=True)
        _run([nvcc(), *ARCH_FLAGS, "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-I", str(INCLUDE_DIR),
              str(API_CHECKS_SRC), "-o", str(API_CHECKS_LIB)])
    return API_CHECKS_LIB


PIPELINE_CHECKS_SRC = REPO_DIR / "tests" / "cuda_api" / "pipeline_checks.cu"
PIPELINE_CHECKS_LIB = REPO_DIR / "tests" / "_build" / "libkg_pipeline_checks.so"


def build_pipeline_checks() -> Path:
    """Compile the device checks of the bounded-wait pipeline primitives (tests only)."""
    deps = [PIPELINE_CHECKS_SRC, CSRC / "kg_ptx.cuh"]
    if _stale(PIPELINE_CHECKS_LIB, deps):
        PIPELINE_CHECKS_LIB.parent.mkdir(exist_ok=True)
        _run([nvcc(), *ARCH_FLAGS, "-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "-cudart", "static", "-I", str(CSRC),
              str(PIPELINE_CHECKS_SRC), "-o", str(PIPELINE_CHECKS_LIB)])
    return PIPELINE_CHECKS_LIB


def clean() -> None:
    shutil.rmtree(OBJ_DIR, ignore_errors=True)
    for p in LIB_DIR.glob("*.so"):
        p.unlink()


if __name__ == "__main__":
    if len(sys.argv) > 1 and sys.argv[1] == "clean":
        clean()
    else:
        build(verbose=True)
