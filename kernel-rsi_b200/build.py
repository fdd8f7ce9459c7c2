"""Build the krsi_b200 native libraries in-tree (no JIT cache, no pip install).

  python kernel-rsi_b200/build.py            # build what is stale
  python kernel-rsi_b200/build.py --force    # rebuild everything
  KRSI_PTXAS_VERBOSE=1 python ...            # print ptxas register/smem usage

Outputs (git-ignored, shipped with the tree):
  lib/libkrsi_b200.so  - the C ABI of include/krsi_b200.h: sm_100a kernels, no torch dependency
  lib/_krsi_torch.so   - thin torch binding registering the krsi::* operators
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = PKG / "_build"
LIB = PKG / "lib"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
NVCC = str(CUDA_HOME / "bin" / "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["capi.cu", "diag.cu", "rmsnorm.cu", "geglu.cu", "relpos_attn_fwd.cu", "relpos_attn_bwd.cu", "t5_bias.cu",
              "linear_geglu.cu"]
C_ABI_LIB = LIB / "libkrsi_b200.so"
TORCH_LIB = LIB / "_krsi_torch.so"


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    p = subprocess.run(cmd, capture_output=True, text=True)
    if p.stdout.strip() or p.stderr.strip():
        out = (p.stdout + p.stderr).strip()
        if p.returncode != 0 or os.environ.get("KRSI_PTXAS_VERBOSE"):
            print(out, file=sys.stderr)
    if p.returncode != 0:
        raise RuntimeError(f"build step failed ({p.returncode}): {' '.join(cmd)}")


def _nvcc_obj(src: Path, obj: Path) -> None:
    cmd = [NVCC, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O3",
           "-I", str(INCLUDE), "-I", str(CSRC), "-c", str(src), "-o", str(obj)]
    if os.environ.get("KRSI_PTXAS_VERBOSE"):
        cmd += ["-Xptxas", "-v"]
    _run(cmd)


def build_c_abi(force: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    LIB.mkdir(exist_ok=True)
    headers = _headers()
    objs, jobs = [], []
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        for name in CU_SOURCES:
            src = CSRC / name
            obj = BUILD / (src.stem + ".o")
            objs.append(obj)
            if force or _stale(obj, [src, *headers]):
                jobs.append(ex.submit(_nvcc_obj, src, obj))
        for j in jobs:
            j.result()
    if force or _stale(C_ABI_LIB, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(C_ABI_LIB), *map(str, objs)])
    return C_ABI_LIB


def build_torch_ext(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension as ce

    src = CSRC / "torch_ext.cpp"
    if not (force or _stale(TORCH_LIB, [src, C_ABI_LIB, *_headers()])):
        return TORCH_LIB
    inc = []
    for p in ce.include_paths(device_type="cuda"):
        inc += ["-I", p]
    libdirs = ce.library_paths(device_type="cuda")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cxx = shutil.which("g++") or "g++"
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *inc, "-I", str(INCLUDE), str(src), "-o", str(TORCH_LIB),
           "-L", str(LIB), "-lkrsi_b200", "-Wl,-rpath,$ORIGIN"]
    for d in libdirs:
        cmd += ["-L", d, f"-Wl,-rpath,{d}"]
    cmd += ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch_cuda", "-ltorch", "-lcudart"]
    _run(cmd)
    return TORCH_LIB


def build(force: bool = False) -> None:
    build_c_abi(force)
    build_torch_ext(force)


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--c-abi-only", action="store_true")
    a = ap.parse_args()
    build_c_abi(a.force)
    if not a.c_abi_only:
        build_torch_ext(a.force)
    print(f"built {C_ABI_LIB} and {TORCH_LIB}")
