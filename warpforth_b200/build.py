"""Builds libwfattn (the sm_100a kernels + C ABI) and the wfattn-runner CLI in-tree.

    python -m warpforth_b200.build          # incremental
    python -m warpforth_b200.build --force  # rebuild everything

Outputs (git-ignored, shipped with the source tree):
    warpforth_b200/lib/libwfattn.so
    warpforth_b200/lib/wfattn-runner
    warpforth_b200/lib/wfattn-mma-probe  (tensor-core issue-rate probe behind the kernel design)
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libwfattn.so"
RUNNER = LIB_DIR / "wfattn-runner"
RUNNER_SRC = PKG / "runner" / "wfattn_runner.cpp"
PROBE = LIB_DIR / "wfattn-mma-probe"
PROBE_SRC = CSRC / "mma_rate_probe.cu"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo", *ARCH,
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(ROOT / "include"),
]
SOURCES = ["wfattn_api.cu", "attn_f32.cu", "attn_f32_tc_sm100.cu", "attn_bf16_sm100.cu",
           "attn_bf16_2q_sm100.cu", "decode_sm100.cu", "tma_map.cu"]
HEADERS = ["wfattn_internal.h", "sm100_ptx.cuh", "tma_map.h", "exp2_poly.cuh"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise FileNotFoundError("nvcc not found; libwfattn needs the CUDA 12.9 toolkit")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every CUDA source for sm_100a and link libwfattn.so and the runner."""
    OBJ.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    cc = nvcc()
    headers = [CSRC / h for h in HEADERS] + [ROOT / "include" / "wfattn.h"]
    jobs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = OBJ / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers]):
            extra = ["-Xptxas", "-v"] if ptxas_info else []
            jobs.append([cc, *NVCC_FLAGS, *extra, "-c", str(s), "-o", str(o)])
    if jobs:
        with ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for cmd, res in zip(jobs, ex.map(
                    lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
                if res.returncode != 0:
                    raise RuntimeError(f"nvcc failed: {' '.join(cmd)}\n{res.stdout}\n{res.stderr}")
                if verbose or ptxas_info:
                    print(res.stderr, end="")
    if force or jobs or _stale(LIB, objs):
        _run([cc, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart_static", "-ldl",
              "-lpthread", "-lrt"])
    if RUNNER_SRC.exists() and (force or _stale(RUNNER, [RUNNER_SRC, LIB,
                                                         ROOT / "include" / "wfattn.h"])):
        _run(["g++", "-std=c++17", "-O2", "-Wall", "-I", str(ROOT / "include"),
              "-I", "/usr/local/cuda/include", str(RUNNER_SRC), "-o", str(RUNNER),
              "-L", str(LIB_DIR), "-lwfattn", "-Wl,-rpath,$ORIGIN",
              "-L", "/usr/local/cuda/lib64", "-lcudart", "-Wl,-rpath,/usr/local/cuda/lib64"])
    if PROBE_SRC.exists() and (force or _stale(PROBE, [PROBE_SRC, CSRC / "sm100_ptx.cuh"])):
        _run([cc, "-std=c++17", "-O3", "-lineinfo", *ARCH, "-I", str(CSRC), "-I",
              str(ROOT / "include"), str(PROBE_SRC), "-o", str(PROBE)])
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
