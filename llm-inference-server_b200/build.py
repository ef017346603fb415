"""Builds the in-tree native libraries of the package with nvcc / g++.

    python llm-inference-server_b200/build.py [--verbose]

Outputs (git-ignored, shipped next to the sources):
    llm-inference-server_b200/lib/libb2decode.so   decode kernels + C-ABI (include/b2_decode.h)
    llm-inference-server_b200/lib/libb2engine.so   GPT-2 decode engine over the C-ABI and cuBLAS
                                                   (include/b2_engine.h)

Every CUDA source is compiled for sm_100a only.  A library is rebuilt when
any of its sources or headers is newer than the .so.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "lib"
INCLUDE = ROOT / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden"]


def _nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build the decode kernels")
    return cand


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str], verbose: bool) -> str:
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout)
        raise RuntimeError(f"build step failed: {' '.join(cmd[:3])} ...")
    return res.stdout


def build_decode(verbose: bool = False, ptxas_info: bool = False) -> Path:
    out = LIB / "libb2decode.so"
    srcs = [CSRC / "b2_decode.cu"]
    deps = srcs + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "b2_decode.h"]
    if _stale(out, deps) or ptxas_info:
        LIB.mkdir(exist_ok=True)
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-shared", "-o", str(out),
               *map(str, srcs)]
        if ptxas_info:
            cmd.insert(1, "-Xptxas=-v")
        log = _run(cmd, verbose)
        if ptxas_info:
            print(log)
    return out


def build_engine(verbose: bool = False) -> Path:
    out = LIB / "libb2engine.so"
    srcs = sorted((CSRC / "engine").glob("*.cu")) + sorted((CSRC / "engine").glob("*.cpp"))
    if not srcs:
        return out
    deps = srcs + sorted((CSRC / "engine").glob("*.h")) + [INCLUDE / "b2_engine.h", INCLUDE / "b2_decode.h",
                                                           LIB / "libb2decode.so"]
    if _stale(out, deps):
        LIB.mkdir(exist_ok=True)
        cmd = [_nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-I", str(CSRC), "-I", str(_json_include()),
               "-shared", "-o", str(out), *map(str, srcs), "-L", str(LIB), "-lb2decode", "-lcublas", "-lcublasLt", "-lnccl",
               "-Xlinker", "-rpath,$ORIGIN"]
        _run(cmd, verbose)
    return out


def _json_include() -> Path:
    """Directory holding nlohmann/json.hpp (header-only; the reference's
    config / manifest parser).  Looked up in the environment: B2_JSON_INCLUDE,
    the system include dirs, then copies vendored by installed Python
    packages."""
    env = os.environ.get("B2_JSON_INCLUDE")
    cands = [Path(env)] if env else []
    cands += [Path("/usr/include"), Path("/usr/local/include")]
    import site
    for sp in site.getsitepackages():
        cands += sorted(Path(sp).glob("include/*/thirdparty"))
        cands += sorted(Path(sp).glob("*/include"))
    for c in cands:
        if (c / "nlohmann" / "json.hpp").exists():
            return c
    raise RuntimeError("nlohmann/json.hpp not found; set B2_JSON_INCLUDE to its include directory")


def build_all(verbose: bool = False) -> list[Path]:
    outs = [build_decode(verbose)]
    if (INCLUDE / "b2_engine.h").exists():
        outs.append(build_engine(verbose))
    return outs


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="rebuild libb2decode with -Xptxas -v")
    args = ap.parse_args()
    if args.ptxas_info:
        build_decode(verbose=args.verbose, ptxas_info=True)
    for p in build_all(args.verbose):
        print(p)
