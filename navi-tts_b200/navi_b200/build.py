"""Builds libnavi_b200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

Objects go to navi-tts_b200/_build/, the library next to this file so it travels
with the repository snapshot.  Rebuilds a translation unit only when it or any
header of csrc/ is newer than its object.
"""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = ROOT / "csrc"
OBJ = ROOT / "_build"
LIB = PKG / "libnavi_b200.so"
CLI_SRC = ROOT / "cli" / "navi_b200_cli.cpp"
CLI = PKG / "navi-b200"          # the command-line front (info / synth), linked against LIB
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++20", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "-I", str(CSRC), "-I", str(ROOT.parent / "include")]


def _sources():
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list((ROOT.parent / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, verbose: bool) -> Path:
    obj = OBJ / (src.name + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, _headers_mtime()):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
        cmd += ["--expt-relaxed-constexpr"]
    else:
        cmd = ["g++", "-O2", "-std=c++20", "-fPIC", "-fvisibility=hidden", "-I", str(CSRC), "-I", str(ROOT.parent / "include"),
               "-I", "/usr/local/cuda/include", "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        print(r.stderr, file=sys.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    OBJ.mkdir(exist_ok=True)
    srcs = _sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcuda"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if not CLI.exists() or CLI.stat().st_mtime < max(LIB.stat().st_mtime, CLI_SRC.stat().st_mtime, _headers_mtime()):
        cmd = ["g++", "-O2", "-std=c++20", "-I", str(ROOT.parent / "include"), str(CLI_SRC), "-o", str(CLI), "-L", str(PKG), "-lnavi_b200",
               "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"CLI build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
