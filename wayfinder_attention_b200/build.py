"""Build libwayfinder_sm100.so in-tree with nvcc (sm_100a only).

Usage: python -m wayfinder_attention_b200.build [--verbose]

The shared library is written next to this file so that it travels with the
source tree; the Python package loads it from there and refuses to run
without it.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_NAME = "libwayfinder_sm100.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["wf_abi.cu", "wf_topk.cu", "wf_topk_tc.cu", "wf_attn.cu", "wf_attn_bf16.cu", "wf_attn_f16.cu",
           "wf_attn_f32.cu", "wf_addr_proj.cu",
           "wf_attn_bwd.cu", "wf_keymask.cu", "wf_bench.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; set NVCC or put /usr/local/cuda/bin on PATH")
    return cand


def _sources() -> list[Path]:
    return [CSRC / s for s in SOURCES]


def _deps() -> list[Path]:
    return _sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [REPO_DIR / "include" / "wayfinder.h"]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    t = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(verbose: bool = False, force: bool = False) -> Path:
    if not force and up_to_date():
        return LIB_PATH
    nvcc = nvcc_path()
    obj_dir = PKG_DIR / "_build"
    obj_dir.mkdir(exist_ok=True)
    common = [
        "-O3",
        "-std=c++17",
        "-lineinfo",
        "-Xcompiler",
        "-fPIC",
        "-Xcompiler",
        "-fvisibility=hidden",
        "-I",
        str(REPO_DIR / "include"),
        *ARCH_FLAGS,
    ]
    if verbose:
        common += ["-Xptxas", "-v"]
    # translation units compile concurrently (the attention instantiations dominate)
    jobs = []
    for src in _sources():
        obj = obj_dir / (src.stem + ".o")
        cmd = [nvcc, *common, "-c", str(src), "-o", str(obj)]
        jobs.append((src, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
    objs = []
    errors = []
    for src, obj, proc in jobs:
        _, err = proc.communicate()
        if proc.returncode != 0:
            errors.append(f"nvcc failed on {src.name}:\n{err}")
        elif verbose and err:
            sys.stderr.write(err)
        objs.append(str(obj))
    if errors:
        raise RuntimeError("\n".join(errors))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *objs, "-cudart", "static"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose=a.verbose, force=a.force))


if __name__ == "__main__":
    main()
