"""Builds the native engine: every CUDA kernel for sm_100a and the C++ host engine, linked into
one in-tree extension, ``furiosa_opt_engine/_native*.so``.

The build is a generated ninja file under ``_build/`` so that a rebuild recompiles only what
changed. ``nvcc`` cross-compiles for sm_100a without a GPU, so the build runs on any host with the
CUDA toolkit. CUDA's runtime is linked statically: the extension needs nothing from the loader
path beyond the driver, which the GPU host provides.

Usage: ``python -m furiosa_opt_models_b200.utils.build [--verbose] [--jobs N]``.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

ROOT = Path(__file__).resolve().parents[2]
CSRC = ROOT / "csrc"
BUILD = ROOT / "_build"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = "-gencode arch=compute_100a,code=sm_100a"


def _pybind_include() -> str:
    import pybind11

    return pybind11.get_include()


def extension_path() -> Path:
    return ROOT / "furiosa_opt_engine" / ("_native" + sysconfig.get_config_var("EXT_SUFFIX"))


def _sources() -> tuple[list[Path], list[Path]]:
    cu = sorted((CSRC / "kernels").glob("*.cu"))
    cc = sorted(p for d in ("engine", "python") for p in (CSRC / d).glob("*.cc"))
    return cu, cc


def _ninja_file(cu: list[Path], cc: list[Path]) -> str:
    nvcc = CUDA_HOME / "bin" / "nvcc"
    inc = f"-I{CSRC} -I{CSRC / 'kernels'} -I{CSRC / 'engine'} -I{CUDA_HOME / 'include'}"
    pyinc = f"-I{sysconfig.get_paths()['include']} -I{_pybind_include()}"
    lines = [
        "ninja_required_version = 1.5",
        f"nvcc = {nvcc}",
        f"cuflags = {ARCH} -O3 -lineinfo -std=c++17 -Xcompiler -fPIC,-fvisibility=hidden "
        f"--expt-relaxed-constexpr -Xptxas -v {inc}",
        f"ccflags = -O2 -g -std=c++17 -fPIC -fvisibility=hidden -Wall -Wno-unused-function "
        f"{inc} {pyinc}",
        f"ldflags = -shared -L{CUDA_HOME / 'lib64'} -lcudart_static -lrt -ldl -lpthread",
        "rule cu",
        "  command = $nvcc $cuflags -c $in -o $out > $out.ptxas.log 2>&1 || "
        "(cat $out.ptxas.log; exit 1)",
        "  description = nvcc $in",
        "rule cc",
        "  command = g++ $ccflags -MMD -MF $out.d -c $in -o $out",
        "  depfile = $out.d",
        "  description = g++ $in",
        "rule link",
        "  command = g++ -o $out $in $ldflags",
        "  description = link $out",
    ]
    objs = []
    headers = sorted((CSRC / "kernels").glob("*.cuh")) + sorted((CSRC / "kernels").glob("*.h"))
    hdeps = " ".join(str(h) for h in headers)
    for src in cu:
        obj = BUILD / "obj" / (src.stem + ".cu.o")
        objs.append(obj)
        lines.append(f"build {obj}: cu {src} | {hdeps}")
    for src in cc:
        obj = BUILD / "obj" / (src.parent.name + "_" + src.stem + ".o")
        objs.append(obj)
        lines.append(f"build {obj}: cc {src}")
    lines.append(f"build {extension_path()}: link {' '.join(str(o) for o in objs)}")
    lines.append(f"default {extension_path()}")
    return "\n".join(lines) + "\n"


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles and links the extension; returns its path. Raises on a failed build."""
    cu, cc = _sources()
    BUILD.mkdir(exist_ok=True)
    (BUILD / "obj").mkdir(exist_ok=True)
    ninja_file = BUILD / "build.ninja"
    text = _ninja_file(cu, cc)
    if not ninja_file.exists() or ninja_file.read_text() != text:
        ninja_file.write_text(text)
    ninja = shutil.which("ninja") or str(Path(sys.executable).parent / "ninja")
    cmd = [ninja, "-C", str(BUILD), "-f", "build.ninja"]
    if jobs:
        cmd += ["-j", str(jobs)]
    if verbose:
        cmd.append("-v")
    result = subprocess.run(cmd, capture_output=not verbose, text=True)
    if result.returncode != 0:
        out = (result.stdout or "") + (result.stderr or "")
        raise RuntimeError(f"native build failed:\n{out[-8000:]}")
    return extension_path()


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--jobs", type=int, default=None)
    args = parser.parse_args()
    print(build(args.verbose, args.jobs))


if __name__ == "__main__":
    main()
