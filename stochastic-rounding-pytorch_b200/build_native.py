"""Build libsrs_b200.so (the sm_100a kernels and their C ABI) in-tree, and the
host helper module _srs_host (C++, CPython API and libtorch headers).

    python stochastic-rounding-pytorch_b200/build_native.py [--force] [--verbose]

Objects go to stochastic-rounding-pytorch_b200/_build/, the shared library to
stochastic-rounding-pytorch_b200/sr_states/_native/libsrs_b200.so.  nvcc
cross-compiles for sm_100a, so the build needs no GPU.  The CUDA runtime is
linked statically; the library needs only the driver at run time.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = REPO / "include"
BUILD = HERE / "_build"
LIBRARY = HERE / "sr_states" / "_native" / "libsrs_b200.so"
# Test-only kernels that check device building blocks (loaded by tests/ only).
SELFTEST = HERE / "sr_states" / "_native" / "libsrs_selftest.so"
# Host helper of the optimizer steps (tensor signatures for the repeated-step check).
HOST = HERE / "sr_states" / "_native" / "_srs_host.so"
HOST_SOURCE = CSRC / "host_signature.cpp"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    # Every FP32 operation of the update is written with an explicit _rn
    # intrinsic; never let the compiler contract anything else into an FMA.
    "-fmad=false",
    "-Xcompiler",
    "-fPIC",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]

# (object name, source, extra defines)
UNITS = [("srs_abi", "srs_abi.cu", []), ("srs_cast", "srs_cast.cu", []),
         ("srs_sgdm", "srs_sgdm.cu", [])]
UNITS += [(f"srs_adamw_m{m}", "srs_adamw.cu", [f"-DSRS_M_FORMAT={m}"]) for m in range(5)]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build")
    return path


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "srs_b200.h"]


def up_to_date() -> bool:
    return _kernels_up_to_date() and _host_up_to_date()


def _kernels_up_to_date() -> bool:
    if not LIBRARY.exists() or not SELFTEST.exists():
        return False
    built = LIBRARY.stat().st_mtime
    return all(src.stat().st_mtime <= built for src in _sources() + [Path(__file__)])


def _host_up_to_date() -> bool:
    return HOST.exists() and HOST.stat().st_mtime >= max(HOST_SOURCE.stat().st_mtime,
                                                         Path(__file__).stat().st_mtime)


def build_host(force: bool = False) -> Path:
    """g++ the _srs_host CPython module against the installed torch (its headers
    for at::Tensor access, its libraries at run time)."""
    if not force and _host_up_to_date():
        return HOST
    import sysconfig

    import torch

    torch_dir = Path(torch.__file__).resolve().parent
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    tmp = HOST.with_suffix(".so.tmp")
    cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           f"-I{sysconfig.get_paths()['include']}", f"-I{torch_dir / 'include'}",
           f"-I{torch_dir / 'include' / 'torch' / 'csrc' / 'api' / 'include'}",
           str(HOST_SOURCE), f"-L{torch_dir / 'lib'}", "-ltorch_python", "-ltorch",
           "-ltorch_cpu", "-lc10", f"-Wl,-rpath,{torch_dir / 'lib'}", "-o", str(tmp)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"g++ failed for {HOST_SOURCE.name}:\n{result.stderr}")
    os.replace(tmp, HOST)
    return HOST


def _compile(unit, verbose: bool) -> str:
    name, source, defines = unit
    out = BUILD / f"{name}.o"
    cmd = [nvcc(), *ARCH, *FLAGS, *defines, "-c", str(CSRC / source), "-o", str(out)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {source} {defines}:\n{result.stderr}")
    return result.stderr


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile and link the library unless it is newer than every source."""
    if not force and not verbose and up_to_date():
        return LIBRARY
    BUILD.mkdir(parents=True, exist_ok=True)
    with ThreadPoolExecutor(1) as host_pool:
        host = host_pool.submit(build_host, force)
        if force or verbose or not _kernels_up_to_date():
            _build_kernels(verbose, jobs)
        host.result()
    return LIBRARY


def _build_kernels(verbose: bool, jobs: int | None) -> None:
    LIBRARY.parent.mkdir(parents=True, exist_ok=True)
    jobs = jobs or min(len(UNITS), os.cpu_count() or 4)
    with ThreadPoolExecutor(jobs) as pool:
        logs = list(pool.map(lambda u: _compile(u, verbose), UNITS))
    if verbose:
        for (name, _, _), log in zip(UNITS, logs):
            print(f"== {name}\n{log}", file=sys.stderr)
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp)]
    cmd += [str(BUILD / f"{name}.o") for name, _, _ in UNITS]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    _link_selftest(verbose)


def _link_selftest(verbose: bool) -> None:
    log = _compile(("srs_selftest", "srs_selftest.cu", []), verbose)
    if verbose:
        print(f"== srs_selftest\n{log}", file=sys.stderr)
    tmp = SELFTEST.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
           str(BUILD / "srs_selftest.o")]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"link failed:\n{result.stderr}")
    os.replace(tmp, SELFTEST)


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))
